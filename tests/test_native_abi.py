"""The C-ABI library builds for sm_100a, loads, and exports exactly what include/*.h declares.
No kernel is launched here (no GPU needed); argument checks that fail before any CUDA call are
exercised through the ABI."""

import ctypes
import glob
import os
import re

import pytest

from decik_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def header_symbols():
    names = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        text = open(h).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        names.update(re.findall(r"\b(decik_\w+)\s*\(", text))
    return names


@pytest.fixture(scope="module")
def built():
    if not os.path.exists(_lib.LIB_PATH):
        from decik_b200 import build
        build.build()
    return ctypes.CDLL(_lib.LIB_PATH)


def test_header_declares_entry_points():
    names = header_symbols()
    assert {"decik_nf4_dequant", "decik_rope_fwd", "decik_rope_bwd", "decik_varlen_attn_fwd",
            "decik_varlen_attn_bwd", "decik_lora_inputs"} <= names


def test_library_exports_every_header_symbol(built):
    for name in header_symbols():
        assert hasattr(built, name), f"{name} declared in include/ but not exported"


def test_bindings_cover_header():
    assert set(_lib.SIGNATURES) == header_symbols()


def test_abi_version_and_error_reporting(built):
    lib = _lib.lib()
    assert lib.decik_abi_version() == 1
    rc = lib.decik_nf4_dequant(None, None, None, None, None, None, None, 16, 1, 64, 256, 0, None)
    assert rc == 1 and b"null" in lib.decik_last_error()
    rc = lib.decik_rope_fwd(None, None, None, None, None, None, None, 4, 12, 2, 100, 0, None)
    assert rc == 1 and b"bad sizes" in lib.decik_last_error()
    T3 = _lib.Tensor3
    z = T3(None, 0, 0)
    rc = lib.decik_varlen_attn_fwd(z, z, z, z, None, None, 1, 4, 4, 12, 2, 64, 0.1, 1, None)
    assert rc == 3 and b"head_dim" in lib.decik_last_error()
    rc = lib.decik_varlen_attn_fwd(z, z, z, z, None, None, 1, 4, 4, 12, 2, 128, 0.1, 1, None)
    assert rc == 1 and b"aligned" in lib.decik_last_error()


def test_empty_inputs_are_no_ops(built):
    lib = _lib.lib()
    assert lib.decik_nf4_dequant(None, None, None, None, None, None, None, 0, 1, 64, 256, 0, None) == 0
    assert lib.decik_rope_fwd(None, None, None, None, None, None, None, 0, 12, 2, 128, 0, None) == 0


def test_workspace_size():
    lib = _lib.lib()
    n = lib.decik_varlen_attn_bwd_workspace(1000, 12, 128)
    assert n >= 1000 * 12 * 128 * 4 + 1000 * 12 * 4 and n % 256 == 0
