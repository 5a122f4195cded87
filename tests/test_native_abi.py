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


def test_step_kernels_reject_bad_arguments_before_any_cuda_call(built):
    """The entry points around the block (residual add + norm, SwiGLU, head statistics) check their
    sizes and pointers first; empty inputs are no-ops."""
    lib = _lib.lib()
    # add + norm: null pointers, then a width that is not a multiple of 4
    rc = lib.decik_add_rmsnorm_fwd(None, None, 0, None, 2, None, None, None, 4, 1536, 1e-6, None)
    assert rc == 1 and b"null" in lib.decik_last_error()
    p = ctypes.c_void_p(16)  # never dereferenced: the size check fails first
    rc = lib.decik_add_rmsnorm_fwd(p, p, 0, p, 2, p, p, None, 4, 1538, 1e-6, None)
    assert rc == 1 and b"n_cols" in lib.decik_last_error()
    rc = lib.decik_add_rmsnorm_bwd(p, None, p, p, 1, p, 7, p, p, None, 4, 1536, None)
    assert rc == 1 and b"w_dtype" in lib.decik_last_error()
    # SwiGLU: inter not a multiple of 8, rows narrower than [gate | up]
    rc = lib.decik_swiglu_fwd(p, 24, p, 12, 4, 12, 1, None)
    assert rc == 1 and b"multiple of 8" in lib.decik_last_error()
    rc = lib.decik_swiglu_bwd(p, 16, p, 24, p, 32, 4, 16, 1, None)
    assert rc == 1 and b"ld" in lib.decik_last_error()
    # head statistics: vocabulary not a multiple of 8
    rc = lib.decik_head_stats(p, 1004, p, p, p, p, p, 2, 1002, 1, None)
    assert rc == 1 and b"n_vocab" in lib.decik_last_error()
    # empty inputs
    assert lib.decik_add_rmsnorm_fwd(None, None, 0, None, 2, None, None, None, 0, 1536, 1e-6, None) == 0
    assert lib.decik_swiglu_fwd(None, 0, None, 0, 0, 8960, 1, None) == 0
    assert lib.decik_head_stats(None, 0, None, None, None, None, None, 0, 151936, 1, None) == 0
