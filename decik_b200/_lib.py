"""ctypes binding of the C ABI in ``include/decik_b200.h`` (``lib/libdecik_b200.so``).

There is no fallback: if the library is missing or a call fails, a RuntimeError says why.
"""

from __future__ import annotations

import ctypes
import os
import threading

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "lib", "libdecik_b200.so")

F16, BF16, F32 = 0, 1, 2

c_void_p, c_int, c_int64, c_float = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_float


class Nf4Job(ctypes.Structure):
    """decik_nf4_job of include/decik_b200.h."""
    _fields_ = [("packed", ctypes.c_void_p), ("absmax", ctypes.c_void_p), ("absmax2", ctypes.c_void_p),
                ("code2", ctypes.c_void_p), ("offset", ctypes.c_void_p), ("code", ctypes.c_void_p),
                ("out", ctypes.c_void_p), ("n_bytes", ctypes.c_int64), ("nested", ctypes.c_int),
                ("blocksize", ctypes.c_int), ("blocksize2", ctypes.c_int)]


class Tensor3(ctypes.Structure):
    """decik_tensor3 / decik_tensor3_mut: (pointer, token stride, head stride), strides in elements."""
    _fields_ = [("ptr", c_void_p), ("tok_stride", c_int64), ("head_stride", c_int64)]


# name -> (restype, argtypes); the exact set of symbols include/decik_b200.h declares
SIGNATURES = {
    "decik_last_error": (ctypes.c_char_p, []),
    "decik_abi_version": (c_int, []),
    "decik_kernel_error": (c_int, [c_int]),
    "decik_wait_limit_selftest": (c_int, [ctypes.c_longlong, c_void_p, c_void_p]),
    "decik_lora_b_ext": (c_int, [c_void_p, c_void_p, c_float, c_void_p, c_void_p, c_int, c_int, c_int, c_void_p]),
    "decik_qkv_proj_fwd": (c_int, [c_void_p, c_int64, c_void_p, c_int64, c_void_p, c_int, c_void_p, c_void_p,
                                   Tensor3, Tensor3, Tensor3, c_void_p, c_int64, c_void_p, c_int64, c_int, c_int,
                                   c_int, c_int, c_int, c_void_p]),
    "decik_qkv_proj_norm_fwd": (c_int, [c_void_p, c_int64, c_void_p, c_int, c_float, c_void_p, c_void_p, c_int64,
                                        c_void_p, c_int, c_void_p, c_void_p, Tensor3, Tensor3, Tensor3, c_void_p,
                                        c_int64, c_void_p, c_int64, c_int, c_int, c_int, c_int, c_int, c_void_p]),
    "decik_proj_dx": (c_int, [c_void_p, c_int64, c_int, c_void_p, c_int64, c_void_p, c_int64, c_int64, c_int, c_int,
                              c_void_p]),
    "decik_lora_grads": (c_int, [c_void_p, c_int64, c_void_p, c_int64, c_void_p, c_int64, c_void_p, c_void_p,
                                 c_float, c_int64, c_int, c_int, c_int, c_int, c_void_p]),
    "decik_transpose16": (c_int, [c_void_p, c_int64, c_void_p, c_int64, c_int64, c_int64, c_void_p]),
    "decik_gemm16": (c_int, [c_void_p, c_int64, c_void_p, c_int64, c_int, c_void_p, c_int64, c_int64, c_int, c_int,
                             c_int, c_void_p]),
    "decik_mlp_gate_up": (c_int, [c_void_p, c_int64, c_void_p, c_int64, c_void_p, c_int64, c_void_p, c_int64,
                                  c_int64, c_int, c_int, c_int, c_void_p]),
    "decik_mlp_down_grad": (c_int, [c_void_p, c_int64, c_void_p, c_int64, c_void_p, c_int64, c_void_p, c_int64,
                                    c_int64, c_int, c_int, c_int, c_void_p]),
    "decik_pack_rows": (c_int, [c_void_p, c_int, c_void_p, c_int64, c_int64, c_void_p, c_void_p, c_void_p,
                                c_void_p, c_void_p, c_void_p]),
    "decik_nf4_dequant_batch": (c_int, [c_void_p, c_int, c_int, c_void_p]),
    "decik_nf4_dequant": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                  c_int64, c_int, c_int, c_int, c_int, c_void_p]),
    "decik_rope_fwd": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                               c_int64, c_int, c_int, c_int, c_int, c_void_p]),
    "decik_rope_bwd": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int64,
                               c_int, c_int, c_int, c_int, c_void_p]),
    "decik_keep_pack": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int, c_void_p]),
    "decik_lora_inputs": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                  c_int64, c_int, c_int, c_void_p]),
    "decik_lora_input_grad": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int,
                                      c_float, c_float, c_int, c_void_p]),
    "decik_rmsnorm_fwd": (c_int, [c_void_p, c_void_p, c_int, c_void_p, c_void_p, c_int64, c_int, c_int64,
                                  c_int64, c_float, c_void_p]),
    "decik_rmsnorm_bwd": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_void_p, c_void_p, c_int64, c_int,
                                  c_void_p]),
    "decik_rmsnorm_bwd_add": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_void_p, c_void_p, c_void_p, c_int64,
                                      c_int, c_void_p]),
    "decik_add_rmsnorm_fwd": (c_int, [c_void_p, c_void_p, c_int, c_void_p, c_int, c_void_p, c_void_p, c_void_p,
                                      c_int64, c_int, c_float, c_void_p]),
    "decik_add_rmsnorm_bwd": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_void_p, c_int, c_void_p,
                                      c_void_p, c_void_p, c_int64, c_int, c_void_p]),
    "decik_add_rmsnorm_fwd16": (c_int, [c_void_p, c_void_p, c_int, c_void_p, c_int, c_void_p, c_void_p, c_void_p,
                                        c_int64, c_int, c_float, c_void_p]),
    "decik_add_rmsnorm_bwd16": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_void_p, c_int, c_void_p,
                                        c_void_p, c_void_p, c_int64, c_int, c_void_p]),
    "decik_swiglu_fwd": (c_int, [c_void_p, c_int64, c_void_p, c_int64, c_int64, c_int, c_int, c_void_p]),
    "decik_swiglu_bwd": (c_int, [c_void_p, c_int64, c_void_p, c_int64, c_void_p, c_int64, c_int64, c_int, c_int,
                                 c_void_p]),
    "decik_head_stats": (c_int, [c_void_p, c_int64, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int64,
                                 c_int, c_int, c_void_p]),
    "decik_varlen_attn_fwd": (c_int, [Tensor3, Tensor3, Tensor3, Tensor3, c_void_p, c_void_p, c_int, c_int,
                                      c_int64, c_int, c_int, c_int, c_float, c_int, c_void_p]),
    "decik_varlen_attn_bwd_workspace": (c_int64, [c_int64, c_int, c_int]),
    "decik_lora_frag_bytes": (c_int64, [c_int, c_int]),
    "decik_lora_pack": (c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_int, c_void_p, c_void_p, c_void_p,
                                c_int, c_int, c_int, c_int, c_int, c_void_p]),
    "decik_qkv_epilogue_fwd": (c_int, [c_void_p, c_int64, c_void_p, c_int64, c_void_p, c_float, c_void_p,
                                       c_void_p, Tensor3, Tensor3, Tensor3, c_void_p, c_int64, c_int, c_int,
                                       c_int, c_int, c_void_p]),
    "decik_qkv_epilogue_bwd": (c_int, [Tensor3, Tensor3, c_void_p, c_void_p, c_void_p, c_float, c_void_p,
                                       c_int64, c_int64, c_int, c_int, c_int, c_int, c_void_p]),
    "decik_varlen_attn_bwd": (c_int, [Tensor3, Tensor3, Tensor3, Tensor3, Tensor3, c_void_p, Tensor3, Tensor3,
                                      Tensor3, c_void_p, c_int, c_int, c_int64, c_int, c_int, c_int, c_float,
                                      c_int, c_void_p, c_void_p]),
    "decik_attn_qkv_bwd_workspace": (c_int64, [c_int64, c_int, c_int, c_int]),
    "decik_set_stage_events": (None, [c_void_p, c_int]),
    "decik_attn_qkv_bwd": (c_int, [Tensor3, Tensor3, Tensor3, Tensor3, Tensor3, c_void_p, c_void_p, c_int, c_int,
                                   c_int64, c_int, c_int, c_int, c_float, c_void_p, c_void_p, c_void_p, c_float,
                                   c_void_p, c_int64, c_int, c_void_p, c_void_p]),
    "decik_varlen_attn_bwd_noalloc": (c_int, [Tensor3, Tensor3, Tensor3, Tensor3, Tensor3, c_void_p, Tensor3,
                                              Tensor3, Tensor3, c_void_p, c_int, c_int, c_int64, c_int, c_int, c_int,
                                              c_float, c_int, c_void_p]),
}

_lib = None
_lock = threading.Lock()


def lib() -> ctypes.CDLL:
    """The loaded library (loads it on first use)."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not os.path.exists(LIB_PATH):
                    raise RuntimeError(
                        f"decik_b200: native library {LIB_PATH} is not built; run "
                        "`python -m decik_b200.build`. There is no CPU or PyTorch fallback.")
                handle = ctypes.CDLL(LIB_PATH)
                for name, (res, args) in SIGNATURES.items():
                    fn = getattr(handle, name)
                    fn.restype = res
                    fn.argtypes = args
                _lib = handle
    return _lib


def check(rc: int, what: str) -> None:
    if rc != 0:
        msg = lib().decik_last_error().decode(errors="replace")
        raise RuntimeError(f"decik_b200 {what} failed (status {rc}): {msg}")
