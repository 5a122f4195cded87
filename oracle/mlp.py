"""The Qwen2 MLP with NF4 projections, forward and backward. TEST INFRASTRUCTURE ONLY.

Restates the reference's MLP node (``RecomputedMLP``, solution/mlp.py:62-110) and its SwiGLU
kernels (solution/swiglu.py:15-37) in numpy:
- x16 = 16-bit(x);
- gate, up = 16-bit(x16 W^T);
- hidden = 16-bit(g * sigmoid(g) * u), computed in fp32;
- out = 16-bit(hidden W_down^T).

The backward computes grad_hidden = 16-bit(g16 W_down), then dgate = grad * u * s * (1 + g (1 - s))
and dup = grad * g * s in fp32, each rounded to 16 bits. The input gradient is
fp32(dgate W_gate) + fp32(dup W_up). Matmuls accumulate in float64 here: the rounding points
match, the accumulation order does not.
"""

from __future__ import annotations

import numpy as np

from .nf4 import dequantize_nf4


def _sigmoid32(x: np.ndarray) -> np.ndarray:
    x = x.astype(np.float32)
    return (np.float32(1.0) / (np.float32(1.0) + np.exp(-x))).astype(np.float32)


def swiglu_fwd(gate, up, dtype=np.float16):
    g = np.asarray(gate).astype(np.float32)
    u = np.asarray(up).astype(np.float32)
    return (g * _sigmoid32(g) * u).astype(np.float32).astype(dtype)


def swiglu_bwd(grad, gate, up, dtype=np.float16):
    gr = np.asarray(grad).astype(np.float32)
    g = np.asarray(gate).astype(np.float32)
    u = np.asarray(up).astype(np.float32)
    s = _sigmoid32(g)
    dup = gr * g * s
    dgate = gr * u * s * (np.float32(1.0) + g * (np.float32(1.0) - s))
    return dgate.astype(np.float32).astype(dtype), dup.astype(np.float32).astype(dtype)


def _mm16(a, b_t, dtype):
    """16-bit(a . b_t^T) with a float64 accumulation."""
    return (np.asarray(a, dtype=np.float64) @ np.asarray(b_t, dtype=np.float64).T).astype(np.float32).astype(dtype)


def mlp_forward(x, states: dict, dtype=np.float16):
    """out (16-bit) and the saved (x16, gate, up) for x [T, H] fp32; states: NF4 state dicts
    gate [I, H], up [I, H], down [H, I] (oracle.nf4 format)."""
    w = {n: dequantize_nf4(st, "f16" if dtype == np.float16 else "f32").astype(np.float32) for n, st in states.items()}
    x16 = np.asarray(x, dtype=np.float32).astype(dtype)
    gate = _mm16(x16, w["gate"], dtype)
    up = _mm16(x16, w["up"], dtype)
    hidden = swiglu_fwd(gate, up, dtype)
    return _mm16(hidden, w["down"], dtype), (x16, gate, up, w)


def mlp_backward(gout, saved, dtype=np.float16):
    """Input gradient (fp32) from the output gradient."""
    _, gate, up, w = saved
    g16 = np.asarray(gout).astype(np.float32).astype(dtype)
    grad_hidden = (np.asarray(g16, np.float64) @ w["down"].astype(np.float64)).astype(np.float32).astype(dtype)
    dgate, dup = swiglu_bwd(grad_hidden, gate, up, dtype)
    a = (np.asarray(dgate, np.float64) @ w["gate"].astype(np.float64)).astype(np.float32).astype(dtype)
    b = (np.asarray(dup, np.float64) @ w["up"].astype(np.float64)).astype(np.float32).astype(dtype)
    return a.astype(np.float32) + b.astype(np.float32)
