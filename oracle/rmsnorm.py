"""Qwen2RMSNorm forward and backward. TEST INFRASTRUCTURE ONLY.

Restates ``skc_rmsnorm_fwd_kernel`` / ``skc_rmsnorm_bwd_kernel`` (solution/rmsnorm.py:17-45):
y = w * (x * rsqrt(mean(x^2) + eps)); dx = rstd * (g - x * rstd^2 * mean(g * x)), g = dy * w.
Computed in float64 here (tolerance oracle: the reduction order differs between any two
implementations).
"""

from __future__ import annotations

import numpy as np


def forward(x, w, eps: float):
    x = np.asarray(x, dtype=np.float64)
    rstd = 1.0 / np.sqrt((x * x).mean(axis=-1, keepdims=True) + eps)
    return np.asarray(w, dtype=np.float64) * (x * rstd), rstd[..., 0]


def backward(dy, x, w, eps: float):
    x = np.asarray(x, dtype=np.float64)
    rstd = 1.0 / np.sqrt((x * x).mean(axis=-1, keepdims=True) + eps)
    g = np.asarray(dy, dtype=np.float64) * np.asarray(w, dtype=np.float64)
    dot = (g * x).mean(axis=-1, keepdims=True)
    return rstd * (g - x * (rstd * rstd * dot))


def add_forward(residual, delta, w, eps: float):
    """AddRMSNormFn.forward (solution/rmsnorm.py:115-122): h = residual + delta with delta widened
    to fp32 and one fp32 rounding (torch's fp32 + fp16 add), y = norm(h). Returns (h fp32, y, rstd)."""
    h = (np.asarray(residual, dtype=np.float32) + np.asarray(delta).astype(np.float32)).astype(np.float32)
    y, rstd = forward(h, w, eps)
    return h, y, rstd


def add_backward(grad_h, grad_y, residual, delta, w, eps: float):
    """AddRMSNormFn.backward (solution/rmsnorm.py:125-144): h rebuilt from residual + delta, the
    norm's input gradient plus grad_h, returned to the residual (fp64 here) and to delta (in delta's
    dtype)."""
    h = (np.asarray(residual, dtype=np.float32) + np.asarray(delta).astype(np.float32)).astype(np.float32)
    total = np.asarray(grad_h, dtype=np.float64) + backward(grad_y, h, w, eps)
    return total, total.astype(np.float32).astype(np.asarray(delta).dtype)
