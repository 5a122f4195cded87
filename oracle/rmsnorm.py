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
