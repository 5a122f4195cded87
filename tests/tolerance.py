"""The floating-point parity bar for 16-bit (bf16 / fp16) results against an fp32/fp64 oracle.

Stated bar: relative L2 error <= 5e-3 and max-abs error <= 2e-2, the max-abs taken on the
result normalised by max(1, max|reference|) (attention outputs are O(1); gradients can be
larger, and the absolute bar is applied at unit scale). The relative-L2 denominator is
max(||reference||, 1), so an exactly-zero reference (the query gradient of a one-token row)
is judged by the absolute error.
"""

import numpy as np

REL_L2 = 5e-3
MAX_ABS = 2e-2


def errors(actual, expected):
    a = np.asarray(actual, dtype=np.float64)
    e = np.asarray(expected, dtype=np.float64)
    assert a.shape == e.shape, (a.shape, e.shape)
    diff = a - e
    rel_l2 = float(np.linalg.norm(diff) / max(np.linalg.norm(e), 1.0))
    scale = max(1.0, float(np.abs(e).max()) if e.size else 1.0)
    max_abs = float(np.abs(diff).max() / scale) if e.size else 0.0
    return rel_l2, max_abs


def assert_close16(actual, expected, what="", rel_l2=REL_L2, max_abs=MAX_ABS):
    r, m = errors(actual, expected)
    assert np.isfinite(np.asarray(actual, dtype=np.float64)).all(), f"{what}: non-finite values"
    assert r <= rel_l2 and m <= max_abs, f"{what}: rel-L2 {r:.3e} (<= {rel_l2}), max-abs {m:.3e} (<= {max_abs})"
