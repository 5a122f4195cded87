"""Padding-free packing plan. TEST INFRASTRUCTURE ONLY.

Restates ``plan`` / ``Packing`` (solution/varlen.py:191-226, :23-40): for a right-padded
attention mask [B, S], the real tokens in row-major order (``index``), each token's position in
its row (``positions``), the rows' (start, length) spans in the packed sequence,
``cu_seqlens`` int32 [rows + 1] and ``max_len``. A mask that is not right-padded or has an empty
row gives None (solution/varlen.py:213-217).
"""

from __future__ import annotations

import numpy as np


def plan(attention_mask: np.ndarray):
    mask = np.asarray(attention_mask).astype(bool)
    B, S = mask.shape
    lengths = mask.sum(axis=1)
    steps = np.arange(S)
    if not np.array_equal(mask, steps[None, :] < lengths[:, None]):
        return None
    if lengths.min() == 0:
        return None
    index = np.nonzero(mask.reshape(-1))[0]
    positions = np.broadcast_to(steps, (B, S)).reshape(-1)[index]
    spans, start = [], 0
    for length in lengths.tolist():
        spans.append((start, int(length)))
        start += int(length)
    cu = np.array([s for s, _ in spans] + [start], dtype=np.int32)
    return dict(index=index, positions=positions, spans=spans, cu_seqlens=cu,
                max_len=int(lengths.max()), n_tokens=int(index.size))


def spans_from_lengths(lengths):
    spans, start = [], 0
    for L in lengths:
        spans.append((start, int(L)))
        start += int(L)
    cu = np.array([s for s, _ in spans] + [start], dtype=np.int32)
    return spans, cu


def positions_from_lengths(lengths) -> np.ndarray:
    return np.concatenate([np.arange(int(L)) for L in lengths]).astype(np.int64)
