"""Packed (padding-free) causal GQA attention over varlen rows. TEST INFRASTRUCTURE ONLY.

Restates ``PackedSDPA`` / ``_row_attention`` (solution/varlen.py:76-121): every row
(start, length) of the packed sequence attends causally (top-left aligned, key j <= query i)
to its own tokens only; query head h reads kv head h // groups (repeat_interleave,
solution/varlen.py:78-80). ``VarlenSDPA`` (solution/varlen.py:134-168) computes the same with
cu_seqlens; its backward sums each kv head's query heads (:165-167), which the GQA backward here
does too.

Two forms:
- ``forward`` / ``backward``: float64 numpy, the tolerance oracle; also returns the natural-log
  logsumexp [Hq, T] of the scaled, masked scores (the reference never exposes it on the CPU).
- ``torch_packed_sdpa``: the reference's own CPU path in torch fp32 (per-row
  ``F.scaled_dot_product_attention`` under autograd), used as the timed CPU baseline.

Layouts (token-major): q [T, Hq, D], k, v [T, Hk, D], out [T, Hq, D], lse [Hq, T].
"""

from __future__ import annotations

import numpy as np


def forward(q, k, v, spans, scale: float):
    q = np.asarray(q, dtype=np.float64)
    k = np.asarray(k, dtype=np.float64)
    v = np.asarray(v, dtype=np.float64)
    T, Hq, D = q.shape
    Hk = k.shape[1]
    g = Hq // Hk
    out = np.zeros((T, Hq, D))
    lse = np.zeros((Hq, T))
    for start, L in spans:
        if L == 0:
            continue
        sl = slice(start, start + L)
        causal = np.tril(np.ones((L, L), dtype=bool))
        for h in range(Hq):
            s = (q[sl, h] @ k[sl, h // g].T) * scale
            s = np.where(causal, s, -np.inf)
            m = s.max(axis=1, keepdims=True)
            p = np.exp(s - m)
            l = p.sum(axis=1, keepdims=True)
            out[sl, h] = (p / l) @ v[sl, h // g]
            lse[h, sl] = (m + np.log(l))[:, 0]
    return out, lse


def backward(dout, q, k, v, spans, scale: float):
    """Returns dq [T, Hq, D], dk, dv [T, Hk, D] (kv grads summed over each group's q heads)."""
    q = np.asarray(q, dtype=np.float64)
    k = np.asarray(k, dtype=np.float64)
    v = np.asarray(v, dtype=np.float64)
    do = np.asarray(dout, dtype=np.float64)
    T, Hq, D = q.shape
    Hk = k.shape[1]
    g = Hq // Hk
    dq = np.zeros_like(q)
    dk = np.zeros_like(k)
    dv = np.zeros_like(v)
    for start, L in spans:
        if L == 0:
            continue
        sl = slice(start, start + L)
        causal = np.tril(np.ones((L, L), dtype=bool))
        for h in range(Hq):
            kh, vh = k[sl, h // g], v[sl, h // g]
            s = np.where(causal, (q[sl, h] @ kh.T) * scale, -np.inf)
            p = np.exp(s - s.max(axis=1, keepdims=True))
            p /= p.sum(axis=1, keepdims=True)
            o = p @ vh
            dv[sl, h // g] += p.T @ do[sl, h]
            dp = do[sl, h] @ vh.T
            delta = (do[sl, h] * o).sum(axis=1, keepdims=True)
            ds = p * (dp - delta)
            dq[sl, h] = (ds @ kh) * scale
            dk[sl, h // g] += (ds.T @ q[sl, h]) * scale
    return dq, dk, dv


def torch_packed_sdpa(q, k, v, spans, scale: float):
    """The reference's CPU path: per-row causal SDPA, GQA by repeat_interleave (solution/varlen.py
    :76-82). Inputs torch [1, H, T, D] head-major (q), k/v [1, Hk, T, D]; returns [1, T, Hq, D].
    Differentiable (autograd), as PackedSDPA's backward re-runs the row under autograd (:106-121)."""
    import torch
    import torch.nn.functional as F

    groups = q.shape[1] // k.shape[1]
    outs = []
    for start, length in spans:
        rows = slice(start, start + length)
        kk = k[:, :, rows].repeat_interleave(groups, dim=1)
        vv = v[:, :, rows].repeat_interleave(groups, dim=1)
        outs.append(F.scaled_dot_product_attention(q[:, :, rows], kk, vv, dropout_p=0.0,
                                                   scale=scale, is_causal=True))
    return torch.cat(outs, dim=2).transpose(1, 2)


def causal_flops(spans, n_heads: int, head_dim: int) -> float:
    """Algorithmic forward FLOPs 4 * D * Hq * sum L(L+1)/2 (QK^T and PV over causal pairs)."""
    pairs = sum(L * (L + 1) // 2 for _, L in spans)
    return 4.0 * head_dim * n_heads * pairs
