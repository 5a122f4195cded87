"""The chunked output head + cross entropy. TEST INFRASTRUCTURE ONLY.

Restates the reference's FusedHeadLoss (solution/head.py:88-139) and its row kernel
(skc_head_stats_kernel, :39-85) in numpy. Per real token the logits are the 16-bit product
h16 . W^T. Then, in float64:
- lse = logsumexp(z) and entropy = lse - sum softmax(z) * z;
- loss = lse - z[target] for a labelled token, 0 for an ignored one (-100);
- hit = (first argmax == target).

The hidden-state gradient is (softmax - onehot), rounded to 16 bits as the reference stores it
over the logits, times W, scaled by 1 / denominator.
"""

from __future__ import annotations

import numpy as np

IGNORE_INDEX = -100


def head_loss(hidden, weight16, targets, denominator):
    """(loss, entropy, token_loss, hit, dhidden) for hidden [T, H] fp32, weight16 [V, H] 16-bit."""
    w = np.asarray(weight16)
    dt = w.dtype
    h16 = np.asarray(hidden, dtype=np.float32).astype(dt)
    z = (h16.astype(np.float64) @ w.astype(np.float64).T).astype(np.float32).astype(dt).astype(np.float64)
    m = z.max(axis=1, keepdims=True)
    e = np.exp(z - m)
    s = e.sum(axis=1, keepdims=True)
    lse = (m + np.log(s))[:, 0]
    p = e / s
    entropy = lse - (p * z).sum(axis=1)
    t = np.asarray(targets)
    labelled = t != IGNORE_INDEX
    tt = np.where(labelled, t, 0)
    token_loss = np.where(labelled, lse - z[np.arange(len(t)), tt], 0.0)
    hit = (labelled & (z.argmax(axis=1) == tt)).astype(np.int32)
    g = p.copy()
    g[np.arange(len(t)), tt] -= 1.0
    g = np.where(labelled[:, None], g, 0.0).astype(np.float32).astype(dt).astype(np.float64)
    dhidden = (g @ w.astype(np.float64)) / float(denominator)
    return token_loss.sum() / float(denominator), entropy, token_loss, hit, dhidden
