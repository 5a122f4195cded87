"""Fused LoRA-add + RoPE, forward and backward, and the cos/sin table. TEST INFRASTRUCTURE ONLY.

Restates ``skc_rope_fwd_kernel`` / ``skc_rope_bwd_kernel`` (solution/attn.py:28-90) in numpy fp32,
where every product and sum is rounded separately (the reference launches with
``enable_fp_fusion=False``, solution/attn.py:107,124):

forward, per token t, head h, dim d (HALF = D/2):
    q[d]   = f32(q_base[d]) + f32(q_lora[d])                            (:39-42)
    rot[d] = -q[d + HALF] if d < HALF else q[d - HALF]                  (:45)
    out[d] = q[d] * cos[t, d] + rot[d] * sin[t, d]                      (:46)
    stored head-major [H, T, D] in the output dtype                      (:47)
k is the same without the LoRA term (:49-60).

backward (token-major out):
    a = g[d] * cos[t, d];  b = g[(d + HALF) % D] * sin[t, (d + HALF) % D]
    dq[d] = a + b if d < HALF else a + (-b)                              (:73-79)

cos/sin: transformers' Qwen2RotaryEmbedding as restated in dev/test_cpu_attn.py:21-24:
``inv = 1 / theta^(arange(0, D, 2) / D)``, ``emb = cat(pos (x) inv, pos (x) inv)``.
"""

from __future__ import annotations

import numpy as np
import torch


def cos_sin(positions, head_dim: int, theta: float = 1e6):
    """fp32 cos, sin [T, head_dim] for integer positions (torch on the CPU, as the reference's
    test builds them)."""
    pos = torch.as_tensor(np.asarray(positions), dtype=torch.float32)
    inv = 1.0 / (theta ** (torch.arange(0, head_dim, 2).float() / head_dim))
    fr = torch.outer(pos, inv)
    emb = torch.cat((fr, fr), -1)
    return emb.cos().numpy(), emb.sin().numpy()


def _rot_fwd(x: np.ndarray, c: np.ndarray, s: np.ndarray) -> np.ndarray:
    """x [T, H, D] fp32 -> rope'd [T, H, D] fp32, each op rounded."""
    half = x.shape[-1] // 2
    rot = np.concatenate([-x[..., half:], x[..., :half]], axis=-1)
    a = (x * c[:, None, :]).astype(np.float32)
    b = (rot * s[:, None, :]).astype(np.float32)
    return (a + b).astype(np.float32)


def rope_fwd(q_base, q_lora, k, cos, sin, n_heads: int, n_kv: int, out_dtype=np.float16):
    """q_base, q_lora [T, Hq*D], k [T, Hk*D] (fp16 or fp32 arrays) -> q [Hq, T, D], k [Hk, T, D]."""
    T = q_base.shape[0]
    D = cos.shape[-1]
    q = (np.asarray(q_base).astype(np.float32) + np.asarray(q_lora).astype(np.float32))
    q = q.astype(np.float32).reshape(T, n_heads, D)
    kk = np.asarray(k).astype(np.float32).reshape(T, n_kv, D)
    c = np.asarray(cos, dtype=np.float32)
    s = np.asarray(sin, dtype=np.float32)
    qo = _rot_fwd(q, c, s).transpose(1, 0, 2)
    ko = _rot_fwd(kk, c, s).transpose(1, 0, 2)
    return _round(qo, out_dtype), _round(ko, out_dtype)


def _rot_bwd(g: np.ndarray, c: np.ndarray, s: np.ndarray) -> np.ndarray:
    """g [T, H, D] fp32 -> input grad [T, H, D] fp32, each op rounded."""
    D = g.shape[-1]
    half = D // 2
    dj = (np.arange(D) + half) % D
    a = (g * c[:, None, :]).astype(np.float32)
    b = (g[..., dj] * s[:, None, dj]).astype(np.float32)
    sign = np.where(np.arange(D) < half, np.float32(1), np.float32(-1)).astype(np.float32)
    return (a + b * sign).astype(np.float32)


def rope_bwd(grad_q, grad_k, cos, sin, out_dtype=np.float16):
    """grad_q [Hq, T, D], grad_k [Hk, T, D] -> dq [T, Hq*D], dk [T, Hk*D]."""
    gq = np.asarray(grad_q).astype(np.float32).transpose(1, 0, 2)
    gk = np.asarray(grad_k).astype(np.float32).transpose(1, 0, 2)
    c = np.asarray(cos, dtype=np.float32)
    s = np.asarray(sin, dtype=np.float32)
    T = gq.shape[0]
    dq = _rot_bwd(gq, c, s).reshape(T, -1)
    dk = _rot_bwd(gk, c, s).reshape(T, -1)
    return _round(dq, out_dtype), _round(dk, out_dtype)


def _round(x: np.ndarray, out_dtype):
    """Round fp32 to the output type; "bf16" returns uint16 bit patterns (round to nearest even)."""
    if out_dtype == "bf16":
        from .nf4 import f32_to_bf16_bits
        return f32_to_bf16_bits(x)
    return x.astype(out_dtype)
