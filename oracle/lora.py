"""LoRA pair of q_proj and v_proj with packed dropout masks. TEST INFRASTRUCTURE ONLY.

Restates solution/attn.py:
- ``keep_pack``:        ``skc_keep_pack_kernel`` (:130-144): bit j of byte c of a row is keep[8c + j];
- ``lora_inputs``:      ``skc_lora_inputs_kernel`` (:154-165): round(x * (keep * scale)) with
                        keep * scale and the product each rounded in fp32;
- ``lora_input_grad``:  ``skc_lora_input_grad_kernel`` (:169-180):
                        (f32(g_q) * keep) * s_q + (f32(g_v) * keep) * s_v in fp32;
- ``pair_forward`` / ``pair_backward``: ``LoRAPairFromNorm`` (:206-273), in fp32 for the
                        tolerance oracle: u = x16 A^T, out = (u B^T) * scaling;
                        g = grad * scaling, dB = g^T u, du = g B, dA = du^T x16, dx = du A
                        through the dropout masks.
"""

from __future__ import annotations

import numpy as np


def keep_pack(keep: np.ndarray) -> np.ndarray:
    """bool/uint8 keep [T, W] (W % 8 == 0) -> uint8 bits [T, W/8]."""
    k = np.asarray(keep).astype(np.uint8).reshape(keep.shape[0], -1, 8)
    weights = (1 << np.arange(8, dtype=np.uint32)).astype(np.uint32)
    return (k.astype(np.uint32) * weights).sum(axis=-1).astype(np.uint8)


def keep_unpack(bits: np.ndarray, width: int) -> np.ndarray:
    b = np.asarray(bits, dtype=np.uint8)
    return ((b[..., None] >> np.arange(8, dtype=np.uint8)) & 1).reshape(b.shape[0], width)


def lora_inputs(x, bits_q, bits_v, scale_q, scale_v, out_dtype=np.float16):
    """x fp32 [T, W] -> (round(x * keep_q * s_q), round(x * keep_v * s_v))."""
    x = np.asarray(x, dtype=np.float32)
    W = x.shape[-1]
    out = []
    for bits, s in ((bits_q, scale_q), (bits_v, scale_v)):
        m = (keep_unpack(bits, W).astype(np.float32) * np.float32(s)).astype(np.float32)
        y = (x * m).astype(np.float32)
        if out_dtype == "bf16":
            from .nf4 import f32_to_bf16_bits
            out.append(f32_to_bf16_bits(y))
        else:
            out.append(y.astype(out_dtype))
    return tuple(out)


def lora_input_grad(g_q, g_v, bits_q, bits_v, scale_q: float, scale_v: float) -> np.ndarray:
    gq = np.asarray(g_q).astype(np.float32)
    gv = np.asarray(g_v).astype(np.float32)
    W = gq.shape[-1]
    kq = keep_unpack(bits_q, W).astype(np.float32)
    kv = keep_unpack(bits_v, W).astype(np.float32)
    tq = ((gq * kq).astype(np.float32) * np.float32(scale_q)).astype(np.float32)
    tv = ((gv * kv).astype(np.float32) * np.float32(scale_v)).astype(np.float32)
    return (tq + tv).astype(np.float32)


def pair_forward(x16, a, b, scaling):
    """One branch in fp32: u = x16 A^T [T, r], out = (u B^T) * scaling [T, N]."""
    x = np.asarray(x16, dtype=np.float64)
    u = x @ np.asarray(a, dtype=np.float64).T
    return u, (u @ np.asarray(b, dtype=np.float64).T) * scaling


def pair_backward(grad, x16, u, a, b, scaling):
    """One branch: returns dA [r, W], dB [N, r], dx16 [T, W] (before the dropout mask)."""
    g = np.asarray(grad, dtype=np.float64) * scaling
    u = np.asarray(u, dtype=np.float64)
    d_b = g.T @ u
    d_u = g @ np.asarray(b, dtype=np.float64)
    d_a = d_u.T @ np.asarray(x16, dtype=np.float64)
    d_x = d_u @ np.asarray(a, dtype=np.float64)
    return d_a, d_b, d_x
