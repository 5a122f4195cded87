"""The whole attention block of the QLoRA step, forward and backward, in torch fp32 on the CPU.

TEST INFRASTRUCTURE ONLY. This is both the tolerance oracle for the block and the reference's
CPU path timed as the baseline (``bench.py --impl reference`` and the ``cpu_baseline`` leg).

It composes, in the reference's order (patched ``Qwen2Attention.forward``,
solution/attn.py:387-418, without o_proj):
1. NF4 double-quant dequant of W_q, W_k, W_v, vectorised in torch following
   solution/nf4.py:36-48 (the bitsandbytes-style CPU dequant);
2. ``F.linear(x, W, b)`` for q, k, v (solution/nf4.py:93-97);
3. LoRA on q and v: ``(dropout(x) A^T) B^T * scaling`` (solution/attn.py:225-228);
4. ``v = v_base + v_lora`` (solution/attn.py:407);
5. RoPE on q = q_base + q_lora and on k (solution/attn.py:39-60);
6. per-row causal GQA attention (``PackedSDPA``, solution/varlen.py:76-121).
Backward is torch autograd over the same graph: dX of the frozen NF4 linears, the LoRA
parameter gradients, and the LoRA input gradient (solution/nf4.py:99-104,
solution/attn.py:235-273).
"""

from __future__ import annotations

import numpy as np
import torch
import torch.nn.functional as F

from .attention import torch_packed_sdpa


def dequant_torch(state: dict) -> torch.Tensor:
    """fp32 [N, K] weights from an NF4 state dict (oracle.nf4.quantize_nf4), torch ops."""
    packed = torch.as_tensor(np.asarray(state["packed"])).to(torch.int64)
    bs = int(state["blocksize"])
    block = (torch.arange(packed.numel(), dtype=torch.int64) * 2) // bs
    if state["nested"]:
        code2 = torch.as_tensor(np.asarray(state["code2"]))
        absmax2 = torch.as_tensor(np.asarray(state["absmax2"]))
        q = torch.as_tensor(np.asarray(state["absmax"])).to(torch.int64)
        scale = code2[q[block]] * absmax2[block // int(state["blocksize2"])]
        scale = scale + float(np.float32(state["offset"]))
    else:
        scale = torch.as_tensor(np.asarray(state["absmax"]))[block]
    code = torch.as_tensor(np.asarray(state["code"]))
    w = torch.stack((code[packed >> 4] * scale, code[packed & 15] * scale), dim=1)
    return w.reshape(state["shape"])


def dequant_torch_qs(packed: torch.Tensor, qs) -> torch.Tensor:
    """fp32 [N, K] weights from packed uint8 bytes and a QuantState-like object (fields absmax,
    code, blocksize, shape, nested, state2.{absmax, code, blocksize}, offset): the arithmetic of
    dequant_torch (solution/nf4.py:36-48: per block scale = code2[absmax] * absmax2, then
    + offset; each weight code[nibble] * scale in fp32, high nibble first), vectorised per byte
    and per block as a CPU dequant would be: a 256-entry table gives each byte's two codes, and one
    scale per block multiplies its bytes."""
    p = packed.reshape(-1).to(torch.int64)
    bs = int(qs.blocksize)
    n_blocks = (p.numel() * 2) // bs
    byte = torch.arange(256, device=p.device)
    pair = torch.stack((qs.code[byte >> 4], qs.code[byte & 15]), dim=1)  # [256, 2]: (hi, lo)
    if qs.nested:
        blk = torch.arange(n_blocks, device=p.device)
        scale = qs.state2.code[qs.absmax.to(torch.int64)] * qs.state2.absmax[blk // int(qs.state2.blocksize)]
        scale = scale + qs.offset.reshape(-1)[0]
    else:
        scale = qs.absmax
    w = pair[p].view(n_blocks, bs // 2, 2) * scale.view(n_blocks, 1, 1)
    return w.reshape(qs.shape)


def rope_torch(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """x [T, H, D] -> x * cos + rotate_half(x) * sin (transformers' apply_rotary_pos_emb)."""
    half = x.shape[-1] // 2
    rot = torch.cat((-x[..., half:], x[..., :half]), dim=-1)
    return x * cos[:, None, :] + rot * sin[:, None, :]


def block_forward(x, w_q, w_k, w_v, b_q, b_k, b_v, a_q, bb_q, a_v, bb_v, scaling, cos, sin,
                  spans, n_heads, n_kv, keep_q=None, keep_v=None, p=0.0):
    """Returns attention output [T, Hq*D] (fp32) for fp32 inputs; differentiable."""
    T = x.shape[0]
    D = cos.shape[-1]
    q_base = F.linear(x, w_q, b_q)
    k = F.linear(x, w_k, b_k)
    v_base = F.linear(x, w_v, b_v)
    xq = x if keep_q is None else x * keep_q * (1.0 / (1.0 - p))
    xv = x if keep_v is None else x * keep_v * (1.0 / (1.0 - p))
    q_lora = F.linear(F.linear(xq, a_q), bb_q) * scaling
    v_lora = F.linear(F.linear(xv, a_v), bb_v) * scaling
    v = v_base + v_lora
    q = rope_torch((q_base + q_lora).view(T, n_heads, D), cos, sin)
    kr = rope_torch(k.view(T, n_kv, D), cos, sin)
    out = torch_packed_sdpa(q.transpose(0, 1)[None], kr.transpose(0, 1)[None],
                            v.view(T, n_kv, D).transpose(0, 1)[None], spans, D ** -0.5)
    return out[0].reshape(T, n_heads * D)


def rmsnorm_torch(h: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    """Qwen2RMSNorm in fp32 (solution/rmsnorm.py:17-28): w * (h * rsqrt(mean(h^2) + eps))."""
    return w * (h * torch.rsqrt(h.pow(2).mean(-1, keepdim=True) + eps))


def block_step(inputs: dict, grad_out: torch.Tensor, weights: dict | None = None):
    """One forward + backward of the block. ``inputs`` holds torch fp32 CPU tensors: x, b_q, b_k,
    b_v, a_q, bb_q, a_v, bb_v, cos, sin and the NF4 states nf4_q/k/v, spans, n_heads, n_kv,
    scaling. Returns (out, dx, dA_q, dB_q, dA_v, dB_v). ``weights`` may carry pre-dequantised
    (w_q, w_k, w_v); otherwise the dequant runs here, as in every reference step. With
    ``inputs["norm_w"]`` (and ``"eps"``) x is the decoder layer's input and the block starts with
    its input RMSNorm; dx is then the gradient for that input."""
    if weights is None:
        w_q, w_k, w_v = (dequant_torch(inputs[n]) for n in ("nf4_q", "nf4_k", "nf4_v"))
    else:
        w_q, w_k, w_v = weights["w_q"], weights["w_k"], weights["w_v"]
    x = inputs["x"].detach().clone().requires_grad_(True)
    params = [inputs[n].detach().clone().requires_grad_(True) for n in ("a_q", "bb_q", "a_v", "bb_v")]
    xn = x if inputs.get("norm_w") is None else rmsnorm_torch(x, inputs["norm_w"], inputs["eps"])
    out = block_forward(xn, w_q, w_k, w_v, inputs["b_q"], inputs["b_k"], inputs["b_v"],
                        params[0], params[1], params[2], params[3], inputs["scaling"],
                        inputs["cos"], inputs["sin"], inputs["spans"], inputs["n_heads"],
                        inputs["n_kv"])
    out.backward(grad_out)
    return (out.detach(), x.grad) + tuple(p.grad for p in params)
