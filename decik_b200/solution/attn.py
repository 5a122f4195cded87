"""Attention inputs and the patched Qwen2Attention.forward on the sm_100a kernels (solution/attn.py).

Keeps the reference's autograd Functions and their arguments:
- ``FusedQKRope`` (solution/attn.py:93-126): q = base + LoRA, RoPE, head-major cast; backward is
  the exact transpose, returned to both the projection and the LoRA branch;
- ``pack_keep`` / ``_lora_inputs`` / ``LoRAPairFromNorm`` (solution/attn.py:183-273): peft's
  q and v LoRA branches with bit-packed dropout masks and the input rebuilt from the norm's input;
- ``patch`` (solution/attn.py:349-421): the padding-free attention forward (q, k, v through the
  NF4 linears, LoRA, RoPE, varlen attention, o_proj).
The element-wise kernels are the bit-exact sm_100a ones in ``decik_b200.ops``.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

from .. import ops
from . import rmsnorm
from ._state import STATE, on_gpu

# keyword under which the patched decoder layer hands its input RMSNorm to the patched attention
INPUT_NORM_KW = "decik_input_norm"
RESIDUAL_LINK_KW = "decik_residual_link"


class FusedQKRope(torch.autograd.Function):
    """(q_base + q_lora, k) -> RoPE'd q [1, HQ, T, D] and k [1, HK, T, D] (solution/attn.py:93-126)."""

    @staticmethod
    def forward(ctx, q_base, q_lora, k, cos, sin, n_heads, n_kv_heads):
        q_out, k_out = ops.rope_fwd(q_base, q_lora, k, cos, sin, n_heads, n_kv_heads)
        ctx.save_for_backward(cos, sin)
        return q_out.unsqueeze(0), k_out.unsqueeze(0)

    @staticmethod
    def backward(ctx, grad_q, grad_k):
        cos, sin = ctx.saved_tensors
        dq, dk = ops.rope_bwd(grad_q[0], grad_k[0], cos, sin)
        # the projection and the LoRA branch both receive round(dq) in the base
        return dq, dq.clone(), dk, None, None, None, None


class FusedAttentionBlock(torch.autograd.Function):
    """x -> packed causal GQA attention output [T, Hq, D] in one autograd node, for q/v LoRA
    without dropout. The arithmetic of the reference's chain (solution/attn.py:395-416: three
    NF4Linear, LoRAPairFromNorm, FusedQKRope, VarlenSDPA), regrouped so each pass over the tokens
    does as much as it can:

    forward   decik_qkv_proj_fwd: x16 = dt(x) and u = [x16 [A_q; A_v]^T | 1] in one pass, then one
              tcgen05 GEMM [x16 | u] [W_q; W_k; W_v | scaling B, bias]^T (the LoRA-up and the bias
              are one more K block) whose epilogue applies RoPE and writes head-major q / k and
              v (the projection never reaches HBM); decik_varlen_attn_fwd.
    backward  decik_attn_qkv_bwd (attention backward, RoPE^T, du) into dy; decik_proj_dx:
              dX = dy . W_cat (one tcgen05 GEMM, fp32 out: the three NF4Linear input gradients and
              both LoRA input gradients); decik_lora_grads: dA = du^T x16, dB = scaling . g^T u.

    ``w_cat`` [(Hq+2Hk)*D + 2r, H] holds this step's dequantised W_q, W_k, W_v in its first rows;
    decik_lora_pack writes A_q, A_v (as dt) into the last 2r rows and the lora_B fragments of both
    epilogues in the same launch. The matrix is kept for backward, where the reference dequantises
    again (solution/nf4.py:99-104).

    With ``w_o`` (the dequantised NF4 o_proj weight [H, Hq*D], optional bias ``b_o``) the node
    also applies o_proj (solution/attn.py:418) and returns [T, H]: the same F.linear the
    reference's NF4Linear runs, with the weight kept for backward instead of dequantised again.

    With ``norm_w`` (the decoder layer's input RMSNorm weight, ``norm_eps`` its epsilon) ``x`` is
    the layer input h and the norm runs inside the forward's first kernel
    (decik_qkv_proj_norm_fwd: the norm's fp32 output is never written); the backward applies the
    norm's backward (decik_rmsnorm_bwd, from the kept rstd) to dX and returns the gradient for h.
    The LoRA gradients use the kept x16, so there is no norm recompute (solution/attn.py:238).
    With ``residual_link`` (rmsnorm.ResidualGradLink, armed here) h's gradient from the residual
    stream, left there by the layer's AddRMSNormFn, is added in the same pass."""

    @staticmethod
    def forward(ctx, x, a_q, b_q, a_v, b_v, w_cat, bias_cat, cos, sin, cu_seqlens, max_len, n_heads,
                n_kv, scaling, scale, w_o=None, b_o=None, norm_w=None, norm_eps=0.0, residual_link=None):
        dt = w_cat.dtype
        ctx.link = residual_link if norm_w is not None else None
        if ctx.link is not None:
            ctx.link.armed = True
        D = cos.shape[-1]
        r = a_q.shape[0]
        n_proj = (n_heads + 2 * n_kv) * D
        frag = ops.lora_pack(a_q, a_v, b_q, b_v, dt, a_out=w_cat[n_proj:])
        ext_b = ops.lora_b_ext(b_q, b_v, scaling, bias_cat, dt, n_heads, n_kv)  # scaled lora_B + bias
        x32 = x if (x.dtype == torch.float32 and x.stride(-1) == 1) else x.float().contiguous()
        if norm_w is None:
            x16, u, q, k, v = ops.qkv_proj_fwd(x32, w_cat, ext_b, True, cos, sin, n_heads, n_kv)
            h = rstd = None
        else:
            x16, u, q, k, v, rstd = ops.qkv_proj_fwd(x32, w_cat, ext_b, True, cos, sin, n_heads, n_kv,
                                                     norm=(norm_w, norm_eps))
            h = x32
        out, lse = ops.varlen_attn_fwd(q.transpose(0, 1), k.transpose(0, 1), v, cu_seqlens, max_len, scale)
        ctx.save_for_backward(x16, w_cat, u, frag, cos, sin, q, k, v, out, lse, cu_seqlens, w_o, h, norm_w, rstd)
        ctx.meta = (int(max_len), n_heads, n_kv, float(scaling), float(scale), r)
        if w_o is not None:
            return F.linear(out.view(out.shape[0], -1), w_o, b_o)
        return out

    @staticmethod
    def backward(ctx, grad_out):
        x16, w_cat, u, frag, cos, sin, q, k, v, out, lse, cu, w_o, h, norm_w, rstd = ctx.saved_tensors
        max_len, n_heads, n_kv, scaling, scale, r = ctx.meta
        if w_o is not None:  # through o_proj first: the attention output's gradient
            grad_out = torch.mm(grad_out.reshape(-1, grad_out.shape[-1]).to(w_o.dtype), w_o).view(out.shape)
        T, D = x16.shape[0], cos.shape[-1]
        n_q, n_kvd = n_heads * D, n_kv * D
        n_proj = n_q + 2 * n_kvd
        dt = x16.dtype
        dy = torch.empty((T, n_proj + 2 * r), dtype=dt, device=x16.device)
        g = grad_out if grad_out.stride(-1) == 1 else grad_out.contiguous()
        # attention backward + RoPE^T + du in one call; dq / dk / dv never exist in 16 bits apart
        # from their place in dy
        ops.attn_qkv_bwd(g, q.transpose(0, 1), k.transpose(0, 1), v, out, lse, cu, max_len, scale, cos, sin,
                         frag, scaling, dy)
        dx = ops.proj_dx(dy, ops.transpose16(w_cat))
        da, db = ops.lora_grads(dy, x16, u, scaling, n_heads, n_kv)
        if norm_w is not None:  # through the input norm: the gradient for the layer input h
            dx = ops.rmsnorm_bwd(dx, h, norm_w, rstd, addend=None if ctx.link is None else ctx.link.take())
        return (dx, da[:r], db[:n_q], da[r:], db[n_q:]) + (None,) * 15


def pack_keep(keep_q, keep_v):
    """Two bool keep-masks [T, W] (W % 8 == 0) -> bit-packed uint8 [T, W / 8] each."""
    return ops.keep_pack(keep_q, keep_v)


def _lora_inputs(x, bits_q, bits_v, scale_q, scale_v, dtype=torch.float16):
    """round(x * dropout values) of the q and v branches, [T, W] each."""
    return ops.lora_inputs(x, bits_q, bits_v, scale_q, scale_v, out_dtype=dtype)


class LoRAPairFromNorm(torch.autograd.Function):
    """peft's LoRA branches of q_proj and v_proj, lora_B(lora_A(dropout(x))) * scaling under 16-bit
    autocast, for x = the output of the RMSNorm (solution/attn.py:206-273). Only the bit-packed
    masks are kept; backward rebuilds the 16-bit inputs from the norm's input with the same norm
    kernel. ``dtype`` is the autocast dtype (fp16 as in the reference, or bf16)."""

    @staticmethod
    def forward(ctx, x, h, norm_weight, eps, scaled_q, mask_q, scale_q, scaled_v, mask_v, scale_v,
                a_q, b_q, a_v, b_v, scaling_q, scaling_v, p_q, p_v, packed, dtype=torch.float16):
        if packed:
            inputs = tuple(t.view(x.shape) for t in _lora_inputs(x, mask_q, mask_v, scale_q, scale_v, dtype))
        else:
            inputs = tuple((x * scaled if scaled is not None else x).to(dtype)
                           for scaled in (scaled_q, scaled_v))
        outs, us = [], []
        for x16, a, b, scaling in zip(inputs, (a_q, a_v), (b_q, b_v), (scaling_q, scaling_v)):
            u = F.linear(x16, a.to(dtype))
            outs.append(F.linear(u, b.to(dtype)) * scaling)
            us.append(u)
        ctx.save_for_backward(h, norm_weight, mask_q, scale_q, mask_v, scale_v, us[0], us[1],
                              a_q, b_q, a_v, b_v)
        ctx.eps, ctx.scalings, ctx.ps, ctx.packed, ctx.dtype = eps, (scaling_q, scaling_v), (p_q, p_v), packed, dtype
        return outs[0], outs[1]

    @staticmethod
    def backward(ctx, grad_q, grad_v):
        h, norm_weight, mask_q, scale_q, mask_v, scale_v, u_q, u_v, a_q, b_q, a_v, b_v = ctx.saved_tensors
        dtype = ctx.dtype
        x = rmsnorm.recompute(h, norm_weight, ctx.eps)
        width = x.shape[-1]
        n_rows = x.numel() // width
        if ctx.packed:
            inputs = _lora_inputs(x, mask_q, mask_v, scale_q, scale_v, dtype)
        else:
            inputs = tuple((x * (m * s) if m is not None else x).to(dtype).reshape(-1, width)
                           for m, s in ((mask_q, scale_q), (mask_v, scale_v)))
        grads, input_grads = [], []
        branches = ((grad_q, u_q, a_q, b_q, ctx.scalings[0]), (grad_v, u_v, a_v, b_v, ctx.scalings[1]))
        for (grad, u, a, b, scaling), x16 in zip(branches, inputs):
            if grad is None:
                grad = torch.zeros(u.shape[:-1] + (b.shape[0],), dtype=dtype, device=u.device)
            g = (grad * scaling).reshape(-1, grad.shape[-1]).to(dtype)
            u2 = u.reshape(-1, u.shape[-1])
            grad_b = g.t().mm(u2)
            grad_u = g.mm(b.to(dtype))
            grads += [grad_u.t().mm(x16).to(torch.float32), grad_b.to(torch.float32)]
            input_grads.append(grad_u.mm(a.to(dtype)))
        if ctx.packed:
            grad_x = ops.lora_input_grad(input_grads[0], input_grads[1], mask_q, mask_v,
                                         1.0 / (1.0 - ctx.ps[0]), 1.0 / (1.0 - ctx.ps[1]))
        else:
            grad_x = None
            for gx16, m, p in zip(input_grads, (mask_q, mask_v), ctx.ps):
                gx = gx16.to(torch.float32)
                if m is not None:
                    gx = gx * m.reshape(-1, width) * (1.0 / (1.0 - p))
                grad_x = gx if grad_x is None else grad_x + gx
        return (grad_x.view(x.shape), None, None, None, None, None, None, None, None, None,
                grads[0], grads[1], grads[2], grads[3], None, None, None, None, None, None)


def _lora_parts(layer, name):
    """(lora_A weight, lora_B weight, scaling, dropout p) of a plain LoRA branch, else None
    (solution/attn.py:276-297)."""
    try:
        lora_a, lora_b = layer.lora_A[name], layer.lora_B[name]
        dropout, scaling = layer.lora_dropout[name], layer.scaling[name]
    except (AttributeError, KeyError, TypeError):
        return None
    if not (type(lora_a) is torch.nn.Linear and type(lora_b) is torch.nn.Linear
            and lora_a.bias is None and lora_b.bias is None
            and isinstance(scaling, (int, float)) and not isinstance(scaling, bool)):
        return None
    if type(dropout) is torch.nn.Identity:
        p = 0.0
    elif (type(dropout) is torch.nn.Dropout and dropout.training and not dropout.inplace
          and 0.0 < dropout.p < 1.0):
        p = float(dropout.p)
    else:
        return None
    a, b = lora_a.weight, lora_b.weight
    if not (a.dtype == torch.float32 and b.dtype == torch.float32 and on_gpu(a) and on_gpu(b)):
        return None
    return a, b, float(scaling), p


def _lora_pair(x, link, parts_q, parts_v, packing, dtype):
    """q and v LoRA deltas through LoRAPairFromNorm; dropout draws in the base's order (q, v)
    (solution/attn.py:300-323)."""
    _, h, norm_weight, eps = link
    width = x.shape[-1]
    packed = parts_q[3] > 0.0 and parts_v[3] > 0.0 and width % 8 == 0
    draws = []
    for _, _, _, p in (parts_q, parts_v):
        if p == 0.0:
            draws.append((None, None, None))
        elif packed:
            keep, scale = packing.dropout_keep(p, width, x.dtype, x.device)
            draws.append((None, keep, scale))
        else:
            scaled, keep = packing.dropout_draw(p, width, x.dtype, x.device)
            draws.append((scaled.view(x.shape), keep, packing.dropout_scale(p, scaled)))
    (sq, kq, cq), (sv, kv, cv) = draws
    if packed:
        mq, mv = pack_keep(kq, kv)
    else:
        mq = kq.view(x.shape) if kq is not None else None
        mv = kv.view(x.shape) if kv is not None else None
    return LoRAPairFromNorm.apply(x, h, norm_weight, eps, sq, mq, cq, sv, mv, cv,
                                  parts_q[0], parts_q[1], parts_v[0], parts_v[1],
                                  parts_q[2], parts_v[2], parts_q[3], parts_v[3], packed, dtype)


def _single_lora(layer, lora_cls):
    """The active adapter name of a plain (unmerged) LoRA layer, else None (solution/attn.py:326-341)."""
    try:
        if not isinstance(layer, lora_cls) or layer.disable_adapters or layer.merged:
            return None
        active = list(layer.active_adapters)
        if len(active) != 1:
            return None
        name = active[0]
        if name not in layer.lora_A or name in getattr(layer, "lora_variant", {}):
            return None
        if getattr(layer, "use_dora", {}).get(name, False):
            return None
        return name
    except AttributeError:
        return None


def _lora_delta(layer, name, x):
    """peft's LoRA branch, unchanged (solution/attn.py:344-346)."""
    return layer.lora_B[name](layer.lora_A[name](layer.lora_dropout[name](x))) * layer.scaling[name]


def _nf4_parts(module, n_in, dtype):
    """(packed weight, QuantState, bias or None) of an NF4 linear the fused block can dequantise."""
    from .nf4 import supported

    weight = getattr(module, "weight", None)
    qs = getattr(weight, "quant_state", None)
    bias = getattr(module, "bias", None)
    if (weight is None or not on_gpu(weight) or weight.dtype != torch.uint8 or weight.requires_grad
            or getattr(module, "compute_dtype", None) != dtype or not supported(qs, n_in)
            or (bias is not None and (bias.requires_grad or not on_gpu(bias)))):
        return None
    return weight.data, qs, bias


def _fused_block(self, x, q_name, v_name, cos, sin, packing, dtype, n_heads, n_kv, head_dim, o_nf4=False,
                 input_norm=None, residual_link=None):
    """(output, o_proj applied) through FusedAttentionBlock, or None when this layer does not
    qualify: both LoRA branches without dropout, rank 16 and one scaling; q, k, v NF4 linears of the
    compute dtype; the varlen attention switched on; head_dim 128. With ``o_nf4`` (o_proj is a plain
    NF4 Linear4bit of the compute dtype) o_proj joins the node: the output is then [1, T, H].
    With ``input_norm`` (the decoder layer's input RMSNorm module, eligible for the fused kernel)
    ``x`` is the layer input and the norm runs inside the node."""
    from .nf4 import dequantize_nf4_many

    pq, pv = _lora_parts(self.q_proj, q_name), _lora_parts(self.v_proj, v_name)
    if not (STATE.varlen_attention and head_dim == 128 and pq is not None and pv is not None
            and pq[3] == 0.0 and pv[3] == 0.0 and pq[2] == pv[2]
            and pq[0].shape[0] == 16 and pv[0].shape[0] == 16
            and (not self.training or getattr(self, "attention_dropout", 0.0) == 0.0)):
        return None
    hidden = x.shape[-1]
    parts = [_nf4_parts(m, hidden, dtype) for m in (self.q_proj.base_layer, self.k_proj, self.v_proj.base_layer)]
    if any(p is None for p in parts):
        return None
    rows = [int(p[1].shape[0]) for p in parts]
    if rows != [n_heads * head_dim, n_kv * head_dim, n_kv * head_dim]:
        return None
    n_tok = x.shape[1]
    w_cat = torch.empty((sum(rows) + 32, hidden), dtype=dtype, device=x.device)
    biases, items, r0 = [], [], 0
    for (packed, qs, bias), nr in zip(parts, rows):
        items.append((packed, qs, w_cat[r0:r0 + nr]))
        biases.append(bias.float() if bias is not None else torch.zeros(nr, device=x.device))
        r0 += nr
    w_o = b_o = None
    po = _nf4_parts(self.o_proj, n_heads * head_dim, dtype) if o_nf4 else None
    if po is not None:
        w_o = torch.empty(tuple(po[1].shape), dtype=dtype, device=x.device)
        items.append((po[0], po[1], w_o))
        b_o = None if po[2] is None else po[2].to(dtype)
    dequantize_nf4_many(items, dtype)  # W_q, W_k, W_v into their rows (and W_o), one launch
    bias_cat = torch.cat(biases + [torch.zeros(32, device=x.device)]).to(dtype)
    out = FusedAttentionBlock.apply(x.reshape(n_tok, hidden), pq[0], pq[1], pv[0], pv[1], w_cat, bias_cat,
                                    cos.reshape(n_tok, -1), sin.reshape(n_tok, -1),
                                    packing.cu_seqlens(x.device), packing.max_len, n_heads, n_kv, pq[2],
                                    self.scaling, w_o, b_o,
                                    None if input_norm is None else input_norm.weight,
                                    0.0 if input_norm is None else float(input_norm.variance_epsilon),
                                    residual_link)
    return out.reshape(1, n_tok, -1), w_o is not None


def patch(recompute_lora=True, linear4bit_cls=None, lora_classes=None, fused_block=True):
    """Patch Qwen2Attention.forward (solution/attn.py:349-421). ``linear4bit_cls`` and
    ``lora_classes`` default to bitsandbytes' Linear4bit and peft's LoRA layers. With
    ``fused_block`` a qualifying layer (LoRA without dropout) runs as one FusedAttentionBlock;
    the others keep the reference's chain of autograd Functions."""
    from transformers.modeling_utils import ALL_ATTENTION_FUNCTIONS
    from transformers.models.qwen2 import modeling_qwen2

    if linear4bit_cls is None:
        import bitsandbytes as bnb
        linear4bit_cls = bnb.nn.Linear4bit
    if lora_classes is None:
        from peft.tuners.lora.bnb import Linear4bit as LoraLinear4bit
        from peft.tuners.lora.layer import Linear as LoraLinear
        lora_classes = (LoraLinear4bit, LoraLinear)
    cls = modeling_qwen2.Qwen2Attention
    if getattr(cls.forward, "_skc", False):
        return
    original = cls.forward

    def nf4_linear(module):
        return (isinstance(module, linear4bit_cls)
                and getattr(module, "compute_dtype", None) in (torch.float16, torch.bfloat16))

    def forward(self, hidden_states, position_embeddings, attention_mask, past_key_values=None, **kwargs):
        # the patched decoder layer may hand over its input RMSNorm with the layer input (instead of
        # the norm's output) so that the fused block runs the norm in its first kernel; any other
        # path applies the norm here first
        input_norm = kwargs.pop(INPUT_NORM_KW, None)
        residual_link = kwargs.pop(RESIDUAL_LINK_KW, None)
        packing = STATE.packing
        q_name = _single_lora(getattr(self, "q_proj", None), lora_classes)
        v_name = _single_lora(getattr(self, "v_proj", None), lora_classes)
        cos, sin = position_embeddings if isinstance(position_embeddings, tuple) else (None, None)
        head_dim = getattr(self, "head_dim", 0)
        if not (STATE.packing_active and packing is not None and attention_mask is None
                and past_key_values is None and isinstance(hidden_states, torch.Tensor)
                and on_gpu(hidden_states) and hidden_states.dtype == torch.float32
                and hidden_states.dim() == 3 and hidden_states.shape[0] == 1
                and hidden_states.shape[1] == packing.n_tokens and torch.is_autocast_enabled("cuda")
                and q_name is not None and v_name is not None
                and nf4_linear(self.q_proj.base_layer) and nf4_linear(self.v_proj.base_layer)
                and nf4_linear(getattr(self, "k_proj", None))
                and isinstance(cos, torch.Tensor) and cos.dtype == torch.float32
                and cos.shape == (1, packing.n_tokens, head_dim) and sin.shape == cos.shape
                and head_dim == 128 and cos.is_contiguous() and sin.is_contiguous()
                and getattr(self, "sliding_window", None) is None):
            if input_norm is not None:
                hidden_states = input_norm(hidden_states)
            return original(self, hidden_states, position_embeddings, attention_mask,
                            past_key_values=past_key_values, **kwargs)
        dtype = self.q_proj.base_layer.compute_dtype
        n_tok = hidden_states.shape[1]
        n_heads = self.config.num_attention_heads
        n_kv = self.config.num_key_value_heads
        x = hidden_states
        if fused_block:
            res = _fused_block(self, x, q_name, v_name, cos, sin, packing, dtype, n_heads, n_kv, head_dim,
                               o_nf4=nf4_linear(getattr(self, "o_proj", None)), input_norm=input_norm,
                               residual_link=residual_link)
            if res is not None:
                out, o_done = res
                return (out if o_done else self.o_proj(out)), None
        if input_norm is not None:
            x = input_norm(x)
        link = STATE.norm_link
        parts_q = parts_v = None
        if (recompute_lora and link is not None and link[0] is x
                and isinstance(link[1], torch.Tensor) and link[1].shape == x.shape):
            parts_q, parts_v = _lora_parts(self.q_proj, q_name), _lora_parts(self.v_proj, v_name)
        # same call order as the base (q, k, v): the LoRA dropout draws stay in step
        q_base = self.q_proj.base_layer(x.to(dtype))
        if parts_q is None or parts_v is None:
            q_lora = _lora_delta(self.q_proj, q_name, x)
        k = self.k_proj(x.to(dtype))
        v_base = self.v_proj.base_layer(x.to(dtype))
        if parts_q is None or parts_v is None:
            v_lora = _lora_delta(self.v_proj, v_name, x)
        else:
            q_lora, v_lora = _lora_pair(x, link, parts_q, parts_v, packing, dtype)
        v = (v_base.float() + v_lora.float()).to(dtype)
        q_rot, k_rot = FusedQKRope.apply(
            q_base.to(dtype).reshape(n_tok, -1).contiguous(), q_lora.to(dtype).reshape(n_tok, -1).contiguous(),
            k.to(dtype).reshape(n_tok, -1).contiguous(), cos.reshape(n_tok, -1), sin.reshape(n_tok, -1),
            n_heads, n_kv)
        v_heads = v.view(1, n_tok, n_kv, head_dim).transpose(1, 2)
        attention = ALL_ATTENTION_FUNCTIONS["sdpa"]
        out, _ = attention(self, q_rot, k_rot, v_heads, None,
                           dropout=0.0 if not self.training else self.attention_dropout,
                           scaling=self.scaling, **kwargs)
        out = out.reshape(1, n_tok, -1).contiguous()
        return self.o_proj(out), None

    forward._skc = True
    cls.forward = forward
