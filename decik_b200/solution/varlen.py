"""Padding-free decoder plumbing and the varlen attention Function (solution/varlen.py).

``Packing`` / ``plan`` keep the reference's packing (solution/varlen.py:23-73, :191-226):
the real tokens of a right-padded [B, S] batch as one [1, T, H] sequence with per-row
positions and ``cu_seqlens``. ``VarlenSDPA`` keeps its arguments and result layout
(solution/varlen.py:134-168) but runs the sm_100a varlen kernels: GQA without expanding K/V,
dK/dV summed over each kv head's query heads inside the kernel, and the forward's logsumexp
kept for the backward instead of a forward recompute.
"""

from __future__ import annotations

import torch

from .. import ops
from ._state import STATE, on_gpu


class Packing:
    def __init__(self, index, positions, spans, batch, seq):
        self.index = index          # [T] flat positions of the real tokens in the [B, S] batch
        self.positions = positions  # [T] position of each real token in its row
        self.spans = spans          # [(start, length)] of each row in the packed sequence
        self.batch, self.seq = batch, seq
        self.n_tokens = int(index.numel())
        self._ones = {}
        self._scales = {}
        self.max_len = max((length for _, length in spans), default=0)
        self._cu = None

    def cu_seqlens(self, device):
        """Cumulative row offsets [rows + 1] (int32) for the varlen kernels (solution/varlen.py:35-40)."""
        if self._cu is None or self._cu.device != device:
            offsets = [start for start, _ in self.spans] + [self.n_tokens]
            self._cu = torch.tensor(offsets, dtype=torch.int32).to(device, non_blocking=True)
        return self._cu

    def dropout_draw(self, p, width, dtype, device):
        """What F.dropout draws for a [B, S, width] input, at the real tokens only
        (solution/varlen.py:42-52): the scaled values and the keep-mask."""
        key = (width, dtype, device)
        ones = self._ones.get(key)
        if ones is None:
            ones = torch.ones((self.batch, self.seq, width), dtype=dtype, device=device)
            self._ones[key] = ones
        scaled, keep = torch.native_dropout(ones, p, True)
        return (scaled.reshape(-1, width).index_select(0, self.index),
                keep.reshape(-1, width).index_select(0, self.index))

    def dropout_keep(self, p, width, dtype, device):
        """The keep-mask of the same draw, and the kept value (solution/varlen.py:54-63)."""
        key = (width, dtype, device)
        ones = self._ones.get(key)
        if ones is None:
            ones = torch.ones((self.batch, self.seq, width), dtype=dtype, device=device)
            self._ones[key] = ones
        scaled, keep = torch.native_dropout(ones, p, True)
        return keep.reshape(-1, width).index_select(0, self.index), self.dropout_scale(p, scaled)

    def dropout_scale(self, p, scaled):
        key = (p, scaled.dtype, scaled.device)
        scale = self._scales.get(key)
        if scale is None:
            scale = scaled.amax()
            self._scales[key] = scale
        return scale


def packing_from_lengths(lengths, device):
    """A Packing for rows of the given lengths (every token real), as plan() builds it."""
    lengths = [int(L) for L in lengths]
    spans, start = [], 0
    for L in lengths:
        spans.append((start, L))
        start += L
    index = torch.arange(start, device=device)
    positions = torch.cat([torch.arange(L, device=device) for L in lengths]) if lengths else index
    return Packing(index, positions, spans, 1, start)


class VarlenSDPA(torch.autograd.Function):
    """Causal attention over all rows of the packed sequence, one kernel launch each way.

    query [1, Hq, T, D] (head-major, as FusedQKRope makes it), key [1, Hk, T, D], value
    [1, Hk, T, D] (any strides with D contiguous) -> out [1, T, Hq, D] contiguous
    (solution/varlen.py:144-151). Backward returns dq, dk, dv with the strides of q, k, v."""

    @staticmethod
    def forward(ctx, query, key, value, cu_seqlens, max_len, groups, scale):
        if scale is None:
            scale = query.shape[-1] ** -0.5
        q3, k3, v3 = query[0].transpose(0, 1), key[0].transpose(0, 1), value[0].transpose(0, 1)
        if q3.shape[1] != k3.shape[1] * groups:
            raise RuntimeError("VarlenSDPA: query heads != kv heads * groups")
        out = torch.empty((1, q3.shape[0], q3.shape[1], q3.shape[2]), dtype=query.dtype, device=query.device)
        _, lse = ops.varlen_attn_fwd(q3, k3, v3, cu_seqlens, max_len, scale, out=out[0])
        ctx.save_for_backward(query, key, value, out, lse, cu_seqlens)
        ctx.max_len, ctx.scale = max_len, scale
        return out

    @staticmethod
    def backward(ctx, grad_out):
        query, key, value, out, lse, cu = ctx.saved_tensors
        dq = torch.empty_like(query)
        dk = torch.empty_like(key)
        dv = torch.empty_like(value)
        g = grad_out[0]
        if g.stride(-1) != 1:
            g = g.contiguous()
        ops.varlen_attn_bwd(g, query[0].transpose(0, 1), key[0].transpose(0, 1), value[0].transpose(0, 1),
                            out[0], lse, cu, ctx.max_len, ctx.scale, dq=dq[0].transpose(0, 1),
                            dk=dk[0].transpose(0, 1), dv=dv[0].transpose(0, 1))
        return dq, dk, dv, None, None, None, None


def plan(model, input_ids, attention_mask, position_ids, past_key_values, inputs_embeds,
         use_cache, kwargs):
    """A Packing for this forward, or None to run the original decoder (solution/varlen.py:191-226)."""
    config = getattr(model, "config", None)
    if not (STATE.request and model.training and torch.is_grad_enabled()
            and isinstance(input_ids, torch.Tensor) and isinstance(attention_mask, torch.Tensor)
            and input_ids.dim() == 2 and attention_mask.shape == input_ids.shape
            and inputs_embeds is None and position_ids is None and past_key_values is None
            and not use_cache and on_gpu(input_ids)
            and getattr(config, "_attn_implementation", None) == "sdpa"
            and not getattr(model, "has_sliding_layers", False)
            and all(t == "full_attention" for t in getattr(config, "layer_types", ["?"]))
            and not kwargs.get("output_attentions") and not kwargs.get("output_hidden_states")
            and not getattr(model, "gradient_checkpointing", False)
            and not any(getattr(layer, "gradient_checkpointing", False)
                        for layer in getattr(model, "layers", []))):
        return None
    batch, seq = input_ids.shape
    mask = attention_mask.to(torch.bool)
    lengths = mask.sum(dim=1)
    steps = torch.arange(seq, device=mask.device)
    if not torch.equal(mask, steps.unsqueeze(0) < lengths.unsqueeze(1)):
        return None  # not right-padded: keep the original path
    lens = lengths.tolist()
    if min(lens) == 0:
        return None  # an empty row
    index = mask.reshape(-1).nonzero().squeeze(1)
    positions = steps.unsqueeze(0).expand(batch, seq).reshape(-1).index_select(0, index)
    spans, start = [], 0
    for length in lens:
        spans.append((start, int(length)))
        start += int(length)
    return Packing(index, positions, spans, batch, seq)


class PackedDropout(torch.autograd.Function):
    """x * mask * scale with a given mask, saved as bool for backward (solution/varlen.py:176-188)."""

    @staticmethod
    def forward(ctx, x, scaled, keep, p):
        ctx.save_for_backward(keep)
        ctx.scale = 1.0 / (1.0 - p)
        return x * scaled

    @staticmethod
    def backward(ctx, grad):
        (keep,) = ctx.saved_tensors
        return grad * keep * ctx.scale, None, None, None


def patch(varlen_attention=True, fuse_residual=True):
    """Patch Qwen2Model.forward (packing), ALL_ATTENTION_FUNCTIONS["sdpa"], Qwen2DecoderLayer.forward
    (with ``fuse_residual``: the residual add + post-attention norm as one AddRMSNormFn) and
    nn.Dropout (solution/varlen.py:229-359). Inputs the packed path is not for go to the original
    code; eligible packed attention always runs the sm_100a kernel (no per-row fallback)."""
    import torch.nn.functional as F
    from transformers.modeling_outputs import BaseModelOutputWithPast
    from transformers.modeling_utils import ALL_ATTENTION_FUNCTIONS
    from transformers.models.qwen2 import modeling_qwen2

    model_cls = modeling_qwen2.Qwen2Model
    if getattr(model_cls.forward, "_skc", False):
        return
    model_forward = model_cls.forward

    def forward(self, input_ids=None, attention_mask=None, position_ids=None,
                past_key_values=None, inputs_embeds=None, use_cache=None, **kwargs):
        packing = plan(self, input_ids, attention_mask, position_ids, past_key_values,
                       inputs_embeds, use_cache, kwargs)
        if packing is None:
            return model_forward(self, input_ids=input_ids, attention_mask=attention_mask,
                                 position_ids=position_ids, past_key_values=past_key_values,
                                 inputs_embeds=inputs_embeds, use_cache=use_cache, **kwargs)
        ids = input_ids.reshape(-1).index_select(0, packing.index).unsqueeze(0)
        positions = packing.positions.unsqueeze(0)
        hidden = self.embed_tokens(ids)
        position_embeddings = self.rotary_emb(hidden, positions)
        STATE.packing, STATE.packing_active = packing, True
        try:
            for layer in self.layers[: self.config.num_hidden_layers]:
                hidden = layer(hidden, attention_mask=None, position_embeddings=position_embeddings,
                               position_ids=positions, past_key_values=None, use_cache=False,
                               **kwargs)
        finally:
            STATE.packing_active = False
            STATE.norm_link = None
        hidden = self.norm(hidden)
        return BaseModelOutputWithPast(last_hidden_state=hidden, past_key_values=None)

    forward._skc = True
    model_cls.forward = forward
    STATE.varlen_attention = bool(varlen_attention)

    sdpa = ALL_ATTENTION_FUNCTIONS["sdpa"]

    def sdpa_packed(module, query, key, value, attention_mask, dropout=0.0, scaling=None,
                    is_causal=None, **kwargs):
        packing = STATE.packing
        if not (varlen_attention and STATE.packing_active and packing is not None
                and attention_mask is None and query.dim() == 4 and query.shape[0] == 1
                and query.shape[2] == packing.n_tokens and key.shape[2] == packing.n_tokens
                and kwargs.get("position_bias") is None and dropout == 0.0 and query.is_cuda
                and query.dtype in (torch.float16, torch.bfloat16)
                and key.dtype == query.dtype and value.dtype == query.dtype
                and query.shape[-1] == 128):
            return sdpa(module, query, key, value, attention_mask, dropout=dropout,
                        scaling=scaling, is_causal=is_causal, **kwargs)
        groups = getattr(module, "num_key_value_groups", 1)
        return VarlenSDPA.apply(query, key, value, packing.cu_seqlens(query.device),
                                packing.max_len, groups, scaling), None

    ALL_ATTENTION_FUNCTIONS["sdpa"] = sdpa_packed

    from . import rmsnorm

    layer_cls = modeling_qwen2.Qwen2DecoderLayer
    layer_forward = layer_cls.forward

    def decoder_layer(self, hidden_states, attention_mask=None, position_ids=None,
                      past_key_values=None, use_cache=False, position_embeddings=None, **kwargs):
        packing = STATE.packing
        post_norm = getattr(self, "post_attention_layernorm", None)
        if not (fuse_residual and STATE.packing_active and packing is not None
                and attention_mask is None and past_key_values is None and not use_cache
                and isinstance(hidden_states, torch.Tensor) and hidden_states.dim() == 3
                and hidden_states.shape[0] == 1 and hidden_states.shape[1] == packing.n_tokens
                and rmsnorm.fusable(post_norm, hidden_states)):
            return layer_forward(self, hidden_states, attention_mask=attention_mask,
                                 position_ids=position_ids, past_key_values=past_key_values,
                                 use_cache=use_cache, position_embeddings=position_embeddings, **kwargs)
        # Qwen2DecoderLayer.forward with the residual add and the post-attention norm as one node
        # (solution/varlen.py:323-343): the norm's input is rebuilt in backward from the layer
        # input and the 16-bit attention output instead of being kept
        residual = hidden_states
        hidden_states = self.input_layernorm(hidden_states)
        attn_out, _ = self.self_attn(hidden_states=hidden_states, attention_mask=attention_mask,
                                     position_ids=position_ids, past_key_values=past_key_values,
                                     use_cache=use_cache, position_embeddings=position_embeddings, **kwargs)
        if (isinstance(attn_out, torch.Tensor) and attn_out.dtype in (torch.float16, torch.bfloat16)
                and attn_out.shape == residual.shape and attn_out.is_cuda):
            eps = float(post_norm.variance_epsilon)
            hidden_states, normed = rmsnorm.AddRMSNormFn.apply(residual, attn_out, post_norm.weight, eps)
            STATE.norm_link = (normed, (residual, attn_out), post_norm.weight, eps)
        else:
            hidden_states = residual + attn_out
            normed = post_norm(hidden_states)
        residual = hidden_states
        hidden_states = self.mlp(normed)
        return residual + hidden_states

    decoder_layer._skc = True
    layer_cls.forward = decoder_layer

    dropout_forward = torch.nn.Dropout.forward

    def dropout(self, input):
        packing = STATE.packing
        if (STATE.packing_active and packing is not None and self.training and 0.0 < self.p < 1.0
                and not self.inplace and isinstance(input, torch.Tensor) and input.dim() == 3
                and input.shape[0] == 1 and input.shape[1] == packing.n_tokens):
            scaled, keep = packing.dropout_draw(self.p, input.shape[-1], input.dtype, input.device)
            return PackedDropout.apply(input, scaled.unsqueeze(0), keep.unsqueeze(0), self.p)
        return dropout_forward(self, input)

    torch.nn.Dropout.forward = dropout
    del F
