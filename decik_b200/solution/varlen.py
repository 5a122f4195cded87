"""Padding-free decoder plumbing and the varlen attention Function (solution/varlen.py).

The reference runs the decoder on the real tokens of a right-padded batch only: they become one
[1, T, H] sequence with per-row RoPE positions and per-row causal attention. Here the packing is
built on the device by one kernel (``decik_pack_rows``) from the attention mask: row lengths,
``cu_seqlens``, the flat index of each real token, its position in its row and the packed token
ids. The host reads back only the kernel's summary (T, the longest row, a right-padding flag and
the row lengths), one copy into pinned memory, where the reference's ``plan()``
(solution/varlen.py:191-226) synchronises three times (``torch.equal``, ``.tolist()``,
``nonzero``).

``VarlenSDPA`` keeps the reference's arguments and result layout (solution/varlen.py:134-168) and
runs the sm_100a varlen kernels: GQA without expanding K/V, dK/dV summed over each kv head's query
heads inside the kernel, and the forward's logsumexp kept for backward (no forward recompute).

LoRA dropout on the packed path draws its random numbers exactly as the unpacked model would:
``torch.native_dropout`` on a [B, S, width] tensor, the op and shape of the base model's draw, of
which only the real tokens' rows are used. So the RNG stream, and the training run, stay the same
as the reference's.
"""

from __future__ import annotations

import itertools

import torch

from .. import ops
from ._state import STATE, on_gpu


class PackedBatch:
    """The real tokens of one right-padded [batch, seq] batch as a single packed sequence.

    Device tensors: ``index`` (flat b * seq + s of each real token), ``positions`` (s), the
    packed token ``ids`` (None when built from lengths) and ``cu_seqlens`` int32 [rows + 1].
    Host values: the row ``lengths``, ``n_tokens`` and ``max_len``; ``spans`` are the rows'
    (start, length) in the packed sequence."""

    def __init__(self, lengths, batch, seq, index, positions, cu_seqlens, ids=None):
        self.lengths = tuple(int(n) for n in lengths)
        self.batch, self.seq = int(batch), int(seq)
        self.index, self.positions, self.ids = index, positions, ids
        self._cu = cu_seqlens
        self.n_tokens = sum(self.lengths)
        self.max_len = max(self.lengths, default=0)
        self._draw_src = {}   # (width, dtype, device) -> ones [batch, seq, width], the draw's input
        self._kept = {}       # (p, dtype, device) -> the kept value of a draw

    @property
    def spans(self):
        starts = itertools.accumulate((0,) + self.lengths[:-1])
        return list(zip(starts, self.lengths))

    def cu_seqlens(self, device):
        """Row offsets int32 [rows + 1] on ``device`` (built by the packing kernel)."""
        if self._cu.device != torch.device(device):
            self._cu = self._cu.to(device)
        return self._cu

    def _sample(self, p, width, dtype, device):
        """One draw of dropout over the padded batch: (values, keep) at the real tokens, and the
        full values tensor (for the kept value)."""
        key = (width, dtype, torch.device(device))
        src = self._draw_src.get(key)
        if src is None:
            src = self._draw_src[key] = torch.ones((self.batch, self.seq, width), dtype=dtype, device=device)
        values, keep = torch.native_dropout(src, p, True)
        at_real = lambda t: t.view(self.batch * self.seq, width).index_select(0, self.index)
        return at_real(values), at_real(keep), values

    def dropout_draw(self, p, width, dtype, device):
        """(scaled values, keep-mask) of the draw F.dropout makes for a [batch, seq, width]
        input, at the real tokens (solution/varlen.py:42-52)."""
        values, keep, _ = self._sample(p, width, dtype, device)
        return values, keep

    def dropout_keep(self, p, width, dtype, device):
        """The keep-mask of the same draw, and its kept value (solution/varlen.py:54-63)."""
        _, keep, full = self._sample(p, width, dtype, device)
        return keep, self.dropout_scale(p, full)

    def dropout_scale(self, p, values):
        """1 / (1 - p) as the dropout kernel rounds it in values.dtype, as a 0-dim device tensor:
        the largest value of a draw (every kept entry holds it)."""
        key = (p, values.dtype, values.device)
        if key not in self._kept:
            self._kept[key] = values.amax()
        return self._kept[key]


# the name the reference's modules use for the packing object
Packing = PackedBatch


def packing_from_lengths(lengths, device):
    """A PackedBatch for rows of the given lengths with no padding (batch = 1 row of all tokens
    for the dropout draws), built with device ops."""
    lengths = [int(n) for n in lengths]
    T = sum(lengths)
    dev = torch.device(device)
    lens = torch.tensor(lengths, dtype=torch.int64, device=dev)
    cu = torch.zeros(len(lengths) + 1, dtype=torch.int32, device=dev)
    if lengths:
        cu[1:] = torch.cumsum(lens, 0).to(torch.int32)
    index = torch.arange(T, device=dev)
    starts = torch.repeat_interleave(cu[:-1].to(torch.int64), lens) if lengths else index
    return PackedBatch(lengths, 1, T, index, index - starts, cu)


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


# ------------------------------------------------------------------------------------------------
# when the decoder may run packed
# ------------------------------------------------------------------------------------------------
def _layers_all_full_attention(model) -> bool:
    config = getattr(model, "config", None)
    return (getattr(config, "_attn_implementation", None) == "sdpa"
            and not getattr(model, "has_sliding_layers", False)
            and all(kind == "full_attention" for kind in getattr(config, "layer_types", ["?"])))


def _checkpointing(model) -> bool:
    # recomputation would replay layers outside the packed step
    return getattr(model, "gradient_checkpointing", False) or any(
        getattr(layer, "gradient_checkpointing", False) for layer in getattr(model, "layers", []))


def _packable_call(model, input_ids, attention_mask, position_ids, past_key_values, inputs_embeds,
                   use_cache, kwargs) -> bool:
    """The reference's eligibility for the padded-free forward (solution/varlen.py:195-206): a
    requested training forward with grad, 2-D ids on the GPU with a mask of the same shape, no
    embeddings, positions, cache or extra outputs, sdpa on full-attention layers only, and no
    gradient checkpointing."""
    call_ok = (STATE.request and model.training and torch.is_grad_enabled()
               and inputs_embeds is None and position_ids is None and past_key_values is None
               and not use_cache and not kwargs.get("output_attentions")
               and not kwargs.get("output_hidden_states"))
    tensors_ok = (isinstance(input_ids, torch.Tensor) and isinstance(attention_mask, torch.Tensor)
                  and input_ids.dim() == 2 and attention_mask.shape == input_ids.shape and on_gpu(input_ids))
    return bool(call_ok and tensors_ok and _layers_all_full_attention(model) and not _checkpointing(model))


def plan(model, input_ids, attention_mask, position_ids, past_key_values, inputs_embeds,
         use_cache, kwargs):
    """A PackedBatch for this forward, or None to run the original decoder: not an eligible call, a
    row that is not right-padded, or an empty row (solution/varlen.py:191-226)."""
    if not _packable_call(model, input_ids, attention_mask, position_ids, past_key_values, inputs_embeds,
                          use_cache, kwargs):
        return None
    mask = attention_mask if attention_mask.dtype in (torch.int64, torch.int32, torch.bool, torch.uint8) \
        else attention_mask.to(torch.int64)
    ids = input_ids if input_ids.dtype == torch.int64 else input_ids.to(torch.int64)
    built = ops.pack_rows(mask, ids)
    if built is None:
        return None  # left padding or holes: the original decoder handles it
    lengths, cu, index, positions, packed_ids = built
    if min(lengths) == 0:
        return None
    batch, seq = input_ids.shape
    return PackedBatch(lengths, batch, seq, index, positions, cu, packed_ids)


class PackedDropout(torch.autograd.Function):
    """Dropout with a draw made outside: x * values forward, grad * keep / (1 - p) backward
    (solution/varlen.py:176-188); only the bool keep-mask is saved."""

    @staticmethod
    def forward(ctx, x, values, keep, p):
        ctx.save_for_backward(keep)
        ctx.inv_keep = 1.0 / (1.0 - p)
        return x * values

    @staticmethod
    def backward(ctx, grad):
        (keep,) = ctx.saved_tensors
        return grad * keep * ctx.inv_keep, None, None, None


# ------------------------------------------------------------------------------------------------
# the patched methods
# ------------------------------------------------------------------------------------------------
class _PackedStep:
    """Marks the packed path active for the layers of one forward, and always clears it."""

    def __init__(self, packing):
        self.packing = packing

    def __enter__(self):
        STATE.packing, STATE.packing_active = self.packing, True
        return self.packing

    def __exit__(self, *exc):
        STATE.packing_active = False
        STATE.norm_link = None
        return False


def _on_packed_path(hidden_states) -> bool:
    """True while a packed forward runs and this tensor is its [1, T, ...] sequence."""
    packing = STATE.packing
    return (STATE.packing_active and packing is not None and isinstance(hidden_states, torch.Tensor)
            and hidden_states.dim() == 3 and hidden_states.shape[0] == 1
            and hidden_states.shape[1] == packing.n_tokens)


def _model_forward(original):
    from transformers.modeling_outputs import BaseModelOutputWithPast

    def forward(self, input_ids=None, attention_mask=None, position_ids=None, past_key_values=None,
                inputs_embeds=None, use_cache=None, **kwargs):
        packing = plan(self, input_ids, attention_mask, position_ids, past_key_values, inputs_embeds,
                       use_cache, kwargs)
        if packing is None:
            return original(self, input_ids=input_ids, attention_mask=attention_mask, position_ids=position_ids,
                            past_key_values=past_key_values, inputs_embeds=inputs_embeds, use_cache=use_cache,
                            **kwargs)
        positions = packing.positions[None]
        hidden = self.embed_tokens(packing.ids[None])
        rope = self.rotary_emb(hidden, positions)
        with _PackedStep(packing):
            for layer in self.layers[: self.config.num_hidden_layers]:
                hidden = layer(hidden, attention_mask=None, position_embeddings=rope, position_ids=positions,
                               past_key_values=None, use_cache=False, **kwargs)
        return BaseModelOutputWithPast(last_hidden_state=self.norm(hidden), past_key_values=None)

    return forward


def _packed_sdpa(original, varlen_attention):
    def sdpa(module, query, key, value, attention_mask, dropout=0.0, scaling=None, is_causal=None, **kwargs):
        packing = STATE.packing
        fits = (varlen_attention and attention_mask is None and dropout == 0.0
                and kwargs.get("position_bias") is None and query.dim() == 4
                and _on_packed_path(query[:, 0]) and key.shape[2] == packing.n_tokens
                and query.is_cuda and query.shape[-1] == 128
                and query.dtype in (torch.float16, torch.bfloat16) and key.dtype == value.dtype == query.dtype)
        if not fits:
            return original(module, query, key, value, attention_mask, dropout=dropout, scaling=scaling,
                            is_causal=is_causal, **kwargs)
        groups = getattr(module, "num_key_value_groups", 1)
        out = VarlenSDPA.apply(query, key, value, packing.cu_seqlens(query.device), packing.max_len, groups,
                               scaling)
        return out, None

    return sdpa


def _decoder_layer(original, fuse_residual, fuse_input_norm=True):
    from . import rmsnorm
    from .attn import INPUT_NORM_KW, RESIDUAL_LINK_KW

    def forward(self, hidden_states, attention_mask=None, position_ids=None, past_key_values=None,
                use_cache=False, position_embeddings=None, **kwargs):
        post_norm = getattr(self, "post_attention_layernorm", None)
        if not (fuse_residual and attention_mask is None and past_key_values is None and not use_cache
                and _on_packed_path(hidden_states) and rmsnorm.fusable(post_norm, hidden_states)):
            return original(self, hidden_states, attention_mask=attention_mask, position_ids=position_ids,
                            past_key_values=past_key_values, use_cache=use_cache,
                            position_embeddings=position_embeddings, **kwargs)
        # the layer with its residual add and post-attention norm as one AddRMSNormFn node
        # (solution/varlen.py:323-343): the norm input is rebuilt in backward from the layer input
        # and the 16-bit attention output, not kept
        layer_in = hidden_states
        norm_in = getattr(self, "input_layernorm", None)
        if (fuse_input_norm and getattr(type(self.self_attn).forward, "_skc", False)
                and rmsnorm.fusable(norm_in, layer_in)):
            # the patched attention takes the layer input and its norm: the fused block then runs
            # the norm inside its first kernel (any other path applies it first)
            # the link carries layer_in's residual gradient into the block's norm backward (armed
            # only if the fused block ran)
            link = rmsnorm.ResidualGradLink()
            attn, _ = self.self_attn(hidden_states=layer_in, attention_mask=None, position_ids=position_ids,
                                     past_key_values=None, use_cache=False, position_embeddings=position_embeddings,
                                     **{INPUT_NORM_KW: norm_in, RESIDUAL_LINK_KW: link}, **kwargs)
        else:
            link = None
            attn, _ = self.self_attn(hidden_states=norm_in(layer_in), attention_mask=None,
                                     position_ids=position_ids, past_key_values=None, use_cache=False,
                                     position_embeddings=position_embeddings, **kwargs)
        if (isinstance(attn, torch.Tensor) and attn.is_cuda and attn.shape == layer_in.shape
                and attn.dtype in (torch.float16, torch.bfloat16)):
            eps = float(post_norm.variance_epsilon)
            # y in the attention output's 16-bit dtype when the patched MLP will compute in that
            # dtype: its cast of an fp32 y (and the fp32 y itself) is then never made
            eligible = getattr(type(self.mlp).forward, "_skc_eligible", None)
            y16 = eligible is not None and eligible(self.mlp, attn) == attn.dtype
            mid, normed = rmsnorm.AddRMSNormFn.apply(layer_in, attn, post_norm.weight, eps, y16, link)
            STATE.norm_link = (normed, (layer_in, attn), post_norm.weight, eps)
        else:
            mid = layer_in + attn
            normed = post_norm(mid)
        if getattr(type(self.mlp).forward, "_skc", False):
            return self.mlp(normed, residual=mid)  # the residual add inside the MLP's down projection
        return mid + self.mlp(normed)

    return forward


def _dropout(original):
    def forward(self, input):
        if (self.training and 0.0 < self.p < 1.0 and not self.inplace and _on_packed_path(input)):
            values, keep = STATE.packing.dropout_draw(self.p, input.shape[-1], input.dtype, input.device)
            return PackedDropout.apply(input, values[None], keep[None], self.p)
        return original(self, input)

    return forward


def patch(varlen_attention=True, fuse_residual=True, fuse_input_norm=True):
    """Install the packed decoder (solution/varlen.py:229-359): Qwen2Model.forward (packing),
    ALL_ATTENTION_FUNCTIONS["sdpa"], Qwen2DecoderLayer.forward (with ``fuse_residual``: the
    residual add + post-attention norm as one AddRMSNormFn; with ``fuse_input_norm`` the input
    RMSNorm is handed to the patched attention, whose fused block runs it in its first kernel) and
    nn.Dropout. Inputs the packed path
    is not for go to the original code; eligible packed attention always runs the sm_100a kernel
    (no per-row fallback). Idempotent."""
    from transformers.modeling_utils import ALL_ATTENTION_FUNCTIONS
    from transformers.models.qwen2 import modeling_qwen2

    model_cls = modeling_qwen2.Qwen2Model
    if getattr(model_cls.forward, "_skc", False):
        return
    STATE.varlen_attention = bool(varlen_attention)
    installs = ((model_cls, "forward", _model_forward(model_cls.forward)),
                (modeling_qwen2.Qwen2DecoderLayer, "forward",
                 _decoder_layer(modeling_qwen2.Qwen2DecoderLayer.forward, fuse_residual, fuse_input_norm)),
                (torch.nn.Dropout, "forward", _dropout(torch.nn.Dropout.forward)))
    ALL_ATTENTION_FUNCTIONS["sdpa"] = _packed_sdpa(ALL_ATTENTION_FUNCTIONS["sdpa"], varlen_attention)
    for cls, name, fn in installs:
        fn._skc = True
        setattr(cls, name, fn)
