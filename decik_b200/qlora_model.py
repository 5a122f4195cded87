"""A random-init Qwen2.5-shaped NF4 QLoRA causal LM: the whole model the reference's QLoRA step
trains, for the full-step benches and tests.

The reference trains Qwen2.5-1.5B-Instruct loaded in 4 bit (nf4, double quant, blocksize 64) with
LoRA r 16 / alpha 32 on q_proj and v_proj (task/task.yaml:3-22), through bitsandbytes' Linear4bit
and peft's LoRA layers. Neither library is a dependency here, so this module builds the same
model from transformers' ``Qwen2ForCausalLM`` (random init, N(0, 0.02) weights) with two module
types that carry exactly the fields the reference's patches read:

- ``Linear4bit``: a uint8 packed NF4 weight with a ``quant_state`` (nested absmax, blocksize 64 /
  256), a bias, ``compute_dtype`` (solution/nf4.py:114-135). Its own forward is the plain
  dequantize + linear on the sm_100a dequant kernel; ``solution.apply()`` replaces it with
  ``NF4Linear`` (same result, dequantised weight not kept).
- ``LoraLinear``: ``base_layer``, ``lora_A`` / ``lora_B`` / ``lora_dropout`` ModuleDicts,
  ``scaling``, ``active_adapters``, ``disable_adapters``, ``merged``, ``use_dora``
  (solution/attn.py:276-346).

``qlora_train_step`` is one training step the way the reference's trainer runs it with the packed
path requested (solution/varlen.py:235-359, solution/head.py:147-171): autocast forward over a
right-padded batch (packed padding-free by the patched Qwen2Model.forward), cross entropy over
the real tokens' shifted labels normalised by the (global) labelled-token count, backward.

    model = build_qlora_qwen2(device="cuda")            # 28 layers, hidden 1536, 12/2 heads
    solution.apply(linear4bit_cls=Linear4bit, lora_classes=(LoraLinear,))
    loss = qlora_train_step(model, ids, mask, labels)
"""

from __future__ import annotations

import math

import numpy as np
import torch
import torch.nn as nn
import torch.nn.functional as F

from .block import QuantState
from .nf4_quant import dynamic_code, nf4_code

# the Qwen2.5-1.5B shape
QWEN25_15B = dict(hidden=1536, intermediate=8960, layers=28, heads=12, kv_heads=2, vocab=151936,
                  rope_theta=1e6, rms_eps=1e-6)


def _nearest(values: torch.Tensor, table: torch.Tensor) -> torch.Tensor:
    """Index of the nearest table entry (ties to the lower one), as numpy.searchsorted over the
    fp64 midpoints in nf4_quant._nearest."""
    t = table.double()
    mids = (t[1:] + t[:-1]) / 2.0
    return torch.bucketize(values.double(), mids, right=False).to(torch.uint8)


@torch.no_grad()
def quantize_nf4_torch(w: torch.Tensor, blocksize: int = 64, blocksize2: int = 256):
    """NF4 double quantisation of ``w`` [N, K] on its own device, the method of
    nf4_quant.quantize_nf4 (QLoRA's NF4 code, per-64 absmax, absmax minus its mean re-quantised per
    256 to the signed dynamic 8-bit map). Returns (packed uint8 [N*K/2], QuantState)."""
    dev = w.device
    flat = w.detach().reshape(-1).float()
    if flat.numel() % blocksize:
        raise ValueError("quantize_nf4_torch: numel must be a multiple of the blocksize")
    blocks = flat.view(-1, blocksize)
    n_blocks = blocks.shape[0]
    absmax = blocks.abs().amax(dim=1)
    safe = torch.where(absmax == 0, torch.ones_like(absmax), absmax)
    code = torch.from_numpy(nf4_code()).to(dev)
    idx = _nearest((blocks / safe[:, None]).reshape(-1), code)
    packed = (idx[0::2] << 4) | idx[1::2]
    offset = absmax.double().mean().float()
    centred = absmax - offset
    n2 = -(-n_blocks // blocksize2)
    padded = torch.zeros(n2 * blocksize2, dtype=torch.float32, device=dev)
    padded[:n_blocks] = centred
    absmax2 = padded.view(n2, blocksize2).abs().amax(dim=1)
    absmax2 = torch.where(absmax2 == 0, torch.ones_like(absmax2), absmax2)
    code2 = torch.from_numpy(dynamic_code()).to(dev)
    scaled = centred / absmax2.repeat_interleave(blocksize2)[:n_blocks]
    qs = QuantState(tuple(w.shape), _nearest(scaled, code2), code, blocksize, None, absmax2=absmax2,
                    code2=code2, offset=offset.reshape(1), blocksize2=blocksize2)
    return packed.contiguous(), qs


class Linear4bit(nn.Module):
    """NF4 linear layer with the fields of bitsandbytes.nn.Linear4bit that the patches read."""

    def __init__(self, linear: nn.Linear, compute_dtype=torch.bfloat16, packed_state=None):
        super().__init__()
        self.in_features, self.out_features = linear.in_features, linear.out_features
        self.compute_dtype = compute_dtype
        packed, qs = packed_state if packed_state is not None else quantize_nf4_torch(linear.weight)
        qs.dtype = compute_dtype
        w = nn.Parameter(packed, requires_grad=False)
        w.quant_state = qs
        self.weight = w
        self.bias = (None if linear.bias is None else
                     nn.Parameter(linear.bias.detach().float().clone(), requires_grad=False))

    def forward(self, x):
        from .solution.nf4 import NF4Linear

        dt = self.compute_dtype
        b = None if self.bias is None else self.bias.to(dt)
        return NF4Linear.apply(x.to(dt), self.weight.data, b, self.weight.quant_state).to(x.dtype)


class LoraLinear(nn.Module):
    """LoRA adapter "default" around a base layer, with the fields of peft's LoRA Linear that the
    patches read: out = base(x) + lora_B(lora_A(dropout(x))) * scaling."""

    def __init__(self, base: nn.Module, r: int = 16, alpha: int = 32, dropout: float = 0.0):
        super().__init__()
        dev = base.weight.device
        self.base_layer = base
        self.lora_A = nn.ModuleDict({"default": nn.Linear(base.in_features, r, bias=False, device=dev)})
        self.lora_B = nn.ModuleDict({"default": nn.Linear(r, base.out_features, bias=False, device=dev)})
        nn.init.kaiming_uniform_(self.lora_A["default"].weight, a=math.sqrt(5))
        nn.init.normal_(self.lora_B["default"].weight, std=0.02)  # random: the LoRA branch is live from step 1
        self.lora_dropout = nn.ModuleDict({"default": nn.Dropout(dropout) if dropout > 0 else nn.Identity()})
        self.scaling = {"default": alpha / r}
        self.active_adapters = ["default"]
        self.disable_adapters = False
        self.merged = False
        self.use_dora = {"default": False}

    @property
    def weight(self):
        return self.base_layer.weight

    def forward(self, x):
        n = "default"
        return self.base_layer(x) + self.lora_B[n](self.lora_A[n](self.lora_dropout[n](x))) * self.scaling[n]


def build_qlora_qwen2(hidden=QWEN25_15B["hidden"], intermediate=QWEN25_15B["intermediate"],
                      layers=QWEN25_15B["layers"], heads=QWEN25_15B["heads"], kv_heads=QWEN25_15B["kv_heads"],
                      vocab=QWEN25_15B["vocab"], rank=16, alpha=32, lora_dropout=0.0, seed=0,
                      compute_dtype=torch.bfloat16, device="cuda", share_layer_weights=False):
    """Random-init Qwen2.5-shaped QLoRA model on ``device``: fp32 embedding (tied head) and norms,
    every decoder linear NF4 (``Linear4bit``), LoRA on q_proj / v_proj, only LoRA trainable.
    ``share_layer_weights``: every layer reuses layer 0's frozen NF4 weights (same shapes and
    compute; for host-memory-bound CPU runs) while LoRA stays per layer."""
    from transformers import Qwen2Config, Qwen2ForCausalLM

    cfg = Qwen2Config(vocab_size=vocab, hidden_size=hidden, intermediate_size=intermediate,
                      num_hidden_layers=layers, num_attention_heads=heads, num_key_value_heads=kv_heads,
                      max_position_embeddings=32768, rope_theta=QWEN25_15B["rope_theta"],
                      rms_norm_eps=QWEN25_15B["rms_eps"], tie_word_embeddings=True, initializer_range=0.02)
    cfg._attn_implementation = "sdpa"
    torch.manual_seed(seed)
    if share_layer_weights:
        # only layer 0's dense weights are ever read: build on the meta device, allocate, and
        # initialise the embedding, norms, rotary table, biases and layer 0's linears (the dense
        # init of all layers dominates a host build otherwise)
        from transformers.models.qwen2.modeling_qwen2 import Qwen2RMSNorm, Qwen2RotaryEmbedding

        with torch.device("meta"):
            model = Qwen2ForCausalLM(cfg)
        model.to_empty(device=device)
        with torch.no_grad():
            model.model.embed_tokens.weight.normal_(0.0, cfg.initializer_range)
            for m in model.modules():
                if isinstance(m, Qwen2RMSNorm):
                    m.weight.fill_(1.0)
                elif isinstance(m, nn.Linear) and m.bias is not None:
                    m.bias.zero_()
            for m in model.model.layers[0].modules():
                if isinstance(m, nn.Linear):
                    m.weight.normal_(0.0, cfg.initializer_range)
        model.model.rotary_emb = Qwen2RotaryEmbedding(config=cfg, device=device)
        model.tie_weights()
    else:
        with torch.device(device):
            model = Qwen2ForCausalLM(cfg)
    shared = {}
    for li, layer in enumerate(model.model.layers):
        attn, mlp = layer.self_attn, layer.mlp
        for owner, names in ((attn, ("q_proj", "k_proj", "v_proj", "o_proj")),
                             (mlp, ("gate_proj", "up_proj", "down_proj"))):
            for name in names:
                lin = getattr(owner, name)
                st = shared.get(name) if share_layer_weights else None
                q = Linear4bit(lin, compute_dtype, packed_state=st)
                if share_layer_weights and li == 0:
                    shared[name] = (q.weight.data, q.weight.quant_state)
                setattr(owner, name, q)
                del lin
        attn.q_proj = LoraLinear(attn.q_proj, rank, alpha, lora_dropout)
        attn.v_proj = LoraLinear(attn.v_proj, rank, alpha, lora_dropout)
    for name, p in model.named_parameters():
        p.requires_grad_("lora_" in name)
    if str(device).startswith("cuda"):
        torch.cuda.empty_cache()
    model.train()
    return model


def lora_parameters(model):
    return [p for n, p in model.named_parameters() if "lora_" in n]


def padded_batch(lengths, vocab, seed, device):
    """Right-padded [rows, max_len] input ids (uniform over the vocabulary), attention mask and
    labels (every real token labelled, padding -100), as the reference's collator hands them to
    the model."""
    g = torch.Generator().manual_seed(seed)
    rows, seq = len(lengths), max(lengths)
    ids = torch.randint(0, vocab, (rows, seq), generator=g)
    mask = torch.zeros(rows, seq, dtype=torch.long)
    for i, L in enumerate(lengths):
        mask[i, :L] = 1
    ids = ids * mask
    labels = torch.where(mask.bool(), ids, torch.full_like(ids, -100))
    return ids.to(device), mask.to(device), labels.to(device)


def qlora_train_step(model, ids, mask, labels, dtype=torch.bfloat16, n_labels=None, fused_head=True):
    """Forward (packed path requested) + loss + backward of one step; returns the loss (a device
    scalar). The loss is the summed cross entropy of the real tokens' shifted labels divided by
    ``n_labels``: this step's labelled-token count, or the global count under data parallelism
    (solution/head.py:157-163). Per-rank losses and gradients then sum to the one-process values.
    On the GPU with ``fused_head`` the head and loss run chunked through ``solution.head.run_head``
    (no [tokens x vocab] fp32 logits); otherwise as lm_head + cross_entropy."""
    from .solution._state import STATE

    STATE.request, STATE.packing = True, None
    try:
        with torch.autocast("cuda", dtype=dtype, enabled=ids.is_cuda):
            hidden = model.model(input_ids=ids, attention_mask=mask, use_cache=False).last_hidden_state
            packing = STATE.packing
            if fused_head and ids.is_cuda:
                from .solution.head import run_head

                if n_labels is None:
                    n_labels = (F.pad(labels, (0, 1), value=-100)[..., 1:] != -100).sum().float()
                loss = run_head(model, hidden, labels, mask, n_labels, packing, dtype)
            else:
                flat = hidden.reshape(-1, hidden.shape[-1])
                if packing is not None:
                    positions = packing.index
                else:
                    positions = mask.reshape(-1).nonzero().squeeze(1)
                    flat = flat.index_select(0, positions)
                targets = F.pad(labels, (0, 1), value=-100)[..., 1:].reshape(-1).index_select(0, positions)
                logits = model.lm_head(flat)
                if n_labels is None:
                    n_labels = (targets != -100).sum()
                loss = F.cross_entropy(logits.float(), targets, ignore_index=-100, reduction="sum") / n_labels
    finally:
        STATE.request, STATE.packing = False, None
    loss.backward()
    return loss.detach()


def lognormal_lengths(seed: int, total: int, median: int, lo: int, hi: int, sigma: float = 1.0):
    """Row lengths drawn log-normal (given median, sigma), clipped to [lo, hi], packed greedily
    until ``total`` tokens; the last row is cut to fit."""
    rng = np.random.default_rng(seed)
    out, s = [], 0
    while s < total:
        L = int(np.clip(round(float(rng.lognormal(math.log(median), sigma))), lo, hi))
        L = min(L, total - s)
        out.append(L)
        s += L
    return out
