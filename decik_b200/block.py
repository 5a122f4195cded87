"""The attention block of one decoder layer of the QLoRA step, as a plain object: the forward and
backward the patched Qwen2Attention.forward runs (solution/attn.py:387-418, without o_proj).
By default one fused autograd node (``FusedAttentionBlock``: one projection GEMM, the sm_100a
epilogues and attention kernels); ``fused=False`` composes the reference-facing autograd
Functions of ``decik_b200.solution`` one by one instead.

    block = QLoRAAttentionBlock.random(hidden=1536, n_heads=12, n_kv=2, device="cuda")
    out = block.forward(x, packing)          # [T, n_heads * 128]
    out.backward(grad)                       # LoRA grads land in block.lora_params()

Weights are NF4 double-quant (blocksize 64 / 256) packed on the device; q/k/v biases and the
LoRA A/B matrices (r = 16, alpha = 32 on q and v) are fp32 parameters, as peft keeps them.
Compute runs in ``dtype`` (bf16 by default; fp16 as in the reference).
"""

from __future__ import annotations

import math

import numpy as np
import torch
import torch.nn.functional as F

from .solution.attn import FusedAttentionBlock, FusedQKRope
from .solution.nf4 import NF4Linear
from .solution.varlen import Packing, VarlenSDPA


class QuantState:
    """The fields of a bitsandbytes QuantState that the NF4 path reads (solution/nf4.py:66-85)."""

    def __init__(self, shape, absmax, code, blocksize, dtype, absmax2=None, code2=None, offset=None,
                 blocksize2=256):
        self.shape = tuple(shape)
        self.absmax, self.code, self.blocksize, self.dtype = absmax, code, blocksize, dtype
        self.quant_type = "nf4"
        self.nested = absmax2 is not None
        self.offset = offset
        if self.nested:
            self.state2 = type("State2", (), {})()
            self.state2.absmax, self.state2.code, self.state2.blocksize = absmax2, code2, blocksize2
        else:
            self.state2 = None


def quant_state_from_arrays(st: dict, device, dtype) -> tuple[torch.Tensor, QuantState]:
    """(packed uint8 tensor, QuantState) on ``device`` from a dict of numpy arrays with the
    fields packed, absmax, code, shape, blocksize, nested, absmax2, code2, offset, blocksize2."""
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(device)
    packed = t(st["packed"])
    if st["nested"]:
        qs = QuantState(st["shape"], t(st["absmax"]), t(st["code"]), st["blocksize"], dtype,
                        absmax2=t(st["absmax2"]), code2=t(st["code2"]),
                        offset=torch.tensor([float(st["offset"])], dtype=torch.float32, device=device),
                        blocksize2=st["blocksize2"])
    else:
        qs = QuantState(st["shape"], t(st["absmax"]), t(st["code"]), st["blocksize"], dtype)
    return packed, qs


def rope_cos_sin(positions: torch.Tensor, head_dim: int, theta: float = 1e6):
    """fp32 cos, sin [T, head_dim] (transformers' Qwen2RotaryEmbedding, attention_scaling 1)."""
    inv = 1.0 / (theta ** (torch.arange(0, head_dim, 2, device=positions.device).float() / head_dim))
    fr = positions.float()[:, None] * inv[None, :]
    emb = torch.cat((fr, fr), dim=-1)
    return emb.cos().contiguous(), emb.sin().contiguous()


class QLoRAAttentionBlock:
    def __init__(self, nf4_states: dict, biases: dict, lora: dict, n_heads: int, n_kv: int,
                 head_dim: int = 128, scaling: float = 2.0, dtype=torch.bfloat16, device="cuda"):
        self.n_heads, self.n_kv, self.head_dim = n_heads, n_kv, head_dim
        self.nf4_states = nf4_states  # the host-side arrays, for checks against the CPU oracle
        self.scaling, self.dtype, self.device = scaling, dtype, device
        self.weights = {n: quant_state_from_arrays(nf4_states[n], device, dtype) for n in ("q", "k", "v")}
        self.bias = {n: biases[n].to(device=device, dtype=torch.float32) for n in ("q", "k", "v")}
        self.lora = {n: lora[n].to(device=device, dtype=torch.float32).requires_grad_(True)
                     for n in ("a_q", "b_q", "a_v", "b_v")}
        rank = self.lora["a_q"].shape[0]
        # frozen biases of the fused projection, zero for the two lora_A output groups
        self.bias_cat = torch.cat([self.bias["q"], self.bias["k"], self.bias["v"],
                                   torch.zeros(2 * rank, device=device)]).to(dtype)

    @classmethod
    def random(cls, hidden=1536, n_heads=12, n_kv=2, head_dim=128, rank=16, alpha=32, seed=0,
               dtype=torch.bfloat16, device="cuda"):
        """Random-init weights of the Qwen2.5 shape: W ~ N(0, 0.02) NF4-quantised (bs 64, double
        quant bs 256), biases ~ N(0, 0.02), LoRA A kaiming-uniform, B ~ N(0, 0.02)."""
        from .nf4_quant import quantize_nf4

        rng = np.random.default_rng(seed)
        states = {}
        for name, n_out in (("q", n_heads * head_dim), ("k", n_kv * head_dim), ("v", n_kv * head_dim)):
            states[name] = quantize_nf4((rng.standard_normal((n_out, hidden)) * 0.02).astype(np.float32))
        g = torch.Generator().manual_seed(seed)
        biases = {n: torch.randn(s, generator=g) * 0.02
                  for n, s in (("q", n_heads * head_dim), ("k", n_kv * head_dim), ("v", n_kv * head_dim))}
        bound = 1.0 / math.sqrt(hidden)  # kaiming_uniform_(a=sqrt(5)) on [rank, hidden]
        lora = {"a_q": (torch.rand(rank, hidden, generator=g) * 2 - 1) * bound,
                "b_q": torch.randn(n_heads * head_dim, rank, generator=g) * 0.02,
                "a_v": (torch.rand(rank, hidden, generator=g) * 2 - 1) * bound,
                "b_v": torch.randn(n_kv * head_dim, rank, generator=g) * 0.02}
        return cls(states, biases, lora, n_heads, n_kv, head_dim, alpha / rank, dtype, device)

    def lora_params(self):
        return [self.lora[n] for n in ("a_q", "b_q", "a_v", "b_v")]

    def dequant_cat(self) -> torch.Tensor:
        """This step's W_q, W_k, W_v (NF4 -> dtype, bit-exact) as the first rows of a fresh
        [(Hq+2Hk)*D + 2r, hidden] matrix; the fused forward fills the last 2r rows with A_q, A_v."""
        from .solution.nf4 import dequantize_nf4_many

        rows = [self.weights[n][1].shape[0] for n in ("q", "k", "v")]
        rank = self.lora["a_q"].shape[0]
        hidden = self.weights["q"][1].shape[1]
        w = torch.empty((sum(rows) + 2 * rank, hidden), dtype=self.dtype, device=self.device)
        items, r0 = [], 0
        for n, nr in zip(("q", "k", "v"), rows):
            packed, qs = self.weights[n]
            items.append((packed, qs, w[r0:r0 + nr]))
            r0 += nr
        dequantize_nf4_many(items, self.dtype)  # one launch for the three
        return w

    def forward(self, x: torch.Tensor, packing: Packing, cos: torch.Tensor, sin: torch.Tensor,
                fused: bool = True, norm: tuple | None = None):
        """x fp32 [T, hidden] (the normed hidden states) -> attention output [T, n_heads*D] (dtype).
        ``fused``: one projection GEMM + the sm_100a epilogues (FusedAttentionBlock); otherwise the
        reference's chain of autograd Functions (NF4Linear x3, LoRA, FusedQKRope, VarlenSDPA).
        With ``norm`` = (weight, eps) x is the decoder layer's input and the block starts with its
        input RMSNorm: inside the fused node's first kernel, or as RMSNormFn before the chain."""
        dt = self.dtype
        T = x.shape[0]
        if fused:
            a_q, b_q, a_v, b_v = self.lora_params()
            norm_w, eps = norm if norm is not None else (None, 0.0)
            out = FusedAttentionBlock.apply(x, a_q, b_q, a_v, b_v, self.dequant_cat(), self.bias_cat, cos, sin,
                                            packing.cu_seqlens(x.device), packing.max_len, self.n_heads,
                                            self.n_kv, self.scaling, self.head_dim ** -0.5, None, None, norm_w,
                                            eps)
            return out.view(T, self.n_heads * self.head_dim)
        if norm is not None:
            from .solution.rmsnorm import RMSNormFn
            x = RMSNormFn.apply(x, norm[0], norm[1])
        x16 = x.to(dt)
        (pq, sq), (pk, sk), (pv, sv) = self.weights["q"], self.weights["k"], self.weights["v"]
        q_base = NF4Linear.apply(x16, pq, self.bias["q"].to(dt), sq)
        k = NF4Linear.apply(x16, pk, self.bias["k"].to(dt), sk)
        v_base = NF4Linear.apply(x16, pv, self.bias["v"].to(dt), sv)
        a_q, b_q, a_v, b_v = self.lora_params()
        q_lora = F.linear(F.linear(x16, a_q.to(dt)), b_q.to(dt)) * self.scaling
        v_lora = F.linear(F.linear(x16, a_v.to(dt)), b_v.to(dt)) * self.scaling
        v = (v_base.float() + v_lora.float()).to(dt)
        q_rot, k_rot = FusedQKRope.apply(q_base.contiguous(), q_lora.to(dt).contiguous(), k.contiguous(),
                                         cos, sin, self.n_heads, self.n_kv)
        v_heads = v.view(1, T, self.n_kv, self.head_dim).transpose(1, 2)
        out = VarlenSDPA.apply(q_rot, k_rot, v_heads, packing.cu_seqlens(x.device), packing.max_len,
                               self.n_heads // self.n_kv, self.head_dim ** -0.5)
        return out.view(T, self.n_heads * self.head_dim)
