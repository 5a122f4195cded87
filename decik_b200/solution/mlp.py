"""Qwen2 MLP with NF4 gate / up / down as one autograd node on the B200 kernels (solution/mlp.py).

The reference (solution/mlp.py:62-163, ``RecomputedMLP``) feeds the three NF4 projections a 16-bit
input and keeps gate and up in 16 bits, since their values are exactly 16-bit matmul outputs. It
runs SwiGLU, returns the 16-bit output, and recomputes gate and up in backward to save memory.
The bitsandbytes base path it replaces casts every projection's output back to the fp32 input
dtype and runs SwiGLU in fp32.

Here, with 180 GB of HBM per GPU, the node:
- dequantises W_gate, W_up (into one [2 * inter, hidden] matrix) and W_down in one launch;
- computes gate | up as ONE tcgen05 GEMM whose epilogue also applies SwiGLU (decik_mlp_gate_up):
  gate and up are rounded to the compute dtype and kept, and silu(gate) * up is computed from them
  with the separate SwiGLU kernel's fp32 arithmetic, rounded once;
- keeps the dequantised weights and gate | up for the backward: no recompute, no second dequant;
- computes grad_hidden = grad . W_down with the SwiGLU backward in the GEMM's epilogue
  (decik_mlp_down_grad: grad_hidden never reaches HBM), then the input gradient as one GEMM over
  [dgate | dup] with fp32 output. That sums the two projections' input gradients in fp32 inside the
  GEMM, where the reference casts each to fp32 and adds.

The two plain GEMMs (down projection, input gradient) have nothing to fuse and run on cuBLAS: at
N = hidden = 1536 cuBLAS's clustered tiles (TMA multicast, which this project's kernels do not use)
are 10-20% faster than decik_gemm16 / decik_proj_dx on these shapes. The MLP sits outside the
attention block.

The output is in the projections' compute dtype, as the reference's node returns fp16.
"""

from __future__ import annotations

import torch

from .. import ops
from ._state import on_gpu
from .nf4 import dequantize_nf4_many, supported


class FusedMLP(torch.autograd.Function):
    """down(silu(gate(x)) * up(x)) with frozen dequantised weights: ``w_gu`` [2 * inter, hidden]
    (W_gate rows then W_up rows) and ``w_down`` [hidden, inter] in the compute dtype (the Qwen2 MLP
    has no biases). Gradient for x (returned in x's dtype).

    With ``residual`` (the decoder layer's fp32 stream, x's shape) the node returns
    residual + mlp(x) in fp32 from the down projection's GEMM (beta = 1, fp32 output): the layer's
    residual add (solution/varlen.py:343) needs no pass of its own, and the MLP output is added
    before any 16-bit rounding. The residual's gradient is the output's. A contiguous residual that
    is not a leaf requiring grad is updated in place and returned (marked dirty): the patched
    decoder layer's stream, which no node keeps for backward."""

    @staticmethod
    def forward(ctx, x, w_gu, w_down, residual=None):
        inter = w_down.shape[1]
        shape = x.shape
        x16 = x.reshape(-1, shape[-1]).to(w_gu.dtype).contiguous()
        gu, hidden = ops.mlp_gate_up(x16, w_gu)            # [T, 2 * inter], [T, inter]
        ctx.save_for_backward(gu, w_gu, w_down)
        ctx.in_dtype, ctx.shape, ctx.inter = x.dtype, shape, inter
        ctx.residual = residual is not None
        if residual is None:
            out = torch.mm(hidden, w_down.t())             # [T, hidden], plain GEMM
            return out.view(*shape[:-1], out.shape[-1])
        r2 = residual.reshape(-1, residual.shape[-1])
        if residual.is_contiguous() and not (residual.is_leaf and residual.requires_grad):
            # into the residual itself (no node keeps it): addmm into a new tensor first copies the
            # residual there (330.7 -> 293.9 us at 16,384 tokens, same bits)
            torch.addmm(r2, hidden, w_down.t(), out_dtype=torch.float32, out=r2)
            ctx.mark_dirty(residual)
            return residual
        out = torch.addmm(r2, hidden, w_down.t(), out_dtype=torch.float32)
        return out.view(*shape[:-1], out.shape[-1])

    @staticmethod
    def backward(ctx, grad_out):
        gu, w_gu, w_down = ctx.saved_tensors
        g16 = grad_out.reshape(-1, grad_out.shape[-1]).to(w_down.dtype).contiguous()
        dgu = ops.mlp_down_grad(g16, w_down, gu)           # [T, 2 * inter] = [dgate | dup]
        if ctx.in_dtype == torch.float32:
            dx = torch.mm(dgu, w_gu, out_dtype=torch.float32)  # both input gradients summed in fp32
        else:  # a 16-bit input: the fp32 sum rounded once to its dtype
            dx = torch.mm(dgu, w_gu)
        return dx.to(ctx.in_dtype).view(ctx.shape), None, None, (grad_out if ctx.residual else None)


def mlp_weights(gate_proj, up_proj, down_proj, dtype):
    """(w_gu, w_down): this step's dequantised weights, one dequant launch."""
    gq, uq, dq = (p.weight.quant_state for p in (gate_proj, up_proj, down_proj))
    inter, hidden = gq.shape
    dev = gate_proj.weight.device
    w_gu = torch.empty((2 * inter, hidden), dtype=dtype, device=dev)
    w_down = torch.empty(tuple(dq.shape), dtype=dtype, device=dev)
    dequantize_nf4_many([(gate_proj.weight.data, gq, w_gu[:inter]), (up_proj.weight.data, uq, w_gu[inter:]),
                         (down_proj.weight.data, dq, w_down)], dtype)
    return w_gu, w_down


def patch(linear4bit_cls=None):
    """Patch Qwen2MLP.forward (solution/mlp.py:113-163). Eligible: an input on the GPU, the silu
    activation, and three bias-free NF4 Linear4bit projections with one 16-bit compute dtype and
    frozen weights, inter a multiple of 256 (the GEMM tiles). Anything else runs the original
    forward."""
    from transformers.models.qwen2 import modeling_qwen2

    if linear4bit_cls is None:
        import bitsandbytes as bnb
        linear4bit_cls = bnb.nn.Linear4bit
    cls = modeling_qwen2.Qwen2MLP
    if getattr(cls.forward, "_skc", False):
        return
    original = cls.forward

    def nf4_projection(module, n_in, dtype):
        weight = getattr(module, "weight", None)
        bias = getattr(module, "bias", None)
        return (isinstance(module, linear4bit_cls) and getattr(module, "compute_dtype", None) == dtype
                and weight is not None and on_gpu(weight) and weight.dtype == torch.uint8
                and not weight.requires_grad and bias is None
                and supported(getattr(weight, "quant_state", None), n_in))

    def eligible(self, x):
        """The node's compute dtype if it runs on x, else None."""
        config = getattr(self, "config", None)
        gate, up, down = (getattr(self, n, None) for n in ("gate_proj", "up_proj", "down_proj"))
        dtype = getattr(gate, "compute_dtype", None)
        ok = (isinstance(x, torch.Tensor) and on_gpu(x) and x.numel() > 0
              and x.dtype in (torch.float32, torch.float16, torch.bfloat16)
              and getattr(config, "hidden_act", None) == "silu" and dtype in (torch.float16, torch.bfloat16)
              and nf4_projection(gate, x.shape[-1], dtype) and nf4_projection(up, x.shape[-1], dtype)
              and gate.weight.quant_state.shape == up.weight.quant_state.shape
              and nf4_projection(down, gate.weight.quant_state.shape[0], dtype)
              and gate.weight.quant_state.shape[0] % 256 == 0 and x.shape[-1] % 8 == 0)
        return dtype if ok else None

    def forward(self, x, residual=None):
        # ``residual``: the patched decoder layer's fp32 stream; the result is then residual + mlp(x)
        dtype = eligible(self, x)
        if dtype is None:
            out = original(self, x)
            return out if residual is None else residual + out
        gate, up, down = self.gate_proj, self.up_proj, self.down_proj
        w_gu, w_down = mlp_weights(gate, up, down, dtype)
        if residual is not None and not (residual.dtype == torch.float32 and residual.shape == x.shape
                                         and residual.is_contiguous()):
            return residual + FusedMLP.apply(x, w_gu, w_down)
        return FusedMLP.apply(x, w_gu, w_down, residual)

    forward._skc = True
    forward._skc_eligible = eligible  # the patched decoder layer asks before choosing its norm's dtype
    cls.forward = forward
