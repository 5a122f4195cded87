"""NF4 4-bit linear layers with the dequant on the B200 kernel (solution/nf4.py).

``dequantize_nf4`` and ``NF4Linear`` keep the reference's names, arguments and results
(solution/nf4.py:66-104): forward = dequantize the whole weight + ``F.linear``, backward =
dequantize again + one matmul for the input gradient (the weight is frozen). The dequant is
``decik_nf4_dequant`` (bit-exact, sm_100a); the weight comes out in the activation's dtype
(fp16 as in the reference, or bf16).
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

from .. import ops
from ._state import on_gpu


def supported(quant_state, n_in=None):
    """Same acceptance test as solution/nf4.py:51-63, plus bf16 as a weight dtype."""
    qs = quant_state
    try:
        ok = (qs is not None and qs.quant_type == "nf4"
              and qs.dtype in (torch.float16, torch.bfloat16)
              and len(qs.shape) == 2 and (qs.shape[0] * qs.shape[1]) % 2 == 0
              and qs.blocksize % 2 == 0 and qs.code is not None)
        if ok and qs.nested:
            ok = qs.state2 is not None and qs.offset is not None and qs.absmax.dtype == torch.uint8
        if ok and n_in is not None:
            ok = qs.shape[1] == n_in
        return bool(ok)
    except AttributeError:
        return False


def dequantize_nf4(packed, quant_state, dtype=torch.float16, out=None):
    """[N, K] weights of a bitsandbytes nf4 tensor (packed uint8 + QuantState), solution/nf4.py:66-85.
    ``out`` (optional, contiguous [N, K] of ``dtype``) receives them, e.g. rows of a larger matrix."""
    qs = quant_state
    code = qs.code if qs.code.device == packed.device else qs.code.to(packed.device)
    if qs.nested:
        offset = qs.offset
        if not torch.is_tensor(offset):
            offset = torch.tensor([float(offset)], dtype=torch.float32, device=packed.device)
        return ops.nf4_dequant(packed, qs.absmax, code, qs.shape, qs.blocksize,
                               absmax2=qs.state2.absmax, code2=qs.state2.code,
                               offset=offset.reshape(1).to(device=packed.device, dtype=torch.float32),
                               blocksize2=qs.state2.blocksize, out_dtype=dtype, out=out)
    return ops.nf4_dequant(packed, qs.absmax, code, qs.shape, qs.blocksize, out_dtype=dtype, out=out)


def dequantize_nf4_many(items, dtype):
    """Several weights at once, one launch: ``items`` = [(packed, quant_state, out)], each out a
    contiguous [N, K] of ``dtype`` (e.g. the row slices of one matrix). Same values as
    dequantize_nf4 per item."""
    jobs = []
    for packed, qs, out in items:
        code = qs.code if qs.code.device == packed.device else qs.code.to(packed.device)
        if qs.nested:
            offset = qs.offset
            if not torch.is_tensor(offset):
                offset = torch.tensor([float(offset)], dtype=torch.float32, device=packed.device)
            jobs.append((packed, qs.absmax, code, qs.shape, qs.blocksize, qs.state2.absmax, qs.state2.code,
                         offset.reshape(1).to(device=packed.device, dtype=torch.float32), qs.state2.blocksize, out))
        else:
            jobs.append((packed, qs.absmax, code, qs.shape, qs.blocksize, None, None, None, 256, out))
    ops.nf4_dequant_batch(jobs, dtype)


class NF4Linear(torch.autograd.Function):
    """F.linear(x, dequant(W), bias) with 16-bit x; the input gradient dequantizes W again, as
    bitsandbytes' MatMul4Bit does (solution/nf4.py:88-104)."""

    @staticmethod
    def forward(ctx, x16, packed, bias16, quant_state):
        weight = dequantize_nf4(packed, quant_state, x16.dtype)
        ctx.packed, ctx.quant_state, ctx.dtype = packed, quant_state, x16.dtype
        return F.linear(x16, weight, bias16)

    @staticmethod
    def backward(ctx, grad_out):
        grad_x = None
        if ctx.needs_input_grad[0]:
            weight = dequantize_nf4(ctx.packed, ctx.quant_state, ctx.dtype)
            grad_x = torch.matmul(grad_out.to(weight.dtype), weight)
        return grad_x, None, None, None


def patch(linear4bit_cls=None):
    """Patch ``bitsandbytes.nn.Linear4bit.forward`` (solution/nf4.py:107-138). The class may be
    passed in (tests use a stand-in with the same fields); by default bitsandbytes is imported."""
    if linear4bit_cls is None:
        import bitsandbytes as bnb
        linear4bit_cls = bnb.nn.Linear4bit
    cls = linear4bit_cls
    if getattr(cls.forward, "_skc", False):
        return
    original = cls.forward

    def forward(self, x):
        weight = getattr(self, "weight", None)
        qs = getattr(weight, "quant_state", None)
        bias = self.bias
        compute = getattr(self, "compute_dtype", None)
        if not (isinstance(x, torch.Tensor) and on_gpu(x) and x.numel() > 0
                and weight is not None and on_gpu(weight) and weight.dtype == torch.uint8
                and not weight.requires_grad and compute in (torch.float16, torch.bfloat16)
                and (bias is None or not bias.requires_grad)
                and supported(qs, x.shape[-1])):
            return original(self, x)
        inp_dtype = x.dtype
        bias16 = None if bias is None else bias.to(compute)
        out = NF4Linear.apply(x.to(compute), weight.data, bias16, qs)
        return out.to(inp_dtype)

    forward._skc = True
    cls.forward = forward
