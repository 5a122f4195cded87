"""Qwen2RMSNorm on the B200 kernel and the norm_link recompute (solution/rmsnorm.py).

The parts on the attention block's path: ``RMSNormFn`` (so the recompute in the LoRA backward
is bit-identical to the forward, same kernel), ``recompute`` (solution/rmsnorm.py:76-80), and
``AddRMSNormFn`` / ``fusable`` (:108-155), the decoder's residual add + post-attention norm that
consumes the block's output.
"""

from __future__ import annotations

import torch

from .. import ops
from ._state import STATE, on_gpu


def _rows(x):
    x2 = x.reshape(-1, x.shape[-1])
    return x2 if x2.stride(-1) == 1 else x2.contiguous()


def _source(source):
    """A norm input given as the tensor or as (residual, delta) with input = residual + delta."""
    if isinstance(source, tuple):
        residual, delta = source
        return residual + delta
    return source


def recompute(source, weight, eps):
    """The norm's output for an input it ran on, bit-identical (same kernel, same launch)."""
    x = _source(source)
    y, _ = ops.rmsnorm_fwd(_rows(x), weight, eps, want_rstd=False)
    return y.view(x.shape)


class RMSNormFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weight, eps):
        x2 = _rows(x)
        y, rstd = ops.rmsnorm_fwd(x2, weight, eps)
        ctx.save_for_backward(x2, weight, rstd)
        ctx.shape = x.shape
        return y.view(x.shape)

    @staticmethod
    def backward(ctx, dy):
        x2, weight, rstd = ctx.saved_tensors
        dx = ops.rmsnorm_bwd(dy.reshape(x2.shape), x2, weight, rstd)
        return dx.view(ctx.shape), None, None


class ResidualGradLink:
    """Hands the residual path's gradient of a decoder layer's input to the fused attention block
    of the same layer, which adds it inside its input norm's backward (decik_rmsnorm_bwd_add)
    instead of autograd summing the two in a separate pass. The block arms the link in its forward
    (so only a block that will consume it gets one); AddRMSNormFn's backward, which runs before the
    block's, leaves the gradient here and returns none for its residual input."""

    def __init__(self):
        self.armed = False
        self.grad = None

    def take(self):
        g, self.grad = self.grad, None
        return g


class AddRMSNormFn(torch.autograd.Function):
    """``h = residual + delta; y = norm(h)``, both returned (solution/rmsnorm.py:108-144). h is not
    kept for backward: it is rebuilt from the residual (the layer input, kept by the input norm
    anyway) and delta (the 16-bit attention output). One sm_100a kernel each way
    (``decik_add_rmsnorm_fwd/bwd``); y equals RMSNormFn on the same h bit for bit, and the input
    gradient is grad_h + the norm's gradient, returned to both inputs (fp32, and in delta's dtype).

    With ``y16`` y comes out in delta's 16-bit dtype, for a consumer that computes in it (the patched
    MLP, whose first step is that cast): the fp32 y is never written, and y's gradient arrives in
    the same dtype and is read as it is. With an armed ``link`` (ResidualGradLink) the residual
    input's gradient goes to the link rather than to autograd."""

    @staticmethod
    def forward(ctx, residual, delta, weight, eps, y16=False, link=None):
        h, y, rstd = ops.add_rmsnorm_fwd(residual, delta, weight, eps, y16=y16)
        ctx.save_for_backward(residual, delta, weight, rstd)
        ctx.eps = eps
        ctx.link = link if (link is not None and link.armed) else None
        return h, y

    @staticmethod
    def backward(ctx, grad_h, grad_y):
        residual, delta, weight, rstd = ctx.saved_tensors
        if grad_y is None:
            if grad_h is None:
                return None, None, None, None, None, None
            total, total16 = grad_h, grad_h.to(delta.dtype)
        else:
            total, total16 = ops.add_rmsnorm_bwd(grad_y, grad_h, residual, delta, weight, rstd)
        if ctx.link is not None:
            ctx.link.grad = total
            total = None
        return total, total16, None, None, None, None


def fusable(module, x):
    """The sm_100a kernel can run this Qwen2RMSNorm on x (the patched forward's conditions,
    solution/rmsnorm.py:147-155)."""
    weight = getattr(module, "weight", None)
    return (isinstance(x, torch.Tensor) and on_gpu(x) and x.dtype == torch.float32 and x.numel() > 0
            and isinstance(weight, torch.Tensor) and on_gpu(weight)
            and weight.dtype in (torch.float32, torch.float16) and not weight.requires_grad
            and weight.dim() == 1 and x.shape[-1] == weight.shape[0] and x.shape[-1] <= 8192
            and x.shape[-1] % 4 == 0 and getattr(type(module).forward, "_skc", False))


def patch(norm_cls=None):
    """Patch Qwen2RMSNorm.forward (solution/rmsnorm.py:157-181); sets STATE.norm_link."""
    if norm_cls is None:
        from transformers.models.qwen2 import modeling_qwen2
        norm_cls = modeling_qwen2.Qwen2RMSNorm
    cls = norm_cls
    if getattr(cls.forward, "_skc", False):
        return
    original = cls.forward

    def forward(self, hidden_states):
        weight = getattr(self, "weight", None)
        if not (isinstance(hidden_states, torch.Tensor) and on_gpu(hidden_states)
                and hidden_states.dtype == torch.float32 and hidden_states.numel() > 0
                and isinstance(weight, torch.Tensor) and on_gpu(weight)
                and weight.dtype in (torch.float32, torch.float16) and not weight.requires_grad
                and weight.dim() == 1 and hidden_states.shape[-1] == weight.shape[0]
                and hidden_states.shape[-1] <= 8192 and hidden_states.shape[-1] % 4 == 0):
            return original(self, hidden_states)
        eps = float(self.variance_epsilon)
        out = RMSNormFn.apply(hidden_states, weight, eps)
        if STATE.packing_active:
            STATE.norm_link = (out, hidden_states, weight, eps)
        return out

    forward._skc = True
    cls.forward = forward
