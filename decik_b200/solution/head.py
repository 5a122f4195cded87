"""Output head + cross entropy without the [tokens x vocab] logits tensor (solution/head.py).

``FusedHeadLoss`` keeps the reference's interface and results (solution/head.py:88-139):
- it takes the real tokens' hidden states, the frozen 16-bit head weight, the shifted targets and
  the loss denominator;
- it returns (loss, entropy, token_loss, hit) and a gradient for the hidden states only.

The labelled tokens go first. The head runs CHUNK_ROWS rows at a time:
1. one cuBLAS GEMM makes a 16-bit logits chunk, the only vocabulary-sized buffer;
2. ``decik_head_stats`` (sm_100a) makes one pass per row for lse, entropy, argmax and the
   target's loss, and a second pass for labelled rows that writes softmax - onehot over the logits;
3. one more GEMM, with fp32 output, turns that into the hidden-state gradient, which backward
   scales by the incoming gradient and 1 / denominator.

The reference hooks ``run_head`` into TRL / Soup's trainer (solution/head.py:178-260). Those
classes are not part of this build; ``decik_b200.qlora_model.qlora_train_step`` calls
``run_head`` instead.
"""

from __future__ import annotations

import types

import torch
import torch.nn.functional as F

from .. import ops
from ._state import STATE

IGNORE_INDEX = -100
CHUNK_ROWS = 2048  # 2048 x 151,936 x 2 bytes = 594 MiB of logits per chunk


class FusedHeadLoss(torch.autograd.Function):
    """(sum of the labelled tokens' cross entropy) / denominator, plus per-token entropy, loss and
    argmax hit; the gradient flows to ``hidden`` only (the head is frozen)."""

    @staticmethod
    def forward(ctx, hidden, weight16, targets, denominator):
        n_tok, n_hidden = hidden.shape
        n_vocab = weight16.shape[0]
        device = hidden.device
        with torch.autocast(device_type=device.type, enabled=False):
            labelled = targets != IGNORE_INDEX
            # labelled tokens first: their gradient matmul then runs on a contiguous prefix
            order = torch.argsort((~labelled).to(torch.int8), stable=True)
            n_lab = int(labelled.sum().item())
            target_sorted = targets.index_select(0, order).contiguous()
            h16 = hidden.detach().index_select(0, order).to(weight16.dtype)
            lse = torch.empty(n_tok, dtype=torch.float32, device=device)
            entropy = torch.empty_like(lse)
            token_loss = torch.empty_like(lse)
            hit = torch.empty(n_tok, dtype=torch.int32, device=device)
            grad = torch.empty((n_lab, n_hidden), dtype=torch.float32, device=device)
            buffer = torch.empty((max(1, min(CHUNK_ROWS, n_tok)), n_vocab), dtype=weight16.dtype, device=device)
            for start in range(0, n_tok, CHUNK_ROWS):
                stop = min(start + CHUNK_ROWS, n_tok)
                logits = buffer[: stop - start]
                torch.mm(h16[start:stop], weight16.t(), out=logits)
                a, b, c, d = ops.head_stats(logits, target_sorted[start:stop])
                lse[start:stop], entropy[start:stop], token_loss[start:stop], hit[start:stop] = a, b, c, d
                with_grad = min(stop, n_lab) - start
                if with_grad > 0:
                    grad[start:start + with_grad] = torch.mm(logits[:with_grad], weight16, out_dtype=torch.float32)
            loss = token_loss.sum() / denominator
            entropy_out = torch.empty_like(entropy).index_copy_(0, order, entropy)
            loss_out = torch.empty_like(token_loss).index_copy_(0, order, token_loss)
            hit_out = torch.empty_like(hit).index_copy_(0, order, hit)
        ctx.save_for_backward(grad, order[:n_lab])
        ctx.n_tok, ctx.dtype, ctx.denominator = n_tok, hidden.dtype, denominator
        ctx.mark_non_differentiable(entropy_out, loss_out, hit_out)
        return loss, entropy_out, loss_out, hit_out

    @staticmethod
    def backward(ctx, grad_loss, *unused):
        grad, positions = ctx.saved_tensors
        grad_hidden = torch.zeros((ctx.n_tok, grad.shape[1]), dtype=torch.float32, device=grad.device)
        grad_hidden.index_copy_(0, positions, grad * (grad_loss.float() / ctx.denominator))
        return grad_hidden.to(ctx.dtype), None, None, None


def shift_labels(labels):
    """Position t is scored against token t + 1, as ForCausalLMLoss does (solution/head.py:142-144)."""
    return F.pad(labels, (0, 1), value=IGNORE_INDEX)[..., 1:]


def run_head(model, hidden, labels, attention_mask, num_items_in_batch, packing, dtype=torch.bfloat16):
    """The loss of one step from the decoder's output (solution/head.py:147-171): the real tokens'
    hidden states (the packed sequence, or the mask's positions of a padded batch) through
    FusedHeadLoss; the per-token statistics go to ``STATE.stats``."""
    batch, seq = labels.shape
    n_hidden = hidden.shape[-1]
    if packing is not None:  # the decoder already ran on the real tokens only
        positions = packing.index
        flat = hidden.reshape(-1, n_hidden)
    else:
        positions = attention_mask.reshape(-1).nonzero().squeeze(1)
        flat = hidden.reshape(-1, n_hidden).index_select(0, positions)
    targets = shift_labels(labels).reshape(-1).index_select(0, positions).to(flat.device)
    weight = model.lm_head.weight
    weight16 = weight if weight.dtype == dtype else weight.to(dtype)
    labelled = (targets != IGNORE_INDEX).sum()
    if num_items_in_batch is None:
        denominator = labelled.to(torch.float32)
    elif torch.is_tensor(num_items_in_batch):
        denominator = num_items_in_batch.to(flat.device)
    else:
        denominator = num_items_in_batch
    loss, entropy, token_loss, hit = FusedHeadLoss.apply(flat, weight16.detach(), targets, denominator)
    loss_grid = torch.zeros(batch * seq, dtype=torch.float32, device=flat.device)
    loss_grid.index_copy_(0, positions, token_loss)
    STATE.stats = types.SimpleNamespace(entropy_sum=entropy.sum(), correct=hit.sum(), labelled=labelled,
                                        token_loss=loss_grid.view(batch, seq))
    return loss
