"""Data parallelism for the attention block: one process per GPU, whole sequences per rank.

The reference trains on one GPU and has no collective. Its rows never mix (each packed sequence
attends only to itself, solution/varlen.py:1-15), so the step shards by whole sequences with no
exchange inside the forward or backward: every rank runs the block on its own ``cu_seqlens``. The
only exchange is once per optimizer step, over the trainable parameters (the LoRA A/B matrices;
the NF4 weights are frozen and replicated):

* ``partition_rows`` splits a global batch of rows across ranks, balancing the two costs of a row:
  its tokens (projections, RoPE, LoRA: linear in L) and its causal attention (quadratic in L).
* ``global_count`` all-reduces the number of labelled tokens, the loss normaliser of the
  reference's head (solution/head.py:157-163), so the per-rank losses sum to the 1-GPU loss.
* ``GradBucket`` lays the LoRA gradients out as views of one flat fp32 buffer, so autograd
  accumulates straight into it and one all-reduce moves them all, with no gather copy.
"""

from __future__ import annotations

import heapq

import torch


def row_cost(length: int, attn_weight: float) -> float:
    """Relative cost of one row: tokens plus ``attn_weight`` x causal score pairs."""
    return float(length) + attn_weight * length * (length + 1) / 2.0


def partition_rows(lengths, world: int, attn_weight: float = 1.0 / 1024.0) -> list[list[int]]:
    """Indices of the rows each rank trains, balanced by ``row_cost``.

    Longest-processing-time greedy: rows in decreasing cost go to the least loaded rank (ties to
    the lower rank), then each rank's rows are put back in batch order. Deterministic, so every
    rank computes the same split without communicating. The default ``attn_weight`` is the 1.5B
    block's ratio of attention FLOPs per score pair (4 x 12 heads x 128) to projection FLOPs per
    token (2 x 1536 x 2048 outputs of q, k, v) = 1/1024: a row of 2047 tokens spends as much on
    attention as on its projections."""
    if world < 1:
        raise ValueError("world must be >= 1")
    lengths = [int(n) for n in lengths]
    if any(n < 0 for n in lengths):
        raise ValueError("row lengths must be >= 0")
    order = sorted(range(len(lengths)), key=lambda i: (-row_cost(lengths[i], attn_weight), i))
    heap = [(0.0, r) for r in range(world)]
    parts: list[list[int]] = [[] for _ in range(world)]
    for i in order:
        load, r = heapq.heappop(heap)
        parts[r].append(i)
        heapq.heappush(heap, (load + row_cost(lengths[i], attn_weight), r))
    return [sorted(p) for p in parts]


def global_count(n_local, group=None) -> torch.Tensor:
    """Sum over ranks of a per-rank count (a tensor or an int), as a float32 tensor on the count's
    device (or the CPU for an int)."""
    import torch.distributed as dist

    t = (n_local.detach().to(torch.float32).reshape(1).clone() if torch.is_tensor(n_local)
         else torch.tensor([float(n_local)], dtype=torch.float32))
    if dist.is_available() and dist.is_initialized() and dist.get_world_size(group) > 1:
        dist.all_reduce(t, group=group)
    return t[0]


class GradBucket:
    """The gradients of ``params`` as views of one flat fp32 buffer.

    ``zero_()`` (before each backward) clears the buffer and points every ``param.grad`` at its
    slice; autograd then accumulates into the slices in place. ``all_reduce()`` sums (and with
    ``average`` divides by the world size) across ranks in one collective, optionally async so it
    overlaps later backward work."""

    def __init__(self, params, device=None):
        self.params = list(params)
        if not self.params:
            raise ValueError("GradBucket needs at least one parameter")
        for p in self.params:
            if p.dtype != torch.float32:
                raise ValueError("GradBucket holds fp32 parameters only")
        device = device if device is not None else self.params[0].device
        self.flat = torch.zeros(sum(p.numel() for p in self.params), dtype=torch.float32, device=device)
        self.views, off = [], 0
        for p in self.params:
            self.views.append(self.flat[off:off + p.numel()].view(p.shape))
            off += p.numel()

    @property
    def nbytes(self) -> int:
        return self.flat.numel() * 4

    def zero_(self):
        self.flat.zero_()
        for p, v in zip(self.params, self.views):
            p.grad = v

    def check_in_place(self):
        """Raise if autograd replaced a view instead of accumulating into it."""
        for p, v in zip(self.params, self.views):
            if p.grad is None or p.grad.data_ptr() != v.data_ptr():
                raise RuntimeError("a gradient left the bucket (was .grad reassigned?)")

    def check_layout(self, group=None):
        """Raise ValueError on every rank unless all ranks hold buckets of the same layout (the
        same number of parameters with the same sizes). Run once before the first all_reduce: a
        rank whose bucket differs would otherwise sum unrelated gradients or wait for a collective
        of another size. Cost: one all-gather of a few integers."""
        import torch.distributed as dist

        if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size(group) == 1:
            return
        sizes = [p.numel() for p in self.params]
        sig = torch.tensor([len(sizes), self.flat.numel(), hash(tuple(sizes)) & 0x7FFFFFFF], dtype=torch.int64,
                           device=self.flat.device)
        every = [torch.empty_like(sig) for _ in range(dist.get_world_size(group))]
        dist.all_gather(every, sig, group=group)
        if any(not torch.equal(e, sig) for e in every):
            rows = ", ".join(f"rank {r}: {int(e[0])} params / {int(e[1])} values" for r, e in enumerate(every))
            raise ValueError(f"GradBucket layouts differ across ranks ({rows})")

    def all_reduce(self, group=None, average: bool = False, async_op: bool = False):
        import torch.distributed as dist

        self.check_in_place()
        if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size(group) == 1:
            return None
        if average:
            self.flat.div_(dist.get_world_size(group))
        return dist.all_reduce(self.flat, group=group, async_op=async_op)
