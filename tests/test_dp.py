"""Data-parallel host logic on the CPU (gloo, world size 2): whole-row partitioning, the global
loss normaliser and the flat LoRA-gradient bucket. Two ranks each run the fp32 oracle block on
their own rows; the all-reduced loss and LoRA gradients must equal one process running every row.
"""

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from decik_b200.dp import GradBucket, global_count, partition_rows, row_cost

HIDDEN, HQ, HK, D = 128, 4, 2, 32
LENGTHS = [37, 5, 80, 12, 60, 3, 25, 1, 44]


def _weights():
    g = torch.Generator().manual_seed(7)
    w = {n: torch.randn(o, HIDDEN, generator=g) * 0.05 for n, o in (("w_q", HQ * D), ("w_k", HK * D), ("w_v", HK * D))}
    w.update({n: torch.randn(o, generator=g) * 0.05 for n, o in (("b_q", HQ * D), ("b_k", HK * D), ("b_v", HK * D))})
    lora = {"a_q": torch.randn(8, HIDDEN, generator=g) * 0.1, "bb_q": torch.randn(HQ * D, 8, generator=g) * 0.1,
            "a_v": torch.randn(8, HIDDEN, generator=g) * 0.1, "bb_v": torch.randn(HK * D, 8, generator=g) * 0.1}
    return w, lora


def _row(i):
    """Row i's inputs, a fixed direction per output token, and its labelled-token mask."""
    L = LENGTHS[i]
    g = torch.Generator().manual_seed(1000 + i)
    x = torch.randn(L, HIDDEN, generator=g)
    r = torch.randn(L, HQ * D, generator=g)
    lab = torch.arange(L) >= L // 3
    return x, r, lab


def _local_loss(rows, w, params, normaliser):
    """Sum over the labelled tokens of rows of out . r, divided by the global labelled count."""
    from oracle.block import block_forward

    x = torch.cat([_row(i)[0] for i in rows])
    r = torch.cat([_row(i)[1] for i in rows])
    lab = torch.cat([_row(i)[2] for i in rows])
    spans, s = [], 0
    for i in rows:
        spans.append((s, LENGTHS[i]))
        s += LENGTHS[i]
    pos = torch.cat([torch.arange(LENGTHS[i]) for i in rows]).float()
    inv = 1.0 / (10000.0 ** (torch.arange(0, D, 2).float() / D))
    ang = pos[:, None] * inv[None]
    ang = torch.cat((ang, ang), dim=-1)
    out = block_forward(x, w["w_q"], w["w_k"], w["w_v"], w["b_q"], w["b_k"], w["b_v"], params[0], params[1],
                        params[2], params[3], 2.0, ang.cos(), ang.sin(), spans, HQ, HK)
    return ((out * r).sum(-1) * lab).sum() / normaliser, int(lab.sum())


def _worker(rank, world, port, out_path):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        w, lora = _weights()
        params = [lora[n].clone().requires_grad_(True) for n in ("a_q", "bb_q", "a_v", "bb_v")]
        rows = partition_rows(LENGTHS, world)[rank]
        n_lab = sum(int(_row(i)[2].sum()) for i in rows)
        normaliser = global_count(n_lab)
        bucket = GradBucket(params)
        for _ in range(2):                 # twice: zero_() must reset the accumulation
            bucket.zero_()
            loss, _ = _local_loss(rows, w, params, normaliser)
            loss.backward()
            bucket.all_reduce()
        total = loss.detach().reshape(1).clone()
        dist.all_reduce(total)
        if rank == 0:
            torch.save({"loss": total[0], "flat": bucket.flat.clone(), "normaliser": normaliser,
                        "rows": partition_rows(LENGTHS, world)}, out_path)
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_partition_covers_rows_and_balances():
    for world in (1, 2, 3, 4, 8):
        parts = partition_rows(LENGTHS, world)
        assert len(parts) == world
        assert sorted(i for p in parts for i in p) == list(range(len(LENGTHS)))
        assert all(p == sorted(p) for p in parts)
        loads = [sum(row_cost(LENGTHS[i], 1 / 1024) for i in p) for p in parts]
        # LPT greedy: no rank exceeds the lightest by more than the costliest row
        assert max(loads) - min(loads) <= max(row_cost(n, 1 / 1024) for n in LENGTHS) + 1e-9
    assert partition_rows([], 2) == [[], []]
    assert partition_rows([5], 3) == [[0], [], []]
    with pytest.raises(ValueError):
        partition_rows([3, -1], 2)
    with pytest.raises(ValueError):
        partition_rows([3], 0)


def test_partition_weighs_attention():
    # one 4096-row against eight 512-rows: by tokens alone 4096 = 8 x 512, by attention the long
    # row is heavier, so it goes alone and the short rows share the other rank
    parts = partition_rows([4096] + [512] * 8, 2)
    assert parts[0] == [0] and parts[1] == list(range(1, 9))
    parts = partition_rows([4096] + [512] * 9, 2)
    assert parts[0] == [0]


def test_grad_bucket_views_take_autograd_in_place():
    a = torch.randn(3, 4, requires_grad=True)
    b = torch.randn(5, requires_grad=True)
    bucket = GradBucket([a, b])
    assert bucket.nbytes == 17 * 4
    bucket.zero_()
    ((a * 2).sum() + (b ** 2).sum()).backward()
    bucket.check_in_place()
    assert torch.equal(bucket.flat[:12], torch.full((12,), 2.0))
    assert torch.allclose(bucket.flat[12:], 2 * b.detach())
    bucket.all_reduce()                     # no process group: a no-op
    a.grad = torch.zeros(3, 4)
    with pytest.raises(RuntimeError):
        bucket.check_in_place()
    with pytest.raises(ValueError):
        GradBucket([torch.zeros(2, dtype=torch.float16, requires_grad=True)])


def test_dp_two_ranks_match_one_process(tmp_path):
    out_path = str(tmp_path / "rank0.pt")
    mp.spawn(_worker, args=(2, _free_port(), out_path), nprocs=2, join=True)
    got = torch.load(out_path)
    assert got["rows"][0] and got["rows"][1]

    w, lora = _weights()
    params = [lora[n].clone().requires_grad_(True) for n in ("a_q", "bb_q", "a_v", "bb_v")]
    n_lab = sum(int(_row(i)[2].sum()) for i in range(len(LENGTHS)))
    assert float(got["normaliser"]) == n_lab
    loss, _ = _local_loss(list(range(len(LENGTHS))), w, params, float(n_lab))
    loss.backward()
    flat = torch.cat([p.grad.reshape(-1) for p in params])
    loss = loss.item()
    assert abs(float(got["loss"]) - loss) <= 1e-5 * abs(loss)
    rel = (got["flat"] - flat).norm() / flat.norm()
    assert rel < 1e-5, rel
