"""Failure detection on the host, with no GPU fault (the data-parallel exchange's error paths).

Two gloo ranks on the CPU, each started with a short process-group timeout, as the bench and a
training loop start theirs:
- a rank that exits after joining: the survivor's LoRA-gradient all-reduce raises instead of
  waiting for good;
- a rank that is late past the timeout: the survivor's all-reduce raises within the timeout;
- ranks whose gradient buckets differ: GradBucket.check_layout raises ValueError on both ranks
  before any gradient is summed.
The reference's analogue is the harness's per-run timeout and process-group kill
(harness/common.py:88-119); the device-side half (a bounded wait that runs out and reports through
the error word) is tests/test_wait_limit_gpu.py.
"""

import datetime
import os
import socket
import time

import pytest
import torch
import torch.multiprocessing as mp

from decik_b200.dp import GradBucket

TIMEOUT_S = 3


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _put(queue, item):
    """Report and flush: os._exit below would drop a queued item its feeder thread has not sent."""
    queue.put(item)
    queue.close()
    queue.join_thread()


def _worker(rank, world, port, mode, queue):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=TIMEOUT_S))
    n_params = 3 if (mode == "mismatch" and rank == 0) else 2
    params = [torch.zeros(16, 8, requires_grad=True) for _ in range(n_params)]
    bucket = GradBucket(params)
    bucket.zero_()
    t0 = time.monotonic()
    try:
        if mode == "mismatch":
            bucket.check_layout()
            _put(queue, (rank, "no error", time.monotonic() - t0))
            return
        if rank == 1:
            if mode == "dead":
                _put(queue, (rank, "left", 0.0))
                os._exit(0)          # leaves without the collective and without a clean shutdown
            time.sleep(4 * TIMEOUT_S)  # "late": past the survivor's timeout
            _put(queue, (rank, "late", 0.0))
            os._exit(0)
        bucket.flat.fill_(1.0)
        bucket.all_reduce()
        _put(queue, (rank, "no error", time.monotonic() - t0))
    except (RuntimeError, ValueError) as e:
        _put(queue, (rank, f"{type(e).__name__}: {str(e)[:200]}", time.monotonic() - t0))
    os._exit(0)


def _run(mode):
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, mode, queue)) for r in range(2)]
    for p in procs:
        p.start()
    results = {}
    deadline = time.monotonic() + 120
    while len(results) < 2 and time.monotonic() < deadline:
        try:
            r, what, dt = queue.get(timeout=5)
            results[r] = (what, dt)
        except Exception:
            if all(not p.is_alive() for p in procs):
                break
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    return results


@pytest.mark.parametrize("mode", ["dead", "late"])
def test_survivor_raises_when_a_rank_is_gone_or_late(mode):
    res = _run(mode)
    assert 0 in res, f"rank 0 reported nothing: {res}"
    what, dt = res[0]
    assert what.startswith("RuntimeError"), f"rank 0 did not raise: {what}"
    # it gave up in bounded time: within the process-group timeout plus slack, not when the late
    # rank finally arrived (4 x the timeout) or never
    assert dt < 3 * TIMEOUT_S + 5, f"rank 0 waited {dt:.1f} s"


def test_mismatched_buckets_raise_on_every_rank():
    res = _run("mismatch")
    assert set(res) == {0, 1}, res
    for r in (0, 1):
        assert res[r][0].startswith("ValueError") and "layouts differ" in res[r][0], res[r]
