"""The device-built packing (decik_pack_rows through solution.varlen.plan) against the oracle's
restatement of the reference's plan() (oracle/packing.py, solution/varlen.py:191-226): index,
positions, cu_seqlens, spans and max_len bit for bit, the packed ids, and None for masks the
reference does not pack (left padding, a hole, an empty row)."""

import numpy as np
import pytest
import torch

from oracle import packing as o_pack

pytestmark = pytest.mark.gpu


def _mask(lengths, seq, dtype=torch.int64):
    m = torch.zeros(len(lengths), seq, dtype=torch.int64)
    for i, L in enumerate(lengths):
        m[i, :L] = 1
    return m.to(dtype)


def _check(mask, ids):
    from decik_b200 import ops

    got = ops.pack_rows(mask.cuda(), ids.cuda())
    ref = o_pack.plan(mask.to(torch.int64).numpy())
    assert got is not None and ref is not None
    lengths, cu, index, positions, packed_ids = got
    assert np.array_equal(index.cpu().numpy(), ref["index"])
    assert np.array_equal(positions.cpu().numpy(), ref["positions"])
    assert np.array_equal(cu.cpu().numpy(), ref["cu_seqlens"])
    assert max(lengths) == ref["max_len"] and sum(lengths) == ref["n_tokens"]
    assert np.array_equal(packed_ids.cpu().numpy(), ids.reshape(-1).numpy()[ref["index"]])


@pytest.mark.parametrize("dtype", [torch.int64, torch.int32, torch.bool, torch.uint8])
def test_pack_rows_reference_spans(cuda_lib, dtype):
    # the reference test's rows (solution/test_solution.py:76: spans of 401, 77, 512, 3 tokens)
    lengths = [401, 77, 512, 3]
    mask = _mask(lengths, 512, dtype)
    ids = torch.randint(0, 151936, mask.shape, generator=torch.Generator().manual_seed(0))
    _check(mask, ids)


def test_pack_rows_random_right_padded_batches(cuda_lib):
    rng = np.random.default_rng(1)
    for B, S in ((1, 1), (3, 33), (25, 4096), (300, 700), (1100, 64)):
        lengths = rng.integers(1, S + 1, size=B).tolist()
        lengths[0] = S  # one full row
        mask = _mask(lengths, S)
        ids = torch.randint(0, 1000, mask.shape, generator=torch.Generator().manual_seed(B))
        _check(mask, ids)


def test_pack_rows_rejects_what_the_reference_does_not_pack(cuda_lib):
    from decik_b200 import ops

    mask = _mask([9, 3, 5, 1], 9)
    left = mask.clone()
    left[1, 0] = 0                                     # left padding
    hole = mask.clone()
    hole[0, 4] = 0                                     # a zero inside a row
    for bad in (left, hole):
        assert o_pack.plan(bad.numpy()) is None
        assert ops.pack_rows(bad.cuda()) is None
    empty = mask.clone()
    empty[3, 0] = 0                                    # an empty row: packed by the kernel, refused by plan()
    got = ops.pack_rows(empty.cuda())
    assert got is not None and got[0][3] == 0 and o_pack.plan(empty.numpy()) is None


def test_plan_builds_the_packed_batch(cuda_lib):
    """solution.varlen.plan on an eligible call: the PackedBatch's spans / cu_seqlens / ids, and
    None for an empty row."""
    from decik_b200.solution import varlen
    from decik_b200.solution._state import STATE

    class Model(torch.nn.Module):
        class config:
            _attn_implementation = "sdpa"
            layer_types = ["full_attention"]

    model = Model().train()
    mask = _mask([5, 2, 7], 8).cuda()
    ids = torch.arange(24, device="cuda").view(3, 8)
    prev = STATE.request
    STATE.request = True
    try:
        with torch.enable_grad():
            p = varlen.plan(model, ids, mask, None, None, None, False, {})
            assert p is not None
            assert p.spans == [(0, 5), (5, 2), (7, 7)] and p.max_len == 7 and p.n_tokens == 14
            assert p.cu_seqlens("cuda").tolist() == [0, 5, 7, 14]
            assert p.ids.tolist() == [0, 1, 2, 3, 4, 8, 9, 16, 17, 18, 19, 20, 21, 22]
            mask[1] = 0
            assert varlen.plan(model, ids, mask, None, None, None, False, {}) is None
    finally:
        STATE.request = prev
