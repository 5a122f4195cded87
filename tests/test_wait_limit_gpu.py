"""The device-side failure path, made to run out on purpose without faulting the GPU: a bounded
mbarrier wait with a short limit (decik_wait_limit_selftest, the same wait the attention kernels
use) gives up, records its code in the error word, frees its TMEM and returns. Afterwards the
context is usable: the attention kernels run and match the oracle."""

import numpy as np
import pytest
import torch

from decik_b200 import _lib
from oracle import attention as o_attn
from tests.tolerance import assert_close16

pytestmark = pytest.mark.gpu


def test_wait_runs_out_reports_and_winds_down(cuda_lib):
    from decik_b200 import ops

    lib = _lib.lib()
    assert lib.decik_kernel_error(1) == 0           # start clean
    done = torch.zeros(1, dtype=torch.int32, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    rc = lib.decik_wait_limit_selftest(2_000_000, done.data_ptr(), stream)  # ~1 ms at 2 GHz
    assert rc == 0, lib.decik_last_error()
    torch.cuda.synchronize()
    assert int(done.item()) == 2                    # the wait ran out and the kernel returned
    assert lib.decik_kernel_error(1) == 901         # ... after recording its code
    assert lib.decik_kernel_error(0) == 0           # reset by the read above
    # the context still works, TMEM included: the tcgen05 attention kernels run and are right
    lengths = [37, 128, 211, 454]
    T = sum(lengths)
    torch.manual_seed(0)
    q = torch.randn(T, 12, 128, device="cuda").bfloat16()
    k = torch.randn(T, 2, 128, device="cuda").bfloat16()
    v = torch.randn(T, 2, 128, device="cuda").bfloat16()
    cu = torch.tensor(np.concatenate([[0], np.cumsum(lengths)]), dtype=torch.int32, device="cuda")
    out, _ = ops.varlen_attn_fwd(q, k, v, cu, max(lengths), 128 ** -0.5)
    f = lambda t: t.float().cpu().numpy()
    spans = [(int(s), int(L)) for s, L in zip(np.cumsum([0] + lengths[:-1]), lengths)]
    ro, _ = o_attn.forward(f(q), f(k), f(v), spans, 128 ** -0.5)
    assert_close16(f(out), ro, "out after the self-test")
    assert lib.decik_kernel_error(1) == 0


def test_selftest_rejects_bad_limits(cuda_lib):
    lib = _lib.lib()
    assert lib.decik_wait_limit_selftest(0, None, None) == 1
    assert lib.decik_wait_limit_selftest(10_000_000_000, None, None) == 1
