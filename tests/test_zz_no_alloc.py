"""The allocation-free attention backward (decik_varlen_attn_bwd_noalloc), called through the
C ABI, against the workspace-taking entry point on the same inputs, two calls in a row.

It is for callers that cannot allocate device memory (hosts whose device memory belongs to their
own pool, or code running where an allocation could block or fail): its scratch is a static
array in the library, so consecutive calls reuse stale contents, which the kernels must clear.
This file is collected last so that a stop-at-first-failure run has run every other test first.
"""

import numpy as np
import pytest
import torch

from decik_b200 import _lib
from oracle import attention as o_attn
from tests.tolerance import assert_close16

pytestmark = pytest.mark.gpu

DTYPES = {"bf16": (torch.bfloat16, _lib.BF16), "fp16": (torch.float16, _lib.F16)}


def _t3(t):
    return _lib.Tensor3(t.data_ptr(), t.stride(0), t.stride(1))


def _case(lengths, seed, dtype, hq=12, hk=2):
    torch.manual_seed(seed)
    T, D = sum(lengths), 128
    dev = "cuda"
    q = torch.randn(hq, T, D, device=dev).to(dtype).transpose(0, 1)
    k = torch.randn(hk, T, D, device=dev).to(dtype).transpose(0, 1)
    v = torch.randn(T, hk, D, device=dev).to(dtype)
    do = torch.randn(T, hq, D, device=dev).to(dtype)
    cu = torch.tensor(np.concatenate([[0], np.cumsum(lengths)]), dtype=torch.int32, device=dev)
    return q, k, v, do, cu


def _noalloc(lib, lengths, q, k, v, do, out, lse, cu, scale, code):
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    stream = torch.cuda.current_stream().cuda_stream
    rc = lib.decik_varlen_attn_bwd_noalloc(_t3(do), _t3(q), _t3(k), _t3(v), _t3(out), lse.data_ptr(),
                                           _t3(dq), _t3(dk), _t3(dv), cu.data_ptr(), len(lengths),
                                           max(lengths), q.shape[0], q.shape[1], k.shape[1], 128, scale, code,
                                           stream)
    assert rc == 0, lib.decik_last_error()
    torch.cuda.synchronize()
    return dq, dk, dv


def test_noalloc_setup_call_with_zero_tokens(cuda_lib):
    """A zero-token call does the per-device set-up only (the start-up call callers make before
    their pool claims the device) and returns success."""
    lib = _lib.lib()
    z = _lib.Tensor3(None, 0, 0)
    rc = lib.decik_varlen_attn_bwd_noalloc(z, z, z, z, z, None, z, z, z, None, 0, 0, 0, 12, 2, 128, 0.088,
                                           _lib.BF16, None)
    assert rc == 0, lib.decik_last_error()


@pytest.mark.parametrize("dt", sorted(DTYPES))
@pytest.mark.parametrize("lengths,hq,hk", [([37, 128, 211, 454], 12, 2),    # 830 x 12 token-heads
                                           ([1000, 24], 16, 2)],          # exactly the 16,384 limit
                         ids=["config1", "at-limit"])
def test_noalloc_backward_matches_workspace_backward(cuda_lib, dt, lengths, hq, hk):
    from decik_b200 import ops

    lib = _lib.lib()
    dtype, code = DTYPES[dt]
    scale = 128 ** -0.5
    assert sum(lengths) * hq <= 16384
    for seed in (0, 1):                                 # two calls in a row on different data
        q, k, v, do, cu = _case(lengths, seed, dtype, hq, hk)
        out, lse = ops.varlen_attn_fwd(q, k, v, cu, max(lengths), scale)
        ref = ops.varlen_attn_bwd(do, q, k, v, out, lse, cu, max(lengths), scale)
        got = _noalloc(lib, lengths, q, k, v, do, out, lse, cu, scale, code)
        for name, a, b in zip(("dq", "dk", "dv"), got, ref):
            assert_close16(a.float().cpu().numpy(), b.float().cpu().numpy(), name)
    assert lib.decik_kernel_error(1) == 0


def test_noalloc_backward_matches_oracle(cuda_lib):
    """The same entry point against the CPU oracle directly (fp16, config-1 lengths)."""
    from decik_b200 import ops

    lib = _lib.lib()
    lengths = [37, 128, 211, 454]
    scale = 128 ** -0.5
    q, k, v, do, cu = _case(lengths, 2, torch.float16)
    out, lse = ops.varlen_attn_fwd(q, k, v, cu, max(lengths), scale)
    dq, dk, dv = _noalloc(lib, lengths, q, k, v, do, out, lse, cu, scale, _lib.F16)
    f = lambda t: t.float().cpu().numpy()
    spans = [(int(s), int(L)) for s, L in zip(np.cumsum([0] + lengths[:-1]), lengths)]
    rdq, rdk, rdv = o_attn.backward(f(do), f(q), f(k), f(v), spans, scale)
    for name, a, r in (("dq", dq, rdq), ("dk", dk, rdk), ("dv", dv, rdv)):
        assert_close16(f(a), r, name)
    assert lib.decik_kernel_error(1) == 0


def test_noalloc_backward_rejects_inputs_beyond_its_scratch(cuda_lib):
    lib = _lib.lib()
    z = _lib.Tensor3(None, 0, 0)
    # 2000 tokens x 12 heads > 16384 token-heads: refused before any pointer is used
    rc = lib.decik_varlen_attn_bwd_noalloc(z, z, z, z, z, None, z, z, z, None, 1, 2000, 2000, 12, 2, 128,
                                           0.088, _lib.BF16, None)
    assert rc == 1 and b"exceeds the static scratch" in lib.decik_last_error()
