"""The allocation-free attention backward (decik_varlen_attn_bwd_noalloc), called through the
C ABI, against the workspace-taking entry point on the same inputs, two calls in a row.

It is for callers that cannot allocate device memory (hosts whose device memory belongs to their
own pool, or code running where an allocation could block or fail): its scratch is a static
array in the library, so consecutive calls reuse stale contents, which the kernels must clear.
This file is collected last so that a stop-at-first-failure run has run every other test first.
"""

import ctypes

import numpy as np
import pytest
import torch

from decik_b200 import _lib
from tests.tolerance import assert_close16

pytestmark = pytest.mark.gpu


def _t3(t):
    return _lib.Tensor3(t.data_ptr(), t.stride(0), t.stride(1))


def _case(lengths, seed):
    torch.manual_seed(seed)
    T, HQ, HK, D = sum(lengths), 12, 2, 128
    dev = "cuda"
    q = torch.randn(HQ, T, D, device=dev).bfloat16().transpose(0, 1)
    k = torch.randn(HK, T, D, device=dev).bfloat16().transpose(0, 1)
    v = torch.randn(T, HK, D, device=dev).bfloat16()
    do = torch.randn(T, HQ, D, device=dev).bfloat16()
    cu = torch.tensor(np.concatenate([[0], np.cumsum(lengths)]), dtype=torch.int32, device=dev)
    return q, k, v, do, cu


def test_noalloc_backward_matches_workspace_backward(cuda_lib):
    from decik_b200 import ops

    lib = _lib.lib()
    lengths = [37, 128, 211, 454]                       # 830 tokens x 12 heads, inside the limit
    scale = 128 ** -0.5
    for seed in (0, 1):                                 # two calls in a row on different data
        q, k, v, do, cu = _case(lengths, seed)
        out, lse = ops.varlen_attn_fwd(q, k, v, cu, max(lengths), scale)
        ref = ops.varlen_attn_bwd(do, q, k, v, out, lse, cu, max(lengths), scale)
        dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
        stream = torch.cuda.current_stream().cuda_stream
        rc = lib.decik_varlen_attn_bwd_noalloc(_t3(do), _t3(q), _t3(k), _t3(v), _t3(out), lse.data_ptr(),
                                               _t3(dq), _t3(dk), _t3(dv), cu.data_ptr(), len(lengths),
                                               max(lengths), q.shape[0], 12, 2, 128, scale, _lib.BF16, stream)
        assert rc == 0, lib.decik_last_error()
        torch.cuda.synchronize()
        for name, a, b in zip(("dq", "dk", "dv"), (dq, dk, dv), ref):
            assert_close16(a.float().cpu().numpy(), b.float().cpu().numpy(), name)
    assert lib.decik_kernel_error(1) == 0


def test_noalloc_backward_rejects_inputs_beyond_its_scratch(cuda_lib):
    lib = _lib.lib()
    z = _lib.Tensor3(None, 0, 0)
    # 2000 tokens x 12 heads > 16384 token-heads: refused before any pointer is used
    rc = lib.decik_varlen_attn_bwd_noalloc(z, z, z, z, z, None, z, z, z, None, 1, 2000, 2000, 12, 2, 128,
                                           0.088, _lib.BF16, None)
    assert rc == 1 and b"exceeds the static scratch" in lib.decik_last_error()
