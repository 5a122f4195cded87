"""The tcgen05 projection GEMMs of the fused block (decik_qkv_proj_fwd, decik_proj_dx,
decik_lora_grads) against the unfused composition of the same arithmetic: torch's GEMMs
(F.linear with bias, torch.mm in fp32) feeding the projection epilogue kernel whose RoPE / LoRA
arithmetic is pinned bit for bit to the reference's kernels (tests/test_qkv_gpu.py). The GEMMs sum
in another order, so the 16-bit outputs agree to rounding, held here at rel-L2 <= 2e-3 and one
16-bit ulp-scale max error; the fp32 products at rel-L2 <= 1e-5."""

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _inputs(T, hidden, hq, hk, dtype, seed):
    from decik_b200.block import rope_cos_sin

    g = torch.Generator(device=DEV).manual_seed(seed)
    D, r = 128, 16
    n_proj = (hq + 2 * hk) * D
    x = torch.randn(T, hidden, device=DEV, generator=g)
    w_cat = (torch.randn(n_proj + 2 * r, hidden, device=DEV, generator=g) * 0.02).to(dtype)
    bias = (torch.randn(n_proj + 2 * r, device=DEV, generator=g) * 0.02).to(dtype)
    bias[n_proj:] = 0
    b_q = torch.randn(hq * D, r, device=DEV, generator=g) * 0.02
    b_v = torch.randn(hk * D, r, device=DEV, generator=g) * 0.02
    pos = torch.arange(T, device=DEV) % 997
    cos, sin = rope_cos_sin(pos, D)
    return x, w_cat, bias, b_q, b_v, cos, sin


def _close(a, e, what, rel=2e-3, mx=2e-2):
    a, e = a.float(), e.float()
    d = a - e
    r = (d.norm() / e.norm().clamp_min(1e-30)).item()
    m = (d.abs().max() / e.abs().max().clamp_min(1.0)).item()
    assert r <= rel and m <= mx, f"{what}: rel-L2 {r:.3e} (<= {rel}), max {m:.3e} (<= {mx})"


CASES = [(830, 1536, 12, 2), (1, 1536, 12, 2), (16384, 1536, 12, 2), (1000, 3584, 28, 4), (257, 1536, 12, 2)]


@pytest.mark.parametrize("T,hidden,hq,hk", CASES, ids=["config1", "one-token", "bench", "7b", "ragged"])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16], ids=["bf16", "fp16"])
def test_qkv_proj_fwd_matches_unfused(cuda_lib, T, hidden, hq, hk, dtype):
    from decik_b200 import ops

    x, w_cat, bias, b_q, b_v, cos, sin = _inputs(T, hidden, hq, hk, dtype, seed=T + hq)
    n_proj = (hq + 2 * hk) * 128
    a_q = torch.randn(16, hidden, device=DEV) * hidden ** -0.5
    a_v = torch.randn(16, hidden, device=DEV) * hidden ** -0.5
    frag = ops.lora_pack(a_q, a_v, b_q, b_v, dtype, a_out=w_cat[n_proj:])
    lora_b = torch.cat((b_q, b_v)).to(dtype)
    x16, u, q, k, v = ops.qkv_proj_fwd(x, w_cat, bias, lora_b, 2.0, cos, sin, hq, hk)
    # unfused: the same GEMM by torch (bias in its epilogue), then the epilogue kernel
    xr = x.to(dtype)
    assert torch.equal(x16, xr)
    y = F.linear(xr, w_cat, bias)
    _close(u, y[:, n_proj:], "u")
    rq, rk, rv, _ = ops.qkv_epilogue_fwd(y, y[:, n_proj:], frag, 2.0, cos, sin, hq, hk)
    _close(q, rq, "q")
    _close(k, rk, "k")
    _close(v, rv, "v")
    assert cuda_lib.decik_kernel_error(1) == 0


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16], ids=["bf16", "fp16"])
def test_qkv_proj_fwd_without_lora(cuda_lib, dtype):
    from decik_b200 import ops

    T, hidden, hq, hk = 700, 1536, 12, 2
    x, w_cat, bias, _, _, cos, sin = _inputs(T, hidden, hq, hk, dtype, seed=3)
    n_proj = (hq + 2 * hk) * 128
    x16, u, q, k, v = ops.qkv_proj_fwd(x, w_cat, bias, None, 2.0, cos, sin, hq, hk)
    assert u is None
    y = F.linear(x.to(dtype), w_cat[:n_proj], bias[:n_proj])
    rq, rk, rv, _ = ops.qkv_epilogue_fwd(y, None, None, 2.0, cos, sin, hq, hk)
    for name, a, e in (("q", q, rq), ("k", k, rk), ("v", v, rv)):
        _close(a, e, name)


@pytest.mark.parametrize("T,hidden,hq,hk", CASES, ids=["config1", "one-token", "bench", "7b", "ragged"])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16], ids=["bf16", "fp16"])
def test_proj_dx_and_lora_grads_match_torch(cuda_lib, T, hidden, hq, hk, dtype):
    from decik_b200 import ops

    g = torch.Generator(device=DEV).manual_seed(T)
    D, r = 128, 16
    n_q, n_kvd = hq * D, hk * D
    n_proj = n_q + 2 * n_kvd
    dy = torch.randn(T, n_proj + 2 * r, device=DEV, generator=g).to(dtype)
    w_cat = (torch.randn(n_proj + 2 * r, hidden, device=DEV, generator=g) * 0.02).to(dtype)
    x16 = torch.randn(T, hidden, device=DEV, generator=g).to(dtype)
    u = torch.randn(T, 2 * r, device=DEV, generator=g).to(dtype)
    dx = ops.proj_dx(dy, w_cat)
    ref = torch.mm(dy.float(), w_cat.float())
    _close(dx, ref, "dx", rel=1e-5, mx=1e-4)
    da, db = ops.lora_grads(dy, x16, u, 2.0, hq, hk)
    rda = torch.mm(dy[:, n_proj:].float().t(), x16.float())
    rdb = torch.mm(dy[:, :n_proj].float().t(), u.float()) * 2.0
    _close(da, rda, "dA", rel=1e-5, mx=1e-4)
    _close(db[:n_q], rdb[:n_q, :r], "dB_q", rel=1e-5, mx=1e-4)
    _close(db[n_q:], rdb[n_q + n_kvd:, r:], "dB_v", rel=1e-5, mx=1e-4)
    assert cuda_lib.decik_kernel_error(1) == 0


def test_proj_entry_points_reject_bad_arguments(cuda_lib):
    from decik_b200 import _lib

    lib = _lib.lib()
    z = _lib.Tensor3(None, 0, 0)
    # hidden not a multiple of 64
    assert lib.decik_qkv_proj_fwd(None, 100, None, 100, None, None, 2.0, None, None, z, z, z, None, 100, None, 5, 100,
                                  12, 2, 128, _lib.BF16, None) == 1
    assert lib.decik_proj_dx(None, 8, 8, None, 8, None, 8, 5, 100, _lib.BF16, None) == 1
    assert lib.decik_lora_grads(None, 8, None, 8, None, None, None, 1.0, 5, 100, 12, 2, _lib.BF16, None) == 1
