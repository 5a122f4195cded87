"""The tcgen05 projection GEMMs of the fused block (decik_qkv_proj_fwd, decik_lora_b_ext,
decik_proj_dx, decik_lora_grads) against the same arithmetic in fp32 by torch on the same 16-bit
operands: the 16-bit outputs (one rounding each) within rel-L2 3e-3, the fp32 products within
rel-L2 1e-5. The whole block, these kernels included, is held to the oracle in
tests/test_block_gpu.py."""

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


def _rope32(x, cos, sin):
    """RoPE of [T, H, 128] fp32 with transformers' rotate_half."""
    half = x.shape[-1] // 2
    rot = torch.cat((-x[..., half:], x[..., :half]), dim=-1)
    return x * cos[:, None, :] + rot * sin[:, None, :]


@pytest.mark.parametrize("T,hidden,hq,hk", CASES, ids=["config1", "one-token", "bench", "7b", "ragged"])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16], ids=["bf16", "fp16"])
@pytest.mark.parametrize("lora", [True, False], ids=["lora", "nolora"])
def test_qkv_proj_fwd_matches_fp32(cuda_lib, T, hidden, hq, hk, dtype, lora):
    """x16 bit for bit; u against torch's GEMM; q, k, v against the same arithmetic in fp32 from the
    same 16-bit operands (x16, W, u, scaling . B, bias): base + LoRA + bias, RoPE, one rounding."""
    from decik_b200 import ops

    x, w_cat, bias, b_q, b_v, cos, sin = _inputs(T, hidden, hq, hk, dtype, seed=T + hq)
    D, n_proj = 128, (hq + 2 * hk) * 128
    a_q = torch.randn(16, hidden, device=DEV) * hidden ** -0.5
    a_v = torch.randn(16, hidden, device=DEV) * hidden ** -0.5
    ops.lora_pack(a_q, a_v, b_q, b_v, dtype, a_out=w_cat[n_proj:])
    ext = ops.lora_b_ext(b_q if lora else None, b_v if lora else None, 2.0, bias, dtype, hq, hk)
    x16, u, q, k, v = ops.qkv_proj_fwd(x, w_cat, ext, lora, cos, sin, hq, hk)
    xr = x.to(dtype)
    assert torch.equal(x16, xr)
    assert torch.equal(u[:, 32].float(), torch.ones_like(u[:, 32].float()))
    assert torch.equal(u[:, 33:], torch.zeros_like(u[:, 33:]))
    assert torch.equal(ext[:, 32], bias[:n_proj].to(dtype))
    if lora:
        _close(u[:, :32], F.linear(xr, w_cat[n_proj:]), "u")
        assert torch.equal(ext[:hq * D, :16], (b_q * 2.0).to(dtype))
        assert torch.equal(ext[hq * D:(hq + hk) * D, :32], torch.zeros_like(ext[hq * D:(hq + hk) * D, :32]))
    else:
        assert torch.equal(u[:, :32], torch.zeros_like(u[:, :32]))
    # the same arithmetic in fp32: base + LoRA-up + bias (through the ones column), RoPE
    y = torch.mm(xr.float(), w_cat[:n_proj].float().t()) + torch.mm(u.float(), ext.float().t())
    rq = _rope32(y[:, :hq * D].view(T, hq, D), cos, sin).transpose(0, 1)
    rk = _rope32(y[:, hq * D:(hq + hk) * D].view(T, hk, D), cos, sin).transpose(0, 1)
    rv = y[:, (hq + hk) * D:].view(T, hk, D)
    _close(q, rq, "q", rel=3e-3)
    _close(k, rk, "k", rel=3e-3)
    _close(v, rv, "v", rel=3e-3)
    assert cuda_lib.decik_kernel_error(1) == 0


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
    w_t = ops.transpose16(w_cat)
    assert torch.equal(w_t, w_cat.t())
    dx = ops.proj_dx(dy, w_t)
    ref = torch.mm(dy.float(), w_cat.float())
    _close(dx, ref, "dx", rel=1e-5, mx=1e-4)
    u64 = torch.cat((u, torch.zeros_like(u)), 1)  # the forward's u rows are 64 wide
    da, db = ops.lora_grads(dy, x16, u64[:, :2 * r], 2.0, hq, hk)
    rda = torch.mm(dy[:, n_proj:].float().t(), x16.float())
    rdb = torch.mm(dy[:, :n_proj].float().t(), u.float()) * 2.0
    _close(da, rda, "dA", rel=1e-5, mx=1e-4)
    _close(db[:n_q], rdb[:n_q, :r], "dB_q", rel=1e-5, mx=1e-4)
    _close(db[n_q:], rdb[n_q + n_kvd:, r:], "dB_v", rel=1e-5, mx=1e-4)
    assert cuda_lib.decik_kernel_error(1) == 0


@pytest.mark.parametrize("T,hidden,hq,hk", [(830, 1536, 12, 2), (1, 1536, 12, 2), (16384, 1536, 12, 2),
                                          (1000, 3584, 28, 4), (257, 1536, 12, 2)],
                         ids=["config1", "one-token", "bench", "7b", "ragged"])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16], ids=["bf16", "fp16"])
@pytest.mark.parametrize("w_dtype", [torch.float32, torch.float16], ids=["w32", "w16"])
def test_qkv_proj_norm_fwd_equals_norm_then_proj(cuda_lib, T, hidden, hq, hk, dtype, w_dtype):
    """The input RMSNorm inside the first kernel (decik_qkv_proj_norm_fwd) against the norm kernel
    followed by decik_qkv_proj_fwd: rstd, x16, u, q, k and v equal bit for bit."""
    from decik_b200 import ops

    h, w_cat, bias, b_q, b_v, cos, sin = _inputs(T, hidden, hq, hk, dtype, seed=3 * T + hq)
    h = h * 3.0 + 0.5
    n_proj = (hq + 2 * hk) * 128
    g = torch.Generator(device=DEV).manual_seed(T)
    w = (1.0 + 0.1 * torch.randn(hidden, device=DEV, generator=g)).to(w_dtype)
    a_q = torch.randn(16, hidden, device=DEV) * hidden ** -0.5
    a_v = torch.randn(16, hidden, device=DEV) * hidden ** -0.5
    ops.lora_pack(a_q, a_v, b_q, b_v, dtype, a_out=w_cat[n_proj:])
    ext = ops.lora_b_ext(b_q, b_v, 2.0, bias, dtype, hq, hk)
    x, rstd_ref = ops.rmsnorm_fwd(h, w, 1e-6)
    ref = ops.qkv_proj_fwd(x, w_cat, ext, True, cos, sin, hq, hk)
    got = ops.qkv_proj_fwd(h, w_cat, ext, True, cos, sin, hq, hk, norm=(w, 1e-6))
    assert torch.equal(got[5], rstd_ref)
    for name, a, e in zip(("x16", "u", "q", "k", "v"), got[:5], ref):
        assert torch.equal(a, e), name
    assert cuda_lib.decik_kernel_error(1) == 0


def test_proj_entry_points_reject_bad_arguments(cuda_lib):
    from decik_b200 import _lib

    lib = _lib.lib()
    z = _lib.Tensor3(None, 0, 0)
    # hidden not a multiple of 64
    assert lib.decik_qkv_proj_fwd(None, 100, None, 100, None, 0, None, None, z, z, z, None, 100, None, 5, 100,
                                  12, 2, 128, _lib.BF16, None) == 1
    assert lib.decik_proj_dx(None, 8, 8, None, 8, None, 8, 5, 100, _lib.BF16, None) == 1
    assert lib.decik_lora_grads(None, 8, None, 8, None, 64, None, None, 1.0, 5, 100, 12, 2, _lib.BF16, None) == 1
    # the norm variant: no norm weight, and a norm weight of an unsupported dtype
    assert lib.decik_qkv_proj_norm_fwd(None, 1536, None, _lib.F32, 1e-6, None, None, 1536, None, 1, None, None,
                                       z, z, z, None, 1536, None, 5, 1536, 12, 2, 128, _lib.BF16, None) == 1
