"""The projection epilogues (decik_qkv_epilogue_fwd / _bwd) against the reference's per-op path:
RoPE and the casts bit for bit (the same kernels' arithmetic as decik_rope_fwd / decik_rope_bwd,
which are pinned to skc_rope_fwd_kernel / skc_rope_bwd_kernel), the rank-16 LoRA products against
cuBLAS in the same dtype (their fp32 sums may be added in another order: rare one-ulp
differences), and everything against an fp64 restatement at the bf16 bar."""

import pytest
import torch
import torch.nn.functional as F

from tests.tolerance import assert_close16

pytestmark = pytest.mark.gpu

HQ, HK, D, R = 12, 2, 128, 16
NQ, NK = HQ * D, HK * D
NPROJ = NQ + 2 * NK


def _ops():
    from decik_b200 import ops

    return ops


def _cos_sin(T):
    from decik_b200.block import rope_cos_sin

    return rope_cos_sin((torch.arange(T, device="cuda") * 7919) % 4096, D)


def _one_ulp_close(a, b, min_equal=0.97):
    """Equal except for rare last-bit differences of the rank-16 sums."""
    a, b = a.float(), b.float()
    assert torch.isfinite(a).all()
    eq = (a == b).float().mean().item()
    assert eq >= min_equal, f"only {eq:.4f} of the values are bit-equal"
    assert ((a - b).abs() <= 2 ** -7 * b.abs() + 1e-6).all()


def _rope64(x, cos, sin):
    half = x.shape[-1] // 2
    rot = torch.cat((-x[..., half:], x[..., :half]), dim=-1)
    return x * cos + rot * sin


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16], ids=["bf16", "fp16"])
@pytest.mark.parametrize("T", [1, 37, 830])
def test_qkv_epilogue_fwd(cuda_lib, dtype, T):
    ops = _ops()
    g = torch.Generator(device="cuda").manual_seed(T)
    y = torch.randn(T, NPROJ + 2 * R, generator=g, device="cuda").to(dtype)
    b_q = torch.randn(NQ, R, generator=g, device="cuda") * 0.05
    b_v = torch.randn(NK, R, generator=g, device="cuda") * 0.05
    a_q = torch.randn(R, 1536, generator=g, device="cuda") * 0.05
    a_v = torch.randn(R, 1536, generator=g, device="cuda") * 0.05
    a_out = torch.zeros(2 * R, 1536 + 8, dtype=dtype, device="cuda")[:, :1536]
    frag = ops.lora_pack(a_q, a_v, b_q, b_v, dtype, a_out=a_out)
    assert torch.equal(a_out, torch.cat([a_q, a_v]).to(dtype))
    s = 2.0
    cos, sin = _cos_sin(T)
    q, k, v, u = ops.qkv_epilogue_fwd(y, y[:, NPROJ:], frag, s, cos, sin, HQ, HK, want_u=True)
    qb, kb, vb = y[:, :NQ].contiguous(), y[:, NQ:NQ + NK].contiguous(), y[:, NQ + NK:NPROJ]
    u_q, u_v = y[:, NPROJ:NPROJ + R], y[:, NPROJ + R:]
    assert torch.equal(u, y[:, NPROJ:])
    # the reference's ops: lora_B(u) * scaling in dt, FusedQKRope, v = dt(f32 + f32)
    q_lora = F.linear(u_q, b_q.to(dtype)) * s
    v_lora = F.linear(u_v, b_v.to(dtype)) * s
    q_ref, k_ref = ops.rope_fwd(qb, q_lora.contiguous(), kb, cos, sin, HQ, HK)
    v_ref = (vb.float() + v_lora.float()).to(dtype).view(T, HK, D)
    assert torch.equal(k, k_ref)
    _one_ulp_close(q, q_ref)
    _one_ulp_close(v, v_ref)
    # fp64 restatement
    c64, s64 = cos.double(), sin.double()
    ql64 = (u_q.double() @ b_q.to(dtype).double().t()) * s
    q64 = _rope64((qb.double() + ql64).view(T, HQ, D).transpose(0, 1), c64, s64)
    v64 = vb.double() + (u_v.double() @ b_v.to(dtype).double().t()) * s
    assert_close16(q.float().cpu().numpy(), q64.cpu().numpy(), "q")
    assert_close16(v.reshape(T, NK).float().cpu().numpy(), v64.cpu().numpy(), "v")
    # no LoRA: RoPE and copies only, bit-exact
    q0, k0, v0, u0 = ops.qkv_epilogue_fwd(y, None, None, s, cos, sin, HQ, HK)
    q0_ref, k0_ref = ops.rope_fwd(qb, None, kb, cos, sin, HQ, HK)
    assert u0 is None
    assert torch.equal(q0, q0_ref) and torch.equal(k0, k0_ref) and torch.equal(v0, vb.reshape(T, HK, D))
    assert cuda_lib.decik_kernel_error(1) == 0


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16], ids=["bf16", "fp16"])
@pytest.mark.parametrize("T", [1, 37, 830])
def test_qkv_epilogue_bwd(cuda_lib, dtype, T):
    ops = _ops()
    g = torch.Generator(device="cuda").manual_seed(100 + T)
    grad_q = torch.randn(T, HQ, D, generator=g, device="cuda").to(dtype)           # token-major view
    grad_k = torch.randn(HK, T, D, generator=g, device="cuda").to(dtype).transpose(0, 1)  # head-major
    dv = torch.randn(T, NK, generator=g, device="cuda").to(dtype)
    b_q = torch.randn(NQ, R, generator=g, device="cuda") * 0.05
    b_v = torch.randn(NK, R, generator=g, device="cuda") * 0.05
    a = torch.zeros(R, 1536, device="cuda")
    frag = ops.lora_pack(a, a, b_q, b_v, dtype)
    s = 2.0
    cos, sin = _cos_sin(T)
    dy = torch.full((T, NPROJ + 2 * R + 8), float("nan"), dtype=dtype, device="cuda")[:, :NPROJ + 2 * R]
    dy[:, NQ + NK:NPROJ] = dv
    ops.qkv_epilogue_bwd(grad_q, grad_k, cos, sin, frag, s, dy, HQ, HK)
    dq_ref, dk_ref = ops.rope_bwd(grad_q.transpose(0, 1), grad_k.transpose(0, 1), cos, sin)
    assert torch.equal(dy[:, :NQ], dq_ref)
    assert torch.equal(dy[:, NQ:NQ + NK], dk_ref)
    assert torch.equal(dy[:, NQ + NK:NPROJ], dv)
    # du = dt(dt(g * scaling) . B16), as LoRAPairFromNorm.backward forms grad_u (solution/attn.py:250-253)
    du_q_ref = (dq_ref * s).mm(b_q.to(dtype))
    du_v_ref = (dv * s).mm(b_v.to(dtype))
    _one_ulp_close(dy[:, NPROJ:NPROJ + R], du_q_ref)
    _one_ulp_close(dy[:, NPROJ + R:], du_v_ref)
    # no LoRA: only the RoPE^T columns are written
    dy0 = torch.zeros((T, NPROJ), dtype=dtype, device="cuda")
    ops.qkv_epilogue_bwd(grad_q, grad_k, cos, sin, None, s, dy0, HQ, HK)
    assert torch.equal(dy0[:, :NQ], dq_ref) and torch.equal(dy0[:, NQ:NQ + NK], dk_ref)
    assert not dy0[:, NQ + NK:].any()
    assert cuda_lib.decik_kernel_error(1) == 0


def test_qkv_epilogue_rejects_bad_arguments(cuda_lib):
    from decik_b200 import _lib

    ops = _ops()
    T = 16
    y = torch.zeros(T, NPROJ + 2 * R, dtype=torch.bfloat16, device="cuda")
    cos, sin = _cos_sin(T)
    b_q = torch.zeros(NQ, R, device="cuda")
    b_v = torch.zeros(NK, R, device="cuda")
    with pytest.raises(RuntimeError, match="rank 16"):
        ops.lora_pack(torch.zeros(8, 1536, device="cuda"), torch.zeros(8, 1536, device="cuda"),
                      torch.zeros(NQ, 8, device="cuda"), torch.zeros(NK, 8, device="cuda"), torch.bfloat16)
    with pytest.raises(RuntimeError, match="leading dimension"):
        short = torch.zeros(T, NPROJ - 8, dtype=torch.bfloat16, device="cuda")
        ops.qkv_epilogue_fwd(short, None, None, 2.0, cos, sin, HQ, HK)
    lib = _lib.lib()
    t3 = _lib.Tensor3(y.data_ptr(), NPROJ, D)
    frag = ops.lora_pack(torch.zeros(R, 1536, device="cuda"), torch.zeros(R, 1536, device="cuda"), b_q, b_v,
                         torch.bfloat16)
    # ldy not a multiple of 8 elements
    assert lib.decik_qkv_epilogue_bwd(t3, t3, cos.data_ptr(), sin.data_ptr(), frag.data_ptr(), 2.0,
                                      y.data_ptr(), NPROJ + 2 * R - 4, T, HQ, HK, D, 1, None) == 1
    assert lib.decik_qkv_epilogue_bwd(t3, t3, cos.data_ptr(), sin.data_ptr(), None, 2.0,
                                      y.data_ptr(), NPROJ + 2 * R, T, HQ, HK, 64, 1, None) == 3
    assert cuda_lib.decik_kernel_error(1) == 0


@pytest.mark.parametrize("lengths,hq,hk,lora", [
    ([37, 128, 211, 454], 12, 2, True),      # config 1: query heads split over CTAs (fp32 dK / dV)
    ([4096, 4096, 4096, 4096], 28, 4, True),  # 7B heads, 16k tokens: dK / dV written directly
    ([300, 1, 129], 12, 2, False),            # no LoRA: dv still rounded into dy
])
def test_attn_qkv_bwd_matches_two_calls(cuda_lib, lengths, hq, hk, lora):
    """decik_attn_qkv_bwd against decik_varlen_attn_bwd + decik_qkv_epilogue_bwd on the same inputs:
    the same roundings, so equal up to the order of the attention's fp32 reduce-adds."""
    import numpy as np

    ops = _ops()
    dtype = torch.bfloat16
    T, nq, nk = sum(lengths), hq * D, hk * D
    nproj = nq + 2 * nk
    g = torch.Generator(device="cuda").manual_seed(len(lengths) + hq)
    q = torch.randn(hq, T, D, generator=g, device="cuda").to(dtype).transpose(0, 1)
    k = torch.randn(hk, T, D, generator=g, device="cuda").to(dtype).transpose(0, 1)
    v = torch.randn(T, hk, D, generator=g, device="cuda").to(dtype)
    do = torch.randn(T, hq, D, generator=g, device="cuda").to(dtype)
    cu = torch.tensor(np.concatenate([[0], np.cumsum(lengths)]), dtype=torch.int32, device="cuda")
    scale = D ** -0.5
    out, lse = ops.varlen_attn_fwd(q, k, v, cu, max(lengths), scale)
    cos, sin = _cos_sin(T)
    frag = None
    if lora:
        frag = ops.lora_pack(torch.zeros(R, 64, device="cuda"), torch.zeros(R, 64, device="cuda"),
                             torch.randn(nq, R, generator=g, device="cuda") * 0.05,
                             torch.randn(nk, R, generator=g, device="cuda") * 0.05, dtype)
    width = nproj + (2 * R if lora else 0)
    dy1 = torch.full((T, width), float("nan"), dtype=dtype, device="cuda")
    dq = torch.empty(T, hq, D, dtype=dtype, device="cuda")
    dk = torch.empty(T, hk, D, dtype=dtype, device="cuda")
    dv = dy1[:, nq + nk:nproj].view(T, hk, D)
    ops.varlen_attn_bwd(do, q, k, v, out, lse, cu, max(lengths), scale, dq=dq, dk=dk, dv=dv)
    ops.qkv_epilogue_bwd(dq, dk, cos, sin, frag, 2.0, dy1, hq, hk)
    dy2 = torch.full((T, width), float("nan"), dtype=dtype, device="cuda")
    ops.attn_qkv_bwd(do, q, k, v, out, lse, cu, max(lengths), scale, cos, sin, frag, 2.0, dy2)
    assert torch.isfinite(dy2).all()
    for name, sl in (("dq", slice(0, nq)), ("dk", slice(nq, nq + nk)), ("dv", slice(nq + nk, nproj)),
                     ("du", slice(nproj, width))):
        a, b = dy2[:, sl].float(), dy1[:, sl].float()
        if a.numel() == 0:
            continue
        assert (a - b).norm() <= 2e-3 * b.norm().clamp_min(1e-6), name
        assert (a == b).float().mean().item() >= 0.5, name
    assert cuda_lib.decik_kernel_error(1) == 0
