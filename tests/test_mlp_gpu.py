"""The MLP node (solution/mlp.py FusedMLP, decik_swiglu_fwd/bwd) on the GPU: the SwiGLU kernels
against the reference's SwiGLU fixture, and the whole node against the reference's RecomputedMLP
fixture (fp16, its compute dtype) and against the unfused bitsandbytes-style chain in bf16."""

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from oracle import mlp as o_mlp
from tests.conftest import golden

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _ulps(a: torch.Tensor, ref: torch.Tensor) -> float:
    """The largest |a - ref| in units of one 16-bit ulp of ref (a's dtype); |ref| * 2^-m is at least
    one ulp, and the floor is the type's smallest subnormal."""
    ref = ref.to(a.dtype).float()
    rel, floor = (2.0 ** -7, 9.2e-41) if a.dtype == torch.bfloat16 else (2.0 ** -10, 5.96e-8)
    return ((a.float() - ref).abs() / (ref.abs() * rel + floor)).max().item()


def test_swiglu_golden(cuda_lib):
    from decik_b200 import ops

    g = golden("mlp_golden.npz")
    gate = torch.from_numpy(g["sw_gate"]).to(DEV)
    up = torch.from_numpy(g["sw_up"]).to(DEV)
    inter = gate.shape[1]
    gu = torch.cat([gate, up], dim=1)
    out = ops.swiglu_fwd(gu, inter)
    assert _ulps(out, torch.from_numpy(g["sw_out"]).to(DEV)) <= 1
    dgu = ops.swiglu_bwd(torch.from_numpy(g["sw_grad"]).to(DEV), gu, inter)
    assert _ulps(dgu[:, :inter], torch.from_numpy(g["sw_dgate"]).to(DEV)) <= 1
    assert _ulps(dgu[:, inter:], torch.from_numpy(g["sw_dup"]).to(DEV)) <= 1


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("rows,inter,pad", [(1, 8, 0), (333, 8960, 0), (64, 256, 24)])
def test_swiglu_vs_fp32_formula(cuda_lib, dtype, rows, inter, pad):
    """Against the reference's formulas in fp32 rounded once (torch), within one 16-bit ulp; gu and
    dgu may be views with a row stride wider than 2 * inter."""
    from decik_b200 import ops

    gen = torch.Generator(device=DEV).manual_seed(rows + inter)
    buf = (torch.randn(rows, 2 * inter + pad, device=DEV, generator=gen) * 3).to(dtype)
    gu = buf[:, : 2 * inter]
    grad = torch.randn(rows, inter, device=DEV, generator=gen).to(dtype)
    g, u = gu[:, :inter].float(), gu[:, inter:].float()
    s = torch.sigmoid(g)
    out = ops.swiglu_fwd(gu, inter)
    assert _ulps(out, (g * s * u).to(dtype)) <= 1
    dbuf = torch.empty(rows, 2 * inter + pad, device=DEV, dtype=dtype)
    ops.swiglu_bwd(grad, gu, inter, dgu=dbuf[:, : 2 * inter])
    gr = grad.float()
    assert _ulps(dbuf[:, :inter], (gr * u * s * (1 + g * (1 - s))).to(dtype)) <= 1
    assert _ulps(dbuf[:, inter: 2 * inter], (gr * g * s).to(dtype)) <= 1


def test_swiglu_rejects_bad_arguments(cuda_lib):
    from decik_b200 import ops

    with pytest.raises(RuntimeError, match="multiple of 8"):
        ops.swiglu_fwd(torch.zeros(4, 12, device=DEV, dtype=torch.bfloat16), 6)


def _nf4_weights(g, dtype):
    from decik_b200.block import quant_state_from_arrays
    from decik_b200.solution.nf4 import dequantize_nf4

    T, H, I = (int(v) for v in g["dims"])
    w = {}
    for n, shape in (("gate", (I, H)), ("up", (I, H)), ("down", (H, I))):
        st = {k: g[f"{n}_{k}"] for k in ("packed", "absmax", "code", "absmax2", "code2")}
        st.update(offset=float(g[f"{n}_offset"]), shape=shape, blocksize=64, blocksize2=256, nested=True)
        packed, qs = quant_state_from_arrays(st, DEV, dtype)
        w[n] = dequantize_nf4(packed, qs, dtype)
    return torch.cat([w["gate"], w["up"]]), w["down"]


def test_fused_mlp_matches_reference_fixture(cuda_lib):
    """FusedMLP in fp16 against the reference's RecomputedMLP on the same NF4 weights and inputs:
    out and the input gradient within rel-L2 5e-3, max-abs 2e-2 (normalised)."""
    from decik_b200.solution.mlp import FusedMLP

    g = golden("mlp_golden.npz")
    T, H, I = (int(v) for v in g["dims"])
    w_gu, w_down = _nf4_weights(g, torch.float16)
    x = torch.from_numpy(g["x"].reshape(T, H)).to(DEV).requires_grad_(True)
    out = FusedMLP.apply(x, w_gu, w_down)
    assert out.dtype == torch.float16
    out.backward(torch.from_numpy(g["gout"].reshape(T, H)).to(DEV))
    for got, ref in ((out.detach().float().cpu().numpy(), g["out"].reshape(T, H).astype(np.float32)),
                     (x.grad.cpu().numpy(), g["dx"].reshape(T, H))):
        assert np.linalg.norm(got - ref) / np.linalg.norm(ref) < 5e-3
        assert np.abs(got - ref).max() / max(1.0, np.abs(ref).max()) < 2e-2


def test_fused_mlp_bf16_vs_unfused_chain(cuda_lib):
    """bf16 at the Qwen2.5-1.5B MLP shape against the chain it replaces (two NF4 projections with
    fp32 outputs, SwiGLU in fp32, the down projection), with the same dequantised weights."""
    from decik_b200.nf4_quant import quantize_nf4
    from decik_b200.block import quant_state_from_arrays
    from decik_b200.solution.mlp import FusedMLP
    from decik_b200.solution.nf4 import dequantize_nf4

    rng = np.random.default_rng(3)
    T, H, I = 257, 1536, 8960
    w = {}
    for n, shape in (("gate", (I, H)), ("up", (I, H)), ("down", (H, I))):
        packed, qs = quant_state_from_arrays(quantize_nf4((rng.standard_normal(shape) * 0.02).astype(np.float32)),
                                             DEV, torch.bfloat16)
        w[n] = dequantize_nf4(packed, qs, torch.bfloat16)
    x = torch.randn(T, H, device=DEV).requires_grad_(True)
    x2 = x.detach().clone().requires_grad_(True)
    gout = torch.randn(T, H, device=DEV).to(torch.bfloat16)
    out = FusedMLP.apply(x, torch.cat([w["gate"], w["up"]]), w["down"])
    out.backward(gout)
    x16 = x2.to(torch.bfloat16)
    gate = F.linear(x16, w["gate"]).float()
    up = F.linear(x16, w["up"]).float()
    ref = F.linear((F.silu(gate) * up).to(torch.bfloat16), w["down"])
    ref.backward(gout)
    for got, exp in ((out.float(), ref.float()), (x.grad, x2.grad)):
        rel = ((got - exp).norm() / exp.norm()).item()
        assert rel < 1e-2, rel


def test_fused_mlp_with_residual(cuda_lib):
    """The node with the decoder layer's residual (fp32): residual + mlp(x) from the down projection's
    GEMM, against residual + the node's own 16-bit output (which rounds the MLP output first: within
    that rounding), and the residual's gradient is the output's gradient, exactly."""
    from decik_b200.solution.mlp import FusedMLP

    g = torch.Generator(device=DEV).manual_seed(5)
    T, H, inter = 700, 1536, 8960
    dt = torch.bfloat16
    x = torch.randn(T, H, device=DEV, generator=g)
    res = torch.randn(T, H, device=DEV, generator=g) * 4.0
    w_gu = (torch.randn(2 * inter, H, device=DEV, generator=g) * 0.02).to(dt)
    w_down = (torch.randn(H, inter, device=DEV, generator=g) * 0.02).to(dt)
    grad = torch.randn(T, H, device=DEV, generator=g)
    xa, ra = x.clone().requires_grad_(True), res.clone().requires_grad_(True)
    out = FusedMLP.apply(xa, w_gu, w_down, ra)
    out.backward(grad)
    xb = x.clone().requires_grad_(True)
    out_b = res + FusedMLP.apply(xb, w_gu, w_down).float()
    out_b.backward(grad)
    assert out.dtype == torch.float32
    d = (out - out_b).abs().max().item()
    assert d <= 2.0 ** -8 * (out_b - res).abs().max().item() + 1e-6, d
    assert torch.equal(ra.grad, grad)
    rel = ((xa.grad - xb.grad).norm() / xb.grad.norm()).item()
    assert rel < 1e-5, rel  # the same kernels on the same 16-bit gradient
    # a residual that is not a leaf (the decoder layer's stream) is updated in place: the same
    # values as into a new tensor, and the same gradients
    rl = res.clone().requires_grad_(True)
    rc = rl * 1.0
    xc = x.clone().requires_grad_(True)
    out_c = FusedMLP.apply(xc, w_gu, w_down, rc)
    assert out_c.data_ptr() == rc.data_ptr() and torch.equal(out_c, out)
    out_c.backward(grad)
    assert torch.equal(rl.grad, grad)
    assert ((xc.grad - xa.grad).norm() / xa.grad.norm()).item() < 1e-6
    assert cuda_lib.decik_kernel_error(1) == 0
