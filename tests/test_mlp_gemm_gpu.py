"""The MLP's tcgen05 GEMMs (decik_gemm16, decik_mlp_gate_up, decik_mlp_down_grad): products against
torch in fp32 on the same 16-bit operands (rel-L2 <= 2e-3 after the one rounding), and the fused
SwiGLU epilogues bit for bit against the separate SwiGLU kernels fed the same GEMM outputs (whose
arithmetic is pinned to the reference's formulas in tests/test_mlp_gpu.py)."""

import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _close(a, e, what, rel=2e-3):
    d = (a.float() - e.float())
    r = (d.norm() / e.float().norm().clamp_min(1e-30)).item()
    m = (d.abs().max() / e.float().abs().max().clamp_min(1.0)).item()
    assert r <= rel and m <= 2e-2, f"{what}: rel-L2 {r:.3e}, max {m:.3e}"


@pytest.mark.parametrize("M,N,K", [(830, 1536, 8960), (16384, 1536, 8960), (257, 1000, 1536), (1, 256, 64),
                                   (3000, 3584, 4608)])
@pytest.mark.parametrize("b_mn", [False, True], ids=["k-major", "mn-major"])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16], ids=["bf16", "fp16"])
def test_gemm16_matches_torch(cuda_lib, M, N, K, b_mn, dtype):
    from decik_b200 import ops

    g = torch.Generator(device=DEV).manual_seed(M + N)
    a = torch.randn(M, K, device=DEV, generator=g).to(dtype)
    b = (torch.randn((K, N) if b_mn else (N, K), device=DEV, generator=g) * K ** -0.5).to(dtype)
    out = ops.gemm16(a, b, b_mn)
    ref = a.float() @ (b.float() if b_mn else b.float().t())
    _close(out, ref, "out")
    assert cuda_lib.decik_kernel_error(1) == 0


@pytest.mark.parametrize("T,hidden,inter", [(830, 1536, 8960), (16384, 1536, 8960), (1, 512, 256), (700, 3584, 18944)])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16], ids=["bf16", "fp16"])
def test_mlp_gate_up_and_down_grad(cuda_lib, T, hidden, inter, dtype):
    from decik_b200 import ops

    g = torch.Generator(device=DEV).manual_seed(T + inter)
    x16 = torch.randn(T, hidden, device=DEV, generator=g).to(dtype)
    w_gu = (torch.randn(2 * inter, hidden, device=DEV, generator=g) * 0.02).to(dtype)
    w_down = (torch.randn(hidden, inter, device=DEV, generator=g) * 0.02).to(dtype)
    gu, h = ops.mlp_gate_up(x16, w_gu)
    _close(gu, x16.float() @ w_gu.float().t(), "gu")
    assert torch.equal(h, ops.swiglu_fwd(gu, inter))               # SwiGLU of the same gu, bit for bit
    grad = torch.randn(T, hidden, device=DEV, generator=g).to(dtype)
    dgu = ops.mlp_down_grad(grad, w_down, gu)
    gh = ops.gemm16(grad, w_down, True)                             # the same product, stored
    _close(gh, grad.float() @ w_down.float(), "grad_hidden")
    assert torch.equal(dgu, ops.swiglu_bwd(gh, gu, inter))          # the SwiGLU backward, bit for bit
    assert cuda_lib.decik_kernel_error(1) == 0


def test_mlp_gemm_entry_points_reject_bad_arguments(cuda_lib):
    from decik_b200 import _lib

    lib = _lib.lib()
    assert lib.decik_gemm16(None, 8, None, 8, 0, None, 8, 5, 7, 8, _lib.BF16, None) == 1      # N % 8
    assert lib.decik_mlp_gate_up(None, 8, None, 8, None, 8, None, 8, 5, 8, 100, _lib.BF16, None) == 1  # inter % 128
    assert lib.decik_mlp_down_grad(None, 8, None, 8, None, 8, None, 8, 5, 8, 128, _lib.BF16, None) == 1  # % 256
