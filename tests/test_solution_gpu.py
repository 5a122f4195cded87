"""The reference-facing autograd Functions (decik_b200.solution) against the oracle and the
reference's golden fixtures, mirroring solution/test_solution.py and dev/test_cpu_*.py."""

import numpy as np
import pytest
import torch

from oracle import attention as o_attn
from oracle import nf4 as o_nf4
from tests.conftest import golden
from tests.tolerance import assert_close16

pytestmark = pytest.mark.gpu
DEV = "cuda"


class _QS:
    pass


def _quant_state(st, dtype=torch.float16):
    qs = _QS()
    qs.shape, qs.nested, qs.blocksize, qs.quant_type, qs.dtype = st["shape"], st["nested"], st["blocksize"], "nf4", dtype
    qs.code = torch.from_numpy(st["code"]).to(DEV)
    if st["nested"]:
        qs.absmax = torch.from_numpy(st["absmax"]).to(DEV)
        qs.state2 = _QS()
        qs.state2.absmax = torch.from_numpy(st["absmax2"]).to(DEV)
        qs.state2.code = torch.from_numpy(st["code2"]).to(DEV)
        qs.state2.blocksize = st["blocksize2"]
        qs.offset = torch.tensor(float(st["offset"]), device=DEV)
    else:
        qs.absmax = torch.from_numpy(st["absmax"]).to(DEV)
    return qs


def test_varlen_sdpa_function_reference_layouts(cuda_lib):
    """VarlenSDPA with the reference's layouts and spans (solution/test_solution.py:164-187)."""
    from decik_b200.solution.varlen import VarlenSDPA

    torch.manual_seed(0)
    hq, hk, d = 12, 2, 128
    spans = [(0, 401), (401, 77), (478, 512), (990, 3)]
    n = sum(L for _, L in spans)
    for dtype in (torch.float16, torch.bfloat16):
        q = torch.randn(1, hq, n, d, device=DEV).to(dtype).requires_grad_(True)
        k = torch.randn(1, hk, n, d, device=DEV).to(dtype).requires_grad_(True)
        v_leaf = torch.randn(1, n, hk, d, device=DEV).to(dtype).requires_grad_(True)
        v = v_leaf.transpose(1, 2)
        g = torch.randn(1, n, hq, d, device=DEV).to(dtype)
        cu = torch.tensor([s for s, _ in spans] + [n], dtype=torch.int32, device=DEV)
        out = VarlenSDPA.apply(q, k, v, cu, 512, hq // hk, d ** -0.5)
        assert out.shape == (1, n, hq, d) and out.is_contiguous()
        out.backward(g)
        f = lambda t: t.detach().float().cpu().numpy()
        ro, _ = o_attn.forward(f(q[0]).transpose(1, 0, 2), f(k[0]).transpose(1, 0, 2), f(v_leaf[0]), spans, d ** -0.5)
        assert_close16(f(out[0]), ro, "out")
        rdq, rdk, rdv = o_attn.backward(f(g[0]), f(q[0]).transpose(1, 0, 2), f(k[0]).transpose(1, 0, 2),
                                        f(v_leaf[0]), spans, d ** -0.5)
        assert_close16(f(q.grad[0]).transpose(1, 0, 2), rdq, "dq")
        assert_close16(f(k.grad[0]).transpose(1, 0, 2), rdk, "dk")
        assert_close16(f(v_leaf.grad[0]), rdv, "dv")


def test_varlen_sdpa_saves_no_expanded_kv(cuda_lib):
    """Only q, k, v, out and lse are kept for backward (no GQA-expanded copies)."""
    from decik_b200.solution.varlen import VarlenSDPA

    n, hq, hk, d = 64, 12, 2, 128
    q = torch.randn(1, hq, n, d, device=DEV, dtype=torch.bfloat16, requires_grad=True)
    k = torch.randn(1, hk, n, d, device=DEV, dtype=torch.bfloat16, requires_grad=True)
    v = torch.randn(1, hk, n, d, device=DEV, dtype=torch.bfloat16, requires_grad=True)
    cu = torch.tensor([0, 40, 64], dtype=torch.int32, device=DEV)
    saved = []
    with torch.autograd.graph.saved_tensors_hooks(lambda t: saved.append(t) or t, lambda t: t):
        VarlenSDPA.apply(q, k, v, cu, 40, 6, None)
    elems = sum(t.numel() for t in saved if t.dtype != torch.int32)
    assert elems == q.numel() * 2 + k.numel() + v.numel() + hq * n


def test_fused_qk_rope_function_golden(cuda_lib):
    from decik_b200.solution.attn import FusedQKRope

    g = golden("rope_golden.npz")
    T, HQ, HK, D = (int(v) for v in g["dims"])
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(DEV)
    qo, ko = FusedQKRope.apply(t(g["qb"]), t(g["ql"]), t(g["kb"]), t(g["cos"]), t(g["sin"]), HQ, HK)
    assert qo.shape == (1, HQ, T, D) and np.array_equal(qo[0].cpu().numpy().view(np.uint16), g["qo"].view(np.uint16))
    ctx = type("C", (), {"saved_tensors": (t(g["cos"]), t(g["sin"]))})()
    dq, dq2, dk, *_ = FusedQKRope.backward(ctx, t(g["gq"])[None], t(g["gk"])[None])
    assert torch.equal(dq, dq2)
    assert np.array_equal(dq.cpu().numpy().view(np.uint16), g["dq"].view(np.uint16))
    assert np.array_equal(dk.cpu().numpy().view(np.uint16), g["dk"].view(np.uint16))


def test_nf4_linear_function(cuda_lib):
    """NF4Linear: bit-exact dequant inside; forward/backward equal F.linear/matmul on that weight."""
    from decik_b200.solution.nf4 import NF4Linear, dequantize_nf4

    rng = np.random.default_rng(0)
    w = (rng.standard_normal((256, 1536)) * 0.02).astype(np.float32)
    st = o_nf4.quantize_nf4(w)
    qs = _quant_state(st)
    packed = torch.from_numpy(st["packed"]).to(DEV)
    w16 = dequantize_nf4(packed, qs, torch.float16)
    assert np.array_equal(w16.cpu().numpy().view(np.uint16), o_nf4.dequantize_nf4(st, "f16").view(np.uint16))
    x = torch.randn(77, 1536, device=DEV).half().requires_grad_(True)
    b = torch.randn(256, device=DEV).half()
    y = NF4Linear.apply(x, packed, b, qs)
    assert torch.equal(y, torch.nn.functional.linear(x.detach(), w16, b))
    gy = torch.randn_like(y)
    y.backward(gy)
    assert torch.equal(x.grad, gy @ w16)


def test_lora_pair_from_norm_golden(cuda_lib):
    """LoRAPairFromNorm with packed masks vs the reference's outputs and grads
    (dev/test_cpu_norm_link.py sizes, tests/golden/lora_golden.npz)."""
    from decik_b200.solution.attn import LoRAPairFromNorm, pack_keep
    from decik_b200.solution.rmsnorm import RMSNormFn

    g = golden("lora_golden.npz")
    T, H, R, HV = (int(v) for v in g["dims"])
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(DEV)
    h = t(g["h"]).requires_grad_(True)
    w = t(g["w"])
    params = [t(g[n]).requires_grad_(True) for n in ("a_q", "b_q", "a_v", "b_v")]
    x = RMSNormFn.apply(h, w, float(g["eps"]))
    bq, bv = pack_keep(t(g["keep_q"].reshape(T, H)), t(g["keep_v"].reshape(T, H)))
    scale = torch.tensor(float(g["scale"]), device=DEV)
    p = float(g["p"])
    oq, ov = LoRAPairFromNorm.apply(x, h, w, float(g["eps"]), None, bq, scale, None, bv, scale,
                                    *params, float(g["scaling"]), float(g["scaling"]), p, p, True)
    torch.autograd.backward([oq, ov], [t(g["gq"]), t(g["gv"])])
    rel = lambda a, b: float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-12))
    assert rel(oq.detach().float().cpu().numpy(), g["oq"].astype(np.float32)) < 5e-3
    assert rel(ov.detach().float().cpu().numpy(), g["ov"].astype(np.float32)) < 5e-3
    for name, prm in zip(("da_q", "db_q", "da_v", "db_v"), params):
        assert rel(prm.grad.cpu().numpy(), g[name]) < 1e-2, name
    assert rel(h.grad.cpu().numpy(), g["dh"]) < 1e-2
