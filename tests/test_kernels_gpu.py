"""Parity of the sm_100a kernels (through the C ABI, via decik_b200.ops) with the CPU oracle and
the reference's golden fixtures. Integer / rounding-defined kernels must be bit-exact; attention
must meet the bf16 bar in tests/tolerance.py."""

import hashlib

import numpy as np
import pytest
import torch

from oracle import attention as o_attn
from oracle import lora as o_lora
from oracle import nf4 as o_nf4
from oracle import rmsnorm as o_norm
from oracle import rope as o_rope
from tests.conftest import golden
from tests.tolerance import assert_close16

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _ops():
    from decik_b200 import ops
    return ops


def _dequant_gpu(st, out_dtype):
    ops = _ops()
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(DEV)
    if st["nested"]:
        return ops.nf4_dequant(t(st["packed"]), t(st["absmax"]), t(st["code"]), st["shape"], st["blocksize"],
                               absmax2=t(st["absmax2"]), code2=t(st["code2"]),
                               offset=torch.tensor([float(st["offset"])], dtype=torch.float32, device=DEV),
                               blocksize2=st["blocksize2"], out_dtype=out_dtype)
    return ops.nf4_dequant(t(st["packed"]), t(st["absmax"]), t(st["code"]), st["shape"], st["blocksize"],
                           out_dtype=out_dtype)


def _golden_state(g, tag):
    nested = bool(g[f"{tag}_nested"])
    st = dict(packed=g[f"{tag}_packed"], absmax=g[f"{tag}_absmax"], code=g[f"{tag}_code"],
              shape=tuple(int(v) for v in g[f"{tag}_shape"]), blocksize=64, blocksize2=256, nested=nested)
    if nested:
        st.update(absmax2=g[f"{tag}_absmax2"], code2=g[f"{tag}_code2"], offset=np.float32(g[f"{tag}_offset"]))
    return st


# ---------------------------------------------------------------------------------------- NF4
@pytest.mark.parametrize("tag", ["a", "b", "c"])
def test_nf4_golden_bit_exact(cuda_lib, tag):
    g = golden("nf4_golden.npz")
    out = _dequant_gpu(_golden_state(g, tag), torch.float16).cpu().numpy()
    assert np.array_equal(out.view(np.uint16), g[f"{tag}_out"].view(np.uint16))


@pytest.mark.parametrize("i", [0, 1, 2, 3])
def test_nf4_reference_shapes_hash(cuda_lib, i):
    """solution/test_solution.py:10 shapes: (1536,1536), (256,1536) nested/not, (1536,8960)."""
    from tests.golden.make_golden import random_nf4_state

    g = golden("nf4_golden.npz")
    shape = tuple(int(v) for v in g[f"hash{i}_shape"])
    st = random_nf4_state(shape, bool(g[f"hash{i}_nested"]), int(g[f"hash{i}_seed"]))
    out = _dequant_gpu(st, torch.float16).cpu().numpy()
    assert hashlib.sha256(out.tobytes()).hexdigest() == str(g[f"hash{i}_sha256"])


@pytest.mark.parametrize("shape,nested,bs", [((1536, 1536), True, 64), ((256, 1536), False, 64),
                                             ((8960, 1536), True, 64), ((96, 64), True, 32),
                                             ((128, 256), True, 128), ((7, 18), False, 2),
                                             ((48, 96), True, 96), ((10, 36), False, 6)])
@pytest.mark.parametrize("dtype", ["f16", "bf16", "f32"])
def test_nf4_vs_oracle_bit_exact(cuda_lib, shape, nested, bs, dtype):
    rng = np.random.default_rng(hash((shape, nested, bs)) % 2**32)
    w = (rng.standard_normal(shape) * 0.05).astype(np.float32)
    st = o_nf4.quantize_nf4(w, blocksize=bs, nested=nested)
    tdt = {"f16": torch.float16, "bf16": torch.bfloat16, "f32": torch.float32}[dtype]
    out = _dequant_gpu(st, tdt).cpu()
    ref = o_nf4.dequantize_nf4(st, dtype)
    if dtype == "bf16":
        assert np.array_equal(out.view(torch.int16).numpy().view(np.uint16), ref)
    elif dtype == "f16":
        assert np.array_equal(out.numpy().view(np.uint16), ref.view(np.uint16))
    else:
        assert np.array_equal(out.numpy().view(np.uint32), ref.view(np.uint32))


def test_nf4_dequant_batch_matches_single_calls(cuda_lib):
    """decik_nf4_dequant_batch over a mixed batch (nested and plain weights, one output slice not
    16-byte aligned, so the jobs go to separate launches by kind) equals one call per weight."""
    ops = _ops()
    rng = np.random.default_rng(11)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(DEV)
    shapes = [((1536, 1536), True), ((256, 1536), True), ((256, 1536), False), ((64, 96), True)]
    states = [o_nf4.quantize_nf4((rng.standard_normal(sh) * 0.02).astype(np.float32), nested=nested)
              for sh, nested in shapes]
    rows = sum(sh[0] for sh, _ in shapes)
    big = torch.zeros(rows * 1536 + 8, dtype=torch.bfloat16, device=DEV)
    jobs, refs, r0 = [], [], 0
    for (sh, nested), st in zip(shapes, states):
        n = sh[0] * sh[1]
        # the last weight's output starts 8 bytes off a 16-byte boundary
        off = r0 + (4 if sh == (64, 96) else 0)
        out = big[off:off + n].view(sh)
        args = (t(st["packed"]), t(st["absmax"]), t(st["code"]), sh, 64)
        if nested:
            extra = (t(st["absmax2"]), t(st["code2"]), torch.tensor([float(st["offset"])], device=DEV), 256)
        else:
            extra = (None, None, None, 256)
        jobs.append(args + extra + (out,))
        refs.append(ops.nf4_dequant(*args, absmax2=extra[0], code2=extra[1], offset=extra[2], blocksize2=256,
                                    out_dtype=torch.bfloat16))
        r0 += n
    ops.nf4_dequant_batch(jobs, torch.bfloat16)
    for job, ref in zip(jobs, refs):
        assert torch.equal(job[-1], ref)
    assert cuda_lib.decik_kernel_error(1) == 0


def test_nf4_unaligned_views(cuda_lib):
    """Packed bytes at an odd offset take the scalar path; results are still bit-exact."""
    ops = _ops()
    rng = np.random.default_rng(3)
    w = (rng.standard_normal((64, 128)) * 0.05).astype(np.float32)
    st = o_nf4.quantize_nf4(w, nested=False)
    buf = torch.zeros(st["packed"].size + 1, dtype=torch.uint8, device=DEV)
    buf[1:] = torch.from_numpy(st["packed"]).to(DEV)
    out = ops.nf4_dequant(buf[1:], torch.from_numpy(st["absmax"]).to(DEV),
                          torch.from_numpy(st["code"]).to(DEV), st["shape"], 64).cpu().numpy()
    assert np.array_equal(out.view(np.uint16), o_nf4.dequantize_nf4(st, "f16").view(np.uint16))


# ---------------------------------------------------------------------------------------- RoPE
def test_rope_golden_bit_exact(cuda_lib):
    ops = _ops()
    g = golden("rope_golden.npz")
    T, HQ, HK, D = (int(v) for v in g["dims"])
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(DEV)
    qo, ko = ops.rope_fwd(t(g["qb"]), t(g["ql"]), t(g["kb"]), t(g["cos"]), t(g["sin"]), HQ, HK)
    assert np.array_equal(qo.cpu().numpy().view(np.uint16), g["qo"].view(np.uint16))
    assert np.array_equal(ko.cpu().numpy().view(np.uint16), g["ko"].view(np.uint16))
    dq, dk = ops.rope_bwd(t(g["gq"]), t(g["gk"]), t(g["cos"]), t(g["sin"]))
    assert np.array_equal(dq.cpu().numpy().view(np.uint16), g["dq"].view(np.uint16))
    assert np.array_equal(dk.cpu().numpy().view(np.uint16), g["dk"].view(np.uint16))


@pytest.mark.parametrize("T,HQ,HK", [(1, 12, 2), (830, 12, 2), (513, 28, 4)])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_rope_vs_oracle_bit_exact(cuda_lib, T, HQ, HK, dtype):
    ops = _ops()
    D = 128
    torch.manual_seed(T)
    qb = (torch.randn(T, HQ * D) * 3).to(dtype)
    ql = (torch.randn(T, HQ * D) * 0.1).to(dtype)
    kb = (torch.randn(T, HK * D) * 3).to(dtype)
    c, s = o_rope.cos_sin(np.arange(T) % 300, D)
    gq = torch.randn(HQ, T, D).to(dtype)
    gk = torch.randn(HK, T, D).to(dtype)
    qo, ko = ops.rope_fwd(qb.to(DEV), ql.to(DEV), kb.to(DEV), torch.from_numpy(c).to(DEV),
                          torch.from_numpy(s).to(DEV), HQ, HK)
    dq, dk = ops.rope_bwd(gq.to(DEV), gk.to(DEV), torch.from_numpy(c).to(DEV), torch.from_numpy(s).to(DEV))
    f = lambda x: x.float().numpy()
    odt = "bf16" if dtype == torch.bfloat16 else np.float16
    rq, rk = o_rope.rope_fwd(f(qb), f(ql), f(kb), c, s, HQ, HK, odt)
    rdq, rdk = o_rope.rope_bwd(f(gq), f(gk), c, s, odt)
    bits = lambda x: x.cpu().view(torch.int16).numpy().view(np.uint16)
    ref_bits = lambda r: r if dtype == torch.bfloat16 else r.view(np.uint16)
    assert np.array_equal(bits(qo), ref_bits(rq)) and np.array_equal(bits(ko), ref_bits(rk))
    assert np.array_equal(bits(dq), ref_bits(rdq)) and np.array_equal(bits(dk), ref_bits(rdk))


# ---------------------------------------------------------------------------------------- LoRA
def test_lora_kernels_golden_bit_exact(cuda_lib):
    ops = _ops()
    g = golden("lora_golden.npz")
    T, H, R, HV = (int(v) for v in g["dims"])
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(DEV)
    bq, bv = ops.keep_pack(t(g["keep_q"].reshape(T, H)), t(g["keep_v"].reshape(T, H)))
    assert np.array_equal(bq.cpu().numpy(), g["bits_q"]) and np.array_equal(bv.cpu().numpy(), g["bits_v"])
    scale = torch.tensor(float(g["scale"]), device=DEV)
    xq, xv = ops.lora_inputs(t(g["x"].reshape(T, H)), bq, bv, scale, scale)
    assert np.array_equal(xq.cpu().numpy().view(np.uint16), g["xq16"].view(np.uint16))
    assert np.array_equal(xv.cpu().numpy().view(np.uint16), g["xv16"].view(np.uint16))
    s = 1.0 / (1.0 - float(g["p"]))
    gin = ops.lora_input_grad(t(g["giq"]), t(g["giv"]), bq, bv, s, s)
    assert np.array_equal(gin.cpu().numpy().view(np.uint32), g["gin"].view(np.uint32))


def test_lora_inputs_bf16_vs_oracle(cuda_lib):
    ops = _ops()
    rng = np.random.default_rng(1)
    T, W = 77, 1536
    x = rng.standard_normal((T, W)).astype(np.float32)
    kq = rng.random((T, W)) > 0.1
    kv = rng.random((T, W)) > 0.1
    bq, bv = o_lora.keep_pack(kq), o_lora.keep_pack(kv)
    sc = np.float32(1 / 0.9)
    xq, xv = ops.lora_inputs(torch.from_numpy(x).to(DEV), torch.from_numpy(bq).to(DEV),
                             torch.from_numpy(bv).to(DEV), torch.tensor(sc, device=DEV),
                             torch.tensor(sc, device=DEV), out_dtype=torch.bfloat16)
    rq, rv = o_lora.lora_inputs(x, bq, bv, sc, sc, out_dtype="bf16")
    assert np.array_equal(xq.cpu().view(torch.int16).numpy().view(np.uint16), rq)
    assert np.array_equal(xv.cpu().view(torch.int16).numpy().view(np.uint16), rv)


# ---------------------------------------------------------------------------------------- RMSNorm
def test_rmsnorm_vs_oracle(cuda_lib):
    ops = _ops()
    g = golden("lora_golden.npz")
    T, H = int(g["dims"][0]), int(g["dims"][1])
    x = torch.from_numpy(g["h"].reshape(T, H)).to(DEV)
    w = torch.from_numpy(g["w"]).to(DEV)
    y, rstd = ops.rmsnorm_fwd(x, w, float(g["eps"]))
    np.testing.assert_allclose(y.cpu().numpy(), g["norm_y"].reshape(T, H), rtol=1e-5, atol=1e-5)
    dx = ops.rmsnorm_bwd(torch.from_numpy(g["norm_gy"].reshape(T, H)).to(DEV), x, w, rstd)
    np.testing.assert_allclose(dx.cpu().numpy(), g["norm_dx"].reshape(T, H), rtol=1e-4, atol=1e-5)
    y2, _ = ops.rmsnorm_fwd(x, w, float(g["eps"]))
    assert torch.equal(y, y2)  # the recompute is bit-identical


def test_add_rmsnorm_golden(cuda_lib):
    """The fused residual add + norm against the reference's AddRMSNormFn fixture (fp16 delta):
    h bit-exact, y and the input gradients within fp32 rounding, the fp16 gradient within one ulp."""
    ops = _ops()
    g = golden("addnorm_golden.npz")
    eps = float(g["eps"])
    r = torch.from_numpy(g["residual"][0]).to(DEV)
    d = torch.from_numpy(g["delta"][0]).to(DEV)
    w = torch.from_numpy(g["w"]).to(DEV)
    h, y, rstd = ops.add_rmsnorm_fwd(r, d, w, eps)
    assert np.array_equal(h.cpu().numpy(), g["h"][0])
    np.testing.assert_allclose(y.cpu().numpy(), g["y"][0], rtol=1e-5, atol=1e-5)
    dx, dx16 = ops.add_rmsnorm_bwd(torch.from_numpy(g["grad_y"][0]).to(DEV), torch.from_numpy(g["grad_h"][0]).to(DEV),
                                   r, d, w, rstd)
    np.testing.assert_allclose(dx.cpu().numpy(), g["d_residual"][0], rtol=1e-4, atol=1e-5)
    ref16 = g["d_delta"][0].astype(np.float32)
    ulp = np.spacing(np.abs(g["d_delta"][0])).astype(np.float32)
    assert dx16.dtype == torch.float16 and np.all(np.abs(dx16.cpu().float().numpy() - ref16) <= ulp)


@pytest.mark.parametrize("rows,cols", [(1, 256), (37, 1536), (1000, 1536), (5, 8192)])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16, torch.float32])
def test_add_rmsnorm_equals_unfused_kernels(cuda_lib, rows, cols, dtype):
    """One pass each way equals the composition it replaces bit for bit: torch's fp32 + 16-bit add,
    decik_rmsnorm_fwd on h, decik_rmsnorm_bwd plus grad_h, and the cast of the sum; also without
    grad_h, and within tolerance of the fp64 oracle."""
    ops = _ops()
    g = torch.Generator().manual_seed(rows + cols)
    r = (torch.randn(rows, cols, generator=g) * 3).to(DEV)
    d = (torch.randn(rows, cols, generator=g) * 2).to(dtype).to(DEV)
    w = (torch.rand(cols, generator=g) + 0.5).to(DEV)
    dy = torch.randn(rows, cols, generator=g).to(DEV)
    gh = torch.randn(rows, cols, generator=g).to(DEV)
    eps = 1e-6
    h, y, rstd = ops.add_rmsnorm_fwd(r, d, w, eps)
    h_ref = r + d.float()
    assert torch.equal(h, h_ref)
    y_ref, rstd_ref = ops.rmsnorm_fwd(h_ref, w, eps)
    assert torch.equal(y, y_ref) and torch.equal(rstd, rstd_ref)
    dx, dx16 = ops.add_rmsnorm_bwd(dy, gh, r, d, w, rstd)
    dx_ref = gh + ops.rmsnorm_bwd(dy, h_ref, w, rstd_ref)
    assert torch.equal(dx, dx_ref)
    assert dx16.dtype == dtype and torch.equal(dx16, dx_ref.to(dtype))
    dx_n, _ = ops.add_rmsnorm_bwd(dy, None, r, d, w, rstd, want_dx16=False)
    assert torch.equal(dx_n, ops.rmsnorm_bwd(dy, h_ref, w, rstd_ref))
    yo, _ = o_norm.forward(h_ref.cpu().numpy(), w.cpu().numpy(), eps)
    np.testing.assert_allclose(y.cpu().numpy(), yo, rtol=1e-5, atol=1e-5)
    tot, _ = o_norm.add_backward(gh.cpu().numpy(), dy.cpu().numpy(), r.cpu().numpy(), d.cpu().float().numpy(),
                                 w.cpu().numpy(), eps)
    np.testing.assert_allclose(dx.cpu().numpy(), tot, rtol=1e-4, atol=1e-4)


@pytest.mark.parametrize("rows,cols", [(1, 256), (1000, 1536), (5, 8192)])
@pytest.mark.parametrize("wdtype", [torch.float32, torch.float16])
def test_rmsnorm_bwd_with_addend(cuda_lib, rows, cols, wdtype):
    """decik_rmsnorm_bwd_add equals the separate norm backward plus the addend (one fp32 add per
    element, as autograd's sum of the two gradients), bit for bit."""
    ops = _ops()
    g = torch.Generator().manual_seed(rows * 7 + cols)
    x = (torch.randn(rows, cols, generator=g) * 2).to(DEV)
    w = (torch.rand(cols, generator=g) + 0.5).to(wdtype).to(DEV)
    dy = torch.randn(rows, cols, generator=g).to(DEV)
    add = torch.randn(rows, cols, generator=g).to(DEV)
    _, rstd = ops.rmsnorm_fwd(x, w, 1e-6)
    assert torch.equal(ops.rmsnorm_bwd(dy, x, w, rstd, addend=add), add + ops.rmsnorm_bwd(dy, x, w, rstd))
    assert cuda_lib.decik_kernel_error(1) == 0


@pytest.mark.parametrize("rows,cols", [(1, 256), (1000, 1536), (5, 8192)])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("wdtype", [torch.float32, torch.float16])
def test_add_rmsnorm_16bit_y_and_dy(cuda_lib, rows, cols, dtype, wdtype):
    """The 16-bit variants (decik_add_rmsnorm_fwd16 / _bwd16) equal the fp32 ones bit for bit: y is
    the fp32 y rounded to delta's dtype (h, rstd unchanged), and the backward of a 16-bit dy is the
    backward of the same dy widened to fp32."""
    ops = _ops()
    g = torch.Generator().manual_seed(rows + cols + 1)
    r = (torch.randn(rows, cols, generator=g) * 3).to(DEV)
    d = (torch.randn(rows, cols, generator=g) * 2).to(dtype).to(DEV)
    w = (torch.rand(cols, generator=g) + 0.5).to(wdtype).to(DEV)
    dy16 = torch.randn(rows, cols, generator=g).to(dtype).to(DEV)
    gh = torch.randn(rows, cols, generator=g).to(DEV)
    h, y, rstd = ops.add_rmsnorm_fwd(r, d, w, 1e-6)
    h16, y16, rstd16 = ops.add_rmsnorm_fwd(r, d, w, 1e-6, y16=True)
    assert y16.dtype == dtype and torch.equal(y16, y.to(dtype))
    assert torch.equal(h16, h) and torch.equal(rstd16, rstd)
    for grad_h in (gh, None):
        dx, dx_16 = ops.add_rmsnorm_bwd(dy16, grad_h, r, d, w, rstd)
        dx_ref, dx_16_ref = ops.add_rmsnorm_bwd(dy16.float(), grad_h, r, d, w, rstd)
        assert torch.equal(dx, dx_ref) and torch.equal(dx_16, dx_16_ref)
    assert cuda_lib.decik_kernel_error(1) == 0
    with pytest.raises(RuntimeError, match="16-bit delta"):
        ops.add_rmsnorm_fwd(r, r.clone(), w, 1e-6, y16=True)


def test_add_rmsnorm_rejects_bad_arguments(cuda_lib):
    ops = _ops()
    r = torch.randn(4, 6, device=DEV)
    with pytest.raises(RuntimeError, match="n_cols"):
        ops.add_rmsnorm_fwd(r, r.half(), torch.ones(6, device=DEV), 1e-6)
    with pytest.raises(RuntimeError, match="same shape"):
        ops.add_rmsnorm_fwd(torch.randn(4, 8, device=DEV), torch.randn(4, 4, device=DEV).half(),
                            torch.ones(8, device=DEV), 1e-6)


# ---------------------------------------------------------------------------------------- attention
def _attn_case(lengths, HQ, HK, dtype, seed=0, layout="token"):
    torch.manual_seed(seed)
    D = 128
    T = int(sum(lengths))
    spans, start = [], 0
    for L in lengths:
        spans.append((start, int(L)))
        start += int(L)
    cu = torch.tensor([s for s, _ in spans] + [T], dtype=torch.int32, device=DEV)
    if layout == "token":
        q = torch.randn(T, HQ, D).to(dtype).to(DEV)
        k = torch.randn(T, HK, D).to(dtype).to(DEV)
        v = torch.randn(T, HK, D).to(dtype).to(DEV)
    else:  # the reference's layouts: q, k head-major, v token-major (solution/attn.py:408-412)
        q = torch.randn(HQ, T, D).to(dtype).to(DEV).transpose(0, 1)
        k = torch.randn(HK, T, D).to(dtype).to(DEV).transpose(0, 1)
        v = torch.randn(T, HK, D).to(dtype).to(DEV)
    do = torch.randn(T, HQ, D).to(dtype).to(DEV)
    return spans, cu, q, k, v, do


def _np(t):
    return t.float().cpu().numpy()


CASES = [
    ([37, 128, 211, 454], 12, 2),                # config 1 lengths
    ([300, 1000, 3], 28, 4),                     # 7B heads: odd group size 7
    ([401, 77, 512, 3], 12, 2),                  # solution/test_solution.py:76 spans
    ([37, 5, 20, 1], 12, 2),                     # dev/test_cpu_sdpa.py:24 spans
    ([1], 12, 2),                                # a single token
    ([129, 64, 65, 127, 191], 28, 4),            # 7B heads, lengths around tile edges
    ([1000], 4, 4),                              # no GQA, one long row
]


@pytest.mark.parametrize("lengths,HQ,HK", CASES)
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_varlen_attention_fwd_bwd_vs_oracle(cuda_lib, lengths, HQ, HK, dtype):
    ops = _ops()
    spans, cu, q, k, v, do = _attn_case(lengths, HQ, HK, dtype, layout="ref")
    scale = 128 ** -0.5
    out, lse = ops.varlen_attn_fwd(q, k, v, cu, max(lengths), scale)
    ro, rl = o_attn.forward(_np(q), _np(k), _np(v), spans, scale)
    assert_close16(_np(out), ro, "out")
    np.testing.assert_allclose(lse.cpu().numpy(), rl, rtol=0, atol=2e-3)
    dq, dk, dv = ops.varlen_attn_bwd(do, q, k, v, out, lse, cu, max(lengths), scale)
    assert dq.stride() == q.stride() and dk.stride() == k.stride() and dv.stride() == v.stride()
    rdq, rdk, rdv = o_attn.backward(_np(do), _np(q), _np(k), _np(v), spans, scale)
    assert_close16(_np(dq), rdq, "dq")
    assert_close16(_np(dk), rdk, "dk")
    assert_close16(_np(dv), rdv, "dv")
    assert cuda_lib.decik_kernel_error(1) == 0


def test_varlen_attention_golden_reference_packed_sdpa(cuda_lib):
    """The reference's own PackedSDPA outputs and grads (tests/golden/sdpa_golden.npz)."""
    ops = _ops()
    g = golden("sdpa_golden.npz")
    HQ, HK, D = (int(v) for v in g["dims"])
    spans = [tuple(int(x) for x in s) for s in g["spans"]]
    T = sum(L for _, L in spans)
    cu = torch.tensor([s for s, _ in spans] + [T], dtype=torch.int32, device=DEV)
    q = torch.from_numpy(g["q"]).to(DEV).transpose(0, 1)      # [T, H, D] view of head-major
    k = torch.from_numpy(g["k"]).to(DEV).transpose(0, 1)
    v = torch.from_numpy(g["v"]).to(DEV)
    do = torch.from_numpy(g["g"][0] if g["g"].ndim == 4 else g["g"]).to(DEV)
    out, lse = ops.varlen_attn_fwd(q, k, v, cu, max(L for _, L in spans), D ** -0.5)
    assert_close16(_np(out), g["out"], "out")
    dq, dk, dv = ops.varlen_attn_bwd(do, q, k, v, out, lse, cu, max(L for _, L in spans), D ** -0.5)
    assert_close16(_np(dq).transpose(1, 0, 2), g["dq"], "dq")
    assert_close16(_np(dk).transpose(1, 0, 2), g["dk"], "dk")
    assert_close16(_np(dv), g["dv"], "dv")


def test_varlen_attention_deterministic_forward(cuda_lib):
    ops = _ops()
    spans, cu, q, k, v, do = _attn_case([300, 700, 5], 12, 2, torch.bfloat16, seed=4)
    a, la = ops.varlen_attn_fwd(q, k, v, cu, 700, 0.088)
    b, lb = ops.varlen_attn_fwd(q, k, v, cu, 700, 0.088)
    assert torch.equal(a, b) and torch.equal(la, lb)
    assert cuda_lib.decik_kernel_error(1) == 0


def test_varlen_attention_large_properties(cuda_lib):
    """Config-3 sized packing (16,384 tokens, L ~ U[64, 4096]): checked on sampled rows against the
    oracle, and for size-independent properties (rows do not interact; finite outputs)."""
    ops = _ops()
    rng = np.random.default_rng(0)
    lengths, total = [], 0
    while total < 16384:
        L = int(min(rng.integers(64, 4097), 16384 - total))
        lengths.append(L)
        total += L
    spans, cu, q, k, v, do = _attn_case(lengths, 12, 2, torch.bfloat16, seed=1)
    scale = 128 ** -0.5
    out, lse = ops.varlen_attn_fwd(q, k, v, cu, max(lengths), scale)
    dq, dk, dv = ops.varlen_attn_bwd(do, q, k, v, out, lse, cu, max(lengths), scale)
    for t in (out, dq, dk, dv, lse):
        assert torch.isfinite(t).all()
    # the shortest row, checked alone against the oracle (rows must not see each other)
    i = int(np.argmin(lengths))
    s, L = spans[i]
    sl = slice(s, s + L)
    ro, _ = o_attn.forward(_np(q[sl]), _np(k[sl]), _np(v[sl]), [(0, L)], scale)
    assert_close16(_np(out[sl]), ro, "out row")
    rdq, rdk, rdv = o_attn.backward(_np(do[sl]), _np(q[sl]), _np(k[sl]), _np(v[sl]), [(0, L)], scale)
    assert_close16(_np(dq[sl]), rdq, "dq row")
    assert_close16(_np(dk[sl]), rdk, "dk row")
    assert_close16(_np(dv[sl]), rdv, "dv row")


def _attn_fp32_rows(q, k, v, do, spans, scale, chunk=512):
    """The math of oracle/attention.py (per-row causal softmax attention, query head h reading kv
    head h // groups, and its gradients with delta = rowsum(dO * O)) restated in fp32 torch on the
    GPU, query-chunked so that rows of 32,768 tokens fit: the full-size reference."""
    T, HQ, D = q.shape
    HK = k.shape[1]
    g = HQ // HK
    dev = q.device
    out = torch.empty(T, HQ, D, device=dev)
    lse = torch.empty(HQ, T, device=dev)
    dq = torch.empty(T, HQ, D, device=dev)
    dk = torch.empty(T, HK, D, device=dev)
    dv = torch.empty(T, HK, D, device=dev)
    for s, L in spans:
        qf = q[s:s + L].float().transpose(0, 1)
        kf = k[s:s + L].float().transpose(0, 1).repeat_interleave(g, 0)
        vf = v[s:s + L].float().transpose(0, 1).repeat_interleave(g, 0)
        dof = do[s:s + L].float().transpose(0, 1)
        dkf = torch.zeros(HQ, L, D, device=dev)
        dvf = torch.zeros(HQ, L, D, device=dev)
        for c0 in range(0, L, chunk):
            c1 = min(L, c0 + chunk)
            sc = torch.bmm(qf[:, c0:c1], kf[:, :c1].transpose(1, 2)) * scale
            qi = torch.arange(c0, c1, device=dev)[:, None]
            kj = torch.arange(c1, device=dev)[None, :]
            sc.masked_fill_(kj > qi, float("-inf"))
            lc = torch.logsumexp(sc, -1)
            p = torch.exp(sc - lc[..., None])
            del sc
            o = torch.bmm(p, vf[:, :c1])
            dp = torch.bmm(dof[:, c0:c1], vf[:, :c1].transpose(1, 2))
            ds = p * (dp - (dof[:, c0:c1] * o).sum(-1, keepdim=True))
            del dp
            dvf[:, :c1] += torch.bmm(p.transpose(1, 2), dof[:, c0:c1])
            del p
            dq[s + c0:s + c1] = (torch.bmm(ds, kf[:, :c1]) * scale).transpose(0, 1)
            dkf[:, :c1] += torch.bmm(ds.transpose(1, 2), qf[:, c0:c1]) * scale
            del ds
            out[s + c0:s + c1] = o.transpose(0, 1)
            lse[:, s + c0:s + c1] = lc
        dk[s:s + L] = dkf.view(HK, g, L, D).sum(1).transpose(0, 1)
        dv[s:s + L] = dvf.view(HK, g, L, D).sum(1).transpose(0, 1)
    return out, lse, dq, dk, dv


def _close_gpu(actual, expected, what):
    """tests/tolerance.py's bar, evaluated on the device (the arrays are GBs)."""
    from tests.tolerance import MAX_ABS, REL_L2

    a, e = actual.float(), expected.float()
    assert torch.isfinite(a).all(), f"{what}: non-finite values"
    d = a - e
    rel = (d.norm() / e.norm().clamp_min(1.0)).item()
    mx = (d.abs().max() / e.abs().max().clamp_min(1.0)).item()
    assert rel <= REL_L2 and mx <= MAX_ABS, f"{what}: rel-L2 {rel:.3e} (<= {REL_L2}), max-abs {mx:.3e} (<= {MAX_ABS})"


def test_varlen_attention_config4_full_size(cuda_lib):
    """The 7B block's attention at full size (28 / 4 heads, 131,072 tokens, rows up to 32,768)
    against the fp32 restatement, every row and every output."""
    from bench import lengths_config4

    ops = _ops()
    lengths = lengths_config4(0)
    assert sum(lengths) == 131072 and max(lengths) == 32768
    spans, cu, q, k, v, do = _attn_case(lengths, 28, 4, torch.bfloat16, seed=7, layout="ref")
    scale = 128 ** -0.5
    out, lse = ops.varlen_attn_fwd(q, k, v, cu, max(lengths), scale)
    dq, dk, dv = ops.varlen_attn_bwd(do, q, k, v, out, lse, cu, max(lengths), scale)
    torch.cuda.synchronize()
    assert cuda_lib.decik_kernel_error(1) == 0
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        ro, rl, rdq, rdk, rdv = _attn_fp32_rows(q, k, v, do, spans, scale)
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    _close_gpu(out, ro, "out")
    assert (lse - rl).abs().max().item() <= 2e-3
    _close_gpu(dq, rdq, "dq")
    _close_gpu(dk, rdk, "dk")
    _close_gpu(dv, rdv, "dv")
    # the longest row alone meets the bar too (not only through the sums over all rows)
    s, L = spans[0]
    for name, a, e in (("out", out, ro), ("dq", dq, rdq), ("dk", dk, rdk), ("dv", dv, rdv)):
        _close_gpu(a[s:s + L], e[s:s + L], f"{name} of the 32,768-token row")


@pytest.mark.parametrize("world,rank", [(1, 0)] + [(8, r) for r in range(8)])
def test_varlen_attention_bench_packings_every_row(cuda_lib, world, rank):
    """The packings bench.py's config-3 block step times: at N = 1 and on each of the 8 ranks at
    N = 8 (bench.block_lengths: one pool of N x 16,384 tokens, rows U[64, 4096], split by
    dp.partition_rows), 12 / 2 heads, bf16, q and k head-major as the projection epilogue writes
    them. This runs the launch order the bench runs (the heavy-first persistent forward and the
    head-split backward with fp32 dK / dV partials). Every row of out, lse, dq, dk and dv is
    checked against the fp32 restatement: the bar holds for the whole packing and for each row."""
    from bench import block_lengths

    ops = _ops()
    lengths = block_lengths("config3", world, rank)
    assert abs(sum(lengths) - 16384) < 4096
    spans, cu, q, k, v, do = _attn_case(lengths, 12, 2, torch.bfloat16, seed=50 + rank, layout="ref")
    scale = 128 ** -0.5
    out, lse = ops.varlen_attn_fwd(q, k, v, cu, max(lengths), scale)
    dq, dk, dv = ops.varlen_attn_bwd(do, q, k, v, out, lse, cu, max(lengths), scale)
    torch.cuda.synchronize()
    assert cuda_lib.decik_kernel_error(1) == 0
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        ro, rl, rdq, rdk, rdv = _attn_fp32_rows(q, k, v, do, spans, scale)
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    assert (lse - rl).abs().max().item() <= 2e-3
    for name, a, e in (("out", out, ro), ("dq", dq, rdq), ("dk", dk, rdk), ("dv", dv, rdv)):
        _close_gpu(a, e, name)
        for i, (s, L) in enumerate(spans):
            _close_gpu(a[s:s + L], e[s:s + L], f"{name} of row {i} (length {L})")


@pytest.mark.parametrize("world,rank", [(1, 0), (8, 3)])
def test_attn_qkv_bwd_bench_packing_every_row(cuda_lib, world, rank):
    """The one-call backward the fused block runs (decik_attn_qkv_bwd: attention backward, then the
    projection epilogue reading its fp32 accumulators) on a bench packing. With cos = 1 and sin = 0
    RoPE^T is the identity, so dy's q, k and v columns are dq, dk and dv rounded to bf16: every row
    is checked against the fp32 restatement."""
    from bench import block_lengths

    ops = _ops()
    lengths = block_lengths("config3", world, rank)
    T, HQ, HK, D = sum(lengths), 12, 2, 128
    spans, cu, q, k, v, do = _attn_case(lengths, HQ, HK, torch.bfloat16, seed=70 + rank, layout="ref")
    scale = D ** -0.5
    out, lse = ops.varlen_attn_fwd(q, k, v, cu, max(lengths), scale)
    cos = torch.ones(T, D, device=DEV)
    sin = torch.zeros(T, D, device=DEV)
    dy = torch.zeros(T, (HQ + 2 * HK) * D + 32, dtype=torch.bfloat16, device=DEV)
    ops.attn_qkv_bwd(do, q, k, v, out, lse, cu, max(lengths), scale, cos, sin, None, 1.0, dy)
    torch.cuda.synchronize()
    assert cuda_lib.decik_kernel_error(1) == 0
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        _, _, rdq, rdk, rdv = _attn_fp32_rows(q, k, v, do, spans, scale)
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    got = {"dq": dy[:, :HQ * D].view(T, HQ, D), "dk": dy[:, HQ * D:(HQ + HK) * D].view(T, HK, D),
           "dv": dy[:, (HQ + HK) * D:(HQ + 2 * HK) * D].view(T, HK, D)}
    for name, e in (("dq", rdq), ("dk", rdk), ("dv", rdv)):
        _close_gpu(got[name], e, name)
        for i, (s, L) in enumerate(spans):
            _close_gpu(got[name][s:s + L], e[s:s + L], f"{name} of row {i} (length {L})")
