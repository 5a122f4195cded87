"""The CPU oracle against the golden fixtures made by running the reference's own modules.

These pin ``oracle/`` before it is trusted as the checker of the CUDA path. Fixtures come from
tests/golden/make_golden.py (reference kernels under the Triton interpreter).
"""

import hashlib

import numpy as np
import pytest
import torch

from tests.conftest import golden
from oracle import attention, lora, nf4, packing, rmsnorm, rope


def _state(g, tag):
    nested = bool(g[f"{tag}_nested"])
    st = dict(packed=g[f"{tag}_packed"], absmax=g[f"{tag}_absmax"], code=g[f"{tag}_code"],
              shape=tuple(int(v) for v in g[f"{tag}_shape"]), blocksize=64, blocksize2=256,
              nested=nested)
    if nested:
        st.update(absmax2=g[f"{tag}_absmax2"], code2=g[f"{tag}_code2"],
                  offset=np.float32(g[f"{tag}_offset"]))
    return st


@pytest.mark.parametrize("tag", ["a", "b", "c"])
def test_nf4_dequant_bit_exact_vs_reference_kernel(tag):
    g = golden("nf4_golden.npz")
    out = nf4.dequantize_nf4(_state(g, tag), "f16")
    assert out.dtype == np.float16
    assert np.array_equal(out.view(np.uint16), g[f"{tag}_out"].view(np.uint16))


@pytest.mark.parametrize("i", [0, 1, 2, 3])
def test_nf4_dequant_reference_shapes_hash(i):
    """The reference test's four shapes (solution/test_solution.py:10), by output hash."""
    from tests.golden.make_golden import random_nf4_state

    g = golden("nf4_golden.npz")
    shape = tuple(int(v) for v in g[f"hash{i}_shape"])
    st = random_nf4_state(shape, bool(g[f"hash{i}_nested"]), int(g[f"hash{i}_seed"]))
    out = nf4.dequantize_nf4(st, "f16")
    assert np.array_equal(out.reshape(-1)[:64].view(np.uint16), g[f"hash{i}_head"].view(np.uint16))
    assert hashlib.sha256(out.tobytes()).hexdigest() == str(g[f"hash{i}_sha256"])


def test_nf4_bf16_is_rne_of_fp32_product():
    g = golden("nf4_golden.npz")
    st = _state(g, "a")
    f32 = nf4.dequant_f32(st)
    bf = nf4.dequantize_nf4(st, "bf16")
    ref = torch.from_numpy(f32).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    assert np.array_equal(bf, ref)


def test_nf4_quantizer_roundtrip_and_table():
    code = nf4.nf4_code()
    assert code.shape == (16,) and code[0] == -1.0 and code[-1] == 1.0 and 0.0 in code
    # the published NF4 values (QLoRA, arXiv:2305.14314, appendix E)
    assert abs(code[1] + 0.6961928) < 1e-5 and abs(code[8] - 0.0795803) < 1e-5
    d = nf4.dynamic_code()
    assert d.shape == (256,) and np.all(np.diff(d) >= 0) and d.max() == 1.0
    rng = np.random.default_rng(0)
    w = (rng.standard_normal((64, 256)) * 0.05).astype(np.float32)
    for nested in (True, False):
        st = nf4.quantize_nf4(w, nested=nested)
        err = np.abs(nf4.dequantize_nf4(st, "f32") - w).mean() / np.abs(w).mean()
        assert err < 0.12


def test_rope_fwd_bwd_bit_exact_vs_reference_kernel():
    g = golden("rope_golden.npz")
    T, HQ, HK, D = (int(v) for v in g["dims"])
    qo, ko = rope.rope_fwd(g["qb"], g["ql"], g["kb"], g["cos"], g["sin"], HQ, HK, np.float16)
    assert np.array_equal(qo.view(np.uint16), g["qo"].view(np.uint16))
    assert np.array_equal(ko.view(np.uint16), g["ko"].view(np.uint16))
    dq, dk = rope.rope_bwd(g["gq"], g["gk"], g["cos"], g["sin"], np.float16)
    assert np.array_equal(dq.view(np.uint16), g["dq"].view(np.uint16))
    assert np.array_equal(dk.view(np.uint16), g["dk"].view(np.uint16))


def test_cos_sin_matches_reference_table():
    g = golden("rope_golden.npz")
    T = int(g["dims"][0])
    c, s = rope.cos_sin(np.arange(T) + 5, 128, 1e6)
    assert np.array_equal(c, g["cos"]) and np.array_equal(s, g["sin"])


def test_packed_attention_vs_reference_packed_sdpa():
    g = golden("sdpa_golden.npz")
    HQ, HK, D = (int(v) for v in g["dims"])
    spans = [tuple(int(x) for x in s) for s in g["spans"]]
    q = g["q"].astype(np.float32).transpose(1, 0, 2)     # [T, H, D]
    k = g["k"].astype(np.float32).transpose(1, 0, 2)
    v = g["v"].astype(np.float32)
    out, lse = attention.forward(q, k, v, spans, D ** -0.5)
    np.testing.assert_allclose(out, g["out"], rtol=1e-5, atol=1e-5)
    dq, dk, dv = attention.backward(g["g"].astype(np.float32), q, k, v, spans, D ** -0.5)
    np.testing.assert_allclose(dq.transpose(1, 0, 2), g["dq"], rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(dk.transpose(1, 0, 2), g["dk"], rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(dv, g["dv"], rtol=1e-4, atol=1e-5)
    # logsumexp: every row's first token attends to itself only
    for start, _ in spans:
        for h in range(HQ):
            s0 = float(q[start, h].astype(np.float64) @ k[start, h // (HQ // HK)]) * D ** -0.5
            assert abs(lse[h, start] - s0) < 1e-9


def test_lora_kernels_vs_reference():
    g = golden("lora_golden.npz")
    T, H, R, HV = (int(v) for v in g["dims"])
    bits_q = lora.keep_pack(g["keep_q"].reshape(T, H))
    bits_v = lora.keep_pack(g["keep_v"].reshape(T, H))
    assert np.array_equal(bits_q, g["bits_q"]) and np.array_equal(bits_v, g["bits_v"])
    xq, xv = lora.lora_inputs(g["x"].reshape(T, H), bits_q, bits_v, g["scale"], g["scale"])
    assert np.array_equal(xq.view(np.uint16), g["xq16"].view(np.uint16))
    assert np.array_equal(xv.view(np.uint16), g["xv16"].view(np.uint16))
    s = np.float32(1.0 / (1.0 - float(g["p"])))
    gin = lora.lora_input_grad(g["giq"], g["giv"], bits_q, bits_v, s, s)
    assert np.array_equal(gin, g["gin"])


def test_lora_pair_math_vs_reference():
    g = golden("lora_golden.npz")
    T, H, R, HV = (int(v) for v in g["dims"])
    scaling = float(g["scaling"])
    xq16, xv16 = g["xq16"].astype(np.float32), g["xv16"].astype(np.float32)
    u_q, oq = lora.pair_forward(xq16, g["a_q"].astype(np.float16), g["b_q"].astype(np.float16), scaling)
    u_v, ov = lora.pair_forward(xv16, g["a_v"].astype(np.float16), g["b_v"].astype(np.float16), scaling)
    np.testing.assert_allclose(oq, g["oq"].reshape(T, H), rtol=2e-2, atol=2e-3)
    np.testing.assert_allclose(ov, g["ov"].reshape(T, HV), rtol=2e-2, atol=2e-3)
    da_q, db_q, _ = lora.pair_backward(g["gq"].reshape(T, H), xq16, u_q,
                                       g["a_q"].astype(np.float16), g["b_q"].astype(np.float16), scaling)
    rel = np.abs(da_q - g["da_q"]).max() / np.abs(g["da_q"]).max()
    assert rel < 2e-2
    rel = np.abs(db_q - g["db_q"]).max() / np.abs(g["db_q"]).max()
    assert rel < 2e-2


def test_rmsnorm_vs_reference():
    g = golden("lora_golden.npz")
    eps = float(g["eps"])
    y, _ = rmsnorm.forward(g["h"], g["w"], eps)
    np.testing.assert_allclose(y, g["norm_y"], rtol=1e-5, atol=1e-5)
    dx = rmsnorm.backward(g["norm_gy"], g["h"], g["w"], eps)
    np.testing.assert_allclose(dx, g["norm_dx"], rtol=1e-4, atol=1e-5)


def test_packing_plan():
    mask = np.zeros((4, 9), dtype=np.int64)
    for i, L in enumerate([9, 3, 5, 1]):
        mask[i, :L] = 1
    p = packing.plan(mask)
    assert p["spans"] == [(0, 9), (9, 3), (12, 5), (17, 1)]
    assert p["cu_seqlens"].tolist() == [0, 9, 12, 17, 18] and p["max_len"] == 9
    assert p["positions"].tolist()[9:12] == [0, 1, 2]
    bad = mask.copy()
    bad[1, 0] = 0                               # left padding: not handled
    assert packing.plan(bad) is None
    empty = mask.copy()
    empty[3, 0] = 0                             # an empty row
    assert packing.plan(empty) is None


def test_add_rmsnorm_oracle_matches_reference_fixture():
    """oracle.rmsnorm.add_forward / add_backward against the reference's AddRMSNormFn
    (solution/rmsnorm.py:108-144, run by tests/golden/make_golden.py): h bit-exact, y and the input
    gradients within fp32 rounding of the reference's Triton kernels."""
    g = golden("addnorm_golden.npz")
    eps = float(g["eps"])
    h, y, _ = rmsnorm.add_forward(g["residual"], g["delta"], g["w"], eps)
    assert np.array_equal(h, g["h"])
    assert np.abs(y - g["y"]).max() <= 1e-5 * max(1.0, np.abs(g["y"]).max())
    total, total16 = rmsnorm.add_backward(g["grad_h"], g["grad_y"], g["residual"], g["delta"], g["w"], eps)
    assert np.abs(total - g["d_residual"]).max() <= 1e-4 * max(1.0, np.abs(g["d_residual"]).max())
    assert total16.dtype == np.float16
    ref16 = g["d_delta"].astype(np.float32)
    # one fp16 ulp at most (the fp32 sums differ by rounding before the cast)
    assert np.all(np.abs(total16.astype(np.float32) - ref16) <= np.spacing(np.abs(ref16).astype(np.float16)).astype(np.float32))


def _mlp_states(g):
    return {n: dict(packed=g[f"{n}_packed"], absmax=g[f"{n}_absmax"], code=g[f"{n}_code"], absmax2=g[f"{n}_absmax2"],
                    code2=g[f"{n}_code2"], offset=np.float32(g[f"{n}_offset"]), blocksize=64, blocksize2=256,
                    nested=True, shape=shape)
            for n, shape in (("gate", (int(g["dims"][2]), int(g["dims"][1]))),
                             ("up", (int(g["dims"][2]), int(g["dims"][1]))),
                             ("down", (int(g["dims"][1]), int(g["dims"][2]))))}


def _ulps16(a, ref):
    a = np.asarray(a, dtype=np.float32)
    ref16 = np.asarray(ref, dtype=np.float16)
    return np.abs(a - ref16.astype(np.float32)) / np.spacing(np.abs(ref16)).astype(np.float32)


def test_mlp_oracle_matches_reference_fixture():
    """oracle.mlp against the reference's SwiGLU kernels and RecomputedMLP (solution/mlp.py:62-110,
    solution/swiglu.py:15-37, run by tests/golden/make_golden.py): SwiGLU within one fp16 ulp (the
    exponential's implementations differ), the whole node within fp16 rounding of its products."""
    from oracle import mlp

    g = golden("mlp_golden.npz")
    assert _ulps16(mlp.swiglu_fwd(g["sw_gate"], g["sw_up"]), g["sw_out"]).max() <= 1
    dgate, dup = mlp.swiglu_bwd(g["sw_grad"], g["sw_gate"], g["sw_up"])
    assert _ulps16(dgate, g["sw_dgate"]).max() <= 1 and _ulps16(dup, g["sw_dup"]).max() <= 1
    T, H, _ = (int(v) for v in g["dims"])
    out, saved = mlp.mlp_forward(g["x"].reshape(T, H), _mlp_states(g))
    ref = g["out"].reshape(T, H).astype(np.float32)
    assert np.linalg.norm(out.astype(np.float32) - ref) / np.linalg.norm(ref) < 2e-3
    dx = mlp.mlp_backward(g["gout"].reshape(T, H), saved)
    dref = g["dx"].reshape(T, H)
    assert np.linalg.norm(dx - dref) / np.linalg.norm(dref) < 2e-3


def test_head_oracle_matches_reference_fixture():
    """oracle.head against the reference's FusedHeadLoss (solution/head.py:88-139): loss, entropy
    and per-token loss within fp32 rounding, the argmax hits equal (with a tie resolved to the first
    index), the hidden-state gradient within the fp16 rounding of its products."""
    from oracle import head

    g = golden("head_golden.npz")
    loss, entropy, token_loss, hit, dh = head.head_loss(g["hidden"], g["weight16"], g["targets"], g["denominator"])
    assert abs(loss - float(g["loss"])) <= 1e-4 * abs(float(g["loss"]))
    np.testing.assert_allclose(entropy, g["entropy"], rtol=1e-4, atol=1e-4)
    np.testing.assert_allclose(token_loss, g["token_loss"], rtol=1e-4, atol=1e-4)
    assert np.array_equal(hit, g["hit"]) and hit[1] == 1
    assert np.linalg.norm(dh - g["dhidden"]) / np.linalg.norm(g["dhidden"]) < 2e-3


def test_packing_from_lengths_matches_the_plan():
    """solution.varlen.packing_from_lengths (device ops, run here on the CPU) gives the positions,
    cu_seqlens and spans of the oracle's plan for the same rows."""
    from decik_b200.solution.varlen import packing_from_lengths

    lengths = [401, 77, 512, 3]
    p = packing_from_lengths(lengths, "cpu")
    mask = np.zeros((4, 512), dtype=np.int64)
    for i, L in enumerate(lengths):
        mask[i, :L] = 1
    ref = packing.plan(mask)
    assert p.spans == ref["spans"] and p.max_len == ref["max_len"] and p.n_tokens == ref["n_tokens"]
    assert np.array_equal(p.positions.numpy(), ref["positions"])
    assert np.array_equal(p.cu_seqlens("cpu").numpy(), ref["cu_seqlens"])
