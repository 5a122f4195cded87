"""Generate the golden fixtures under tests/golden/ by running the REFERENCE's own modules.

Run in a container where the reference checkout exists (it is read, never modified):

    python tests/golden/make_golden.py <reference checkout>

The reference's Triton kernels run on the CPU through the Triton interpreter
(``TRITON_INTERPRET=1``) with its ``on_gpu`` guards stubbed to True, as the reference's own CPU
checks do (dev/test_cpu_attn.py:2-9, dev/test_cpu_norm_link.py:12-21). bitsandbytes is not
installed, so the NF4 states come from ``oracle.nf4.quantize_nf4`` (and from seeded random bytes,
which are valid NF4 data); the reference's ``dequantize_nf4`` reads them through a stand-in
object with the QuantState fields it uses (solution/nf4.py:66-85).

Fixtures written (numpy .npz):
- nf4_golden.npz      solution/nf4.py dequantize_nf4 (skc_nf4_dequant_kernel): small shapes in
                      full, nested and not, and the sha256 of larger shapes' outputs
- rope_golden.npz     solution/attn.py FusedQKRope forward and backward (shapes of
                      dev/test_cpu_attn.py:18 with fewer tokens)
- sdpa_golden.npz     solution/varlen.py PackedSDPA forward and backward in fp32 (spans of
                      dev/test_cpu_sdpa.py:24)
- lora_golden.npz     solution/attn.py pack_keep, _lora_inputs, LoRAPairFromNorm and
                      solution/rmsnorm.py RMSNormFn (sizes of dev/test_cpu_norm_link.py:32-45)
- mlp_golden.npz      solution/swiglu.py SwiGLU kernels (fp16) and solution/mlp.py RecomputedMLP
                      forward and backward over three NF4 projections (fp32 input, fp16 compute)
- head_golden.npz     solution/head.py FusedHeadLoss (skc_head_stats_kernel + the gradient matmul)
                      forward and backward, fp16 head, some targets ignored, a tie for the argmax
- addnorm_golden.npz  solution/rmsnorm.py AddRMSNormFn (the decoder's residual add + post-attention
                      norm, solution/varlen.py:323-337) forward and backward, fp16 delta

``python tests/golden/make_golden.py <reference> addnorm`` writes only the named fixture files.
"""

from __future__ import annotations

import hashlib
import os
import sys

os.environ["TRITON_INTERPRET"] = "1"

import numpy as np  # noqa: E402
import torch  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))  # the repo, for oracle.nf4


class _QS:
    """The QuantState fields solution/nf4.py:66-85 reads."""


class _State2:
    pass


def _quant_state(st: dict) -> _QS:
    qs = _QS()
    qs.shape = st["shape"]
    qs.nested = st["nested"]
    qs.blocksize = st["blocksize"]
    qs.code = torch.from_numpy(np.asarray(st["code"], dtype=np.float32))
    qs.quant_type = "nf4"
    qs.dtype = torch.float16
    if st["nested"]:
        qs.absmax = torch.from_numpy(np.asarray(st["absmax"], dtype=np.uint8))
        qs.state2 = _State2()
        qs.state2.absmax = torch.from_numpy(np.asarray(st["absmax2"], dtype=np.float32))
        qs.state2.code = torch.from_numpy(np.asarray(st["code2"], dtype=np.float32))
        qs.state2.blocksize = st["blocksize2"]
        qs.offset = torch.tensor(np.float32(st["offset"]))
    else:
        qs.absmax = torch.from_numpy(np.asarray(st["absmax"], dtype=np.float32))
        qs.state2 = None
        qs.offset = None
    return qs


def random_nf4_state(shape, nested: bool, seed: int) -> dict:
    """Seeded random NF4 data (any bytes are valid): the large-shape hash cases."""
    from oracle.nf4 import dynamic_code, nf4_code

    rng = np.random.default_rng(seed)
    n = shape[0] * shape[1]
    n_blocks = n // 64
    st = dict(shape=tuple(shape), nested=nested, blocksize=64, blocksize2=256,
              packed=rng.integers(0, 256, n // 2, dtype=np.uint8), code=nf4_code())
    if nested:
        st.update(absmax=rng.integers(0, 256, n_blocks, dtype=np.uint8),
                  absmax2=(rng.random(-(-n_blocks // 256)) * 0.1 + 0.01).astype(np.float32),
                  code2=dynamic_code(), offset=np.float32(0.0421))
    else:
        st.update(absmax=(rng.random(n_blocks) * 0.2 + 0.01).astype(np.float32), absmax2=None,
                  code2=None, offset=None)
    return st


def nf4_fixtures(nf4) -> dict:
    from oracle.nf4 import quantize_nf4

    out = {}
    for tag, shape, nested in (("a", (64, 512), True), ("b", (64, 512), False),
                               ("c", (24, 1536), True)):
        torch.manual_seed(0)
        w = (torch.randn(shape) * 0.05).half().numpy()          # solution/test_solution.py:17
        st = quantize_nf4(w, blocksize=64, nested=nested)
        ref = nf4.dequantize_nf4(torch.from_numpy(st["packed"]), _quant_state(st)).numpy()
        out[f"{tag}_packed"] = st["packed"]
        out[f"{tag}_absmax"] = st["absmax"]
        out[f"{tag}_code"] = st["code"]
        out[f"{tag}_shape"] = np.array(shape)
        out[f"{tag}_nested"] = np.array(nested)
        if nested:
            out[f"{tag}_absmax2"] = st["absmax2"]
            out[f"{tag}_code2"] = st["code2"]
            out[f"{tag}_offset"] = np.array(st["offset"], dtype=np.float32)
        out[f"{tag}_out"] = ref
    # the reference test's shapes (solution/test_solution.py:10), random NF4 data, output hashes
    for i, (shape, nested) in enumerate((((1536, 1536), True), ((256, 1536), True),
                                         ((256, 1536), False), ((1536, 8960), True))):
        st = random_nf4_state(shape, nested, seed=100 + i)
        ref = nf4.dequantize_nf4(torch.from_numpy(st["packed"]), _quant_state(st)).numpy()
        out[f"hash{i}_shape"] = np.array(shape)
        out[f"hash{i}_nested"] = np.array(nested)
        out[f"hash{i}_seed"] = np.array(100 + i)
        out[f"hash{i}_sha256"] = np.array(hashlib.sha256(ref.tobytes()).hexdigest())
        out[f"hash{i}_head"] = ref.reshape(-1)[:64].copy()
    return out


def rope_fixtures(attn) -> dict:
    torch.manual_seed(0)
    T, HQ, HK, D = 16, 12, 2, 128                                  # dev/test_cpu_attn.py:18
    qb = (torch.randn(T, HQ * D) * 3).half()
    ql = (torch.randn(T, HQ * D) * 0.1).half()
    kb = (torch.randn(T, HK * D) * 3).half()
    pos = torch.arange(T).float() + 5.0                            # not starting at 0
    inv = 1.0 / (1e6 ** (torch.arange(0, D, 2).float() / D))
    fr = torch.outer(pos, inv)
    emb = torch.cat((fr, fr), -1)
    cos, sin = emb.cos(), emb.sin()
    qo, ko = attn.FusedQKRope.apply(qb, ql, kb, cos, sin, HQ, HK)
    gq = torch.randn(1, HQ, T, D).half()
    gk = torch.randn(1, HK, T, D).half()
    ctx = type("C", (), {"saved_tensors": (cos, sin), "shape": (T, HQ, HK, D)})()
    dq, dq2, dk, *_ = attn.FusedQKRope.backward(ctx, gq, gk)
    assert torch.equal(dq, dq2)
    return dict(qb=qb.numpy(), ql=ql.numpy(), kb=kb.numpy(), cos=cos.numpy(), sin=sin.numpy(),
                qo=qo[0].numpy(), ko=ko[0].numpy(), gq=gq[0].numpy(), gk=gk[0].numpy(),
                dq=dq.numpy(), dk=dk.numpy(), dims=np.array([T, HQ, HK, D]))


def sdpa_fixtures(varlen) -> dict:
    torch.manual_seed(0)
    HQ, HK, D = 4, 2, 128
    spans = [(0, 37), (37, 5), (42, 20), (62, 1)]                  # dev/test_cpu_sdpa.py:24
    T = sum(L for _, L in spans)
    groups = HQ // HK
    scale = D ** -0.5
    q16 = torch.randn(1, HQ, T, D).half()
    k16 = torch.randn(1, HK, T, D).half()
    v16 = torch.randn(1, T, HK, D).half()
    g16 = torch.randn(1, T, HQ, D).half()
    q, k = q16.float().requires_grad_(True), k16.float().requires_grad_(True)
    v_leaf = v16.float().requires_grad_(True)
    out = varlen.PackedSDPA.apply(q, k, v_leaf.transpose(1, 2), spans, groups, scale)
    out.backward(g16.float())
    return dict(q=q16[0].numpy(), k=k16[0].numpy(), v=v16[0].numpy(), g=g16[0].numpy(),
                out=out.detach()[0].numpy(), dq=q.grad[0].numpy(), dk=k.grad[0].numpy(),
                dv=v_leaf.grad[0].numpy(), spans=np.array(spans), dims=np.array([HQ, HK, D]))


def lora_fixtures(attn, rmsnorm) -> dict:
    torch.manual_seed(0)
    T, H, R, HV = 29, 256, 8, 64                                   # dev/test_cpu_norm_link.py:32
    eps = 1e-6
    h = (torch.randn(1, T, H) * 3).requires_grad_(True)
    w = torch.rand(H) + 0.5
    a_q = (torch.randn(R, H) * 0.05).requires_grad_(True)
    b_q = (torch.randn(H, R) * 0.05).requires_grad_(True)
    a_v = (torch.randn(R, H) * 0.05).requires_grad_(True)
    b_v = (torch.randn(HV, R) * 0.05).requires_grad_(True)
    p, scaling = 0.05, 2.0
    ones = torch.ones(1, T, H)
    scaled_q, keep_q = torch.native_dropout(ones, p, True)
    scaled_v, keep_v = torch.native_dropout(ones, p, True)
    gq = torch.randn(1, T, H).half() * 64
    gv = torch.randn(1, T, HV).half() * 64
    gy = torch.randn(1, T, H)

    # RMSNorm forward/backward on its own
    hn = h.detach().clone().requires_grad_(True)
    y = rmsnorm.RMSNormFn.apply(hn, w, eps)
    y.backward(gy)
    norm = dict(norm_y=y.detach().numpy(), norm_dx=hn.grad.numpy(), norm_gy=gy.numpy())

    x = rmsnorm.RMSNormFn.apply(h, w, eps)
    bits_q, bits_v = attn.pack_keep(keep_q.reshape(T, H).contiguous(), keep_v.reshape(T, H).contiguous())
    scale = scaled_q.amax()
    xq16, xv16 = attn._lora_inputs(x.detach().reshape(T, H).contiguous(), bits_q, bits_v, scale, scale)
    oq, ov = attn.LoRAPairFromNorm.apply(x, h, w, eps, scaled_q, bits_q, scale, scaled_v, bits_v,
                                         scale, a_q, b_q, a_v, b_v, scaling, scaling, p, p, True)
    torch.autograd.backward([oq, ov], [gq, gv])
    # the kernel the backward uses for the input gradient through both masks
    giq = (torch.randn(T, H) * 4).half()
    giv = (torch.randn(T, H) * 4).half()
    gin = torch.empty(T, H)
    attn.skc_lora_input_grad_kernel[(T,)](giq, giv, bits_q, bits_v, gin, T, 1.0 / (1.0 - p),
                                          1.0 / (1.0 - p), WIDTH=H, BLOCK=H, num_warps=4,
                                          enable_fp_fusion=False)
    return dict(h=h.detach().numpy(), w=w.numpy(), a_q=a_q.detach().numpy(),
                b_q=b_q.detach().numpy(), a_v=a_v.detach().numpy(), b_v=b_v.detach().numpy(),
                keep_q=keep_q.numpy(), keep_v=keep_v.numpy(), scale=np.float32(scale.item()),
                gq=gq.numpy(), gv=gv.numpy(), x=x.detach().numpy(), bits_q=bits_q.numpy(),
                bits_v=bits_v.numpy(), xq16=xq16.numpy(), xv16=xv16.numpy(),
                oq=oq.detach().numpy(), ov=ov.detach().numpy(), dh=h.grad.numpy(),
                da_q=a_q.grad.numpy(), db_q=b_q.grad.numpy(), da_v=a_v.grad.numpy(),
                db_v=b_v.grad.numpy(), giq=giq.numpy(), giv=giv.numpy(), gin=gin.numpy(),
                dims=np.array([T, H, R, HV]), p=np.float32(p), scaling=np.float32(scaling),
                eps=np.float32(eps), **norm)


def addnorm_fixtures(rmsnorm) -> dict:
    torch.manual_seed(0)
    T, H = 29, 256
    eps = 1e-6
    residual = (torch.randn(1, T, H) * 3).requires_grad_(True)
    delta = (torch.randn(1, T, H) * 2).half().requires_grad_(True)  # the fp16 attention output
    w = torch.rand(H) + 0.5
    grad_h = torch.randn(1, T, H)
    grad_y = torch.randn(1, T, H)
    h, y = rmsnorm.AddRMSNormFn.apply(residual, delta, w, eps)
    torch.autograd.backward([h, y], [grad_h, grad_y])
    return dict(residual=residual.detach().numpy(), delta=delta.detach().numpy(), w=w.numpy(),
                grad_h=grad_h.numpy(), grad_y=grad_y.numpy(), h=h.detach().numpy(), y=y.detach().numpy(),
                d_residual=residual.grad.numpy(), d_delta=delta.grad.numpy(), eps=np.float32(eps))


class _Proj(torch.nn.Module):
    """The fields of a bitsandbytes Linear4bit that solution/mlp.py reads (weight.quant_state, bias)."""

    def __init__(self, st):
        super().__init__()
        self.weight = torch.nn.Parameter(torch.from_numpy(st["packed"]), requires_grad=False)
        self.weight.quant_state = _quant_state(st)
        self.bias = None


def mlp_fixtures(mlp) -> dict:
    from oracle.nf4 import quantize_nf4

    from solution import swiglu

    torch.manual_seed(0)
    T, H, I = 23, 128, 256
    gate = (torch.randn(T, I) * 3).half()
    up = (torch.randn(T, I) * 2).half()
    grad = torch.randn(T, I).half()
    hidden = swiglu.SwiGLU.apply(gate, up)
    dgate, dup = swiglu.SwiGLU.backward(type("Ctx", (), {"saved_tensors": (gate, up)})(), grad)
    rng = np.random.default_rng(0)
    states = {n: quantize_nf4((rng.standard_normal(shape) * 0.05).astype(np.float32))
              for n, shape in (("gate", (I, H)), ("up", (I, H)), ("down", (H, I)))}
    x = torch.randn(1, T, H).requires_grad_(True)
    gout = torch.randn(1, T, H).half()
    out = mlp.RecomputedMLP.apply(x, _Proj(states["gate"]), _Proj(states["up"]), _Proj(states["down"]))
    out.backward(gout)
    res = dict(sw_gate=gate.numpy(), sw_up=up.numpy(), sw_grad=grad.numpy(), sw_out=hidden.numpy(),
               sw_dgate=dgate.numpy(), sw_dup=dup.numpy(), x=x.detach().numpy(), gout=gout.numpy(),
               out=out.detach().numpy(), dx=x.grad.numpy(), dims=np.array([T, H, I]))
    for n, st in states.items():
        for k in ("packed", "absmax", "code", "absmax2", "code2"):
            res[f"{n}_{k}"] = st[k]
        res[f"{n}_offset"] = np.float32(st["offset"])
    return res


def head_fixtures(head) -> dict:
    torch.manual_seed(0)
    T, H, V = 37, 64, 1000
    hidden = (torch.randn(T, H) * 2).requires_grad_(True)
    weight16 = (torch.randn(V, H) * 0.5).half()
    weight16[7] = weight16[3]  # two identical rows: equal logits, the argmax takes the first
    targets = torch.randint(0, V, (T,))
    targets[::5] = -100
    targets[1] = 3
    with torch.no_grad():
        hidden[1] = weight16[3].float() * 4  # rows 3 and 7 tie for the maximum of token 1
    denominator = torch.tensor(float((targets != -100).sum()))
    loss, entropy, token_loss, hit = head.FusedHeadLoss.apply(hidden, weight16, targets, denominator)
    loss.backward()
    return dict(hidden=hidden.detach().numpy(), weight16=weight16.numpy(), targets=targets.numpy(),
                denominator=denominator.numpy(), loss=loss.detach().numpy(), entropy=entropy.numpy(),
                token_loss=token_loss.numpy(), hit=hit.numpy(), dhidden=hidden.grad.numpy())


def main(reference: str, only=None) -> None:
    sys.path.insert(0, reference)
    import solution._state as st
    from solution import attn, head, mlp, nf4, rmsnorm, varlen

    for m in (st, attn, head, mlp, nf4, rmsnorm, varlen):
        m.on_gpu = lambda t: True
    makers = {"nf4": lambda: nf4_fixtures(nf4), "rope": lambda: rope_fixtures(attn),
              "sdpa": lambda: sdpa_fixtures(varlen), "lora": lambda: lora_fixtures(attn, rmsnorm),
              "addnorm": lambda: addnorm_fixtures(rmsnorm), "mlp": lambda: mlp_fixtures(mlp),
              "head": lambda: head_fixtures(head)}
    for name, make in makers.items():
        if only is None or name in only:
            np.savez_compressed(os.path.join(HERE, f"{name}_golden.npz"), **make())
    print("fixtures written to", HERE)


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else "../reference", sys.argv[2:] or None)
