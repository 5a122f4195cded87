"""The full-model QLoRA builder (decik_b200.qlora_model) on the CPU: its NF4 quantizer against the
oracle's, its torch dequant against the oracle's, the module structure the reference's patches
expect, the bench packings, and one step of the reference's CPU path (original transformers code,
torch dequant) over a tiny model."""

import numpy as np
import pytest
import torch

from decik_b200 import qlora_model as qm
from oracle import block as ob
from oracle.nf4 import quantize_nf4


@pytest.mark.parametrize("shape", [(64, 256), (96, 128), (3, 4096)])
def test_torch_quantizer_matches_oracle(shape):
    rng = np.random.default_rng(7)
    w = (rng.standard_normal(shape) * 0.02).astype(np.float32)
    w[0, :64] = 0.0  # an all-zero block
    ref = quantize_nf4(w)
    packed, qs = qm.quantize_nf4_torch(torch.from_numpy(w))
    assert np.array_equal(packed.numpy(), ref["packed"])
    assert np.array_equal(qs.absmax.numpy(), ref["absmax"])
    assert np.array_equal(qs.state2.absmax.numpy(), ref["absmax2"])
    assert np.array_equal(qs.code.numpy(), ref["code"]) and np.array_equal(qs.state2.code.numpy(), ref["code2"])
    assert abs(float(qs.offset) - float(ref["offset"])) <= 1e-9 * max(1.0, abs(float(ref["offset"])))
    # the dequant used by the CPU reference arm equals the oracle's on the same state
    assert torch.equal(ob.dequant_torch_qs(torch.from_numpy(ref["packed"]), _qs_from(ref)), ob.dequant_torch(ref))


def _qs_from(st):
    from decik_b200.block import QuantState

    t = torch.from_numpy
    return QuantState(st["shape"], t(st["absmax"]), t(st["code"]), st["blocksize"], torch.float16,
                      absmax2=t(st["absmax2"]), code2=t(st["code2"]),
                      offset=torch.tensor([float(st["offset"])]), blocksize2=st["blocksize2"])


def _tiny(**kw):
    args = dict(hidden=256, intermediate=512, layers=2, heads=2, kv_heads=1, vocab=512, device="cpu")
    args.update(kw)
    return qm.build_qlora_qwen2(**args)


def test_model_structure():
    model = _tiny()
    for layer in model.model.layers:
        a, m = layer.self_attn, layer.mlp
        assert isinstance(a.q_proj, qm.LoraLinear) and isinstance(a.v_proj, qm.LoraLinear)
        for mod in (a.q_proj.base_layer, a.k_proj, a.v_proj.base_layer, a.o_proj, m.gate_proj, m.up_proj,
                    m.down_proj):
            assert isinstance(mod, qm.Linear4bit)
            assert mod.weight.dtype == torch.uint8 and not mod.weight.requires_grad
            assert mod.weight.numel() * 2 == mod.in_features * mod.out_features
            assert mod.weight.quant_state.dtype == torch.bfloat16 and mod.weight.quant_state.nested
        assert a.q_proj.lora_A["default"].weight.shape == (16, 256)
        assert a.q_proj.lora_B["default"].weight.shape == (256, 16)
        assert a.v_proj.lora_B["default"].weight.shape == (128, 16)
        assert a.q_proj.scaling["default"] == 2.0
    trainable = {n for n, p in model.named_parameters() if p.requires_grad}
    assert trainable and all("lora_" in n for n in trainable)
    assert len(qm.lora_parameters(model)) == 4 * 2
    shared = _tiny(share_layer_weights=True)
    l0, l1 = shared.model.layers[0].mlp.up_proj, shared.model.layers[1].mlp.up_proj
    assert l0.weight.data_ptr() == l1.weight.data_ptr()


@pytest.mark.parametrize("total,median,lo,hi", [(830, 180, 16, 1024), (16384, 512, 16, 4096)])
def test_lognormal_lengths(total, median, lo, hi):
    lengths = qm.lognormal_lengths(1000, total, median, lo, hi)
    assert sum(lengths) == total
    assert all(1 <= L <= hi for L in lengths) and all(L >= lo for L in lengths[:-1])
    assert lengths == qm.lognormal_lengths(1000, total, median, lo, hi)


def test_padded_batch():
    ids, mask, labels = qm.padded_batch([5, 3, 7], 100, 0, "cpu")
    assert ids.shape == mask.shape == labels.shape == (3, 7)
    assert mask.sum(1).tolist() == [5, 3, 7]
    assert torch.equal(labels[mask.bool()], ids[mask.bool()])
    assert (labels[~mask.bool()] == -100).all() and (ids[~mask.bool()] == 0).all()


@pytest.mark.parametrize("share", [False, True])
def test_reference_cpu_step_trains(share):
    """The bench's reference arm: the original transformers forward on the host in fp32, each NF4
    weight dequantised with torch ops; three AdamW steps lower the loss of a fixed batch (also with
    the layers sharing layer 0's frozen weights, the host build the arm uses)."""
    model = _tiny(layers=2, share_layer_weights=share)
    for n, p in model.named_parameters():
        assert torch.isfinite(p.float()).all(), n
    saved = qm.Linear4bit.forward

    def cpu_forward(self, x):
        w = ob.dequant_torch_qs(self.weight.data, self.weight.quant_state)
        return torch.nn.functional.linear(x.float(), w, None if self.bias is None else self.bias.float())

    qm.Linear4bit.forward = cpu_forward
    try:
        ids, mask, labels = qm.padded_batch([9, 4, 6], 512, 3, "cpu")
        opt = torch.optim.AdamW(qm.lora_parameters(model), lr=1e-2)
        losses = []
        for _ in range(3):
            model.zero_grad(set_to_none=True)
            losses.append(float(qm.qlora_train_step(model, ids, mask, labels)))
            opt.step()
    finally:
        qm.Linear4bit.forward = saved
    assert all(np.isfinite(losses)) and losses[-1] < losses[0]
