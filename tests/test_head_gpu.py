"""The chunked head + cross entropy (solution/head.py FusedHeadLoss over decik_head_stats) on the
GPU: against the reference's FusedHeadLoss fixture (fp16), against torch's cross entropy on the
same bf16 logits at the Qwen2.5 vocabulary (151,936), and one training step of a small QLoRA
model with the fused head against the same step with lm_head + cross_entropy."""

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from oracle import head as o_head
from tests.conftest import golden

pytestmark = pytest.mark.gpu
DEV = "cuda"


def test_fused_head_matches_reference_fixture(cuda_lib):
    from decik_b200.solution.head import FusedHeadLoss

    g = golden("head_golden.npz")
    hidden = torch.from_numpy(g["hidden"]).to(DEV).requires_grad_(True)
    w16 = torch.from_numpy(g["weight16"]).to(DEV)
    targets = torch.from_numpy(g["targets"]).to(DEV)
    den = torch.from_numpy(g["denominator"]).to(DEV)
    loss, entropy, token_loss, hit = FusedHeadLoss.apply(hidden, w16, targets, den)
    loss.backward()
    assert abs(loss.item() - float(g["loss"])) <= 1e-4 * abs(float(g["loss"]))
    np.testing.assert_allclose(entropy.cpu().numpy(), g["entropy"], rtol=1e-4, atol=1e-4)
    np.testing.assert_allclose(token_loss.cpu().numpy(), g["token_loss"], rtol=1e-4, atol=1e-4)
    assert np.array_equal(hit.cpu().numpy(), g["hit"])  # includes the tie at token 1
    dh = hidden.grad.cpu().numpy()
    assert np.linalg.norm(dh - g["dhidden"]) / np.linalg.norm(g["dhidden"]) < 5e-3
    _, _, _, _, dh_o = o_head.head_loss(g["hidden"], g["weight16"], g["targets"], g["denominator"])
    assert np.linalg.norm(dh - dh_o) / np.linalg.norm(dh_o) < 5e-3


@pytest.mark.parametrize("n_tok", [1, 300, 2600])
def test_fused_head_vs_torch_cross_entropy(cuda_lib, n_tok):
    """bf16 at the Qwen2.5 vocabulary, more tokens than one chunk at 2600: the same loss, entropy,
    argmax hits and hidden-state gradient as torch on the same bf16 logits (cast to fp32)."""
    from decik_b200.solution import head

    gen = torch.Generator(device=DEV).manual_seed(n_tok)
    V, H = 151936, 1536
    w16 = (torch.randn(V, H, device=DEV, generator=gen) * 0.05).to(torch.bfloat16)
    hidden = torch.randn(n_tok, H, device=DEV, generator=gen).requires_grad_(True)
    targets = torch.randint(0, V, (n_tok,), device=DEV, generator=gen)
    targets[::7] = -100
    if n_tok > 1:
        targets[0] = -100
    den = (targets != -100).sum().float().clamp(min=1)
    loss, entropy, token_loss, hit = head.FusedHeadLoss.apply(hidden, w16, targets, den)
    loss.backward()
    h2 = hidden.detach().clone().requires_grad_(True)
    logits = (h2.to(torch.bfloat16) @ w16.t()).float()
    ref = F.cross_entropy(logits, targets, ignore_index=-100, reduction="sum") / den
    ref.backward()
    assert abs(loss.item() - ref.item()) <= 1e-4 * max(1.0, abs(ref.item()))
    lp = torch.log_softmax(logits, dim=1)
    ent = -(lp.exp() * lp).sum(1)
    assert torch.allclose(entropy, ent.detach(), rtol=1e-3, atol=1e-3)
    lab = targets != -100
    exp_hit = (lab & (logits.argmax(1) == targets.clamp(min=0))).int()
    assert (hit != exp_hit).sum().item() <= max(1, n_tok // 1000)  # bf16 logit ties aside
    if den.item() > 0 and lab.any():
        rel = ((hidden.grad - h2.grad).norm() / h2.grad.norm()).item()
        assert rel < 1e-2, rel


def test_head_stats_rejects_bad_arguments(cuda_lib):
    from decik_b200 import ops

    with pytest.raises(RuntimeError, match="multiple of 8"):
        ops.head_stats(torch.zeros(2, 12, device=DEV, dtype=torch.bfloat16), torch.zeros(2, device=DEV))


@pytest.fixture()
def patched_classes():
    from transformers.modeling_utils import ALL_ATTENTION_FUNCTIONS
    from transformers.models.qwen2 import modeling_qwen2 as mq

    from decik_b200 import qlora_model as qm

    saved = [(mq.Qwen2Model, "forward", mq.Qwen2Model.forward),
             (mq.Qwen2DecoderLayer, "forward", mq.Qwen2DecoderLayer.forward),
             (mq.Qwen2MLP, "forward", mq.Qwen2MLP.forward),
             (mq.Qwen2Attention, "forward", mq.Qwen2Attention.forward),
             (mq.Qwen2RMSNorm, "forward", mq.Qwen2RMSNorm.forward),
             (torch.nn.Dropout, "forward", torch.nn.Dropout.forward),
             (qm.Linear4bit, "forward", qm.Linear4bit.forward)]
    sdpa = ALL_ATTENTION_FUNCTIONS["sdpa"]
    yield
    for cls, name, fn in saved:
        setattr(cls, name, fn)
    ALL_ATTENTION_FUNCTIONS["sdpa"] = sdpa


def test_train_step_fused_head_matches_plain_head(cuda_lib, patched_classes):
    from decik_b200 import qlora_model as qm
    from decik_b200 import solution

    solution.apply(linear4bit_cls=qm.Linear4bit, lora_classes=(qm.LoraLinear,))
    ids, mask, labels = qm.padded_batch([300, 77, 512, 9], 4096, 4, DEV)
    grads = []
    losses = []
    for fused in (False, True):
        model = qm.build_qlora_qwen2(hidden=512, intermediate=1024, layers=2, heads=4, kv_heads=2, vocab=4096,
                                     seed=0, device=DEV)
        losses.append(qm.qlora_train_step(model, ids, mask, labels, fused_head=fused).item())
        grads.append(torch.cat([p.grad.reshape(-1) for p in qm.lora_parameters(model)]))
    assert abs(losses[0] - losses[1]) <= 1e-3 * abs(losses[0]), losses
    rel = ((grads[0] - grads[1]).norm() / grads[0].norm()).item()
    assert rel < 1e-2, rel
    assert cuda_lib.decik_kernel_error(1) == 0
