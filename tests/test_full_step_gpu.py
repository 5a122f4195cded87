"""The full QLoRA train step of a small Qwen2-shaped model (decik_b200.qlora_model) through
``solution.apply()`` on the GPU: data-parallel loss parity by emulation on one GPU. The rows of a
batch are split over two "ranks" by ``dp.partition_rows``; each rank's loss is normalised by the
global labelled-token count and the ranks' LoRA gradients are summed (what the NCCL all-reduce
does), against one process over all rows. Losses must agree at every step of a 32-step AdamW run
at lr 2e-4 (the baseline's data-parallel configuration runs 32 steps)."""

import pytest
import torch

from decik_b200 import qlora_model as qm

pytestmark = pytest.mark.gpu


@pytest.fixture()
def patched_classes():
    from transformers.modeling_utils import ALL_ATTENTION_FUNCTIONS
    from transformers.models.qwen2 import modeling_qwen2 as mq

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


def _model():
    return qm.build_qlora_qwen2(hidden=512, intermediate=1024, layers=2, heads=4, kv_heads=2, vocab=1000,
                                seed=0, device="cuda")


def test_data_parallel_loss_parity_emulated(cuda_lib, patched_classes):
    from decik_b200 import solution
    from decik_b200.dp import GradBucket, partition_rows

    solution.apply(linear4bit_cls=qm.Linear4bit, lora_classes=(qm.LoraLinear,))
    lengths = qm.lognormal_lengths(5, 2048, 256, 16, 700)
    n_labels = torch.tensor(float(sum(lengths) - len(lengths)), device="cuda")
    ids, mask, labels = qm.padded_batch(lengths, 1000, 11, "cuda")
    parts = partition_rows(lengths, 2)
    assert all(parts) and sorted(i for p in parts for i in p) == list(range(len(lengths)))

    def sub_batch(rows):
        sub = [lengths[i] for i in rows]
        idx = torch.tensor(rows, device="cuda")
        seq = max(sub)
        return ids[idx, :seq], mask[idx, :seq], labels[idx, :seq]

    def train(model, split, n_steps=32):
        params = qm.lora_parameters(model)
        bucket = GradBucket(params)
        opt = torch.optim.AdamW(params, lr=2e-4)
        losses = []
        for _ in range(n_steps):
            bucket.zero_()
            if split:
                loss = sum(qm.qlora_train_step(model, *sub_batch(p), n_labels=n_labels) for p in parts)
            else:
                loss = qm.qlora_train_step(model, ids, mask, labels, n_labels=n_labels)
            bucket.check_in_place()
            opt.step()
            losses.append(float(loss))
        return losses, bucket.flat.clone()

    one, g1 = train(_model(), split=False)
    dp, g2 = train(_model(), split=True)
    print("one process", one)
    print("two ranks  ", dp)
    assert one[-1] < one[0]  # it trains
    for i, (a, b) in enumerate(zip(one, dp)):
        assert abs(a - b) <= 1e-3 * abs(a), (i, a, b)
    rel = ((g1 - g2).norm() / g1.norm()).item()
    print("last-step LoRA gradient rel-L2", rel)
    assert rel < 2e-2
    assert cuda_lib.decik_kernel_error(1) == 0
