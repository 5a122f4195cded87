"""End to end through the reference's patch surface: a tiny Qwen2 (head_dim 128) with NF4 q/k/v/o
and LoRA on q and v, trained one step on a right-padded batch, with ``decik_b200.solution.apply()``
(padding-free packing, patched Qwen2Attention.forward / sdpa / RMSNorm / Linear4bit on the sm_100a
kernels) against the same model on the original transformers code. Mirrors the reference's
dev/test_cpu_attn.py section 2 (loss and LoRA gradients vs the unpatched path, and every new path
taken once per layer)."""

import pytest
import torch
import torch.nn.functional as F

from tests.qlora_stubs import Linear4bit, LoraLayer

pytestmark = pytest.mark.gpu


def _model(device, dtype, lora_dropout):
    from transformers import Qwen2Config, Qwen2ForCausalLM

    torch.manual_seed(0)
    cfg = Qwen2Config(vocab_size=300, hidden_size=512, intermediate_size=256, num_hidden_layers=2,
                      num_attention_heads=4, num_key_value_heads=2, max_position_embeddings=512,
                      tie_word_embeddings=False, rope_theta=1e6)
    cfg._attn_implementation = "sdpa"
    model = Qwen2ForCausalLM(cfg).to(device)
    for layer in model.model.layers:
        a = layer.self_attn
        a.q_proj = LoraLayer(Linear4bit(a.q_proj, dtype, device), 16, 32, lora_dropout, device)
        a.k_proj = Linear4bit(a.k_proj, dtype, device)
        a.v_proj = LoraLayer(Linear4bit(a.v_proj, dtype, device), 16, 32, lora_dropout, device)
        a.o_proj = Linear4bit(a.o_proj, dtype, device)
        m = layer.mlp
        m.gate_proj = Linear4bit(m.gate_proj, dtype, device)
        m.up_proj = Linear4bit(m.up_proj, dtype, device)
        m.down_proj = Linear4bit(m.down_proj, dtype, device)
    for name, p in model.named_parameters():
        p.requires_grad_("lora_" in name)
    model.train()
    return model


def _batch(device, lengths, vocab=300):
    g = torch.Generator().manual_seed(1)
    B, S = len(lengths), max(lengths)
    ids = torch.randint(0, vocab, (B, S), generator=g)
    am = torch.zeros(B, S, dtype=torch.long)
    lab = torch.full((B, S), -100)
    for i, L in enumerate(lengths):
        am[i, :L] = 1
        lab[i, L // 3:L] = ids[i, L // 3:L]
    return ids.to(device), am.to(device), lab.to(device)


def _step(model, batch, state, dtype, autocast=True):
    """One training step. The loss is taken on the real tokens as the reference's fused head does
    (solution/head.py:147-171, shifted labels gathered at packing.index when the decoder ran
    packed, at the mask's positions otherwise); the head itself is not part of this path."""
    ids, am, lab = batch
    model.zero_grad(set_to_none=True)
    torch.manual_seed(5)
    state.request, state.packing = True, None
    try:
        with torch.autocast("cuda", dtype=dtype, enabled=autocast):
            hidden = model.model(input_ids=ids, attention_mask=am, use_cache=False).last_hidden_state
            packing = state.packing
            flat = hidden.reshape(-1, hidden.shape[-1])
            if packing is not None:
                positions = packing.index
            else:
                positions = am.reshape(-1).nonzero().squeeze(1)
                flat = flat.index_select(0, positions)
            targets = F.pad(lab, (0, 1), value=-100)[..., 1:].reshape(-1).index_select(0, positions)
            logits = model.lm_head(flat).float()
    finally:
        state.request, state.packing = False, None
    loss = F.cross_entropy(logits, targets, ignore_index=-100, reduction="sum") / (targets != -100).sum()
    loss.backward()
    grads = {n: p.grad.detach().float().clone() for n, p in model.named_parameters() if p.grad is not None}
    return loss.detach().float(), grads, packing is not None


@pytest.fixture()
def patched_classes():
    """Saves and restores every class attribute apply() patches."""
    from transformers.modeling_utils import ALL_ATTENTION_FUNCTIONS
    from transformers.models.qwen2 import modeling_qwen2 as mq

    saved = [(mq.Qwen2Model, "forward", mq.Qwen2Model.forward),
             (mq.Qwen2DecoderLayer, "forward", mq.Qwen2DecoderLayer.forward),
             (mq.Qwen2MLP, "forward", mq.Qwen2MLP.forward),
             (mq.Qwen2Attention, "forward", mq.Qwen2Attention.forward),
             (mq.Qwen2RMSNorm, "forward", mq.Qwen2RMSNorm.forward),
             (torch.nn.Dropout, "forward", torch.nn.Dropout.forward),
             (Linear4bit, "forward", Linear4bit.forward)]
    sdpa = ALL_ATTENTION_FUNCTIONS["sdpa"]
    yield
    for cls, name, fn in saved:
        setattr(cls, name, fn)
    ALL_ATTENTION_FUNCTIONS["sdpa"] = sdpa


@pytest.mark.parametrize("lengths,lora_dropout", [([17, 6, 11], 0.0), ([300, 129, 64, 1], 0.0),
                                                  ([40, 33, 7], 0.1)])
def test_patched_qwen2_matches_original(cuda_lib, patched_classes, lengths, lora_dropout):
    """With LoRA dropout the packed path draws its keep-masks with the base's op on the base's
    [B, S, H] shape (solution/varlen.py:42-63), so the same seed gives the same masks."""
    from decik_b200 import solution
    from decik_b200.solution import _state, attn, mlp, nf4, rmsnorm, varlen

    dtype = torch.bfloat16
    base = _model("cuda", dtype, lora_dropout)
    batch = _batch("cuda", lengths)
    l0, g0, packed0 = _step(base, batch, _state.STATE, dtype)   # original transformers + stub modules
    assert not packed0
    # the same model in fp32 on the original code: the truth both bf16 paths approximate
    _, g32, _ = _step(_model("cuda", torch.float32, lora_dropout), batch, _state.STATE, torch.float32,
                      autocast=False)

    model = _model("cuda", dtype, lora_dropout)    # same seeds: identical weights
    solution.apply(linear4bit_cls=Linear4bit, lora_classes=(LoraLayer,))
    fns = (("rope", attn.FusedQKRope), ("varlen", varlen.VarlenSDPA), ("pair", attn.LoRAPairFromNorm),
           ("fused", attn.FusedAttentionBlock), ("addnorm", rmsnorm.AddRMSNormFn), ("mlp", mlp.FusedMLP),
           ("nf4linear", nf4.NF4Linear), ("rmsnorm", rmsnorm.RMSNormFn))
    calls = {n: 0 for n, _ in fns}
    orig = {n: getattr(c, "forward") for n, c in fns}

    def counting(name):
        def fwd(ctx, *a):
            calls[name] += 1
            return orig[name](ctx, *a)
        return staticmethod(fwd)

    # the fused layers' input-norm backward takes the residual stream's gradient of the layer input
    # as its addend (rmsnorm.ResidualGradLink) instead of autograd summing the two
    from decik_b200 import ops
    orig_bwd, added = ops.rmsnorm_bwd, []

    def counting_bwd(*a, **kw):
        added.append(kw.get("addend") is not None)
        return orig_bwd(*a, **kw)

    try:
        for n, c in fns:
            c.forward = counting(n)
        ops.rmsnorm_bwd = counting_bwd
        l1, g1, packed1 = _step(model, batch, _state.STATE, dtype)
    finally:
        for n, c in fns:
            c.forward = orig[n]
        ops.rmsnorm_bwd = orig_bwd
    assert packed1
    n_layers = len(model.model.layers)
    # without LoRA dropout every layer runs as one fused node (o_proj and the input norm included);
    # with it, the reference's chain, whose q, k, v and o projections are NF4Linear calls and whose
    # input norm is an RMSNormFn. The model's final norm is one more RMSNormFn.
    chain = n_layers if lora_dropout > 0 else 0
    assert calls == {"rope": chain, "varlen": chain, "pair": chain, "fused": n_layers - chain,
                     "addnorm": n_layers, "mlp": n_layers, "nf4linear": 4 * chain,
                     "rmsnorm": chain + 1}, calls
    assert sum(added) == n_layers - chain, added
    print(f"loss {l0.item():.6f} -> {l1.item():.6f}")
    assert abs(l1.item() - l0.item()) / abs(l0.item()) < 2e-3, (l1.item(), l0.item())
    assert set(g1) == set(g0)
    rel = lambda a, b: ((a - b).norm() / b.norm().clamp(min=1e-12)).item()
    for name in g0:
        d, e1, e0 = rel(g1[name], g0[name]), rel(g1[name], g32[name]), rel(g0[name], g32[name])
        print(f"{name}: patched vs original {d:.3e}; vs fp32: patched {e1:.3e}, original {e0:.3e}")
        # the two bf16 paths round differently (the fused block adds the LoRA product to the
        # projection in fp32 before one rounding; the original rounds each term): within 2e-2 of
        # each other, or the patched gradient no further from fp32 than the original's
        assert d < 2e-2 or e1 <= 1.1 * e0, f"{name}: {d:.3e} apart; vs fp32 {e1:.3e} (original {e0:.3e})"
    assert cuda_lib.decik_kernel_error(1) == 0


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_loss_after_steps_matches_original(cuda_lib, patched_classes, dtype):
    """Eight AdamW steps (lr 2e-4, as the reference's task config) of the same tiny QLoRA Qwen2 on
    the original code and through ``solution.apply()``: the losses agree step by step. The bar is
    1e-3 absolute on every step in fp16 (the reference's compute dtype); bf16 keeps 8 bits of
    mantissa, so its two paths round differently from the first step and are held to 1e-2."""
    from decik_b200 import solution
    from decik_b200.solution import _state

    lengths = [96, 37, 211, 5]
    batch = _batch("cuda", lengths)

    def train(model, n_steps=8):
        params = [p for p in model.parameters() if p.requires_grad]
        opt = torch.optim.AdamW(params, lr=2e-4)
        losses = []
        for _ in range(n_steps):
            loss, _, _ = _step(model, batch, _state.STATE, dtype)
            opt.step()
            losses.append(loss.item())
        return losses

    base = train(_model("cuda", dtype, 0.0))
    model = _model("cuda", dtype, 0.0)
    solution.apply(linear4bit_cls=Linear4bit, lora_classes=(LoraLayer,))
    ours = train(model)
    print("original", base)
    print("patched ", ours)
    tol = 1e-3 if dtype == torch.float16 else 1e-2
    assert base[-1] < base[0]  # it trains
    for i, (a, b) in enumerate(zip(base, ours)):
        assert abs(a - b) <= tol, (i, a, b)
    assert cuda_lib.decik_kernel_error(1) == 0
