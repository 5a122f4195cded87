"""The reference's patch surface, on the B200 kernels: ``apply()`` (solution/__init__.py:30-51).

``apply()`` installs, once and idempotently, class-level patches gated by the reference's
``SKC_<NAME>=0`` switches:
- ``SKC_NF4``         bitsandbytes Linear4bit forward -> sm_100a NF4 dequant + linear (nf4.py)
- ``SKC_RMSNORM``     Qwen2RMSNorm -> sm_100a RMSNorm, recorded as the LoRA input link (rmsnorm.py)
- ``SKC_MLP``         Qwen2MLP with NF4 gate/up/down -> one node: one gate|up GEMM, sm_100a SwiGLU (mlp.py)
- ``SKC_VARLEN``      padding-free decoder + varlen attention (varlen.py); ``SKC_VARLEN_ATTN``;
                      ``SKC_ADDNORM`` (residual add + post-attention norm as one node);
                      ``SKC_FUSED_NORM`` (this build's addition: the input RMSNorm runs inside the
                      fused block's first kernel)
- ``SKC_ATTN``        Qwen2Attention forward: LoRA + RoPE + varlen attention (attn.py);
                      ``SKC_LORA_RECOMPUTE``; ``SKC_FUSED_BLOCK`` (this build's addition: LoRA
                      without dropout runs as one fused projection + attention node)
The reference's head, embedding and warm-up patches are outside this build's scope.
Patches whose third-party library is not installed (bitsandbytes, peft) are skipped with a
warning; an eligible input never falls back to a CPU or per-row path.
"""

import os
import warnings


def _enabled(name):
    return os.environ.get(f"SKC_{name}", "1") != "0"


def apply(linear4bit_cls=None, lora_classes=None):
    from . import attn, mlp, nf4, rmsnorm, varlen

    def _try(fn, what, *args, **kw):
        try:
            fn(*args, **kw)
        except ImportError as e:
            warnings.warn(f"decik_b200.solution.apply: {what} not patched ({e})")

    if _enabled("NF4"):
        _try(nf4.patch, "Linear4bit", linear4bit_cls)
    if _enabled("RMSNORM"):
        _try(rmsnorm.patch, "Qwen2RMSNorm")
    if _enabled("MLP"):
        _try(mlp.patch, "Qwen2MLP", linear4bit_cls)
    if _enabled("VARLEN"):
        _try(varlen.patch, "Qwen2Model", varlen_attention=_enabled("VARLEN_ATTN"),
             fuse_residual=_enabled("ADDNORM"), fuse_input_norm=_enabled("FUSED_NORM"))
        if _enabled("ATTN"):
            _try(attn.patch, "Qwen2Attention", recompute_lora=_enabled("LORA_RECOMPUTE"),
                 linear4bit_cls=linear4bit_cls, lora_classes=lora_classes,
                 fused_block=_enabled("FUSED_BLOCK"))
