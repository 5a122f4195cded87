"""CPU oracle for the attention block of decik's NF4 QLoRA step. TEST INFRASTRUCTURE ONLY.

This package restates, in numpy (and torch fp32 on the CPU for the floating-point attention
and block compositions), the reference's algorithm for the hot path:

- ``oracle.nf4``       NF4 double-quant dequant (solution/nf4.py:28-49) plus an NF4 quantizer
                       restated from the published method (QLoRA, arXiv:2305.14314; dynamic
                       8-bit map of arXiv:2110.02861) that produces packed weights to test with;
- ``oracle.rope``      fused LoRA-add + RoPE forward/backward (solution/attn.py:28-90) and the
                       cos/sin producer (transformers Qwen2RotaryEmbedding, restated as in
                       dev/test_cpu_attn.py:21-24);
- ``oracle.lora``      keep-mask packing, masked LoRA inputs, LoRA input gradient
                       (solution/attn.py:130-180) and the LoRA pair math (solution/attn.py:206-273);
- ``oracle.rmsnorm``   Qwen2RMSNorm (solution/rmsnorm.py:17-45) and the residual add + norm
                       (AddRMSNormFn, :108-144);
- ``oracle.mlp``       the MLP with NF4 gate / up / down and SwiGLU (solution/mlp.py:62-110,
                       solution/swiglu.py:15-37), fp16 rounding points;
- ``oracle.packing``   padding-free packing plan (solution/varlen.py:23-40, :191-226);
- ``oracle.attention`` per-row causal GQA attention, forward (out, logsumexp) and backward
                       (solution/varlen.py:76-121, PackedSDPA);
- ``oracle.block``     the whole attention block, forward and backward, in fp32.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py`` (its ``cpu_baseline`` leg and its
``--impl reference`` arm) may import this package, and only as the checker or the timed CPU
baseline. The product path (``decik_b200``) never imports it.

Pinning: ``tests/golden/make_golden.py`` runs the reference's own modules (Triton interpreter on
the CPU) on seeded inputs and stores the results under ``tests/golden/``; ``tests/test_oracle.py``
checks this oracle against those fixtures.
"""
