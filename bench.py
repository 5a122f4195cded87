#!/usr/bin/env python
"""Benchmark of the hot path: the attention block of the NF4 QLoRA step, forward + backward.

One step = one pass of the block over one packed batch per GPU: NF4 double-quant dequant of
W_q/W_k/W_v + q/k/v GEMMs with bias + LoRA r=16 (alpha 32) on q and v + RoPE + packed varlen causal
GQA attention, then the backward (attention, RoPE, LoRA A/B grads, the projections' input
gradient), then, on N > 1 GPUs, the NCCL all-reduce of the LoRA gradients (data-parallel by whole
packed sequences). Shapes: Qwen2.5-1.5B layer (hidden 1536, 12 q / 2 kv heads, head_dim 128).
Packing: config 3 of the baseline, 16,384 tokens per GPU, row lengths uniform in [64, 4096].
``--workload config4`` runs the baseline's 7B block instead (hidden 3584, 28 q / 4 kv heads,
131,072 tokens per GPU, log-normal lengths of median 4096 up to 32,768).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload config3|config4]

Prints one JSON line (rank 0). ``value`` is whole-job tokens/s with inputs resident in HBM;
``e2e`` is the same step with the inputs copied from pinned host memory and the LoRA gradients
read back inside the timed region (each step's input copy runs on a second stream during the
previous step, as a training loop's prefetch would); ``roofline`` is the varlen attention kernels
(forward + backward) timed live with CUDA events inside the timed steps, against the measured bf16
peak.
``--impl reference`` times the reference's CPU path (the oracle's torch fp32 port of
solution/nf4.py + attn.py + varlen.py PackedSDPA) on a bounded sample, on rank 0 only.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np
import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "QLoRA step tokens/s at 1/2/4/8 B200; varlen attn fwd+bwd TFLOP/s vs BF16 peak"
HIDDEN, HQ, HK, D = 1536, 12, 2, 128
TOKENS = 16384
WORKLOAD = ("attention block fwd+bwd of one Qwen2.5-1.5B QLoRA layer (input RMSNorm, NF4 dq q/k/v + bias, "
            "LoRA r16 q,v, RoPE, varlen causal GQA attention) over config-3 packing")
WORKLOAD7B = ("attention block fwd+bwd of one Qwen2.5-7B QLoRA layer (input RMSNorm, NF4 dq q/k/v + bias, "
              "LoRA r16 q,v, RoPE, varlen causal GQA attention) over config-4 packing")


def lengths_for(seed: int, total: int = TOKENS, lo: int = 64, hi: int = 4096) -> list[int]:
    """Row lengths uniform in [lo, hi], packed greedily to ``total`` tokens (last row truncated)."""
    rng = np.random.default_rng(seed)
    out, t = [], 0
    while t < total:
        L = int(min(rng.integers(lo, hi + 1), total - t))
        out.append(L)
        t += L
    return out


def lengths_config4(seed: int, total: int = 131072, median: int = 4096, sigma: float = 1.0, lo: int = 16,
                    hi: int = 32768, first_max: bool = True) -> list[int]:
    """The 7B block's packing: log-normal lengths (median 4096, sigma 1, clipped to [16, 32768]),
    packed greedily to ``total`` tokens (last row truncated). With ``first_max`` the first row has
    the maximum length, so the longest case is always present."""
    rng = np.random.default_rng(seed)
    out, t = ([hi], hi) if first_max else ([], 0)
    while t < total:
        L = int(np.clip(round(rng.lognormal(np.log(median), sigma)), lo, hi))
        L = min(L, total - t)
        out.append(L)
        t += L
    return out


# name -> (hidden, q heads, kv heads, lengths(seed), workload text, lengths text)
WORKLOADS = {
    "config3": (HIDDEN, HQ, HK, lambda seed: lengths_for(seed), WORKLOAD, "U[64,4096]"),
    "config4": (3584, 28, 4, lambda seed: lengths_config4(seed), WORKLOAD7B,
                "log-normal median 4096 sigma 1 in [16,32768], first row 32768"),
}


# full QLoRA train steps of the 28-layer Qwen2.5-1.5B shape (decik_b200.qlora_model):
# name -> (tokens per GPU, log-normal median, min, max length, workload text)
FULL_STEP = {
    "config2": (830, 180, 16, 1024,
                "28-layer Qwen2.5-1.5B NF4 QLoRA train step (fwd + loss + bwd + AdamW lr 2e-4, LoRA r16 q,v) "
                "over ~830 packed tokens, through solution.apply()"),
    "config5": (16384, 512, 16, 4096,
                "28-layer Qwen2.5-1.5B NF4 QLoRA train step (fwd + loss + bwd + LoRA-grad all-reduce + AdamW "
                "lr 2e-4) over 16,384 packed tokens per GPU, through solution.apply()"),
}


def causal_flops(lengths, n_heads=HQ, head_dim=D) -> float:
    return 4.0 * head_dim * n_heads * sum(L * (L + 1) // 2 for L in lengths)


def peaks() -> dict:
    """Roofline denominators: MEASURED_PEAKS.json (driver-measured on this pool's B200s: bf16 GEMM
    burst and sustained, HBM copy), else the pool's earlier measurement as a labelled fallback."""
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return {"bf16_tflops": float(p["bf16_tflops"]), "hbm_gbs": float(p["hbm_gbs"]),
                "bf16_tflops_sustained": float(p.get("bf16_tflops_sustained", p["bf16_tflops"])),
                "source": "MEASURED_PEAKS.json (measured; bf16 burst)",
                "source_sustained": "MEASURED_PEAKS.json (measured; bf16 sustained: the kernels run inside a "
                                    "long step)"}
    except Exception:
        return {"bf16_tflops": 1590.0, "hbm_gbs": 6650.0, "bf16_tflops_sustained": 1400.0,
                "source": "fallback (earlier pool measurement)",
                "source_sustained": "fallback (earlier pool measurement, sustained)"}


class ClockSampler:
    """SM clocks and clock-event (throttle) reasons sampled every 5 ms through NVML (read-only
    queries) in a background thread while the timed region runs; nvidia-smi at 200 ms as a
    fallback when NVML is unavailable."""

    REASONS = (("hw_slowdown", "nvmlClocksEventReasonHwSlowdown"),
               ("hw_thermal_slowdown", "nvmlClocksEventReasonHwThermalSlowdown"),
               ("sw_thermal_slowdown", "nvmlClocksEventReasonSwThermalSlowdown"),
               ("sw_power_cap", "nvmlClocksEventReasonSwPowerCap"),
               ("hw_power_brake", "nvmlClocksEventReasonHwPowerBrakeSlowdown"))

    def __init__(self, cuda_index: int):
        self.cuda_index = cuda_index
        self.samples, self.max_mhz, self.reasons = [], None, set()
        self.thread = None
        self.stop = False
        self.error = None
        import threading
        self.started = threading.Event()  # set once the first sample is in (or sampling failed)

    def _nvml_index(self) -> int:
        try:
            return int(torch.cuda._get_nvml_device_index(self.cuda_index))
        except Exception:
            return self.cuda_index

    def _run(self):
        try:
            import pynvml as nv
            nv.nvmlInit()
            h = nv.nvmlDeviceGetHandleByIndex(self._nvml_index())
            self.max_mhz = float(nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM))
            masks = [(name, getattr(nv, attr)) for name, attr in self.REASONS if hasattr(nv, attr)]
            while True:
                self.samples.append(float(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)))
                active = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
                for name, m in masks:
                    if active & m:
                        self.reasons.add(name)
                self.started.set()
                if self.stop:
                    break
                time.sleep(0.005)
            nv.nvmlShutdown()
        except Exception as e:  # NVML missing: one nvidia-smi reading instead
            self.error = repr(e)
            try:
                out = subprocess.run(["nvidia-smi", "--query-gpu=clocks.sm,clocks.max.sm", "--format=csv,noheader,nounits",
                                      "-i", str(self._nvml_index())], capture_output=True, text=True, timeout=10).stdout
                cur, mx = out.strip().split(", ")[:2]
                self.samples.append(float(cur))
                self.max_mhz = float(mx)
            except Exception:
                pass
            self.started.set()

    def __enter__(self):
        import threading
        self.thread = threading.Thread(target=self._run, daemon=True)
        self.thread.start()
        self.started.wait(timeout=30)  # the first sample precedes the timed region
        return self

    def __exit__(self, *exc):
        self.stop = True
        self.thread.join(timeout=10)
        return False

    def summary(self) -> dict:
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None, "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples), "source": "nvml" if not self.error else "nvidia-smi"}


def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        import torch.distributed as dist
        backend = "nccl" if torch.cuda.is_available() else "gloo"
        if backend == "nccl":
            torch.cuda.set_device(local)
        dist.init_process_group(backend, timeout=datetime.timedelta(seconds=300))
    return world, rank, local


def block_flops(lengths, hidden=HIDDEN, n_heads=HQ, n_kv=HK) -> float:
    """Algorithmic FLOPs of one attention-block step over these rows: the q/k/v projections'
    forward and input-gradient GEMMs, the LoRA r16 products (forward, input and parameter
    gradients) and the causal attention (3 x the forward's 4 . D . Hq . L(L+1)/2)."""
    T = sum(lengths)
    proj = hidden * (n_heads + 2 * n_kv) * D
    lora = 16 * (2 * hidden + (n_heads + n_kv) * D)
    return 4.0 * proj * T + 6.0 * lora * T + 3.0 * causal_flops(lengths, n_heads=n_heads)


def cpu_reference_steps(lengths, n_steps: int, sample_tokens: int, seed: int = 0, hidden: int = HIDDEN,
                        n_heads: int = HQ, n_kv: int = HK):
    """Times the reference's CPU path (oracle.block, torch fp32) on the first rows of the packing,
    ``sample_tokens`` tokens (last row truncated). Returns (tokens/s of the whole packing
    extrapolated from the sample by block_flops, sample description, threads, step times)."""
    from decik_b200.nf4_quant import quantize_nf4
    from oracle import block as ob

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    rows, t = [], 0
    for L in lengths:
        if t >= sample_tokens:
            break
        L = min(L, sample_tokens - t)
        rows.append(L)
        t += L
    spans, s = [], 0
    for L in rows:
        spans.append((s, L))
        s += L
    T = s
    rng = np.random.default_rng(seed)
    g = torch.Generator().manual_seed(seed)
    inputs = dict(x=torch.randn(T, hidden, generator=g), spans=spans, n_heads=n_heads, n_kv=n_kv, scaling=2.0,
                  norm_w=1.0 + 0.1 * torch.randn(hidden, generator=g), eps=1e-6)
    for name, n_out in (("q", n_heads * D), ("k", n_kv * D), ("v", n_kv * D)):
        inputs[f"nf4_{name}"] = quantize_nf4((rng.standard_normal((n_out, hidden)) * 0.02).astype(np.float32))
        inputs[f"b_{name}"] = torch.randn(n_out, generator=g) * 0.02
    inputs.update(a_q=torch.randn(16, hidden, generator=g) * 0.02,
                  bb_q=torch.randn(n_heads * D, 16, generator=g) * 0.02,
                  a_v=torch.randn(16, hidden, generator=g) * 0.02, bb_v=torch.randn(n_kv * D, 16, generator=g) * 0.02)
    pos = torch.cat([torch.arange(L) for L in rows]).float()
    inv = 1.0 / (1e6 ** (torch.arange(0, D, 2).float() / D))
    fr = torch.outer(pos, inv)
    emb = torch.cat((fr, fr), -1)
    inputs["cos"], inputs["sin"] = emb.cos(), emb.sin()
    grad = torch.randn(T, n_heads * D, generator=g)
    times = []
    for _ in range(n_steps):
        t0 = time.perf_counter()
        ob.block_step(inputs, grad)
        times.append(time.perf_counter() - t0)
    ratio = block_flops(lengths, hidden, n_heads, n_kv) / block_flops(rows, hidden, n_heads, n_kv)
    value = sum(lengths) / (statistics.mean(times) * ratio)
    desc = (f"{len(rows)} rows, {T} tokens (first rows of the packing) timed, fwd+bwd incl. NF4 dequant, fp32 "
            f"({T / statistics.mean(times):.1f} tokens/s); value = the packing's {sum(lengths)} tokens / (sample "
            f"step time x FLOP ratio {ratio:.2f}, block_flops)")
    return value, desc, threads, times


REF_BUDGET_S = 90.0  # the reference arm's timed steps, seconds

# DRAM bytes (read + write) of the two attention kernels per step, from one-pass ncu captures
# (dram__bytes_read.sum + dram__bytes_write.sum). Not measured by this run: the second field says
# which kernel build they describe. config3: one block step (N = 1 packing), forward 68.1 + 14.5 MB,
# backward 432.4 + 181.3 MB. config5: 28 layers x the means of two layers of a timed step at N = 1.
FULL_STEP_ATTN_DRAM_BYTES = {
    "config5": (28 * (81.1e6 + 373.1e6),
                "ncu captures (dram__bytes_read + write, one pass) of attn_fwd_sm100_kernel (83.0, 79.2 MB) and "
                "attn_bwd_sm100_kernel (374.7, 371.5 MB) of two layers of a timed config-5 step at N=1, x 28 "
                "layers; kernels as of commit 1f5d442; not this run's")}
ATTN_DRAM_BYTES = {"config3": (696.3e6, "ncu capture (dram__bytes_read + write) of attn_fwd_sm100_kernel "
                                        "(82.6 MB) and attn_bwd_sm100_kernel (613.7 MB), one launch each, "
                                        "kernels as of commit 1f5d442; not this run's")}


def run_reference(args, world, rank):
    if rank != 0:
        return
    hidden, hq, hk, _, workload, _ = WORKLOADS[args.workload]
    lengths = block_lengths(args.workload, 1, 0)
    sample = args.ref_tokens
    # warm-up step (untimed), then K timed steps, each one bounded sample of the workload; the
    # sample shrinks (attention is superlinear in it, so it is stated in the line) when K steps of
    # it would run past the time budget
    if args.warmup:
        _, _, _, warm = cpu_reference_steps(lengths, 1, sample, hidden=hidden, n_heads=hq, n_kv=hk)
        if args.steps * warm[0] > REF_BUDGET_S:
            sample = max(512, int(sample * REF_BUDGET_S / (args.steps * warm[0])) // 128 * 128)
    value, desc, threads, times = cpu_reference_steps(lengths, args.steps, sample, hidden=hidden, n_heads=hq, n_kv=hk)
    line = {"metric": METRIC, "value": round(value, 2), "unit": "tokens/s", "impl": "reference",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(1e3 * statistics.mean(times), 3), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": workload + " (bounded CPU sample)", "tokens_per_gpu": sum(lengths),
                       "sample": desc, "parallelism": "cpu"},
            "cpu_baseline": {"value": round(value, 2), "unit": "tokens/s", "cores": threads, "kind": "port",
                             "sample": desc},
            "e2e": {"value": round(value, 2), "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def block_lengths(workload: str, world: int, rank: int) -> list[int]:
    """This rank's rows of the block workload. Config 3: one global pool of world x 16,384 tokens
    (lengths U[64, 4096], seed 1000) split across the ranks by whole rows with dp.partition_rows
    (balanced by tokens + causal pairs); at N = 1 the pool is lengths_for(1000). Config 4: each
    rank its own 131,072-token packing (seed 1000 + rank)."""
    from decik_b200.dp import partition_rows

    if workload != "config3":
        return WORKLOADS[workload][3](1000 + rank)
    pool = lengths_for(1000, total=world * TOKENS)
    return [pool[i] for i in partition_rows(pool, world)[rank]]


def measure_block(args, world, rank, local, n_steps, workload=None, e2e=True, cpu=True):
    """The attention block step (config 3 or 4) on this rank; returns rank 0's JSON line (None on
    other ranks). ``e2e`` adds the end-to-end leg, ``cpu`` the CPU baseline leg (rank 0, N=1)."""
    from decik_b200 import ops
    from decik_b200.block import QLoRAAttentionBlock, rope_cos_sin
    from decik_b200.dp import GradBucket
    from decik_b200.solution.varlen import packing_from_lengths

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    name = workload or args.workload
    hidden, hq, hk, _, workload, lengths_text = WORKLOADS[name]
    block = QLoRAAttentionBlock.random(hidden=hidden, n_heads=hq, n_kv=hk, seed=0, device=dev)  # frozen + LoRA
    lengths = block_lengths(name, world, rank)                        # this rank's whole rows
    T = sum(lengths)
    T_all = T
    if world > 1:
        import torch.distributed as dist
        t = torch.tensor([float(T)], device=dev)
        dist.all_reduce(t)
        T_all = int(t.item())
    packing = packing_from_lengths(lengths, dev)
    cos, sin = rope_cos_sin(packing.positions, D)
    g = torch.Generator(device=dev).manual_seed(100 + rank)
    # x is the decoder layer's input h: the block starts with the layer's input RMSNorm (weight
    # ~ 1 + 0.1 N(0, 1), frozen), which the fused node runs inside its first kernel
    x = torch.randn(T, hidden, device=dev, generator=g).requires_grad_(True)
    norm_w = 1.0 + 0.1 * torch.randn(hidden, device=dev, generator=g)
    dout = torch.randn(T, hq * D, device=dev, generator=g).to(torch.bfloat16)
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)  # > 126 MB L2
    bucket = GradBucket(block.lora_params())                         # LoRA grads: views of one fp32 buffer
    if world > 1:
        import torch.distributed as dist

    def step(xin, din):
        bucket.zero_()
        xin.grad = None
        out = block.forward(xin, packing, cos, sin, norm=(norm_w, 1e-6))
        out.backward(din)
        bucket.all_reduce()   # data-parallel exchange: one flat NCCL all-reduce (no-op at N=1)
        return out

    for _ in range(args.warmup):
        step(x, dout)
    torch.cuda.synchronize()

    def timed(n, fn):
        starts = [torch.cuda.Event(enable_timing=True) for _ in range(n)]
        ends = [torch.cuda.Event(enable_timing=True) for _ in range(n)]
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        for i in range(n):
            flush.zero_()                      # L2 flushed between timed steps (not timed)
            starts[i].record()
            fn()
            ends[i].record()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        return [a.elapsed_time(b) for a, b in zip(starts, ends)]

    # the timed steps carry no instrumentation; this library's launches are counted (no events)
    counter = ops.OpTimer(names=())
    ops.install_timer(counter)
    with ClockSampler(local) as clocks:
        step_ms = timed(n_steps, lambda: step(x, dout))
    ops.install_timer(None)
    launches = counter.launches
    # the same steps again with CUDA events around the two attention kernels only (the roofline
    # figure), then a few with events around every op of this library (the kernel table)
    timer = ops.OpTimer(names=("varlen_attn_fwd", "varlen_attn_bwd"))
    ops.install_timer(timer)
    timed(n_steps, lambda: step(x, dout))
    ops.install_timer(None)
    attn_ms = timer.elapsed_ms()
    timer = ops.OpTimer()
    ops.install_timer(timer)
    timed(min(n_steps, 5), lambda: step(x, dout))
    ops.install_timer(None)
    op_ms = timer.elapsed_ms()
    total_ms = sum(step_ms)
    if world > 1:
        t = torch.tensor([total_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        total_ms = float(t.item())
    value = T_all * n_steps / (total_ms / 1e3)

    e2e_value = None
    if e2e:
        # end to end through the same public API: every step's x and dOut are copied from pinned host
        # memory and its LoRA gradients read back inside the timed region. As a training loop's input
        # prefetch would, step i + 1's inputs are copied on a second stream (into the other of two
        # device buffers) while step i computes. Inputs (151 MB) exceed L2 and are new every step.
        x_host = x.detach().cpu().pin_memory()
        d_host = dout.cpu().pin_memory()
        g_host = torch.empty(bucket.flat.numel(), dtype=torch.float32).pin_memory()
        bufs = [(torch.empty_like(x.detach()), torch.empty_like(dout)) for _ in range(2)]
        copy_stream = torch.cuda.Stream(device=dev)
        compute = torch.cuda.current_stream(dev)

        def e2e_run(n):
            copied = [torch.cuda.Event() for _ in range(2)]
            consumed = [torch.cuda.Event() for _ in range(2)]

            def copy_in(i):
                b = i % 2
                with torch.cuda.stream(copy_stream):
                    if i >= 2:
                        copy_stream.wait_event(consumed[b])  # step i - 2 is done with this buffer
                    bufs[b][0].copy_(x_host, non_blocking=True)
                    bufs[b][1].copy_(d_host, non_blocking=True)
                    copied[b].record(copy_stream)

            copy_in(0)
            for i in range(n):
                b = i % 2
                if i + 1 < n:
                    copy_in(i + 1)
                compute.wait_event(copied[b])
                step(bufs[b][0].detach().requires_grad_(True), bufs[b][1])
                consumed[b].record(compute)
                g_host.copy_(bucket.flat, non_blocking=True)

        e2e_run(2)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ev0.record(compute)
        e2e_run(n_steps)
        ev1.record(compute)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        e2e_ms = ev0.elapsed_time(ev1)
        if world > 1:
            t = torch.tensor([e2e_ms], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            e2e_ms = float(t.item())
        e2e_value = T_all * n_steps / (e2e_ms / 1e3)

    if rank != 0:
        return None
    pk = peaks()
    f_fwd = causal_flops(lengths, n_heads=hq)
    fwd_ms = statistics.mean(attn_ms.get("varlen_attn_fwd", [float("nan")]))
    bwd_ms = statistics.mean(attn_ms.get("varlen_attn_bwd", [float("nan")]))
    attn_tflops = 3.0 * f_fwd / ((fwd_ms + bwd_ms) / 1e3) / 1e12
    kernels = {name: {"ms_mean": round(statistics.mean(v), 4), "calls_per_step": len(v) // min(n_steps, 5)}
               for name, v in op_ms.items()}
    kernels["varlen_attn_fwd"]["tflops"] = round(f_fwd / (fwd_ms / 1e3) / 1e12, 2)
    kernels["varlen_attn_bwd"]["tflops"] = round(2 * f_fwd / (bwd_ms / 1e3) / 1e12, 2)
    line = {
        "metric": METRIC, "value": round(value, 1), "unit": "tokens/s", "n_gpus": world,
        "steps": n_steps, "warmup": args.warmup, "ms_per_step": round(total_ms / n_steps, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded lengths, N(0,1) activations, random-init NF4/LoRA weights)",
        "config": {"workload": workload, "tokens_per_gpu": T, "tokens_all_ranks": T_all, "rows_rank0": len(lengths),
                   "lengths": f"{lengths_text}; " + ("one pool of N x 16,384 tokens (seed 1000) split by "
                                                     "dp.partition_rows" if name == "config3" else
                                                     "numpy default_rng(1000 + rank)"), "hidden": hidden,
                   "heads": f"{hq}/{hk}", "head_dim": D, "lora": "r16 alpha32 q,v", "nf4": "bs64, double quant bs256",
                   "l2": "flushed between timed steps (256 MiB write, untimed)", "parallelism": f"dp{world}"},
        "roofline": {"bound": "tensor", "kernel": "varlen attention fwd+bwd (decik_varlen_attn_fwd/bwd)",
                     "achieved": round(attn_tflops, 2), "peak": pk["bf16_tflops"], "unit": "TFLOP/s",
                     "frac": round(attn_tflops / pk["bf16_tflops"], 4),
                     "traffic": ATTN_DRAM_BYTES.get(name, (None, None))[0],
                     "traffic_source": ATTN_DRAM_BYTES.get(name, (None, None))[1],
                     "flops_per_step": 3.0 * f_fwd, "peak_source": pk["source"]},
        "attn_tflops": round(attn_tflops, 2),
        "kernels": kernels,
        "kernels_note": "CUDA events around every op of this library, 5 extra steps (host-inclusive: an op "
                        "whose launch the GPU waited for includes the wait); the roofline uses events around "
                        "the attention kernels only, over a second pass of the timed steps",
        "gpu_launches": launches,
        "clocks": clocks.summary(),
    }
    if e2e:
        line["e2e"] = {"value": round(e2e_value, 1), "unit": "tokens/s",
                       "h2d_bytes_per_step": x_host.numel() * 4 + d_host.numel() * 2,
                       "d2h_bytes_per_step": g_host.numel() * 4,
                       "pipelining": "step i+1's inputs copied on a second stream while step i computes"}
    if cpu and world == 1 and not args.no_cpu_baseline:
        cv, desc, threads, _ = cpu_reference_steps(lengths, 1, args.ref_tokens, hidden=hidden, n_heads=hq, n_kv=hk)
        line["cpu_baseline"] = {"value": round(cv, 2), "unit": "tokens/s", "cores": threads, "kind": "port",
                                "sample": desc}
    return line


def run_ours(args, world, rank, local):
    line = measure_block(args, world, rank, local, args.steps)
    if line is not None:
        print(json.dumps(line), flush=True)


def full_step_attn_weight(cfg=None) -> float:
    """Causal score pairs -> token-equivalents for dp.partition_rows on the full step: attention
    FLOPs per score pair over the linear-layer FLOPs per token of the 28-layer model (its 7 NF4
    linears per layer and the head), doubled because the attention kernels run at about half the
    GEMMs' fraction of peak."""
    from decik_b200.qlora_model import QWEN25_15B

    c = cfg or QWEN25_15B
    h, hq, hk, inter, vocab = c["hidden"], c["heads"], c["kv_heads"], c["intermediate"], c["vocab"]
    per_token = c["layers"] * h * ((hq + 2 * hk) * D + hq * D + 3 * inter) + h * vocab
    per_pair = c["layers"] * 2 * hq * D
    return 2.0 * per_pair / per_token


def full_step_lengths(workload: str, world: int, rank: int) -> list[int]:
    """This rank's rows of a full-step workload: one global pool of world x (tokens per GPU) rows
    (log-normal lengths, seed 1000) split across the ranks by whole rows with dp.partition_rows."""
    from decik_b200.dp import partition_rows
    from decik_b200.qlora_model import lognormal_lengths

    total, median, lo, hi, _ = FULL_STEP[workload]
    pool = lognormal_lengths(1000, world * total, median, lo, hi)
    if world == 1:
        return pool
    return [pool[i] for i in partition_rows(pool, world, attn_weight=full_step_attn_weight())[rank]]


def full_step_flops(lengths, cfg=None) -> float:
    """Algorithmic FLOPs of one QLoRA train step over these rows: the frozen linears' forward and
    input-gradient GEMMs (2 x 2 x MACs per token), the head's the same, the LoRA r16 products
    (forward, input and parameter gradients) and the causal attention (3 x the forward's
    4 . D . Hq . L(L+1)/2 per layer). The basis of the CPU arm's extrapolation from its sample."""
    from decik_b200.qlora_model import QWEN25_15B

    c = cfg or QWEN25_15B
    h, hq, hk, inter, vocab, layers = c["hidden"], c["heads"], c["kv_heads"], c["intermediate"], c["vocab"], c["layers"]
    T = sum(lengths)
    lin = layers * h * ((hq + 2 * hk) * D + hq * D + 3 * inter) + h * vocab
    lora = layers * 16 * (2 * h + (hq + hk) * D)
    return 4.0 * lin * T + 6.0 * lora * T + layers * 3.0 * causal_flops(lengths, n_heads=hq)


def run_full_step(args, world, rank, local):
    """The whole QLoRA train step of the 28-layer model through the reference-facing surface:
    solution.apply() patches the model; each step is forward + loss + backward + the LoRA-grad
    all-reduce (N > 1) + AdamW. The rows of one global pool are split across the ranks by
    dp.partition_rows; the loss is normalised by the global labelled-token count."""
    from decik_b200 import ops, solution
    from decik_b200.dp import GradBucket, global_count
    from decik_b200.qlora_model import (QWEN25_15B, Linear4bit, LoraLinear, build_qlora_qwen2,
                                        lora_parameters, padded_batch, qlora_train_step)

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    total, median, lo, hi, workload = FULL_STEP[args.workload]
    model = build_qlora_qwen2(device=dev, seed=0)
    solution.apply(linear4bit_cls=Linear4bit, lora_classes=(LoraLinear,))
    n_layers = QWEN25_15B["layers"]
    lengths = full_step_lengths(args.workload, world, rank)
    T = sum(lengths)
    ids, mask, labels = padded_batch(lengths, QWEN25_15B["vocab"], 2000 + rank, dev)
    params = lora_parameters(model)
    bucket = GradBucket(params)
    bucket.check_layout()
    opt = torch.optim.AdamW(params, lr=2e-4)
    # labelled tokens of this step over all ranks (each row's last token has no next-token label)
    n_labels = global_count(torch.tensor(float(T - len(lengths)), device=dev)).to(dev)
    T_all = int(global_count(torch.tensor(float(T), device=dev)).item())
    if world > 1:
        import torch.distributed as dist
    ar_events = []  # (start, end) around the LoRA-gradient all-reduce of each timed step

    def step(i_ids, i_mask, i_labels, time_ar=False):
        bucket.zero_()
        loss = qlora_train_step(model, i_ids, i_mask, i_labels, n_labels=n_labels)
        if time_ar:
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            bucket.all_reduce()
            b.record()
            ar_events.append((a, b))
        else:
            bucket.all_reduce()
        opt.step()
        return loss

    for _ in range(args.warmup):
        step(ids, mask, labels)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    counter = ops.OpTimer(names=())  # counts this library's launches; no events in the timed steps
    ops.install_timer(counter)
    with ClockSampler(local) as clocks:
        for i in range(args.steps):
            starts[i].record()
            step(ids, mask, labels, time_ar=True)
            ends[i].record()
        torch.cuda.synchronize()
    ops.install_timer(None)
    step_ms = [a.elapsed_time(b) for a, b in zip(starts, ends)]
    # a second pass of the same steps with events around the attention kernels only (the
    # roofline), then a few with events around every op of this library (the kernel table)
    n_inst = min(args.steps, 5)
    timer = ops.OpTimer(names=("varlen_attn_fwd", "varlen_attn_bwd"))
    ops.install_timer(timer)
    for i in range(args.steps):
        step(ids, mask, labels)
    ops.install_timer(None)
    attn_ms = timer.elapsed_ms()
    timer = ops.OpTimer()
    ops.install_timer(timer)
    for i in range(n_inst):
        step(ids, mask, labels)
    ops.install_timer(None)
    op_ms = timer.elapsed_ms()
    ar_ms = statistics.mean(a.elapsed_time(b) for a, b in ar_events) if ar_events else 0.0
    total_ms = sum(step_ms)
    rank_ms = [total_ms / args.steps]
    if world > 1:
        every = [torch.zeros(2, device=dev) for _ in range(world)]
        dist.all_gather(every, torch.tensor([total_ms / args.steps, ar_ms], device=dev))
        rank_ms = [float(e[0]) for e in every]
        rank_ar = [float(e[1]) for e in every]
        total_ms = max(rank_ms) * args.steps
    else:
        rank_ar = [ar_ms]
    value = T_all * args.steps / (total_ms / 1e3)

    # end to end: each step's token ids, mask and labels copied from pinned host memory and its loss
    # read back into pinned host memory, all inside the timed region
    h_ids, h_mask, h_labels = (t.cpu().pin_memory() for t in (ids, mask, labels))
    h_loss = torch.empty(args.steps, dtype=torch.float32).pin_memory()
    d_ids, d_mask, d_labels = torch.empty_like(ids), torch.empty_like(mask), torch.empty_like(labels)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(args.steps):
        d_ids.copy_(h_ids, non_blocking=True)
        d_mask.copy_(h_mask, non_blocking=True)
        d_labels.copy_(h_labels, non_blocking=True)
        loss = step(d_ids, d_mask, d_labels)
        h_loss[i:i + 1].copy_(loss.reshape(1), non_blocking=True)
    e1.record()
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([e2e_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())
    e2e_value = T_all * args.steps / (e2e_ms / 1e3)

    # the block step of config 3 (the path alone, L2 flushed between steps), as an extra key
    block = None
    if not args.no_block:
        block = measure_block(args, world, rank, local, min(args.steps, 20), workload="config3", e2e=False,
                              cpu=False)
    if rank != 0:
        return
    pk = peaks()
    f_fwd = causal_flops(lengths, n_heads=QWEN25_15B["heads"]) * n_layers
    fwd_ms = sum(attn_ms.get("varlen_attn_fwd", [float("nan")])) / args.steps
    bwd_ms = sum(attn_ms.get("varlen_attn_bwd", [float("nan")])) / args.steps
    attn_tflops = 3.0 * f_fwd / ((fwd_ms + bwd_ms) / 1e3) / 1e12
    kernels = {name: {"ms_per_step": round(sum(v) / n_inst, 4), "calls_per_step": len(v) // n_inst}
               for name, v in op_ms.items()}
    line = {
        "metric": METRIC, "value": round(value, 1), "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(total_ms / args.steps, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded log-normal lengths, uniform token ids, random-init NF4 weights and LoRA)",
        "config": {"workload": workload, "tokens_per_gpu": T, "tokens_all_ranks": T_all, "rows_rank0": len(lengths),
                   "lengths": f"log-normal median {median} sigma 1 in [{lo},{hi}]: one pool of N x {total} tokens "
                              "(numpy default_rng(1000)) split across ranks by dp.partition_rows",
                   "model": "Qwen2.5-1.5B shape: 28 layers, hidden 1536, inter 8960, 12/2 heads, vocab 151936",
                   "lora": "r16 alpha32 q,v", "nf4": "bs64, double quant bs256 (all 7 linears per layer)",
                   "l2": "not flushed: each step streams the 0.7 GB of NF4 weights and the 0.9 GB embedding (> L2)",
                   "parallelism": f"dp{world}"},
        "roofline": {"bound": "tensor", "kernel": "varlen attention fwd+bwd of the 28 layers (decik_varlen_attn_fwd/bwd)",
                     "achieved": round(attn_tflops, 2), "peak": pk["bf16_tflops_sustained"], "unit": "TFLOP/s",
                     "frac": round(attn_tflops / pk["bf16_tflops_sustained"], 4),
                     "traffic": FULL_STEP_ATTN_DRAM_BYTES.get(args.workload, (None, None))[0],
                     "traffic_source": FULL_STEP_ATTN_DRAM_BYTES.get(args.workload, (None, None))[1],
                     "flops_per_step": 3.0 * f_fwd,
                     "peak_source": pk["source_sustained"]},
        "attn_tflops": round(attn_tflops, 2),
        "rank_ms_per_step": [round(v, 3) for v in rank_ms],
        "allreduce_ms_per_step": [round(v, 4) for v in rank_ar],
        "allreduce_bytes": bucket.nbytes,
        "kernels": kernels,
        "kernels_note": "CUDA events around every op of this library over 5 extra steps (host-inclusive: an op "
                        "whose launch the GPU waited for includes the wait); the roofline uses events around the "
                        "attention kernels only, over a second pass of the timed steps",
        "gpu_launches": counter.launches,
        "clocks": clocks.summary(),
        "loss_last": round(float(h_loss[-1]), 5),
        "e2e": {"value": round(e2e_value, 1), "unit": "tokens/s",
                "h2d_bytes_per_step": sum(t.numel() * t.element_size() for t in (h_ids, h_mask, h_labels)),
                "d2h_bytes_per_step": 4},
    }
    if block is not None:
        line["block_config3"] = {k: block[k] for k in ("value", "ms_per_step", "roofline", "kernels", "config")}
    if world == 1 and not args.no_cpu_baseline:
        cv, cv_sample, desc, threads, _ = cpu_full_step(args.workload, lengths, 2, args.full_ref_tokens)
        line["cpu_baseline"] = {"value": round(cv, 4), "unit": "tokens/s", "cores": threads, "kind": "port",
                                "sample": desc, "sample_value": round(cv_sample, 3)}
    print(json.dumps(line), flush=True)
    if args.profile and world == 1:  # one GPU only: a step would all-reduce with ranks that have left
        from torch.profiler import ProfilerActivity, profile

        with profile(activities=[ProfilerActivity.CUDA, ProfilerActivity.CPU]) as prof:
            step(ids, mask, labels)
            torch.cuda.synchronize()
        avg = prof.key_averages()
        print(avg.table(sort_by="self_cuda_time_total", row_limit=30, max_name_column_width=60), file=sys.stderr)
        print(avg.table(sort_by="self_cpu_time_total", row_limit=40, max_name_column_width=60), file=sys.stderr,
              flush=True)


def cpu_full_step(workload, lengths, n_steps, sample_tokens, warmup=0, budget_s=None):
    """The reference's CPU path for the full step, timed on bounded samples: the same model on the
    host in fp32 with the original transformers code (no patches), NF4 weights dequantised by the
    torch restatement of solution/nf4.py:36-48 on every call, over the first rows of ``lengths``
    cut to a sample. The timed steps alternate between two samples (``sample_tokens`` / 4 and
    ``sample_tokens``) so that the step time can be split into a part fixed per step (the NF4
    dequant of every linear call, the optimizer) and a part proportional to the step's FLOPs
    (full_step_flops); that affine fit extrapolates the step time to ``lengths``. ``budget_s``
    stops the timed steps early (at least two) once their time would pass it.
    Returns (tokens/s of ``lengths`` extrapolated, tokens/s of the larger sample, description,
    threads, step times)."""
    from decik_b200.qlora_model import (QWEN25_15B, Linear4bit, build_qlora_qwen2, lora_parameters,
                                        padded_batch, qlora_train_step)
    from oracle.block import dequant_torch_qs

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    t_build = time.perf_counter()
    model = build_qlora_qwen2(device="cpu", seed=0, share_layer_weights=True)
    build_s = time.perf_counter() - t_build
    original = Linear4bit.forward

    def cpu_forward(self, x):
        w = dequant_torch_qs(self.weight.data, self.weight.quant_state)
        return torch.nn.functional.linear(x.float(), w, None if self.bias is None else self.bias.float())

    def first_rows(n_tok):
        rows, t = [], 0
        for L in lengths:
            if t >= n_tok:
                break
            rows.append(min(L, n_tok - t))
            t += rows[-1]
        return rows

    samples = [first_rows(max(8, sample_tokens // 4)), first_rows(sample_tokens)]
    batches = [padded_batch(rows, QWEN25_15B["vocab"], 2000, "cpu") for rows in samples]
    Linear4bit.forward = cpu_forward
    times = {0: [], 1: []}
    all_times = []
    try:
        opt = torch.optim.AdamW(lora_parameters(model), lr=2e-4)
        n_run = 0
        for i in range(warmup + max(n_steps, 2)):
            which = i % 2
            t0 = time.perf_counter()
            model.zero_grad(set_to_none=True)
            qlora_train_step(model, *batches[which])
            opt.step()
            dt = time.perf_counter() - t0
            if i >= warmup:
                times[which].append(dt)
                all_times.append(dt)
                n_run += 1
                if (budget_s is not None and n_run >= 2 and n_run < n_steps
                        and sum(all_times) * (n_run + 1) / n_run > budget_s):
                    break
    finally:
        Linear4bit.forward = original
    t_small, t_large = statistics.mean(times[0]), statistics.mean(times[1])
    f_small, f_large, f_full = (full_step_flops(r) for r in (samples[0], samples[1], lengths))
    per_flop = (t_large - t_small) / (f_large - f_small) if f_large > f_small else 0.0
    if per_flop > 0:
        fixed = max(0.0, t_large - per_flop * f_large)
        full_s = fixed + per_flop * f_full
        how = (f"affine fit over the two samples: {fixed:.2f} s per step fixed + {per_flop * 1e12:.2f} s per "
               f"TFLOP x {f_full / 1e12:.1f} TFLOP (full_step_flops of the workload)")
    else:  # the two samples did not separate: proportional to FLOPs from the larger one
        full_s = t_large * f_full / f_large
        how = f"larger sample's step time x FLOP ratio {f_full / f_large:.1f} (full_step_flops)"
    value = sum(lengths) / full_s
    sample_value = sum(samples[1]) / t_large
    desc = (f"two samples of the workload's first rows timed alternately ({sum(samples[0])} tokens: "
            f"{t_small:.2f} s/step, {sum(samples[1])} tokens: {t_large:.2f} s/step; {len(all_times)} steps): full "
            f"28-layer step fwd+bwd+AdamW in fp32 with NF4 dequant per call, frozen NF4 weights shared by the "
            f"layers (model build {build_s:.0f} s, untimed); value = the workload's {sum(lengths)} tokens / "
            f"{full_s:.1f} s, the step time extrapolated by an {how}")
    return value, sample_value, desc, threads, all_times


def run_reference_full(args, world, rank):
    """The reference arm for the full step: the reference's CPU path (cpu_full_step) on rank 0,
    with the value extrapolated from its timed sample to this configuration's rows by FLOPs."""
    if rank != 0:
        return
    *_, workload = FULL_STEP[args.workload]
    lengths = full_step_lengths(args.workload, 1, 0)
    value, sample_value, desc, threads, times = cpu_full_step(args.workload, lengths, args.steps,
                                                              args.full_ref_tokens, warmup=min(args.warmup, 1),
                                                              budget_s=REF_BUDGET_S)
    line = {"metric": METRIC, "value": round(value, 4), "unit": "tokens/s", "impl": "reference",
            "n_gpus": args.gpus, "steps": len(times), "warmup": min(args.warmup, 1),
            "steps_note": f"{len(times)} of the {args.steps} requested timed CPU steps ran (stopped at the "
                          f"{REF_BUDGET_S:.0f} s CPU budget, at least 2); one warm-up step",
            "ms_per_step": round(1e3 * statistics.mean(times), 1), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": workload.replace("through solution.apply()",
                                                    "on the original transformers code with torch NF4 dequant"),
                       "tokens_per_gpu": sum(lengths), "sample": desc, "parallelism": "cpu",
                       "extrapolated": True, "sample_value": round(sample_value, 3)},
            "cpu_baseline": {"value": round(value, 4), "unit": "tokens/s", "cores": threads, "kind": "port",
                             "sample": desc},
            "e2e": {"value": round(value, 4), "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None, help="timed steps (default 100; 10 with --impl reference)")
    ap.add_argument("--warmup", type=int, default=None, help="untimed steps (default 10; 1 with --impl reference)")
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--ref-tokens", type=int, default=4096, help="tokens of the bounded CPU sample")
    ap.add_argument("--full-ref-tokens", type=int, default=512,
                    help="tokens of the bounded CPU sample of the full step (cpu_baseline and --impl reference)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-block", action="store_true", help="full step: skip the extra config-3 block measurement")
    ap.add_argument("--profile", action="store_true",
                    help="full-step workloads, one GPU: after the JSON line, one more step under torch.profiler; "
                         "its device-time and host-time tables go to stderr")
    ap.add_argument("--workload", choices=sorted(WORKLOADS) + sorted(FULL_STEP), default="config5",
                    help="config5: the full 28-layer QLoRA train step over 16,384 tokens per GPU (default, "
                         "with the config-3 block step as an extra key); config2: the same over ~830 tokens; "
                         "config3: the 1.5B attention block over 16,384 tokens; config4: the 7B block over 131,072")
    args = ap.parse_args()
    if args.steps is None:
        args.steps = 10 if args.impl == "reference" else (20 if args.workload in FULL_STEP else 100)
    if args.warmup is None:
        args.warmup = 1 if args.impl == "reference" else (5 if args.workload in FULL_STEP else 10)
    world, rank, local = dist_setup()
    try:
        if args.workload in FULL_STEP:
            if args.impl == "reference":
                run_reference_full(args, world, rank)
            else:
                run_full_step(args, world, rank, local)
        elif args.impl == "reference":
            run_reference(args, world, rank)
        else:
            run_ours(args, world, rank, local)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
