"""Torch-tensor front end of the C ABI: each function checks its tensors, allocates the outputs
with the PyTorch caching allocator and enqueues the kernels on the current CUDA stream.

These are the operators the reference-facing modules in ``decik_b200.solution`` call. They run
only on CUDA tensors; anything else raises (there is no CPU fallback).
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib
from ._lib import BF16, F16, F32, Tensor3

_DT = {torch.float16: F16, torch.bfloat16: BF16, torch.float32: F32}


def _dt(t: torch.Tensor) -> int:
    try:
        return _DT[t.dtype]
    except KeyError:
        raise RuntimeError(f"decik_b200: unsupported dtype {t.dtype}") from None


def _cuda(*ts: torch.Tensor | None) -> None:
    for t in ts:
        if t is not None and not t.is_cuda:
            raise RuntimeError("decik_b200: tensors must be on a CUDA device (no CPU fallback)")


def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def _p(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


# ------------------------------------------------------------------------------------------------
# padding-free packing
# ------------------------------------------------------------------------------------------------
_MASK_CODES = {torch.int64: 0, torch.int32: 1, torch.uint8: 2, torch.bool: 2}
_pinned: dict = {}


def _pinned_i32(n: int) -> torch.Tensor:
    """A reused page-locked int32 host buffer of at least n values (this thread's packing reads)."""
    buf = _pinned.get("summary")
    if buf is None or buf.numel() < n:
        buf = torch.empty(max(n, 1024), dtype=torch.int32, pin_memory=True)
        _pinned["summary"] = buf
    return buf


def pack_rows(mask: torch.Tensor, input_ids: torch.Tensor | None = None):
    """The packing of a right-padded [B, S] batch built on the device (decik_pack_rows).

    Returns None when some row is not right-padded, else ``(lengths, cu_seqlens, index,
    positions, ids)``: the row lengths as host ints, cu_seqlens int32 [B + 1], index / positions
    int64 [T] and the packed ids int64 [T] (None without ``input_ids``), all on the mask's device.
    The only host read is the summary of 4 + B int32, copied into pinned memory."""
    _cuda(mask, input_ids)
    if mask.dim() != 2:
        raise RuntimeError("decik_b200 pack_rows: mask must be [batch, seq]")
    code = _MASK_CODES.get(mask.dtype)
    if code is None:
        raise RuntimeError(f"decik_b200 pack_rows: mask dtype {mask.dtype}")
    mask = mask.contiguous()
    B, S = mask.shape
    dev = mask.device
    if input_ids is not None:
        if input_ids.shape != mask.shape or input_ids.dtype != torch.int64:
            raise RuntimeError("decik_b200 pack_rows: input_ids must be int64 [batch, seq]")
        input_ids = input_ids.contiguous()
    cu = torch.empty(B + 1, dtype=torch.int32, device=dev)
    index = torch.empty(B * S, dtype=torch.int64, device=dev)
    positions = torch.empty(B * S, dtype=torch.int64, device=dev)
    ids = torch.empty(B * S, dtype=torch.int64, device=dev) if input_ids is not None else None
    summary = torch.empty(4 + B, dtype=torch.int32, device=dev)
    rc = _lib.lib().decik_pack_rows(_p(mask), code, _p(input_ids), B, S, _p(cu), _p(index), _p(positions),
                                    _p(ids), _p(summary), _stream(mask))
    _lib.check(rc, "pack_rows")
    host = _pinned_i32(4 + B)[:4 + B]
    host.copy_(summary, non_blocking=True)
    done = torch.cuda.Event()
    done.record(torch.cuda.current_stream(dev))
    done.synchronize()  # the step's one device -> host read
    vals = host.tolist()
    T, right_padded = vals[0], vals[2]
    if not right_padded:
        return None
    lengths = vals[4:4 + B]
    return lengths, cu, index[:T], positions[:T], (ids[:T] if ids is not None else None)


# ------------------------------------------------------------------------------------------------
# NF4
# ------------------------------------------------------------------------------------------------
def nf4_dequant(packed: torch.Tensor, absmax: torch.Tensor, code: torch.Tensor, shape,
                blocksize: int, absmax2: torch.Tensor | None = None, code2: torch.Tensor | None = None,
                offset: torch.Tensor | None = None, blocksize2: int = 256,
                out_dtype: torch.dtype = torch.float16, out: torch.Tensor | None = None) -> torch.Tensor:
    """[N, K] weights from packed NF4 (solution/nf4.py:66-85). ``nested`` iff absmax is uint8."""
    nested = absmax.dtype == torch.uint8
    _cuda(packed, absmax, code, absmax2, code2, offset)
    n_out, n_in = int(shape[0]), int(shape[1])
    n_bytes = n_out * n_in // 2
    if packed.numel() < n_bytes:
        raise RuntimeError("decik_b200 nf4_dequant: packed tensor smaller than shape")
    if out is None:
        out = torch.empty((n_out, n_in), dtype=out_dtype, device=packed.device)
    elif not (out.is_contiguous() and out.numel() == n_out * n_in and out.dtype == out_dtype):
        raise RuntimeError("decik_b200 nf4_dequant: out must be contiguous [N, K] of out_dtype")
    with _timed("nf4_dequant", 1):
        rc = _lib.lib().decik_nf4_dequant(
            _p(packed), _p(absmax), _p(absmax2) if nested else None, _p(code2) if nested else None,
            _p(offset) if nested else None, _p(code), _p(out), n_bytes, int(nested), int(blocksize),
            int(blocksize2), _dt(out), _stream(packed))
    _lib.check(rc, "nf4_dequant")
    return out


def nf4_dequant_batch(jobs, out_dtype: torch.dtype) -> None:
    """Several NF4 weights in one launch (decik_nf4_dequant_batch). ``jobs``: tuples (packed, absmax,
    code, shape, blocksize, absmax2, code2, offset, blocksize2, out) with nf4_dequant's meaning; each
    ``out`` a contiguous [N, K] of ``out_dtype`` (e.g. row slices of one matrix)."""
    arr = (_lib.Nf4Job * len(jobs))()
    stream = None
    for i, (packed, absmax, code, shape, blocksize, absmax2, code2, offset, blocksize2, out) in enumerate(jobs):
        nested = absmax.dtype == torch.uint8
        _cuda(packed, absmax, code, absmax2, code2, offset, out)
        n_out, n_in = int(shape[0]), int(shape[1])
        if packed.numel() < n_out * n_in // 2:
            raise RuntimeError("decik_b200 nf4_dequant: packed tensor smaller than shape")
        if not (out.is_contiguous() and out.numel() == n_out * n_in and out.dtype == out_dtype):
            raise RuntimeError("decik_b200 nf4_dequant: out must be contiguous [N, K] of out_dtype")
        arr[i] = _lib.Nf4Job(_p(packed), _p(absmax), _p(absmax2) if nested else None, _p(code2) if nested else None,
                             _p(offset) if nested else None, _p(code), _p(out), n_out * n_in // 2, int(nested),
                             int(blocksize), int(blocksize2))
        stream = _stream(packed)
    if not jobs:
        return
    with _timed("nf4_dequant", 1):
        rc = _lib.lib().decik_nf4_dequant_batch(ctypes.addressof(arr), len(jobs), _DT[out_dtype], stream)
    _lib.check(rc, "nf4_dequant_batch")


# ------------------------------------------------------------------------------------------------
# RoPE
# ------------------------------------------------------------------------------------------------
def rope_fwd(q_base: torch.Tensor, q_lora: torch.Tensor | None, k: torch.Tensor, cos: torch.Tensor,
             sin: torch.Tensor, n_heads: int, n_kv: int):
    """q_base, q_lora [T, Hq*D], k [T, Hk*D] (contiguous, fp16/bf16), cos/sin fp32 [T, D] ->
    q [Hq, T, D], k [Hk, T, D] (solution/attn.py:97-111)."""
    _cuda(q_base, q_lora, k, cos, sin)
    T = q_base.shape[0]
    D = cos.shape[-1]
    for t in (q_base, q_lora, k, cos, sin):
        if t is not None and not t.is_contiguous():
            raise RuntimeError("decik_b200 rope_fwd: inputs must be contiguous")
    q_out = torch.empty((n_heads, T, D), dtype=q_base.dtype, device=q_base.device)
    k_out = torch.empty((n_kv, T, D), dtype=q_base.dtype, device=q_base.device)
    with _timed("rope_fwd", 1):
        rc = _lib.lib().decik_rope_fwd(_p(q_base), _p(q_lora), _p(k), _p(cos), _p(sin), _p(q_out),
                                       _p(k_out), T, n_heads, n_kv, D, _dt(q_base), _stream(q_base))
    _lib.check(rc, "rope_fwd")
    return q_out, k_out


def rope_bwd(grad_q: torch.Tensor, grad_k: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor):
    """grad_q [Hq, T, D], grad_k [Hk, T, D] -> dq [T, Hq*D], dk [T, Hk*D] (solution/attn.py:113-126)."""
    _cuda(grad_q, grad_k, cos, sin)
    grad_q = grad_q.contiguous()
    grad_k = grad_k.contiguous()
    Hq, T, D = grad_q.shape
    Hk = grad_k.shape[0]
    dq = torch.empty((T, Hq * D), dtype=grad_q.dtype, device=grad_q.device)
    dk = torch.empty((T, Hk * D), dtype=grad_q.dtype, device=grad_q.device)
    with _timed("rope_bwd", 1):
        rc = _lib.lib().decik_rope_bwd(_p(grad_q), _p(grad_k), _p(cos.contiguous()), _p(sin.contiguous()),
                                       _p(dq), _p(dk), T, Hq, Hk, D, _dt(grad_q), _stream(grad_q))
    _lib.check(rc, "rope_bwd")
    return dq, dk


# ------------------------------------------------------------------------------------------------
# LoRA dropout helpers
# ------------------------------------------------------------------------------------------------
def keep_pack(keep_q: torch.Tensor, keep_v: torch.Tensor):
    _cuda(keep_q, keep_v)
    n, w = keep_q.shape
    kq = keep_q.contiguous().view(torch.uint8)
    kv = keep_v.contiguous().view(torch.uint8)
    bq = torch.empty((n, w // 8), dtype=torch.uint8, device=keep_q.device)
    bv = torch.empty_like(bq)
    _lib.check(_lib.lib().decik_keep_pack(_p(kq), _p(kv), _p(bq), _p(bv), n, w, _stream(kq)), "keep_pack")
    return bq, bv


def lora_inputs(x: torch.Tensor, bits_q, bits_v, scale_q, scale_v, out_dtype=torch.float16):
    _cuda(x, bits_q, bits_v, scale_q, scale_v)
    w = x.shape[-1]
    x2 = x.reshape(-1, w).contiguous()
    n = x2.shape[0]
    xq = torch.empty((n, w), dtype=out_dtype, device=x.device)
    xv = torch.empty_like(xq)
    sq = scale_q.reshape(1).to(torch.float32).contiguous()
    sv = scale_v.reshape(1).to(torch.float32).contiguous()
    rc = _lib.lib().decik_lora_inputs(_p(x2), _p(bits_q), _p(bits_v), _p(sq), _p(sv), _p(xq), _p(xv),
                                      n, w, _dt(xq), _stream(x))
    _lib.check(rc, "lora_inputs")
    return xq, xv


def lora_input_grad(g_q, g_v, bits_q, bits_v, scale_q: float, scale_v: float):
    _cuda(g_q, g_v, bits_q, bits_v)
    w = g_q.shape[-1]
    gq = g_q.reshape(-1, w).contiguous()
    gv = g_v.reshape(-1, w).to(gq.dtype).contiguous()
    n = gq.shape[0]
    out = torch.empty((n, w), dtype=torch.float32, device=g_q.device)
    rc = _lib.lib().decik_lora_input_grad(_p(gq), _p(gv), _p(bits_q), _p(bits_v), _p(out), n, w,
                                          float(scale_q), float(scale_v), _dt(gq), _stream(gq))
    _lib.check(rc, "lora_input_grad")
    return out


# ------------------------------------------------------------------------------------------------
# RMSNorm
# ------------------------------------------------------------------------------------------------
def rmsnorm_fwd(x2: torch.Tensor, w: torch.Tensor, eps: float, want_rstd: bool = True):
    _cuda(x2, w)
    n, c = x2.shape
    if x2.stride(-1) != 1:
        x2 = x2.contiguous()
    y = torch.empty((n, c), dtype=torch.float32, device=x2.device)
    rstd = torch.empty(n, dtype=torch.float32, device=x2.device) if want_rstd else None
    rc = _lib.lib().decik_rmsnorm_fwd(_p(x2), _p(w.contiguous()), _dt(w), _p(y), _p(rstd), n, c,
                                      x2.stride(0), y.stride(0), float(eps), _stream(x2))
    _lib.check(rc, "rmsnorm_fwd")
    return y, rstd


def rmsnorm_bwd(dy2: torch.Tensor, x2: torch.Tensor, w: torch.Tensor, rstd: torch.Tensor,
                addend: torch.Tensor | None = None):
    """The RMSNorm input gradient [n, c] fp32; with ``addend`` (fp32 [n, c]) it is added in the same
    pass (decik_rmsnorm_bwd_add): addend + norm_bwd, one rounding, as autograd's sum."""
    _cuda(dy2, x2, w, rstd, addend)
    n, c = x2.shape
    dy2 = dy2.contiguous()
    x2 = x2.contiguous()
    dx = torch.empty((n, c), dtype=torch.float32, device=x2.device)
    if addend is None:
        rc = _lib.lib().decik_rmsnorm_bwd(_p(dy2), _p(x2), _p(w.contiguous()), _dt(w), _p(rstd), _p(dx), n, c,
                                          _stream(x2))
    else:
        a2 = addend.reshape(n, c).contiguous().float()
        rc = _lib.lib().decik_rmsnorm_bwd_add(_p(dy2), _p(x2), _p(w.contiguous()), _dt(w), _p(rstd), _p(a2), _p(dx),
                                              n, c, _stream(x2))
    _lib.check(rc, "rmsnorm_bwd")
    return dx


def add_rmsnorm_fwd(residual: torch.Tensor, delta: torch.Tensor, w: torch.Tensor, eps: float, y16: bool = False):
    """h = residual + delta (fp32), y = RMSNorm(h) * w, rstd [rows]; residual fp32 and delta
    fp32 / fp16 / bf16 of the same shape (last dim the normalised one). y is fp32, or with ``y16``
    in delta's 16-bit dtype (decik_add_rmsnorm_fwd16: the fp32 y rounded, never written)."""
    _cuda(residual, delta, w)
    if residual.dtype != torch.float32 or residual.shape != delta.shape:
        raise RuntimeError("decik_b200 add_rmsnorm_fwd: residual fp32 and delta of the same shape")
    n_cols = residual.shape[-1]
    r2 = residual.reshape(-1, n_cols).contiguous()
    d2 = delta.reshape(-1, n_cols).contiguous()
    if y16 and d2.dtype not in (torch.float16, torch.bfloat16):
        raise RuntimeError("decik_b200 add_rmsnorm_fwd: a 16-bit y needs a 16-bit delta")
    # h and y in the caller's shape (not views: the decoder layer's stream h may be updated in place)
    h = torch.empty(residual.shape, dtype=torch.float32, device=r2.device)
    y = torch.empty(residual.shape, dtype=d2.dtype if y16 else torch.float32, device=r2.device)
    rstd = torch.empty(r2.shape[0], dtype=torch.float32, device=r2.device)
    fn = _lib.lib().decik_add_rmsnorm_fwd16 if y16 else _lib.lib().decik_add_rmsnorm_fwd
    with _timed("add_rmsnorm_fwd", 1):
        rc = fn(_p(r2), _p(d2), _dt(d2), _p(w.contiguous()), _dt(w), _p(h), _p(y), _p(rstd), r2.shape[0], n_cols,
                float(eps), _stream(r2))
    _lib.check(rc, "add_rmsnorm_fwd")
    return h, y, rstd


def add_rmsnorm_bwd(dy, grad_h, residual, delta, w, rstd, want_dx16: bool = True):
    """(dx fp32, dx in delta's dtype or None): dx = grad_h + RMSNorm backward of dy at
    h = residual + delta (rebuilt, not stored); grad_h may be None. dy fp32, or in delta's 16-bit
    dtype (the gradient of a 16-bit y: decik_add_rmsnorm_bwd16 reads it as it is)."""
    _cuda(dy, residual, delta, w, rstd)
    n_cols = residual.shape[-1]
    r2 = residual.reshape(-1, n_cols).contiguous()
    d2 = delta.reshape(-1, n_cols).contiguous()
    dy16 = dy.dtype == d2.dtype and dy.dtype in (torch.float16, torch.bfloat16)
    g2 = dy.reshape(-1, n_cols).contiguous()
    if not dy16:
        g2 = g2.float()
    gh = None if grad_h is None else grad_h.reshape(-1, n_cols).contiguous().float()
    dx = torch.empty_like(r2)
    dx16 = torch.empty_like(d2) if want_dx16 else None
    fn = _lib.lib().decik_add_rmsnorm_bwd16 if dy16 else _lib.lib().decik_add_rmsnorm_bwd
    with _timed("add_rmsnorm_bwd", 1):
        rc = fn(_p(g2), _p(gh), _p(r2), _p(d2), _dt(d2), _p(w.contiguous()), _dt(w), _p(rstd), _p(dx), _p(dx16),
                r2.shape[0], n_cols, _stream(r2))
    _lib.check(rc, "add_rmsnorm_bwd")
    return dx.view(residual.shape), None if dx16 is None else dx16.view(delta.shape)


def swiglu_fwd(gu: torch.Tensor, inter: int, out: torch.Tensor | None = None) -> torch.Tensor:
    """silu(gate) * up of gu = [gate | up] ([T, 2 * inter], 16-bit, rows 16-byte aligned) -> [T, inter]."""
    _cuda(gu)
    if gu.dim() != 2 or gu.stride(1) != 1 or gu.shape[1] < 2 * inter:
        raise RuntimeError("decik_b200 swiglu_fwd: gu must be [T, >= 2 * inter] with unit column stride")
    if out is None:
        out = torch.empty((gu.shape[0], inter), dtype=gu.dtype, device=gu.device)
    with _timed("swiglu_fwd", 1):
        rc = _lib.lib().decik_swiglu_fwd(_p(gu), gu.stride(0), _p(out), out.stride(0), gu.shape[0], inter, _dt(gu),
                                         _stream(gu))
    _lib.check(rc, "swiglu_fwd")
    return out


def swiglu_bwd(grad: torch.Tensor, gu: torch.Tensor, inter: int, dgu: torch.Tensor | None = None) -> torch.Tensor:
    """[dgate | dup] ([T, 2 * inter], laid out like gu) from grad [T, inter] and gu."""
    _cuda(grad, gu)
    if grad.stride(1) != 1:
        grad = grad.contiguous()
    if dgu is None:
        dgu = torch.empty((gu.shape[0], 2 * inter), dtype=gu.dtype, device=gu.device)
    with _timed("swiglu_bwd", 1):
        rc = _lib.lib().decik_swiglu_bwd(_p(grad), grad.stride(0), _p(gu), gu.stride(0), _p(dgu), dgu.stride(0),
                                         gu.shape[0], inter, _dt(gu), _stream(gu))
    _lib.check(rc, "swiglu_bwd")
    return dgu


def head_stats(logits: torch.Tensor, target: torch.Tensor):
    """(lse, entropy, token_loss, hit) of each row of 16-bit logits [rows, vocab]; labelled rows'
    logits are replaced by softmax - onehot (in place)."""
    _cuda(logits, target)
    if logits.dim() != 2 or logits.stride(1) != 1:
        raise RuntimeError("decik_b200 head_stats: logits must be [rows, vocab] with unit column stride")
    n = logits.shape[0]
    target = target.to(torch.int64).contiguous()
    f = lambda: torch.empty(n, dtype=torch.float32, device=logits.device)
    lse, entropy, loss = f(), f(), f()
    hit = torch.empty(n, dtype=torch.int32, device=logits.device)
    with _timed("head_stats", 1):
        rc = _lib.lib().decik_head_stats(_p(logits), logits.stride(0), _p(target), _p(lse), _p(entropy), _p(loss),
                                         _p(hit), n, logits.shape[1], _dt(logits), _stream(logits))
    _lib.check(rc, "head_stats")
    return lse, entropy, loss, hit


# ------------------------------------------------------------------------------------------------
# varlen attention
# ------------------------------------------------------------------------------------------------
def _t3(t: torch.Tensor) -> Tensor3:
    """A [T, H, D] view (last dim contiguous) -> decik_tensor3."""
    if t.dim() != 3 or t.stride(2) != 1:
        raise RuntimeError("decik_b200: attention tensors must be [T, H, D] views with D contiguous")
    return Tensor3(t.data_ptr(), t.stride(0), t.stride(1))


def varlen_attn_fwd(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, cu_seqlens: torch.Tensor,
                    max_len: int, scale: float, out: torch.Tensor | None = None):
    """q [T, Hq, D], k/v [T, Hk, D] views -> out [T, Hq, D] (contiguous unless given), lse fp32 [Hq, T]."""
    _cuda(q, k, v, cu_seqlens)
    T, Hq, D = q.shape
    Hk = k.shape[1]
    if cu_seqlens.dtype != torch.int32:
        raise RuntimeError("decik_b200 varlen_attn_fwd: cu_seqlens must be int32")
    if out is None:
        out = torch.empty((T, Hq, D), dtype=q.dtype, device=q.device)
    lse = torch.empty((Hq, T), dtype=torch.float32, device=q.device)
    with _timed("varlen_attn_fwd", 1):
        rc = _lib.lib().decik_varlen_attn_fwd(_t3(q), _t3(k), _t3(v), _t3(out), _p(lse), _p(cu_seqlens),
                                              cu_seqlens.numel() - 1, int(max_len), T, Hq, Hk, D,
                                              float(scale), _dt(q), _stream(q))
    _lib.check(rc, "varlen_attn_fwd")
    return out, lse


def varlen_attn_bwd_workspace(n_tok: int, n_heads: int, head_dim: int) -> int:
    return int(_lib.lib().decik_varlen_attn_bwd_workspace(n_tok, n_heads, head_dim))


def varlen_attn_bwd(dout, q, k, v, out, lse, cu_seqlens, max_len: int, scale: float,
                    dq=None, dk=None, dv=None, workspace: torch.Tensor | None = None):
    """Returns (dq, dk, dv) shaped and strided like q, k, v (dk/dv GQA-summed)."""
    _cuda(dout, q, k, v, out, lse, cu_seqlens)
    T, Hq, D = q.shape
    Hk = k.shape[1]
    dq = torch.empty_like(q) if dq is None else dq
    dk = torch.empty_like(k) if dk is None else dk
    dv = torch.empty_like(v) if dv is None else dv
    nbytes = varlen_attn_bwd_workspace(T, Hq, D)
    if workspace is None or workspace.numel() < nbytes:
        workspace = torch.empty(nbytes, dtype=torch.uint8, device=q.device)
    with _timed("varlen_attn_bwd", 3):
        rc = _lib.lib().decik_varlen_attn_bwd(_t3(dout), _t3(q), _t3(k), _t3(v), _t3(out), _p(lse), _t3(dq),
                                              _t3(dk), _t3(dv), _p(cu_seqlens), cu_seqlens.numel() - 1,
                                              int(max_len), T, Hq, Hk, D, float(scale), _dt(q),
                                              _p(workspace), _stream(q))
    _lib.check(rc, "varlen_attn_bwd")
    return dq, dk, dv


# ------------------------------------------------------------------------------------------------
# projection epilogues (around one fused q|k|v|LoRA-down GEMM)
# ------------------------------------------------------------------------------------------------
LORA_RANK = 16


def _t3any(t: torch.Tensor) -> Tensor3:
    """Any 3-D [T, H, D] view with D contiguous (strides in elements)."""
    if t.dim() != 3 or t.stride(2) != 1:
        raise RuntimeError("decik_b200: expected a [T, H, D] view with D contiguous")
    return Tensor3(t.data_ptr(), t.stride(0), t.stride(1))


def lora_pack(a_q: torch.Tensor, a_v: torch.Tensor, b_q: torch.Tensor, b_v: torch.Tensor, dtype: torch.dtype,
              a_out: torch.Tensor | None = None) -> torch.Tensor:
    """One step's LoRA operands: A_q, A_v rounded to ``dtype`` into the rows of ``a_out`` [32, hidden]
    (a row slice of the projection weight; optional) and the lora_B fragments both projection
    epilogues read (a uint8 buffer; keep it from forward to backward)."""
    _cuda(a_q, a_v, b_q, b_v, a_out)
    for t in (a_q, a_v, b_q, b_v):
        if t.dtype != torch.float32 or not t.is_contiguous():
            raise RuntimeError("decik_b200 lora_pack: LoRA weights must be contiguous fp32")
    rank, hidden = a_q.shape
    D = 128
    n_heads, n_kv = b_q.shape[0] // D, b_v.shape[0] // D
    frag = torch.empty(int(_lib.lib().decik_lora_frag_bytes(n_heads, n_kv)), dtype=torch.uint8, device=a_q.device)
    if a_out is not None and (a_out.dtype != dtype or a_out.stride(1) != 1 or tuple(a_out.shape) != (2 * rank, hidden)):
        raise RuntimeError("decik_b200 lora_pack: a_out must be [2r, hidden] rows of dtype")
    with _timed("lora_pack", 1):
        rc = _lib.lib().decik_lora_pack(_p(a_q), _p(a_v), _p(a_out), a_out.stride(0) if a_out is not None else 0,
                                        hidden, _p(b_q), _p(b_v), _p(frag), n_heads, n_kv, D, rank,
                                        _DT[dtype], _stream(a_q))
    _lib.check(rc, "lora_pack")
    return frag


def qkv_epilogue_fwd(y: torch.Tensor, u: torch.Tensor | None, frag: torch.Tensor | None, scaling: float,
                     cos: torch.Tensor, sin: torch.Tensor, n_heads: int, n_kv: int, want_u: bool = False):
    """From y [T, >= (Hq+2Hk)*D] (q_base | k | v_base) and u [T, >= 32] (u_q | u_v): q [Hq, T, D]
    and k [Hk, T, D] head-major with RoPE, v [T, Hk, D], and (want_u) a compact u copy [T, 32]."""
    _cuda(y, u, frag, cos, sin)
    T = y.shape[0]
    D = cos.shape[-1]
    if y.stride(1) != 1 or (u is not None and u.stride(1) != 1):
        raise RuntimeError("decik_b200 qkv_epilogue_fwd: y and u need contiguous rows")
    q = torch.empty((n_heads, T, D), dtype=y.dtype, device=y.device)
    k = torch.empty((n_kv, T, D), dtype=y.dtype, device=y.device)
    v = torch.empty((T, n_kv, D), dtype=y.dtype, device=y.device)
    lora = frag is not None
    u_out = torch.empty((T, 2 * LORA_RANK), dtype=y.dtype, device=y.device) if (lora and want_u) else None
    with _timed("qkv_epilogue_fwd", 1):
        rc = _lib.lib().decik_qkv_epilogue_fwd(
            _p(y), y.stride(0), _p(u) if lora else None, u.stride(0) if lora else 0, _p(frag),
            float(scaling), _p(cos), _p(sin), _t3any(q.transpose(0, 1)), _t3any(k.transpose(0, 1)), _t3any(v),
            _p(u_out), T, n_heads, n_kv, D, _dt(y), _stream(y))
    _lib.check(rc, "qkv_epilogue_fwd")
    return q, k, v, u_out


def lora_b_ext(b_q: torch.Tensor | None, b_v: torch.Tensor | None, scaling: float, bias: torch.Tensor,
               dtype: torch.dtype, n_heads: int, n_kv: int) -> torch.Tensor:
    """The B operand of the projection GEMM's extra K block [(Hq+2Hk)*D, 64] (decik_lora_b_ext):
    scaling . B_q rows against u_q (columns 0..15), scaling . B_v rows against u_v (16..31), the
    bias in column 32 of every row, zero elsewhere. b_q / b_v None: no LoRA."""
    _cuda(b_q, b_v, bias)
    D = 128
    n_proj = (n_heads + 2 * n_kv) * D
    bias16 = bias[:n_proj].to(dtype).contiguous()
    out = torch.empty((n_proj, 4 * LORA_RANK), dtype=dtype, device=bias.device)
    with _timed("lora_b_ext", 1):
        rc = _lib.lib().decik_lora_b_ext(_p(b_q.contiguous()) if b_q is not None else None,
                                         _p(b_v.contiguous()) if b_v is not None else None, float(scaling),
                                         _p(bias16), _p(out), n_heads, n_kv, _DT[dtype], _stream(bias))
    _lib.check(rc, "lora_b_ext")
    return out


def qkv_proj_fwd(x: torch.Tensor, w_cat: torch.Tensor, ext_b: torch.Tensor, lora: bool, cos: torch.Tensor,
                 sin: torch.Tensor, n_heads: int, n_kv: int, norm: tuple | None = None):
    """The block's forward projections on tcgen05 (decik_qkv_proj_fwd): from x fp32 [T, H], w_cat
    [(Hq+2Hk)*D (+ 32 with ``lora``), H] (W_q, W_k, W_v rows, then A_q, A_v as lora_pack wrote them)
    and the extra K block's B operand (lora_b_ext: scaled lora_B and the bias) returns x16 [T, H],
    u [T, 64] (u_q | u_v | 1 | zeros), q [Hq, T, D] and k [Hk, T, D] head-major with RoPE,
    v [T, Hk, D]. With ``norm`` = (weight, eps) x is the decoder layer's input h and the input
    RMSNorm runs inside the first kernel (decik_qkv_proj_norm_fwd); then rstd [T] comes back as a
    sixth value."""
    _cuda(x, w_cat, ext_b, cos, sin)
    T, H = x.shape
    D = cos.shape[-1]
    dt, dev = w_cat.dtype, x.device
    if x.dtype != torch.float32 or x.stride(1) != 1 or w_cat.stride(1) != 1:
        raise RuntimeError("decik_b200 qkv_proj_fwd: x fp32 and w_cat with contiguous rows")
    x16 = torch.empty((T, H), dtype=dt, device=dev)
    u = torch.empty((T, 4 * LORA_RANK), dtype=dt, device=dev)
    q = torch.empty((n_heads, T, D), dtype=dt, device=dev)
    k = torch.empty((n_kv, T, D), dtype=dt, device=dev)
    v = torch.empty((T, n_kv, D), dtype=dt, device=dev)
    outs = (_t3any(q.transpose(0, 1)), _t3any(k.transpose(0, 1)), _t3any(v), _p(x16), x16.stride(0), _p(u), T, H,
            n_heads, n_kv, D, _dt(w_cat), _stream(x))
    tail = (_p(w_cat), w_cat.stride(0), _p(ext_b), 1 if lora else 0, _p(cos.contiguous()), _p(sin.contiguous()))
    if norm is None:
        with _timed("qkv_proj_fwd", 2):
            rc = _lib.lib().decik_qkv_proj_fwd(_p(x), x.stride(0), *tail, *outs)
        _lib.check(rc, "qkv_proj_fwd")
        return x16, u, q, k, v
    w, eps = norm
    _cuda(w)
    w = w.contiguous()
    rstd = torch.empty(T, dtype=torch.float32, device=dev)
    with _timed("qkv_proj_fwd", 2):
        rc = _lib.lib().decik_qkv_proj_norm_fwd(_p(x), x.stride(0), _p(w), _dt(w), float(eps), _p(rstd), *tail,
                                                *outs)
    _lib.check(rc, "qkv_proj_norm_fwd")
    return x16, u, q, k, v, rstd


def transpose16(src: torch.Tensor) -> torch.Tensor:
    """src [R, C] (16-bit, contiguous rows) -> a new [C, R] tensor (decik_transpose16)."""
    _cuda(src)
    R, C = src.shape
    if src.stride(1) != 1:
        src = src.contiguous()
    dst = torch.empty((C, R), dtype=src.dtype, device=src.device)
    with _timed("transpose16", 1):
        rc = _lib.lib().decik_transpose16(_p(src), src.stride(0), _p(dst), dst.stride(0), R, C, _stream(src))
    _lib.check(rc, "transpose16")
    return dst


def proj_dx(dy: torch.Tensor, w_t: torch.Tensor, k_cols: int | None = None) -> torch.Tensor:
    """dx = dy[:, :K] . w_t[:, :K]^T in fp32 [T, H] on tcgen05 CTA pairs (decik_proj_dx); w_t [H, >= K]
    is the transposed weight (transpose16 of a [K, H] weight)."""
    _cuda(dy, w_t)
    T = dy.shape[0]
    H = w_t.shape[0]
    K = int(k_cols if k_cols is not None else w_t.shape[1])
    if dy.stride(1) != 1 or w_t.stride(1) != 1:
        raise RuntimeError("decik_b200 proj_dx: dy and w_t need contiguous rows")
    dx = torch.empty((T, H), dtype=torch.float32, device=dy.device)
    with _timed("proj_dx", 1):
        rc = _lib.lib().decik_proj_dx(_p(dy), dy.stride(0), K, _p(w_t), w_t.stride(0), _p(dx), dx.stride(0), T, H,
                                      _dt(dy), _stream(dy))
    _lib.check(rc, "proj_dx")
    return dx


def gemm16(a: torch.Tensor, b: torch.Tensor, b_mn: bool, out: torch.Tensor | None = None) -> torch.Tensor:
    """a [M, K] . b^T (b [N, K], ``b_mn`` False) or a . b (b [K, N], ``b_mn`` True) in a's 16-bit dtype
    on tcgen05 CTA pairs (decik_gemm16)."""
    _cuda(a, b, out)
    M, K = a.shape
    N = b.shape[1] if b_mn else b.shape[0]
    if a.stride(1) != 1 or b.stride(1) != 1:
        raise RuntimeError("decik_b200 gemm16: operands need contiguous rows")
    if out is None:
        out = torch.empty((M, N), dtype=a.dtype, device=a.device)
    with _timed("gemm16", 1):
        rc = _lib.lib().decik_gemm16(_p(a), a.stride(0), _p(b), b.stride(0), 1 if b_mn else 0, _p(out), out.stride(0),
                                     M, N, K, _dt(a), _stream(a))
    _lib.check(rc, "gemm16")
    return out


def mlp_gate_up(x16: torch.Tensor, w_gu: torch.Tensor):
    """(gu [T, 2 inter], h [T, inter]) = (x16 . w_gu^T, SwiGLU of it) in one tcgen05 GEMM
    (decik_mlp_gate_up)."""
    _cuda(x16, w_gu)
    T, H = x16.shape
    inter = w_gu.shape[0] // 2
    gu = torch.empty((T, 2 * inter), dtype=x16.dtype, device=x16.device)
    h = torch.empty((T, inter), dtype=x16.dtype, device=x16.device)
    with _timed("mlp_gate_up", 1):
        rc = _lib.lib().decik_mlp_gate_up(_p(x16), x16.stride(0), _p(w_gu), w_gu.stride(0), _p(gu), gu.stride(0), _p(h),
                                          h.stride(0), T, H, inter, _dt(x16), _stream(x16))
    _lib.check(rc, "mlp_gate_up")
    return gu, h


def mlp_down_grad(grad16: torch.Tensor, w_down: torch.Tensor, gu: torch.Tensor) -> torch.Tensor:
    """[dgate | dup] [T, 2 inter] of SwiGLU for grad_hidden = grad16 . w_down, computed in the
    GEMM's epilogue (decik_mlp_down_grad)."""
    _cuda(grad16, w_down, gu)
    T, H = grad16.shape
    inter = w_down.shape[1]
    dgu = torch.empty((T, 2 * inter), dtype=grad16.dtype, device=grad16.device)
    with _timed("mlp_down_grad", 1):
        rc = _lib.lib().decik_mlp_down_grad(_p(grad16), grad16.stride(0), _p(w_down), w_down.stride(0), _p(gu),
                                            gu.stride(0), _p(dgu), dgu.stride(0), T, H, inter, _dt(grad16),
                                            _stream(grad16))
    _lib.check(rc, "mlp_down_grad")
    return dgu


def lora_grads(dy: torch.Tensor, x16: torch.Tensor, u: torch.Tensor, scaling: float, n_heads: int, n_kv: int):
    """(dA [32, H], dB [(Hq+Hk)*D, 16]) fp32 of the fused block (decik_lora_grads): dA = du^T x16 with
    du = dy's last 32 columns; dB = scaling g^T u over dy's q columns (u_q) and v columns (u_v)."""
    _cuda(dy, x16, u)
    T, H = x16.shape
    D = 128
    da = torch.empty((2 * LORA_RANK, H), dtype=torch.float32, device=dy.device)
    db = torch.empty(((n_heads + n_kv) * D, LORA_RANK), dtype=torch.float32, device=dy.device)
    with _timed("lora_grads", 1):
        if u.stride(1) != 1:
            u = u.contiguous()
        rc = _lib.lib().decik_lora_grads(_p(dy), dy.stride(0), _p(x16), x16.stride(0), _p(u), u.stride(0), _p(da),
                                         _p(db), float(scaling), T, H, n_heads, n_kv, _dt(dy), _stream(dy))
    _lib.check(rc, "lora_grads")
    return da, db


def qkv_epilogue_bwd(grad_q: torch.Tensor, grad_k: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor,
                     frag: torch.Tensor | None, scaling: float, dy: torch.Tensor, n_heads: int,
                     n_kv: int) -> torch.Tensor:
    """grad_q/grad_k: [T, H, D] views. dy [T, ld] must hold dv in its v columns; fills the rest."""
    _cuda(grad_q, grad_k, cos, sin, frag, dy)
    T = dy.shape[0]
    D = cos.shape[-1]
    if dy.stride(1) != 1:
        raise RuntimeError("decik_b200 qkv_epilogue_bwd: dy needs contiguous rows")
    with _timed("qkv_epilogue_bwd", 1):
        rc = _lib.lib().decik_qkv_epilogue_bwd(
            _t3any(grad_q), _t3any(grad_k), _p(cos), _p(sin), _p(frag), float(scaling), _p(dy), dy.stride(0),
            T, n_heads, n_kv, D, _dt(dy), _stream(dy))
    _lib.check(rc, "qkv_epilogue_bwd")
    return dy


def attn_qkv_bwd(dout, q, k, v, out, lse, cu_seqlens, max_len: int, scale: float, cos: torch.Tensor,
                 sin: torch.Tensor, frag: torch.Tensor | None, scaling: float, dy: torch.Tensor,
                 workspace: torch.Tensor | None = None) -> torch.Tensor:
    """The attention backward and the projection epilogue backward in one call
    (decik_attn_qkv_bwd): fills dy [T, ld] (dq, dk after RoPE^T, dv, du) from the attention's
    fp32 accumulators. q, k, v, out, dout: [T, H, D] views as for varlen_attn_bwd."""
    _cuda(dout, q, k, v, out, lse, cu_seqlens, cos, sin, frag, dy)
    T, Hq, D = q.shape
    Hk = k.shape[1]
    if dy.stride(1) != 1:
        raise RuntimeError("decik_b200 attn_qkv_bwd: dy needs contiguous rows")
    nbytes = int(_lib.lib().decik_attn_qkv_bwd_workspace(T, Hq, Hk, D))
    if workspace is None or workspace.numel() < nbytes:
        workspace = torch.empty(nbytes, dtype=torch.uint8, device=q.device)
    lib = _lib.lib()
    args = (_t3(dout), _t3(q), _t3(k), _t3(v), _t3(out), _p(lse), _p(cu_seqlens), cu_seqlens.numel() - 1,
            int(max_len), T, Hq, Hk, D, float(scale), _p(cos), _p(sin), _p(frag), float(scaling), _p(dy),
            dy.stride(0), _dt(q), _p(workspace), _stream(q))
    if _timer is None or (_timer.names is not None and "varlen_attn_bwd" not in _timer.names):
        rc = lib.decik_attn_qkv_bwd(*args)
        if _timer is not None:
            _timer.launches += 3
    else:  # the two stages timed apart: an event recorded between them by the library
        a, mid, b = (torch.cuda.Event(enable_timing=True) for _ in range(3))
        mid.record()  # creates the event; the library records it again between the stages
        handles = (ctypes.c_void_p * 1)(mid.cuda_event)
        lib.decik_set_stage_events(handles, 1)
        a.record()
        rc = lib.decik_attn_qkv_bwd(*args)
        b.record()
        lib.decik_set_stage_events(None, 0)
        _timer.events.append(("varlen_attn_bwd", a, mid))
        _timer.events.append(("qkv_epilogue_bwd", mid, b))
        _timer.launches += 3
    _lib.check(rc, "attn_qkv_bwd")
    return dy


# ------------------------------------------------------------------------------------------------
# instrumentation (off unless a caller installs a recorder): CUDA events around named ops on the
# stream they launch on, and a count of this library's kernel launches.
# ------------------------------------------------------------------------------------------------
class OpTimer:
    """Records (name, start event, end event) around ops while installed with ``install``, and
    counts this library's kernel launches. With ``names`` only those ops get events (fewer host-side
    event records, so the timed GPU work is not starved by the instrumentation)."""

    def __init__(self, names=None):
        self.events = []
        self.launches = 0
        self.names = None if names is None else set(names)

    def elapsed_ms(self) -> dict:
        torch.cuda.synchronize()
        out: dict = {}
        for name, a, b in self.events:
            out.setdefault(name, []).append(a.elapsed_time(b))
        return out


_timer: OpTimer | None = None


def install_timer(t: OpTimer | None) -> None:
    global _timer
    _timer = t


class _timed:
    def __init__(self, name: str, launches: int):
        self.name, self.launches = name, launches

    def __enter__(self):
        self.on = _timer is not None and (_timer.names is None or self.name in _timer.names)
        if self.on:
            self.a = torch.cuda.Event(enable_timing=True)
            self.a.record()
        return self

    def __exit__(self, *exc):
        if _timer is not None:
            if self.on:
                b = torch.cuda.Event(enable_timing=True)
                b.record()
                _timer.events.append((self.name, self.a, b))
            _timer.launches += self.launches
        return False
