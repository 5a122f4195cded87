/*
 * decik_b200: C ABI of the B200 (sm_100a) kernels for the attention block of decik's NF4 QLoRA
 * training step.
 *
 * Every entry point takes plain device pointers, sizes and a CUDA stream (cudaStream_t passed as
 * void*, NULL = the legacy default stream), enqueues its kernels on that stream and returns a
 * status code. Nothing here allocates device memory: outputs and workspaces are the caller's.
 * On a non-zero status, decik_last_error() returns a message for the calling thread.
 *
 * Layout conventions: "token-major" [T, H*D] means row t holds all heads of token t;
 * "head-major" [H, T, D] means head h is one contiguous [T, D] block. Strides are in ELEMENTS.
 * dtype codes: DECIK_F16, DECIK_BF16, DECIK_F32.
 *
 * Reference citations are paths inside the tokha-t/decik repository.
 */
#ifndef DECIK_B200_H
#define DECIK_B200_H

#include <stdint.h>

#if defined(__GNUC__)
#define DECIK_API __attribute__((visibility("default")))
#else
#define DECIK_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define DECIK_OK 0
#define DECIK_ERR_INVALID 1      /* bad argument: size, alignment, dtype, null pointer */
#define DECIK_ERR_CUDA 2         /* a CUDA runtime error while launching */
#define DECIK_ERR_UNSUPPORTED 3  /* a shape or option this build has no kernel for */

#define DECIK_F16 0
#define DECIK_BF16 1
#define DECIK_F32 2

/* Message of the last failed call on this thread ("" if none). */
DECIK_API const char* decik_last_error(void);

/* ABI version of this library (bumped on any signature change). */
DECIK_API int decik_abi_version(void);

/* Error code recorded on the current device by a kernel whose bounded wait gave up (0 = none;
 * -1 if it could not be read). Synchronizes with the device. reset != 0 clears it. Kernels that
 * wait on mbarriers never spin forever: they record a code here and return. */
DECIK_API int decik_kernel_error(int reset);

/* Failure-path self-test (no counterpart in the reference, whose Triton kernels have no bounded
 * waits): launches one warp that holds 32 TMEM columns and waits on an mbarrier nothing arrives
 * on, giving up after limit_cycles (at most 4e9) exactly as the attention kernels give up after
 * theirs. It then records 901 in the error word read by decik_kernel_error(), frees its TMEM and
 * returns; *done (device int) becomes 2 when the wait ran out (1 if it had completed). */
DECIK_API int decik_wait_limit_selftest(long long limit_cycles, int* done, void* stream);

/* ---------------------------------------------------------------------------------------------
 * Padding-free packing of a right-padded batch, on the device.
 * Replaces plan() / Packing of solution/varlen.py:191-226 and :23-40 (mask.sum, the right-padding
 * torch.equal check, lengths.tolist(), mask.nonzero(), the positions and cu_seqlens), which read
 * the device three times; here the caller reads only `summary` (one copy of 4 + batch int32).
 *   mask       [batch, seq], contiguous; mask_dtype 0 = int64, 1 = int32, 2 = uint8 / bool
 *   input_ids  int64 [batch, seq] contiguous, or NULL (then ids_out must be NULL)
 *   cu_seqlens int32 [batch + 1]: row starts in the packed sequence, then T
 *   index      int64 [>= T]: b * seq + s of each real token, row-major (capacity batch * seq)
 *   positions  int64 [>= T]: s (the token's position in its row)
 *   ids_out    int64 [>= T]: input_ids at index, or NULL
 *   summary    int32 [4 + batch]: T, max row length, 1 if every row is right-padded (else 0: the
 *              other outputs are then meaningless), min row length, then the row lengths.
 * batch <= 8192, seq <= 2^30, batch * seq < 2^31. One kernel on `stream`. */
DECIK_API int decik_pack_rows(const void* mask, int mask_dtype, const int64_t* input_ids, int64_t batch,
                              int64_t seq, int32_t* cu_seqlens, int64_t* index, int64_t* positions,
                              int64_t* ids_out, int32_t* summary, void* stream);

/* ---------------------------------------------------------------------------------------------
 * NF4 double-quant dequant.
 * Replaces solution/nf4.py:66-85 (dequantize_nf4) and its kernel skc_nf4_dequant_kernel
 * (solution/nf4.py:28-49). Bit-exact: for packed byte i, the high nibble is weight 2i and the low
 * nibble weight 2i+1; block = (2i) / blocksize; with nested=1 the block scale is
 * code2[absmax_u8[block]] * absmax2[block / blocksize2] then + *offset (two fp32 roundings, no
 * FMA); each weight is code[nibble] * scale in fp32, rounded to out_dtype (F16, BF16 or F32).
 *   packed  uint8 [n_bytes]                 (row-major [N_out, K_in] weights, 2 per byte)
 *   absmax  uint8 [n_blocks] if nested, else fp32 [n_blocks]
 *   absmax2 fp32 [ceil(n_blocks / blocksize2)] (nested only, else may be NULL)
 *   code2   fp32 [256] (nested only), offset fp32 [1] device scalar (nested only)
 *   code    fp32 [16]
 *   out     [2 * n_bytes] of out_dtype
 * ------------------------------------------------------------------------------------------- */
DECIK_API int decik_nf4_dequant(const uint8_t* packed, const void* absmax, const float* absmax2,
                      const float* code2, const float* offset, const float* code, void* out,
                      int64_t n_bytes, int nested, int blocksize, int blocksize2, int out_dtype,
                      void* stream);

/* Several NF4 weights in one launch (the block's W_q, W_k, W_v into the row slices of one matrix):
 * each job has decik_nf4_dequant's arguments; all share the output dtype. Jobs whose form differs
 * (nested or not, 16-byte aligned or not) go to separate launches. Same results as one
 * decik_nf4_dequant call per job. */
typedef struct {
  const uint8_t* packed;
  const void* absmax;
  const float* absmax2;
  const float* code2;
  const float* offset;
  const float* code;
  void* out;
  int64_t n_bytes;
  int nested;
  int blocksize;
  int blocksize2;
} decik_nf4_job;
DECIK_API int decik_nf4_dequant_batch(const decik_nf4_job* jobs, int n_jobs, int out_dtype, void* stream);

/* ---------------------------------------------------------------------------------------------
 * LoRA add + RoPE + cast, forward. Replaces FusedQKRope.forward / skc_rope_fwd_kernel
 * (solution/attn.py:28-61, :97-111). Bit-exact (each fp32 product and sum rounded, no FMA):
 *   q = f32(q_base) + f32(q_lora);  q_out = q * cos + rotate_half(q) * sin
 *   k_out = k * cos + rotate_half(k) * sin
 *   q_base, q_lora  [T, n_heads*head_dim] token-major, dtype (q_lora may be NULL: no LoRA term)
 *   k               [T, n_kv*head_dim] token-major, dtype
 *   cos, sin        fp32 [T, head_dim]
 *   q_out           [n_heads, T, head_dim] head-major, dtype;  k_out [n_kv, T, head_dim]
 * dtype: DECIK_F16 or DECIK_BF16. head_dim % 16 == 0.
 * ------------------------------------------------------------------------------------------- */
DECIK_API int decik_rope_fwd(const void* q_base, const void* q_lora, const void* k, const float* cos,
                   const float* sin, void* q_out, void* k_out, int64_t n_tok, int n_heads,
                   int n_kv, int head_dim, int dtype, void* stream);

/* RoPE backward. Replaces FusedQKRope.backward / skc_rope_bwd_kernel (solution/attn.py:64-90,
 * :113-126): dq[d] = g[d]*cos[d] + (d < D/2 ? g[d+D/2]*sin[d+D/2] : -(g[d-D/2]*sin[d-D/2])).
 *   grad_q [n_heads, T, head_dim] head-major, grad_k [n_kv, T, head_dim]  (dtype)
 *   dq [T, n_heads*head_dim], dk [T, n_kv*head_dim] token-major (dtype)                        */
DECIK_API int decik_rope_bwd(const void* grad_q, const void* grad_k, const float* cos, const float* sin,
                   void* dq, void* dk, int64_t n_tok, int n_heads, int n_kv, int head_dim,
                   int dtype, void* stream);

/* ---------------------------------------------------------------------------------------------
 * LoRA dropout helpers (p > 0 only).
 * decik_keep_pack replaces skc_keep_pack_kernel / pack_keep (solution/attn.py:130-144, :195-203):
 *   keep_q, keep_v bool (one byte 0/1) [n_rows, width] -> bits_q, bits_v uint8 [n_rows, width/8],
 *   bit j of byte c = keep[8c + j]. width % 8 == 0.
 * decik_lora_inputs replaces skc_lora_inputs_kernel / _lora_inputs (solution/attn.py:154-165,
 *   :183-192): xq = round(x * (keep_q * scale_q)), xv likewise; x fp32 [n_rows, width];
 *   scale_q, scale_v fp32 device scalars; xq, xv of out_dtype (F16/BF16).
 * decik_lora_input_grad replaces skc_lora_input_grad_kernel (solution/attn.py:169-180):
 *   out = (f32(g_q) * keep_q) * scale_q + (f32(g_v) * keep_v) * scale_v, fp32 [n_rows, width];
 *   g_q, g_v of in_dtype (F16/BF16).
 * ------------------------------------------------------------------------------------------- */
DECIK_API int decik_keep_pack(const uint8_t* keep_q, const uint8_t* keep_v, uint8_t* bits_q,
                    uint8_t* bits_v, int64_t n_rows, int width, void* stream);
DECIK_API int decik_lora_inputs(const float* x, const uint8_t* bits_q, const uint8_t* bits_v,
                      const float* scale_q, const float* scale_v, void* xq, void* xv,
                      int64_t n_rows, int width, int out_dtype, void* stream);
DECIK_API int decik_lora_input_grad(const void* g_q, const void* g_v, const uint8_t* bits_q,
                          const uint8_t* bits_v, float* out, int64_t n_rows, int width,
                          float scale_q, float scale_v, int in_dtype, void* stream);

/* [T, H, D] views: (pointer, token stride, head stride) in elements; D contiguous. */
typedef struct {
  const void* ptr;
  int64_t tok_stride;
  int64_t head_stride;
} decik_tensor3;

typedef struct {
  void* ptr;
  int64_t tok_stride;
  int64_t head_stride;
} decik_tensor3_mut;

/* ---------------------------------------------------------------------------------------------
 * Projection epilogues: the per-token work between one fused q|k|v|LoRA-down GEMM and attention.
 * No single reference counterpart: together they replace what the reference's patched
 * Qwen2Attention.forward (solution/attn.py:395-411) does between its three NF4Linear calls
 * (solution/nf4.py:93-97), LoRAPairFromNorm (solution/attn.py:217-228) and FusedQKRope
 * (solution/attn.py:97-111), and the matching backward (solution/attn.py:113-126, :235-273).
 * head_dim == 128, LoRA rank == 16, dtype F16 or BF16 (dt below).
 *
 * decik_lora_pack prepares one step's LoRA operands: A_q, A_v (fp32 [16, hidden]) rounded to dt
 * into rows 0..15 and 16..31 of a_out (row stride lda; may be NULL to skip), and the lora_B
 * weights b_q (fp32 [Hq*D, 16]) and b_v (fp32 [Hk*D, 16]) rounded to dt (as peft's b.to(dt)) in
 * the mma fragment order both epilogues read, into frag (decik_lora_frag_bytes() bytes, 16-byte
 * aligned). Keep frag from the forward for the backward of the same step.
 *
 * Forward: y [T, ldy] of dt holds q_base | k | v_base in columns [0, Hq*D), [Hq*D, (Hq+Hk)*D),
 * [(Hq+Hk)*D, (Hq+2Hk)*D) (biases already added); u [T, ldu] of dt holds u_q = x16 A16_q^T in
 * columns [0, 16) and u_v in [16, 32) (u may point into y). frag = NULL: no LoRA term.
 *   q = rope(f32(q_base) + f32(dt(dt(u_q B16_q^T) * scaling)))   (RoPE exactly as decik_rope_fwd)
 *   k = rope(k);   v = dt(f32(v_base) + f32(dt(dt(u_v B16_v^T) * scaling)))
 * q, k, v are [T, H, D] views (8-byte aligned, strides % 4 == 0; head-major q, k for attention).
 * y and cos/sin 16-byte aligned, ldy % 8 == 0. u_out (may be NULL): a compact [T, 32] copy of u.
 *
 * Backward: grad_q, grad_k are the gradients of q and k ([T, H, D] views, 16-byte aligned,
 * strides % 8 == 0). dy [T, ldy] of dt must hold dv in its v columns on entry; this writes
 * rope^T(grad_q) and rope^T(grad_k) (exactly as decik_rope_bwd) into the q and k columns and,
 * with frag, du_q = dt(dt(rope^T(grad_q) * scaling) B16_q) and du_v = dt(dt(dv * scaling) B16_v)
 * into columns [(Hq+2Hk)*D, +32). Then dX = dy . [W_q; W_k; W_v; A_q; A_v] is one GEMM.
 * ------------------------------------------------------------------------------------------- */
DECIK_API int64_t decik_lora_frag_bytes(int n_heads, int n_kv);
DECIK_API int decik_lora_pack(const float* a_q, const float* a_v, void* a_out, int64_t lda, int hidden,
                    const float* b_q, const float* b_v, void* frag, int n_heads, int n_kv,
                    int head_dim, int rank, int dtype, void* stream);
DECIK_API int decik_qkv_epilogue_fwd(const void* y, int64_t ldy, const void* u, int64_t ldu,
                           const void* frag, float scaling, const float* cos, const float* sin,
                           decik_tensor3_mut q, decik_tensor3_mut k, decik_tensor3_mut v, void* u_out,
                           int64_t n_tok, int n_heads, int n_kv, int head_dim, int dtype, void* stream);
DECIK_API int decik_qkv_epilogue_bwd(decik_tensor3 grad_q, decik_tensor3 grad_k, const float* cos,
                           const float* sin, const void* frag, float scaling, void* dy, int64_t ldy,
                           int64_t n_tok, int n_heads, int n_kv, int head_dim, int dtype, void* stream);

/* The fused block's backward in one call: decik_varlen_attn_bwd followed by
 * decik_qkv_epilogue_bwd, without the 16-bit dq / dk / dv in between. The epilogue reads the
 * attention backward's fp32 accumulators and rounds them exactly as decik_varlen_attn_bwd's cast
 * pass does (dq = bf16/fp16(scale * acc)), so the results are those of the two calls up to the
 * order of the attention's fp32 reduce-adds. q, k, v, dout, out, lse, cu_seqlens: as for
 * decik_varlen_attn_bwd; cos, sin, frag, scaling, dy, ldy: as for decik_qkv_epilogue_bwd, except
 * that dy's v columns are written here (dv) instead of being supplied. workspace:
 * decik_attn_qkv_bwd_workspace() bytes, 256-byte aligned. Replaces, for one fused node, the
 * backward of VarlenSDPA (solution/varlen.py:154-168), FusedQKRope (solution/attn.py:113-126) and
 * LoRAPairFromNorm's grad_u (solution/attn.py:250-253). */
/* Profiling hook: calls made on this host thread with n > 0 events set record them between their
 * stages, on their stream (decik_attn_qkv_bwd: events[0] after the attention backward, before the
 * projection epilogue). events are cudaEvent_t handles; n = 0 or NULL clears the hook. */
DECIK_API void decik_set_stage_events(void* const* events, int n);
DECIK_API int64_t decik_attn_qkv_bwd_workspace(int64_t n_tok, int n_heads, int n_kv, int head_dim);
DECIK_API int decik_attn_qkv_bwd(decik_tensor3 dout, decik_tensor3 q, decik_tensor3 k, decik_tensor3 v,
                       decik_tensor3 out, const float* lse, const int32_t* cu_seqlens, int n_rows,
                       int max_len, int64_t n_tok, int n_heads, int n_kv, int head_dim, float scale,
                       const float* cos, const float* sin, const void* frag, float scaling, void* dy,
                       int64_t ldy, int dtype, void* workspace, void* stream);

/* ---------------------------------------------------------------------------------------------
 * RMSNorm (Qwen2RMSNorm), the producer of the LoRA input (norm_link recompute).
 * Replaces skc_rmsnorm_fwd_kernel / skc_rmsnorm_bwd_kernel (solution/rmsnorm.py:17-45) and
 * rmsnorm.recompute (:76-80): y = w * (x * rsqrt(mean(x^2) + eps)), fp32 rows.
 *   x fp32 [n_rows, n_cols] (row stride stride_x), w of w_dtype (F32 or F16) [n_cols],
 *   y fp32 (row stride stride_y), rstd fp32 [n_rows] (may be NULL).
 * Backward: dx = rstd * (g - x * rstd^2 * mean(g * x)), g = dy * w. n_cols % 4 == 0, <= 8192.
 * ------------------------------------------------------------------------------------------- */
DECIK_API int decik_rmsnorm_fwd(const float* x, const void* w, int w_dtype, float* y, float* rstd,
                      int64_t n_rows, int n_cols, int64_t stride_x, int64_t stride_y, float eps,
                      void* stream);
DECIK_API int decik_rmsnorm_bwd(const float* dy, const float* x, const void* w, int w_dtype,
                      const float* rstd, float* dx, int64_t n_rows, int n_cols, void* stream);
/* decik_rmsnorm_bwd plus an fp32 addend [n_rows, n_cols] (16-byte aligned): dx = addend +
 * norm_bwd(dy, x), the one fp32 rounding of the sum autograd forms when x also reaches the loss by
 * another path (the decoder layer's residual stream: the input norm's gradient plus the residual
 * gradient of the layer input, in one pass instead of a separate add). */
DECIK_API int decik_rmsnorm_bwd_add(const float* dy, const float* x, const void* w, int w_dtype, const float* rstd,
                      const float* addend, float* dx, int64_t n_rows, int n_cols, void* stream);

/* ---------------------------------------------------------------------------------------------
 * The decoder's residual add + post-attention RMSNorm, one pass each way.
 * Replaces AddRMSNormFn (solution/rmsnorm.py:108-144) as the patched Qwen2DecoderLayer.forward
 * calls it (solution/varlen.py:323-337).
 *   forward:  h = residual + f32(delta) (one fp32 rounding), y = w * (h * rsqrt(mean(h^2) + eps));
 *             writes h, y (fp32) and rstd [n_rows] (may be NULL).
 *   backward: h rebuilt from residual and delta (not kept), dx = grad_h + norm_bwd(dy, h) in fp32
 *             (grad_h may be NULL: dx = norm_bwd), and dx16 = dx in delta's type (may be NULL).
 * residual, h, y, dy, grad_h, dx: fp32 [n_rows, n_cols] contiguous, 16-byte aligned; delta and
 * dx16 of delta_dtype (F32, F16 or BF16), 8-byte aligned (16 for F32); w of w_dtype (F32 or F16).
 * y and the norm gradient equal decik_rmsnorm_fwd / _bwd applied to the same h bit for bit.
 * n_cols % 4 == 0, <= 8192.
 * ------------------------------------------------------------------------------------------- */
DECIK_API int decik_add_rmsnorm_fwd(const float* residual, const void* delta, int delta_dtype, const void* w,
                      int w_dtype, float* h, float* y, float* rstd, int64_t n_rows, int n_cols, float eps,
                      void* stream);
DECIK_API int decik_add_rmsnorm_bwd(const float* dy, const float* grad_h, const float* residual,
                      const void* delta, int delta_dtype, const void* w, int w_dtype, const float* rstd,
                      float* dx, void* dx16, int64_t n_rows, int n_cols, void* stream);
/* The same with y (forward) and dy (backward) in delta's 16-bit type (delta F16 or BF16; y, dy
 * 8-byte aligned): for a consumer of y that computes in that type (the patched MLP), which would
 * otherwise cast the fp32 y, and whose input gradient is then of that type. y equals
 * decik_add_rmsnorm_fwd's y rounded to the type, and the backward equals decik_add_rmsnorm_bwd on
 * the widened dy, bit for bit. */
DECIK_API int decik_add_rmsnorm_fwd16(const float* residual, const void* delta, int delta_dtype, const void* w,
                      int w_dtype, float* h, void* y16, float* rstd, int64_t n_rows, int n_cols, float eps,
                      void* stream);
DECIK_API int decik_add_rmsnorm_bwd16(const void* dy16, const float* grad_h, const float* residual,
                      const void* delta, int delta_dtype, const void* w, int w_dtype, const float* rstd,
                      float* dx, void* dx16, int64_t n_rows, int n_cols, void* stream);

/* ---------------------------------------------------------------------------------------------
 * SwiGLU of the Qwen2 MLP, for the fused MLP node.
 * Replaces the SwiGLU of RecomputedMLP (solution/mlp.py:36-59, kernels solution/swiglu.py:15-37):
 * gu = [gate | up] is one [n_rows, 2*inter] projection output (row stride ld) in dtype (F16/BF16);
 *   forward:  out[r, c] = g * sigmoid(g) * u in fp32, rounded to dtype (row stride ldo)
 *   backward: dup = grad * g * s, dgate = grad * u * s * (1 + g (1 - s)), s = sigmoid(g), written
 *             as dgu = [dgate | dup] laid out like gu (row stride ldd); grad row stride ldg.
 * inter % 8 == 0; every row start 16-byte aligned.
 * ------------------------------------------------------------------------------------------- */
DECIK_API int decik_swiglu_fwd(const void* gu, int64_t ld, void* out, int64_t ldo, int64_t n_rows, int inter,
                      int dtype, void* stream);
DECIK_API int decik_swiglu_bwd(const void* grad, int64_t ldg, const void* gu, int64_t ld, void* dgu, int64_t ldd,
                      int64_t n_rows, int inter, int dtype, void* stream);

/* ---------------------------------------------------------------------------------------------
 * LM-head cross entropy over one chunk of logits (the chunked fused head + loss).
 * Replaces skc_head_stats_kernel (solution/head.py:39-85): per row of logits ([n_rows, n_vocab],
 * 16-bit of dtype, row stride ld) lse, entropy = lse - sum(p z), token_loss = lse - z[target]
 * (0 for target < 0, NaN for target >= n_vocab), hit = (argmax == target, first maximal index);
 * then, for rows with a label, softmax - onehot written over the logits in place (the operand of
 * the hidden-state gradient matmul). target int64 [n_rows]; n_vocab, ld multiples of 8.
 * ------------------------------------------------------------------------------------------- */
DECIK_API int decik_head_stats(void* logits, int64_t ld, const int64_t* target, float* lse, float* entropy,
                      float* token_loss, int* hit, int64_t n_rows, int n_vocab, int dtype, void* stream);

/* ---------------------------------------------------------------------------------------------
 * Packed (padding-free) varlen causal GQA attention.
 * Replaces VarlenSDPA (solution/varlen.py:134-168), i.e. aten::_efficient_attention_forward /
 * _backward over cu_seqlens with the 6x GQA expansion (_expand_kv, :124-131) and the
 * dk/dv group sum (:165-167); same result as PackedSDPA (:85-121). Query head h reads kv head
 * h / (n_heads / n_kv); row r spans tokens [cu_seqlens[r], cu_seqlens[r+1]); key j is visible to
 * query i of the same row iff j <= i (top-left causal).
 *
 * Tensors are 3-D views [T, H, head_dim] given by (pointer, token stride, head stride) in
 * elements; head_dim is contiguous. dtype F16 or BF16, head_dim == 128. Strides and pointers must
 * be 16-byte aligned.
 *   cu_seqlens int32 [n_rows + 1] (device), max_len = the longest row.
 *   out [T, n_heads, D]; lse fp32 [n_heads, T] (natural-log logsumexp of the scaled scores).
 * ------------------------------------------------------------------------------------------- */
DECIK_API int decik_varlen_attn_fwd(decik_tensor3 q, decik_tensor3 k, decik_tensor3 v, decik_tensor3_mut out,
                          float* lse, const int32_t* cu_seqlens, int n_rows, int max_len,
                          int64_t n_tok, int n_heads, int n_kv, int head_dim, float scale,
                          int dtype, void* stream);

/* Bytes of device workspace decik_varlen_attn_bwd needs for these sizes (fp32 dq accumulator
 * [T, n_heads, D] and the fp32 rowsum(dO * O) [n_heads, T]). */
DECIK_API int64_t decik_varlen_attn_bwd_workspace(int64_t n_tok, int n_heads, int head_dim);

/* Backward: dq, dk, dv (dk/dv already summed over each kv head's query heads). Uses the forward's
 * out and lse (no forward recompute). workspace: decik_varlen_attn_bwd_workspace() bytes,
 * 256-byte aligned; its contents on entry do not matter. */
DECIK_API int decik_varlen_attn_bwd(decik_tensor3 dout, decik_tensor3 q, decik_tensor3 k, decik_tensor3 v,
                          decik_tensor3 out, const float* lse, decik_tensor3_mut dq,
                          decik_tensor3_mut dk, decik_tensor3_mut dv, const int32_t* cu_seqlens,
                          int n_rows, int max_len, int64_t n_tok, int n_heads, int n_kv,
                          int head_dim, float scale, int dtype, void* workspace, void* stream);

/* ---------------------------------------------------------------------------------------------
 * The same backward for callers that cannot allocate device memory. No counterpart in the
 * reference (its backward runs inside PyTorch, which allocates freely).
 *
 * Arguments and results are those of decik_varlen_attn_bwd without the workspace: the scratch is
 * a static device array inside this library, sized for n_tok * n_heads <= 16384 (about 8.5 MB,
 * held on every GPU that loads the library until the process exits). Larger inputs return
 * DECIK_ERR_INVALID with a message. It is meant for callers whose device memory is owned by a
 * host framework's pool that forbids raw allocations, or that run where an allocation could
 * block or fail. The first call on a device looks up the array's address; under CUDA's default
 * lazy module loading that is also when the driver loads the array's module and reserves its
 * 8.5 MB on that device. So make the first call on each device at start-up, before the host's
 * pool takes the device memory and before any stream capture: a call with n_tok = 0 does only
 * this set-up (no kernel runs). Every call reuses the same array, so calls whose kernels overlap
 * on the GPU (different streams with no ordering) race with each other: order them on one stream
 * or with events. This entry point itself allocates and frees nothing.
 * ------------------------------------------------------------------------------------------- */
DECIK_API int decik_varlen_attn_bwd_noalloc(decik_tensor3 dout, decik_tensor3 q, decik_tensor3 k, decik_tensor3 v,
                          decik_tensor3 out, const float* lse, decik_tensor3_mut dq,
                          decik_tensor3_mut dk, decik_tensor3_mut dv, const int32_t* cu_seqlens,
                          int n_rows, int max_len, int64_t n_tok, int n_heads, int n_kv,
                          int head_dim, float scale, int dtype, void* stream);

/* ---------------------------------------------------------------------------------------------
 * The projection GEMMs of the attention block on tcgen05, with their epilogues fused.
 *
 * decik_lora_b_ext writes the B operand of the GEMM's extra K block, out dt [n_proj, 64]
 * (n_proj = (n_heads + 2 n_kv) 128): row c of a q head = scaling . B_q[c] in columns 0..15, row c
 * of a v head = scaling . B_v[c] in columns 16..31, every row its bias (dt [n_proj]) in column 32,
 * zero elsewhere. b_q fp32 [n_heads 128, 16] and b_v fp32 [n_kv 128, 16] are peft's lora_B weights,
 * or both NULL (no LoRA). */
DECIK_API int decik_lora_b_ext(const float* b_q, const float* b_v, float scaling, const void* bias, void* out,
                               int n_heads, int n_kv, int dtype, void* stream);

/* decik_qkv_proj_fwd replaces, for one layer, the reference's three NF4Linear forwards
 * (solution/nf4.py:93-97: F.linear(x16, W, b16)), the LoRA pair's forward (solution/attn.py:217-228)
 * and FusedQKRope.forward (solution/attn.py:97-111, skc_rope_fwd_kernel :28-61). Two kernels:
 *   1. x16 = dt(x) [T, hidden] (ldx16) and u [T, 64] = [u_q | u_v | 1 | 0 ...] with
 *      u_q | u_v = dt(x16 . w_cat[n_proj : n_proj + 32]^T) (zero when lora is 0);
 *   2. one persistent tcgen05 GEMM on CTA pairs over K = hidden + 64:
 *      acc = x16 . w_cat[0 : n_proj]^T + u . ext_b^T = base + LoRA-up + bias   (fp32, in TMEM)
 *      q = rope(acc_q) head-major, k = rope(acc_k) head-major, v = acc_v, each rounded once to dt;
 *      RoPE in fp32 with separate roundings (no FMA). The projection never leaves the chip. The
 *      reference rounds the biased projection and the LoRA product to dt before adding them; here
 *      they meet in the fp32 accumulator (one rounding, at the end).
 *   x       fp32 [T, hidden] (ldx)
 *   w_cat   dt [n_proj (+ 32 with lora), hidden] (ldw): dequantised W_q, W_k, W_v rows, then A_q, A_v
 *   ext_b   decik_lora_b_ext's output (required: it carries the bias)
 *   cos/sin fp32 [T, 128]; q, k, v: [T, H, 128] views (any 16-byte aligned strides)
 * hidden % 128 == 0, head_dim 128, an even n_heads + 2 n_kv. */
DECIK_API int decik_qkv_proj_fwd(const float* x, int64_t ldx, const void* w_cat, int64_t ldw, const void* ext_b,
                                 int lora, const float* cosp, const float* sinp, decik_tensor3_mut q,
                                 decik_tensor3_mut k, decik_tensor3_mut v, void* x16, int64_t ldx16, void* u,
                                 int64_t n_tok, int hidden, int n_heads, int n_kv, int head_dim, int dtype,
                                 void* stream);

/* decik_qkv_proj_norm_fwd: decik_qkv_proj_fwd with the decoder layer's input RMSNorm fused into its
 * first kernel (the reference's Qwen2RMSNorm, solution/rmsnorm.py:17-28, whose fp32 output the
 * attention casts to 16 bits). h fp32 [T, hidden] (ldh) is the layer input; the pass computes
 * x = norm_w * (h * rstd), rstd = rsqrt(mean(h^2) + eps), exactly as decik_rmsnorm_fwd does (the
 * same reduction order: x16 equals decik_rmsnorm_fwd's output cast to dt), and writes rstd fp32
 * [T] for the norm's backward (decik_rmsnorm_bwd). x never exists in fp32. norm_w of norm_dtype
 * (F32, 16-byte aligned, or F16) [hidden]. The other arguments are decik_qkv_proj_fwd's. */
DECIK_API int decik_qkv_proj_norm_fwd(const float* h, int64_t ldh, const void* norm_w, int norm_dtype, float eps,
                                      float* rstd, const void* w_cat, int64_t ldw, const void* ext_b, int lora,
                                      const float* cosp, const float* sinp, decik_tensor3_mut q, decik_tensor3_mut k,
                                      decik_tensor3_mut v, void* x16, int64_t ldx16, void* u, int64_t n_tok,
                                      int hidden, int n_heads, int n_kv, int head_dim, int dtype, void* stream);

/* dx = dy[:, 0:k_cols] . w_t[:, 0:k_cols]^T in fp32 [T, hidden] (ld_dx), w_t dt [hidden, >= k_cols]
 * (ldw) the TRANSPOSED weight (decik_transpose16 of W_cat [k_cols, hidden]): the three NF4Linear
 * input gradients (solution/nf4.py:99-104: g16 @ W16) and both LoRA input gradients
 * (solution/attn.py:264-273) summed in one tcgen05 GEMM on CTA pairs; also the MLP's input gradient
 * ([dgate | dup] . [W_gate; W_up]). dy dt [T, >= k_cols]. hidden, k_cols multiples of 8. */
DECIK_API int decik_proj_dx(const void* dy, int64_t ld_dy, int k_cols, const void* w_t, int64_t ldw, float* dx,
                            int64_t ld_dx, int64_t n_tok, int hidden, int dtype, void* stream);

/* dst [cols, rows] = src [rows, cols]^T for 16-bit values (rows, cols multiples of 8). */
DECIK_API int decik_transpose16(const void* src, int64_t lds, void* dst, int64_t ldd, int64_t rows, int64_t cols,
                                void* stream);

/* The LoRA parameter gradients of the fused block (solution/attn.py:255-262):
 *   da [32, hidden] fp32 = du^T x16 (du = dy[:, n_proj : n_proj + 32]; rows 0-15 dA_q, 16-31 dA_v)
 *   db [(n_heads + n_kv) 128, 16] fp32 = scaling . g^T u (g = dy's q columns with u_q, then its v
 *      columns with u_v)
 * dy dt [T, >= n_proj + 32] (ld_dy), x16 dt [T, hidden], u dt [T, >= 32] (ldu). Zeroes da and db,
 * then adds token-chunked tensor-core partial products into them. */
DECIK_API int decik_lora_grads(const void* dy, int64_t ld_dy, const void* x16, int64_t ldx, const void* u,
                               int64_t ldu, float* da, float* db, float scaling, int64_t n_tok, int hidden,
                               int n_heads, int n_kv, int dtype, void* stream);

/* ---------------------------------------------------------------------------------------------
 * The MLP's GEMMs on tcgen05 CTA pairs (the same kernel as the projections), with SwiGLU fused.
 * They replace the four F.linear / torch.mm calls of the MLP node and its separate SwiGLU kernels:
 * the reference's RecomputedMLP (solution/mlp.py:62-110: gate and up projections, SwiGLU, down
 * projection, and their input gradients) and skc_swiglu (solution/swiglu.py:15-37).
 *
 * decik_gemm16: out[M, N] (dt, ldo) = a[M, K] . b^T with b dt [N, K] (b_mn = 0), or a . b with
 * b [K, N] (b_mn = 1); fp32 accumulation, one rounding. N, K multiples of 8. */
DECIK_API int decik_gemm16(const void* a, int64_t lda, const void* b, int64_t ldb, int b_mn, void* out, int64_t ldo,
                           int64_t m, int n, int k, int dtype, void* stream);

/* gu [M, 2 inter] = x16 . w_gu^T (w_gu dt [2 inter, hidden]: W_gate rows then W_up rows), each
 * value rounded to dt, and h [M, inter] = dt(gate * sigmoid(gate) * up) from those rounded values
 * (the separate SwiGLU kernel's arithmetic, decik_swiglu_fwd). inter % 128 == 0. */
DECIK_API int decik_mlp_gate_up(const void* x16, int64_t ldx, const void* w_gu, int64_t ldw, void* gu, int64_t ldgu,
                                void* h, int64_t ldh, int64_t m, int hidden, int inter, int dtype, void* stream);

/* dgu [M, 2 inter] = [dgate | dup] of SwiGLU for grad_hidden = dt(grad . w_down) (grad dt [M, hidden],
 * w_down dt [hidden, inter]) and the forward's gu: dup = g' g s, dgate = g' u s (1 + g (1 - s)),
 * s = sigmoid(g) (decik_swiglu_bwd's arithmetic); grad_hidden never reaches HBM. inter % 256 == 0. */
DECIK_API int decik_mlp_down_grad(const void* grad, int64_t ldg, const void* w_down, int64_t ldw, const void* gu,
                                  int64_t ldgu, void* dgu, int64_t lddgu, int64_t m, int hidden, int inter, int dtype,
                                  void* stream);

#ifdef __cplusplus
}
#endif

#endif /* DECIK_B200_H */
