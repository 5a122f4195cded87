// C entry points of the packed varlen causal GQA attention (VarlenSDPA, solution/varlen.py:134-168)
// and the two element-wise passes around the tcgen05 backward: delta = rowsum(dO * O) with the fp32
// dq accumulator zeroed, and the final dq = scale * dq_acc cast into dq's layout. The tensor-core
// kernels are in attn_fwd_sm100.cu and attn_bwd_sm100.cu.
#include "attn_common.cuh"

namespace decik {
namespace attn {
namespace {

// ------------------------------------------------------------------------------------------------
// backward
// ------------------------------------------------------------------------------------------------
// delta[h, t] = sum_d dO * O (fp32), dq_acc = 0 and, when dK / dV are reduced in fp32, their
// accumulators = 0. kPrepItems (token, head) rows per warp, 4 dims per lane.
constexpr int kPrepItems = 4;  // (token, head) rows per warp in the prep kernel

template <typename T>
__global__ void __launch_bounds__(256)
attn_bwd_prep_kernel(Tensor3 dout, Tensor3 out, float* __restrict__ delta, float* __restrict__ dq_acc,
                     float* __restrict__ dk_acc, float* __restrict__ dv_acc, int64_t n_tok, int n_heads, int n_kv) {
  // kPrepItems (token, head) rows per warp, all their loads issued before any arithmetic (one row
  // per warp left too few bytes in flight: ~0.68 of HBM); lane l holds dims 4l .. 4l + 3 of a row
  const int lane = threadIdx.x & 31;
  const int64_t first = (static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5)) * kPrepItems;
  const int64_t n_items = n_tok * n_heads;
  uint2 a[kPrepItems], b[kPrepItems];
#pragma unroll
  for (int i = 0; i < kPrepItems; ++i) {
    const int64_t item = first + i;
    if (item < n_items) {
      const int64_t tok = item / n_heads;
      const int h = static_cast<int>(item % n_heads);
      a[i] = *reinterpret_cast<const uint2*>(static_cast<const T*>(dout.ptr) + tok * dout.tok + h * dout.head + lane * 4);
      b[i] = *reinterpret_cast<const uint2*>(static_cast<const T*>(out.ptr) + tok * out.tok + h * out.head + lane * 4);
    }
  }
#pragma unroll
  for (int i = 0; i < kPrepItems; ++i) {
    const int64_t item = first + i;
    if (item >= n_items) break;  // uniform across the warp
    const int64_t tok = item / n_heads;
    const int h = static_cast<int>(item % n_heads);
    float acc = Dt<T>::lo_f(a[i].x) * Dt<T>::lo_f(b[i].x) + Dt<T>::hi_f(a[i].x) * Dt<T>::hi_f(b[i].x) +
                Dt<T>::lo_f(a[i].y) * Dt<T>::lo_f(b[i].y) + Dt<T>::hi_f(a[i].y) * Dt<T>::hi_f(b[i].y);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) delta[static_cast<int64_t>(h) * n_tok + tok] = acc;
    const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
    reinterpret_cast<float4*>(dq_acc + (tok * n_heads + h) * D)[lane] = z;
    if (dk_acc != nullptr && h < n_kv) {
      reinterpret_cast<float4*>(dk_acc + (tok * n_kv + h) * D)[lane] = z;
      reinterpret_cast<float4*>(dv_acc + (tok * n_kv + h) * D)[lane] = z;
    }
  }
}

// dq = scale * dq_acc and, with fp32 dK / dV accumulators, dk = scale * dk_acc and dv = dv_acc,
// cast into the callers' strided layouts. One thread per 8 dims.
template <typename T>
__global__ void __launch_bounds__(256)
attn_bwd_post_kernel(const float* __restrict__ dq_acc, Tensor3Mut dq, const float* __restrict__ dk_acc, Tensor3Mut dk,
                     const float* __restrict__ dv_acc, Tensor3Mut dv, int64_t n_tok, int n_heads, int n_kv, float scale) {
  int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t nq = n_tok * n_heads * (D / 8);
  const int64_t nkv = dk_acc != nullptr ? n_tok * n_kv * (D / 8) : 0;
  const float* src;
  Tensor3Mut dst;
  int heads;
  float mul;
  if (i < nq) {
    src = dq_acc; dst = dq; heads = n_heads; mul = scale;
  } else if (i < nq + nkv) {
    i -= nq; src = dk_acc; dst = dk; heads = n_kv; mul = scale;
  } else if (i < nq + 2 * nkv) {
    i -= nq + nkv; src = dv_acc; dst = dv; heads = n_kv; mul = 1.f;
  } else {
    return;
  }
  const int c = static_cast<int>(i % (D / 8));
  const int64_t th = i / (D / 8);
  const int h = static_cast<int>(th % heads);
  const int64_t tok = th / heads;
  const float4 a = reinterpret_cast<const float4*>(src + th * D + c * 8)[0];
  const float4 b = reinterpret_cast<const float4*>(src + th * D + c * 8)[1];
  const float f[8] = {a.x * mul, a.y * mul, a.z * mul, a.w * mul, b.x * mul, b.y * mul, b.z * mul, b.w * mul};
  stg16(static_cast<T*>(dst.ptr) + tok * dst.tok + h * dst.head + c * 8, pack8<T>(f));
}

bool ok3(const void* p, int64_t tok, int64_t head) {
  return p != nullptr && aligned16(p) && (tok % 8) == 0 && (head % 8) == 0;
}

}  // namespace
}  // namespace attn
}  // namespace decik

using namespace decik;
using namespace decik::attn;

namespace decik {
namespace attn {
int fwd_sm100(const decik_tensor3& q, const decik_tensor3& k, const decik_tensor3& v, const decik_tensor3_mut& out,
              float* lse, const int32_t* cu, int n_rows, int max_len, int64_t n_tok, int n_heads, int n_kv,
              float scale, int dtype, cudaStream_t stream);
int bwd_sm100(const decik_tensor3& q, const decik_tensor3& k, const decik_tensor3& v, const decik_tensor3& dout,
              const decik_tensor3_mut& dk, const decik_tensor3_mut& dv, const float* lse, const float* delta,
              float* dq_acc, float* dk_acc, float* dv_acc, int n_split, const int32_t* cu, int n_rows,
              int max_len, int64_t n_tok, int n_heads, int n_kv, float scale, int dtype, cudaStream_t stream);
int bwd_sm100_splits(int64_t n_tok, int n_rows, int n_heads, int n_kv);
}
}  // namespace decik

extern "C" int decik_varlen_attn_fwd(decik_tensor3 q, decik_tensor3 k, decik_tensor3 v,
                                     decik_tensor3_mut out, float* lse, const int32_t* cu_seqlens,
                                     int n_rows, int max_len, int64_t n_tok, int n_heads, int n_kv,
                                     int head_dim, float scale, int dtype, void* stream) {
  if (n_rows == 0 || n_tok == 0 || max_len == 0) return DECIK_OK;
  if (head_dim != D) return set_error(DECIK_ERR_UNSUPPORTED, "varlen_attn_fwd: head_dim %d (only 128)", head_dim);
  if (n_rows < 0 || max_len < 0 || n_tok < 0 || n_heads <= 0 || n_kv <= 0 || n_heads % n_kv ||
      n_tok > INT32_MAX - 256)
    return set_error(DECIK_ERR_INVALID, "varlen_attn_fwd: bad sizes (rows %d, heads %d/%d)", n_rows, n_heads, n_kv);
  if (!ok3(q.ptr, q.tok_stride, q.head_stride) || !ok3(k.ptr, k.tok_stride, k.head_stride) ||
      !ok3(v.ptr, v.tok_stride, v.head_stride) || !ok3(out.ptr, out.tok_stride, out.head_stride))
    return set_error(DECIK_ERR_INVALID, "varlen_attn_fwd: tensors need 16-byte aligned pointers and strides");
  if (!lse || !cu_seqlens) return set_error(DECIK_ERR_INVALID, "varlen_attn_fwd: null lse / cu_seqlens");
  if (dtype != DECIK_F16 && dtype != DECIK_BF16) return set_error(DECIK_ERR_INVALID, "varlen_attn_fwd: dtype");
  return fwd_sm100(q, k, v, out, lse, cu_seqlens, n_rows, max_len, n_tok, n_heads, n_kv, scale, dtype,
                   as_stream(stream));
}

namespace {
int64_t up256(int64_t b) { return ((b + 255) / 256) * 256; }
}  // namespace

namespace decik {
namespace attn {

// Workspace bytes: the fp32 dq accumulator and delta; with `kv_acc`, also fp32 dK / dV
// accumulators, sized for n_kv = n_heads (the largest a caller can have).
int64_t bwd_workspace_bytes(int64_t n_tok, int n_heads, bool kv_acc) {
  const int64_t acc = up256(n_tok * n_heads * D * 4);
  return acc + up256(n_tok * n_heads * 4) + (kv_acc ? 2 * acc : 0);
}

// Where the attention backward left its results: dq always in the fp32 accumulator (unscaled),
// dk (unscaled) / dv in fp32 accumulators when a key block's query heads were split over CTAs,
// else already in the caller's dk (scaled) / dv.
struct BwdAcc {
  float* dq;
  float* dk;
  float* dv;
  int n_split;
};

int check_bwd_args(const decik_tensor3& dout, const decik_tensor3& q, const decik_tensor3& k, const decik_tensor3& v,
                   const decik_tensor3& out, const float* lse, const decik_tensor3_mut& dk,
                   const decik_tensor3_mut& dv, const int32_t* cu_seqlens, int n_rows, int max_len, int64_t n_tok,
                   int n_heads, int n_kv, int head_dim, int dtype, void* workspace) {
  if (head_dim != D) return set_error(DECIK_ERR_UNSUPPORTED, "varlen_attn_bwd: head_dim %d (only 128)", head_dim);
  if (n_rows < 0 || max_len < 0 || n_tok < 0 || n_heads <= 0 || n_kv <= 0 || n_heads % n_kv ||
      n_tok > INT32_MAX - 256)
    return set_error(DECIK_ERR_INVALID, "varlen_attn_bwd: bad sizes");
  if (dtype != DECIK_F16 && dtype != DECIK_BF16) return set_error(DECIK_ERR_INVALID, "varlen_attn_bwd: dtype");
  if (!ok3(dout.ptr, dout.tok_stride, dout.head_stride) || !ok3(q.ptr, q.tok_stride, q.head_stride) ||
      !ok3(k.ptr, k.tok_stride, k.head_stride) || !ok3(v.ptr, v.tok_stride, v.head_stride) ||
      !ok3(out.ptr, out.tok_stride, out.head_stride) || !ok3(dk.ptr, dk.tok_stride, dk.head_stride) ||
      !ok3(dv.ptr, dv.tok_stride, dv.head_stride))
    return set_error(DECIK_ERR_INVALID, "varlen_attn_bwd: tensors need 16-byte aligned pointers and strides");
  if (!lse || !cu_seqlens || !workspace || (reinterpret_cast<uintptr_t>(workspace) & 255))
    return set_error(DECIK_ERR_INVALID, "varlen_attn_bwd: null lse/cu_seqlens or workspace not 256-byte aligned");
  return DECIK_OK;
}

// delta / accumulator zeroing, then the tcgen05 backward (no cast pass); validated arguments
int varlen_attn_bwd_core(const decik_tensor3& dout, const decik_tensor3& q, const decik_tensor3& k,
                         const decik_tensor3& v, const decik_tensor3& out, const float* lse,
                         const decik_tensor3_mut& dk, const decik_tensor3_mut& dv, const int32_t* cu_seqlens,
                         int n_rows, int max_len, int64_t n_tok, int n_heads, int n_kv, float scale, int dtype,
                         void* workspace, bool allow_split, cudaStream_t s, BwdAcc* acc_out) {
  const int n_split = allow_split ? bwd_sm100_splits(n_tok, n_rows, n_heads, n_kv) : 1;
  char* ws = static_cast<char*>(workspace);
  const int64_t acc = up256(n_tok * n_heads * D * 4);
  float* dq_acc = reinterpret_cast<float*>(ws);
  float* delta = reinterpret_cast<float*>(ws + acc);
  float* dk_acc = n_split > 1 ? reinterpret_cast<float*>(ws + acc + up256(n_tok * n_heads * 4)) : nullptr;
  float* dv_acc = n_split > 1 ? reinterpret_cast<float*>(ws + 2 * acc + up256(n_tok * n_heads * 4)) : nullptr;
  *acc_out = BwdAcc{dq_acc, dk_acc, dv_acc, n_split};
  return DECIK_DISPATCH_16(dtype, [&] {
    const int64_t items = n_tok * n_heads;
    attn_bwd_prep_kernel<T><<<static_cast<unsigned>((items + 8 * kPrepItems - 1) / (8 * kPrepItems)), 256, 0, s>>>(
        Tensor3{dout.ptr, dout.tok_stride, dout.head_stride}, Tensor3{out.ptr, out.tok_stride, out.head_stride},
        delta, dq_acc, dk_acc, dv_acc, n_tok, n_heads, n_kv);
    int rc = check_launch("varlen_attn_bwd prep");
    if (rc) return rc;
    return bwd_sm100(q, k, v, dout, dk, dv, lse, delta, dq_acc, dk_acc, dv_acc, n_split, cu_seqlens, n_rows,
                     max_len, n_tok, n_heads, n_kv, scale, dtype, s);
  });
}

// The backward with a workspace of bwd_workspace_bytes(n_tok, n_heads, allow_split) bytes.
int varlen_attn_bwd_impl(const decik_tensor3& dout, const decik_tensor3& q, const decik_tensor3& k,
                         const decik_tensor3& v, const decik_tensor3& out, const float* lse,
                         const decik_tensor3_mut& dq, const decik_tensor3_mut& dk, const decik_tensor3_mut& dv,
                         const int32_t* cu_seqlens, int n_rows, int max_len, int64_t n_tok, int n_heads,
                         int n_kv, int head_dim, float scale, int dtype, void* workspace, bool allow_split,
                         cudaStream_t s) {
  if (n_rows == 0 || n_tok == 0 || max_len == 0) return DECIK_OK;
  int rc = check_bwd_args(dout, q, k, v, out, lse, dk, dv, cu_seqlens, n_rows, max_len, n_tok, n_heads, n_kv,
                          head_dim, dtype, workspace);
  if (rc) return rc;
  if (!ok3(dq.ptr, dq.tok_stride, dq.head_stride))
    return set_error(DECIK_ERR_INVALID, "varlen_attn_bwd: tensors need 16-byte aligned pointers and strides");
  BwdAcc acc;
  rc = varlen_attn_bwd_core(dout, q, k, v, out, lse, dk, dv, cu_seqlens, n_rows, max_len, n_tok, n_heads, n_kv,
                            scale, dtype, workspace, allow_split, s, &acc);
  if (rc) return rc;
  return DECIK_DISPATCH_16(dtype, [&] {
    const int64_t n8 = n_tok * (n_heads + (acc.n_split > 1 ? 2 * n_kv : 0)) * (D / 8);
    attn_bwd_post_kernel<T><<<static_cast<unsigned>((n8 + 255) / 256), 256, 0, s>>>(
        acc.dq, Tensor3Mut{dq.ptr, dq.tok_stride, dq.head_stride}, acc.dk,
        Tensor3Mut{dk.ptr, dk.tok_stride, dk.head_stride}, acc.dv, Tensor3Mut{dv.ptr, dv.tok_stride, dv.head_stride},
        n_tok, n_heads, n_kv, scale);
    return check_launch("varlen_attn_bwd post");
  });
}

}  // namespace attn
}  // namespace decik

extern "C" int64_t decik_varlen_attn_bwd_workspace(int64_t n_tok, int n_heads, int head_dim) {
  (void)head_dim;
  return decik::attn::bwd_workspace_bytes(n_tok, n_heads, true);
}

extern "C" int decik_varlen_attn_bwd(decik_tensor3 dout, decik_tensor3 q, decik_tensor3 k,
                                     decik_tensor3 v, decik_tensor3 out, const float* lse,
                                     decik_tensor3_mut dq, decik_tensor3_mut dk,
                                     decik_tensor3_mut dv, const int32_t* cu_seqlens, int n_rows,
                                     int max_len, int64_t n_tok, int n_heads, int n_kv,
                                     int head_dim, float scale, int dtype, void* workspace,
                                     void* stream) {
  return decik::attn::varlen_attn_bwd_impl(dout, q, k, v, out, lse, dq, dk, dv, cu_seqlens, n_rows, max_len, n_tok,
                                           n_heads, n_kv, head_dim, scale, dtype, workspace, true,
                                           decik::as_stream(stream));
}

// ------------------------------------------------------------------------------------------------
// the fused block's backward: attention backward + projection epilogue backward
// ------------------------------------------------------------------------------------------------
namespace decik {
int qkv_epilogue_bwd_acc(const float* q_acc, float q_mul, const decik_tensor3& grad_k, const float* k_acc,
                         float k_mul, const float* v_acc, const float* cos, const float* sin, const void* frag,
                         float scaling, void* dy, int64_t ldy, int64_t n_tok, int n_heads, int n_kv, int dtype,
                         cudaStream_t stream);
}  // namespace decik

namespace {
// events a multi-stage call records between its stages on its stream (profiling; none by default)
thread_local cudaEvent_t g_stage_events[4];
thread_local int g_n_stage_events = 0;
}  // namespace

extern "C" void decik_set_stage_events(void* const* events, int n) {
  g_n_stage_events = events == nullptr ? 0 : (n < 0 ? 0 : (n > 4 ? 4 : n));
  for (int i = 0; i < g_n_stage_events; ++i) g_stage_events[i] = static_cast<cudaEvent_t>(events[i]);
}

extern "C" int64_t decik_attn_qkv_bwd_workspace(int64_t n_tok, int n_heads, int n_kv, int head_dim) {
  (void)head_dim;
  return decik::attn::bwd_workspace_bytes(n_tok, n_heads, true) + up256(n_tok * n_kv * D * 2);
}

extern "C" int decik_attn_qkv_bwd(decik_tensor3 dout, decik_tensor3 q, decik_tensor3 k, decik_tensor3 v,
                                  decik_tensor3 out, const float* lse, const int32_t* cu_seqlens, int n_rows,
                                  int max_len, int64_t n_tok, int n_heads, int n_kv, int head_dim, float scale,
                                  const float* cos, const float* sin, const void* frag, float scaling, void* dy,
                                  int64_t ldy, int dtype, void* workspace, void* stream) {
  using namespace decik::attn;
  if (n_rows == 0 || n_tok == 0 || max_len == 0) return DECIK_OK;
  if (!dy || (ldy % 8) || ldy < static_cast<int64_t>(n_heads + 2 * n_kv) * D)
    return set_error(DECIK_ERR_INVALID, "attn_qkv_bwd: dy needs a leading dimension >= (Hq + 2 Hk) D, % 8 == 0");
  char* ws = static_cast<char*>(workspace);
  // dk (scaled, 16-bit) when it is written directly goes to the end of the workspace; dv to dy's v columns
  const decik_tensor3_mut dk{ws + bwd_workspace_bytes(n_tok, n_heads, true), static_cast<int64_t>(n_kv) * D, D};
  const int elem = 2;
  const decik_tensor3_mut dv{static_cast<char*>(dy) + static_cast<int64_t>(n_heads + n_kv) * D * elem, ldy, D};
  int rc = check_bwd_args(dout, q, k, v, out, lse, dk, dv, cu_seqlens, n_rows, max_len, n_tok, n_heads, n_kv,
                          head_dim, dtype, workspace);
  if (rc) return rc;
  const cudaStream_t s = decik::as_stream(stream);
  BwdAcc acc;
  rc = varlen_attn_bwd_core(dout, q, k, v, out, lse, dk, dv, cu_seqlens, n_rows, max_len, n_tok, n_heads, n_kv,
                            scale, dtype, workspace, true, s, &acc);
  if (rc) return rc;
  if (g_n_stage_events > 0) cudaEventRecord(g_stage_events[0], s);  // attention done, epilogue next
  const decik_tensor3 dk_in{dk.ptr, dk.tok_stride, dk.head_stride};
  return decik::qkv_epilogue_bwd_acc(acc.dq, scale, dk_in, acc.dk, scale, acc.dv, cos, sin, frag, scaling, dy, ldy,
                                     n_tok, n_heads, n_kv, dtype, s);
}
