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
// delta[h, t] = sum_d dO * O (fp32) and dq_acc = 0. One warp per (token, head), 4 dims per lane.
template <typename T>
__global__ void __launch_bounds__(256)
attn_bwd_prep_kernel(Tensor3 dout, Tensor3 out, float* __restrict__ delta, float* __restrict__ dq_acc,
                     int64_t n_tok, int n_heads) {
  const int lane = threadIdx.x & 31;
  const int64_t item = static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5);
  if (item >= n_tok * n_heads) return;
  const int64_t tok = item / n_heads;
  const int h = static_cast<int>(item % n_heads);
  const uint2 a = *reinterpret_cast<const uint2*>(static_cast<const T*>(dout.ptr) + tok * dout.tok + h * dout.head + lane * 4);
  const uint2 b = *reinterpret_cast<const uint2*>(static_cast<const T*>(out.ptr) + tok * out.tok + h * out.head + lane * 4);
  float acc = Dt<T>::lo_f(a.x) * Dt<T>::lo_f(b.x) + Dt<T>::hi_f(a.x) * Dt<T>::hi_f(b.x) +
              Dt<T>::lo_f(a.y) * Dt<T>::lo_f(b.y) + Dt<T>::hi_f(a.y) * Dt<T>::hi_f(b.y);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if (lane == 0) delta[static_cast<int64_t>(h) * n_tok + tok] = acc;
  reinterpret_cast<float4*>(dq_acc + (tok * n_heads + h) * D)[lane] = make_float4(0.f, 0.f, 0.f, 0.f);
}

// dq = dq_acc * scale, cast, into dq's strided layout. One thread per 8 dims.
template <typename T>
__global__ void __launch_bounds__(256)
attn_bwd_post_kernel(const float* __restrict__ dq_acc, Tensor3Mut dq, int64_t n_tok, int n_heads, float scale) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n_tok * n_heads * (D / 8)) return;
  const int c = static_cast<int>(i % (D / 8));
  const int64_t th = i / (D / 8);
  const int h = static_cast<int>(th % n_heads);
  const int64_t tok = th / n_heads;
  const float4 a = reinterpret_cast<const float4*>(dq_acc + th * D + c * 8)[0];
  const float4 b = reinterpret_cast<const float4*>(dq_acc + th * D + c * 8)[1];
  const float f[8] = {a.x * scale, a.y * scale, a.z * scale, a.w * scale,
                      b.x * scale, b.y * scale, b.z * scale, b.w * scale};
  stg16(static_cast<T*>(dq.ptr) + tok * dq.tok + h * dq.head + c * 8, pack8<T>(f));
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
              float* dq_acc, const int32_t* cu, int n_rows, int max_len, int64_t n_tok, int n_heads, int n_kv,
              float scale, int dtype, cudaStream_t stream);
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

extern "C" int64_t decik_varlen_attn_bwd_workspace(int64_t n_tok, int n_heads, int head_dim) {
  const int64_t dq = n_tok * n_heads * head_dim * 4;
  const int64_t delta = n_tok * n_heads * 4;
  return ((dq + 255) / 256) * 256 + ((delta + 255) / 256) * 256;
}

extern "C" int decik_varlen_attn_bwd(decik_tensor3 dout, decik_tensor3 q, decik_tensor3 k,
                                     decik_tensor3 v, decik_tensor3 out, const float* lse,
                                     decik_tensor3_mut dq, decik_tensor3_mut dk,
                                     decik_tensor3_mut dv, const int32_t* cu_seqlens, int n_rows,
                                     int max_len, int64_t n_tok, int n_heads, int n_kv,
                                     int head_dim, float scale, int dtype, void* workspace,
                                     void* stream) {
  if (n_rows == 0 || n_tok == 0 || max_len == 0) return DECIK_OK;
  if (head_dim != D) return set_error(DECIK_ERR_UNSUPPORTED, "varlen_attn_bwd: head_dim %d (only 128)", head_dim);
  if (n_rows < 0 || max_len < 0 || n_tok < 0 || n_heads <= 0 || n_kv <= 0 || n_heads % n_kv ||
      n_tok > INT32_MAX - 256)
    return set_error(DECIK_ERR_INVALID, "varlen_attn_bwd: bad sizes");
  if (dtype != DECIK_F16 && dtype != DECIK_BF16) return set_error(DECIK_ERR_INVALID, "varlen_attn_bwd: dtype");
  if (!ok3(dout.ptr, dout.tok_stride, dout.head_stride) || !ok3(q.ptr, q.tok_stride, q.head_stride) ||
      !ok3(k.ptr, k.tok_stride, k.head_stride) || !ok3(v.ptr, v.tok_stride, v.head_stride) ||
      !ok3(out.ptr, out.tok_stride, out.head_stride) || !ok3(dq.ptr, dq.tok_stride, dq.head_stride) ||
      !ok3(dk.ptr, dk.tok_stride, dk.head_stride) || !ok3(dv.ptr, dv.tok_stride, dv.head_stride))
    return set_error(DECIK_ERR_INVALID, "varlen_attn_bwd: tensors need 16-byte aligned pointers and strides");
  if (!lse || !cu_seqlens || !workspace || (reinterpret_cast<uintptr_t>(workspace) & 255))
    return set_error(DECIK_ERR_INVALID, "varlen_attn_bwd: null lse/cu_seqlens or workspace not 256-byte aligned");
  float* dq_acc = static_cast<float*>(workspace);
  float* delta = reinterpret_cast<float*>(static_cast<char*>(workspace) + ((n_tok * n_heads * D * 4 + 255) / 256) * 256);
  cudaStream_t s = as_stream(stream);
  return DECIK_DISPATCH_16(dtype, [&] {
    const int64_t items = n_tok * n_heads;
    attn_bwd_prep_kernel<T><<<static_cast<unsigned>((items + 7) / 8), 256, 0, s>>>(
        Tensor3{dout.ptr, dout.tok_stride, dout.head_stride}, Tensor3{out.ptr, out.tok_stride, out.head_stride},
        delta, dq_acc, n_tok, n_heads);
    int rc = check_launch("varlen_attn_bwd prep");
    if (rc) return rc;
    rc = bwd_sm100(q, k, v, dout, dk, dv, lse, delta, dq_acc, cu_seqlens, n_rows, max_len, n_tok, n_heads, n_kv,
                   scale, dtype, s);
    if (rc) return rc;
    const int64_t n8 = n_tok * n_heads * (D / 8);
    attn_bwd_post_kernel<T><<<static_cast<unsigned>((n8 + 255) / 256), 256, 0, s>>>(
        dq_acc, Tensor3Mut{dq.ptr, dq.tok_stride, dq.head_stride}, n_tok, n_heads, scale);
    return check_launch("varlen_attn_bwd post");
  });
}
