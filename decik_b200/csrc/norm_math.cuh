// The per-element and per-row arithmetic of Qwen2RMSNorm (solution/rmsnorm.py:17-45), shared by
// the norm kernels (rmsnorm.cu) and the projection's fused norm + cast pass (proj_sm100.cu). One
// source for every caller keeps their outputs equal bit for bit: a row's mean square is each
// lane's running sum of sumsq4 over its 16-byte pieces (columns 4 lane + 128 j, in j order), then
// the warp_sum tree; y = w * (x * rstd) per element.
#pragma once

#include "common.cuh"

namespace decik {
namespace norm {

template <typename W>
__device__ __forceinline__ float wload(const W* w, int i);
template <> __device__ __forceinline__ float wload<float>(const float* w, int i) { return __ldg(w + i); }
template <> __device__ __forceinline__ float wload<__half>(const __half* w, int i) { return __half2float(w[i]); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// x . x of four values and the weighted dot g . (w x) of four, the per-step row terms of the
// forward and backward reductions
__device__ __forceinline__ float sumsq4(float4 v) { return v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w; }
template <typename W>
__device__ __forceinline__ float wdot4(float4 g, float4 v, const W* w, int c) {
  return g.x * wload<W>(w, c) * v.x + g.y * wload<W>(w, c + 1) * v.y + g.z * wload<W>(w, c + 2) * v.z +
         g.w * wload<W>(w, c + 3) * v.w;
}
// rstd of a row from the warp's per-lane partial sums
__device__ __forceinline__ float row_rstd(float lane_acc, int n_cols, float eps) {
  const float mean_sq = warp_sum(lane_acc) / static_cast<float>(n_cols);
  return rsqrtf(mean_sq + eps);
}
// w * (x * rstd) of four values, with the four weights already loaded
__device__ __forceinline__ float4 norm_out4w(float4 v, float4 w, float rstd) {
  float4 o;
  o.x = w.x * (v.x * rstd);
  o.y = w.y * (v.y * rstd);
  o.z = w.z * (v.z * rstd);
  o.w = w.w * (v.w * rstd);
  return o;
}
template <typename W>
__device__ __forceinline__ float4 wload4(const W* w, int c) {
  return make_float4(wload<W>(w, c), wload<W>(w, c + 1), wload<W>(w, c + 2), wload<W>(w, c + 3));
}
template <typename W>
__device__ __forceinline__ float4 norm_out4(float4 v, const W* w, int c, float rstd) {
  return norm_out4w(v, wload4<W>(w, c), rstd);
}
template <typename W>
__device__ __forceinline__ float4 norm_grad4(float4 g, float4 v, const W* w, int c, float rstd, float k) {
  float4 o;
  o.x = rstd * (g.x * wload<W>(w, c) - v.x * k);
  o.y = rstd * (g.y * wload<W>(w, c + 1) - v.y * k);
  o.z = rstd * (g.z * wload<W>(w, c + 2) - v.z * k);
  o.w = rstd * (g.w * wload<W>(w, c + 3) - v.w * k);
  return o;
}

}  // namespace norm
}  // namespace decik
