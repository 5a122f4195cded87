// Qwen2RMSNorm forward and backward over fp32 rows (solution/rmsnorm.py:17-45). The forward is
// also the norm_link recompute of the LoRA input in the block's backward (solution/attn.py:238):
// the same kernel on the same input gives bit-identical output.
//
// One warp per row; each lane reads 4 consecutive floats per step (16-byte loads) and the row
// reductions (mean of x^2, mean of g*x) are warp-shuffle trees.
#include "common.cuh"

namespace decik {
namespace {

template <typename W>
__device__ __forceinline__ float wload(const W* w, int i);
template <> __device__ __forceinline__ float wload<float>(const float* w, int i) { return __ldg(w + i); }
template <> __device__ __forceinline__ float wload<__half>(const __half* w, int i) { return __half2float(w[i]); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

constexpr int kMaxCols = 8192;

template <typename W>
__global__ void __launch_bounds__(256)
rmsnorm_fwd_kernel(const float* __restrict__ x, const W* __restrict__ w, float* __restrict__ y,
                   float* __restrict__ rstd_out, int64_t n_rows, int n_cols, int64_t sx, int64_t sy,
                   float eps) {
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= n_rows) return;
  const float* xr = x + row * sx;
  float acc = 0.f;
  for (int c = lane * 4; c < n_cols; c += 128) {
    const float4 v = __ldg(reinterpret_cast<const float4*>(xr + c));
    acc += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
  }
  const float mean_sq = warp_sum(acc) / static_cast<float>(n_cols);
  const float rstd = rsqrtf(mean_sq + eps);
  float* yr = y + row * sy;
  for (int c = lane * 4; c < n_cols; c += 128) {
    const float4 v = __ldg(reinterpret_cast<const float4*>(xr + c));
    float4 o;
    o.x = wload<W>(w, c) * (v.x * rstd);
    o.y = wload<W>(w, c + 1) * (v.y * rstd);
    o.z = wload<W>(w, c + 2) * (v.z * rstd);
    o.w = wload<W>(w, c + 3) * (v.w * rstd);
    *reinterpret_cast<float4*>(yr + c) = o;
  }
  if (rstd_out != nullptr && lane == 0) rstd_out[row] = rstd;
}

template <typename W>
__global__ void __launch_bounds__(256)
rmsnorm_bwd_kernel(const float* __restrict__ dy, const float* __restrict__ x,
                   const W* __restrict__ w, const float* __restrict__ rstd_in,
                   float* __restrict__ dx, int64_t n_rows, int n_cols) {
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= n_rows) return;
  const float* xr = x + row * n_cols;
  const float* gr = dy + row * n_cols;
  const float rstd = rstd_in[row];
  float acc = 0.f;
  for (int c = lane * 4; c < n_cols; c += 128) {
    const float4 v = __ldg(reinterpret_cast<const float4*>(xr + c));
    const float4 g = __ldg(reinterpret_cast<const float4*>(gr + c));
    acc += g.x * wload<W>(w, c) * v.x + g.y * wload<W>(w, c + 1) * v.y +
           g.z * wload<W>(w, c + 2) * v.z + g.w * wload<W>(w, c + 3) * v.w;
  }
  const float dot = warp_sum(acc) / static_cast<float>(n_cols);
  const float k = rstd * rstd * dot;
  float* dr = dx + row * n_cols;
  for (int c = lane * 4; c < n_cols; c += 128) {
    const float4 v = __ldg(reinterpret_cast<const float4*>(xr + c));
    const float4 g = __ldg(reinterpret_cast<const float4*>(gr + c));
    float4 o;
    o.x = rstd * (g.x * wload<W>(w, c) - v.x * k);
    o.y = rstd * (g.y * wload<W>(w, c + 1) - v.y * k);
    o.z = rstd * (g.z * wload<W>(w, c + 2) - v.z * k);
    o.w = rstd * (g.w * wload<W>(w, c + 3) - v.w * k);
    *reinterpret_cast<float4*>(dr + c) = o;
  }
}

}  // namespace
}  // namespace decik

extern "C" int decik_rmsnorm_fwd(const float* x, const void* w, int w_dtype, float* y, float* rstd,
                                 int64_t n_rows, int n_cols, int64_t stride_x, int64_t stride_y,
                                 float eps, void* stream) {
  using namespace decik;
  if (n_rows == 0) return DECIK_OK;
  if (n_rows < 0 || n_cols <= 0 || n_cols % 4 != 0 || n_cols > kMaxCols || stride_x % 4 || stride_y % 4)
    return set_error(DECIK_ERR_INVALID, "rmsnorm_fwd: n_cols %d (multiple of 4, <= 8192), strides multiples of 4", n_cols);
  if (!x || !w || !y) return set_error(DECIK_ERR_INVALID, "rmsnorm_fwd: null pointer");
  if (!aligned16(x) || !aligned16(y)) return set_error(DECIK_ERR_INVALID, "rmsnorm_fwd: x, y must be 16-byte aligned");
  const int grid = static_cast<int>((n_rows + 7) / 8);
  if (w_dtype == DECIK_F32)
    rmsnorm_fwd_kernel<float><<<grid, 256, 0, as_stream(stream)>>>(x, static_cast<const float*>(w), y, rstd, n_rows, n_cols, stride_x, stride_y, eps);
  else if (w_dtype == DECIK_F16)
    rmsnorm_fwd_kernel<__half><<<grid, 256, 0, as_stream(stream)>>>(x, static_cast<const __half*>(w), y, rstd, n_rows, n_cols, stride_x, stride_y, eps);
  else
    return set_error(DECIK_ERR_INVALID, "rmsnorm_fwd: w_dtype must be F32 or F16");
  return check_launch("rmsnorm_fwd");
}

extern "C" int decik_rmsnorm_bwd(const float* dy, const float* x, const void* w, int w_dtype,
                                 const float* rstd, float* dx, int64_t n_rows, int n_cols,
                                 void* stream) {
  using namespace decik;
  if (n_rows == 0) return DECIK_OK;
  if (n_rows < 0 || n_cols <= 0 || n_cols % 4 != 0 || n_cols > kMaxCols)
    return set_error(DECIK_ERR_INVALID, "rmsnorm_bwd: n_cols %d", n_cols);
  if (!dy || !x || !w || !rstd || !dx) return set_error(DECIK_ERR_INVALID, "rmsnorm_bwd: null pointer");
  if (!aligned16(dy) || !aligned16(x) || !aligned16(dx))
    return set_error(DECIK_ERR_INVALID, "rmsnorm_bwd: dy, x, dx must be 16-byte aligned");
  const int grid = static_cast<int>((n_rows + 7) / 8);
  if (w_dtype == DECIK_F32)
    rmsnorm_bwd_kernel<float><<<grid, 256, 0, as_stream(stream)>>>(dy, x, static_cast<const float*>(w), rstd, dx, n_rows, n_cols);
  else if (w_dtype == DECIK_F16)
    rmsnorm_bwd_kernel<__half><<<grid, 256, 0, as_stream(stream)>>>(dy, x, static_cast<const __half*>(w), rstd, dx, n_rows, n_cols);
  else
    return set_error(DECIK_ERR_INVALID, "rmsnorm_bwd: w_dtype must be F32 or F16");
  return check_launch("rmsnorm_bwd");
}
