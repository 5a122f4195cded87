// Qwen2RMSNorm forward and backward over fp32 rows (solution/rmsnorm.py:17-45). The forward is
// also the norm_link recompute of the LoRA input in the block's backward (solution/attn.py:238):
// the same kernel on the same input gives bit-identical output.
//
// One warp per row; each lane reads 4 consecutive floats per step (16-byte loads) and the row
// reductions (mean of x^2, mean of g*x) are warp-shuffle trees.
//
// The decoder's residual add + post-attention norm (AddRMSNormFn, solution/rmsnorm.py:108-144,
// called from the patched decoder layer, solution/varlen.py:323-337) is one pass each way:
// forward h = residual + f32(delta), y = norm(h), writing h, y and rstd; backward rebuilds h from
// residual and delta (h is not kept, as in the reference), then total = grad_h + norm_bwd(dy, h)
// and its copy in delta's 16-bit type. The per-element and per-row arithmetic is the same source
// as the plain kernels (sumsq4 / wdot4 / the output lines), so y and the norm gradient equal
// rmsnorm_fwd / rmsnorm_bwd applied to the same h bit for bit.
#include <type_traits>

#include "common.cuh"
#include "norm_math.cuh"

namespace decik {
namespace {

using norm::norm_grad4;
using norm::norm_out4;
using norm::sumsq4;
using norm::warp_sum;
using norm::wdot4;
using norm::wload;

constexpr int kMaxCols = 8192;

// four consecutive values of the delta operand as fp32, and four fp32 values stored in its type
template <typename D>
__device__ __forceinline__ float4 dload4(const D* p);
template <> __device__ __forceinline__ float4 dload4<float>(const float* p) {
  return __ldg(reinterpret_cast<const float4*>(p));
}
template <typename D>
__device__ __forceinline__ float4 dload4(const D* p) {
  const uint2 u = __ldg(reinterpret_cast<const uint2*>(p));
  return make_float4(Dt<D>::lo_f(u.x), Dt<D>::hi_f(u.x), Dt<D>::lo_f(u.y), Dt<D>::hi_f(u.y));
}
template <typename D>
__device__ __forceinline__ void dstore4(D* p, float4 v);
template <> __device__ __forceinline__ void dstore4<float>(float* p, float4 v) {
  *reinterpret_cast<float4*>(p) = v;
}
template <typename D>
__device__ __forceinline__ void dstore4(D* p, float4 v) {
  *reinterpret_cast<uint2*>(p) = make_uint2(Dt<D>::pack2(v.x, v.y), Dt<D>::pack2(v.z, v.w));
}
// residual + f32(delta), one fp32 rounding per element (the reference's fp32 + fp16 add)
__device__ __forceinline__ float4 add4(float4 r, float4 d) {
  return make_float4(__fadd_rn(r.x, d.x), __fadd_rn(r.y, d.y), __fadd_rn(r.z, d.z), __fadd_rn(r.w, d.w));
}

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
  for (int c = lane * 4; c < n_cols; c += 128) acc += sumsq4(__ldg(reinterpret_cast<const float4*>(xr + c)));
  const float rstd = norm::row_rstd(acc, n_cols, eps);
  float* yr = y + row * sy;
  for (int c = lane * 4; c < n_cols; c += 128)
    *reinterpret_cast<float4*>(yr + c) = norm_out4<W>(__ldg(reinterpret_cast<const float4*>(xr + c)), w, c, rstd);
  if (rstd_out != nullptr && lane == 0) rstd_out[row] = rstd;
}

template <typename W>
__global__ void __launch_bounds__(256)
rmsnorm_bwd_kernel(const float* __restrict__ dy, const float* __restrict__ x,
                   const W* __restrict__ w, const float* __restrict__ rstd_in, const float* __restrict__ addend,
                   float* __restrict__ dx, int64_t n_rows, int n_cols) {
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= n_rows) return;
  const float* xr = x + row * n_cols;
  const float* gr = dy + row * n_cols;
  const float rstd = rstd_in[row];
  float acc = 0.f;
  for (int c = lane * 4; c < n_cols; c += 128)
    acc += wdot4<W>(__ldg(reinterpret_cast<const float4*>(gr + c)), __ldg(reinterpret_cast<const float4*>(xr + c)), w, c);
  const float dot = warp_sum(acc) / static_cast<float>(n_cols);
  const float k = rstd * rstd * dot;
  float* dr = dx + row * n_cols;
  for (int c = lane * 4; c < n_cols; c += 128) {
    float4 o = norm_grad4<W>(__ldg(reinterpret_cast<const float4*>(gr + c)), __ldg(reinterpret_cast<const float4*>(xr + c)),
                             w, c, rstd, k);
    if (addend != nullptr) o = add4(__ldg(reinterpret_cast<const float4*>(addend + row * n_cols + c)), o);
    *reinterpret_cast<float4*>(dr + c) = o;
  }
}

// h = residual + f32(delta); y = w * (h * rstd) stored as Y (fp32, or delta's 16-bit type for a
// consumer that computes in it: the same rounding as casting the fp32 y); rows contiguous
template <typename W, typename D, typename Y>
__global__ void __launch_bounds__(256)
add_rmsnorm_fwd_kernel(const float* __restrict__ residual, const D* __restrict__ delta, const W* __restrict__ w,
                       float* __restrict__ h, Y* __restrict__ y, float* __restrict__ rstd_out, int64_t n_rows,
                       int n_cols, float eps) {
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= n_rows) return;
  const int64_t off = row * n_cols;
  float acc = 0.f;
  for (int c = lane * 4; c < n_cols; c += 128) {
    const float4 v = add4(__ldg(reinterpret_cast<const float4*>(residual + off + c)), dload4<D>(delta + off + c));
    *reinterpret_cast<float4*>(h + off + c) = v;
    acc += sumsq4(v);
  }
  const float rstd = norm::row_rstd(acc, n_cols, eps);
  for (int c = lane * 4; c < n_cols; c += 128) {
    const float4 v = add4(__ldg(reinterpret_cast<const float4*>(residual + off + c)), dload4<D>(delta + off + c));
    dstore4<Y>(y + off + c, norm_out4<W>(v, w, c, rstd));
  }
  if (rstd_out != nullptr && lane == 0) rstd_out[row] = rstd;
}

// total = grad_h + norm_bwd(dy, h) with h = residual + f32(delta) rebuilt; total in fp32 and,
// when dx16 is set, in delta's type (the delta input's gradient); dy of type G (fp32, or the 16-bit
// gradient of a 16-bit y)
template <typename W, typename D, typename G>
__global__ void __launch_bounds__(256)
add_rmsnorm_bwd_kernel(const G* __restrict__ dy, const float* __restrict__ grad_h,
                       const float* __restrict__ residual, const D* __restrict__ delta, const W* __restrict__ w,
                       const float* __restrict__ rstd_in, float* __restrict__ dx, D* __restrict__ dx16,
                       int64_t n_rows, int n_cols) {
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= n_rows) return;
  const int64_t off = row * n_cols;
  const float rstd = rstd_in[row];
  float acc = 0.f;
  for (int c = lane * 4; c < n_cols; c += 128) {
    const float4 v = add4(__ldg(reinterpret_cast<const float4*>(residual + off + c)), dload4<D>(delta + off + c));
    acc += wdot4<W>(dload4<G>(dy + off + c), v, w, c);
  }
  const float dot = warp_sum(acc) / static_cast<float>(n_cols);
  const float k = rstd * rstd * dot;
  for (int c = lane * 4; c < n_cols; c += 128) {
    const float4 v = add4(__ldg(reinterpret_cast<const float4*>(residual + off + c)), dload4<D>(delta + off + c));
    float4 o = norm_grad4<W>(dload4<G>(dy + off + c), v, w, c, rstd, k);
    if (grad_h != nullptr) o = add4(__ldg(reinterpret_cast<const float4*>(grad_h + off + c)), o);
    *reinterpret_cast<float4*>(dx + off + c) = o;
    if (dx16 != nullptr) dstore4<D>(dx16 + off + c, o);
  }
}

}  // namespace
// The same four kernels for rows of NC * 128 columns (NC a compile-time count): the lane keeps its
// NC 16-byte pieces of each row in registers between the reduction and the output pass instead
// of reading them again. Same per-element and per-row arithmetic in the same order as the loops
// above, so the outputs are equal bit for bit.
template <typename W, int NC>
__global__ void __launch_bounds__(256)
rmsnorm_fwd_reg_kernel(const float* __restrict__ x, const W* __restrict__ w, float* __restrict__ y,
                       float* __restrict__ rstd_out, int64_t n_rows, int64_t sx, int64_t sy, float eps) {
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= n_rows) return;
  const float* xr = x + row * sx;
  float4 v[NC];
#pragma unroll
  for (int j = 0; j < NC; ++j) v[j] = __ldg(reinterpret_cast<const float4*>(xr + lane * 4 + 128 * j));
  float acc = 0.f;
#pragma unroll
  for (int j = 0; j < NC; ++j) acc += sumsq4(v[j]);
  const float rstd = norm::row_rstd(acc, NC * 128, eps);
  float* yr = y + row * sy;
#pragma unroll
  for (int j = 0; j < NC; ++j)
    *reinterpret_cast<float4*>(yr + lane * 4 + 128 * j) = norm_out4<W>(v[j], w, lane * 4 + 128 * j, rstd);
  if (rstd_out != nullptr && lane == 0) rstd_out[row] = rstd;
}

// The backward kernels hold two register rows per thread (dy and x); uncapped they took 129-158
// registers, one 256-thread CTA per SM. Capped at two CTAs per SM (128 registers, no spills with
// fp32 weights): 70 -> 57 us (rmsnorm) and 107 -> 86 us (add + norm) at 16,384 x 1536, same bits.
template <typename W, int NC>
__global__ void __launch_bounds__(256, 2)
rmsnorm_bwd_reg_kernel(const float* __restrict__ dy, const float* __restrict__ x, const W* __restrict__ w,
                       const float* __restrict__ rstd_in, const float* __restrict__ addend, float* __restrict__ dx,
                       int64_t n_rows) {
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= n_rows) return;
  const int64_t off = row * (NC * 128);
  const float rstd = rstd_in[row];
  float4 g[NC], v[NC];
#pragma unroll
  for (int j = 0; j < NC; ++j) {
    g[j] = __ldg(reinterpret_cast<const float4*>(dy + off + lane * 4 + 128 * j));
    v[j] = __ldg(reinterpret_cast<const float4*>(x + off + lane * 4 + 128 * j));
  }
  float acc = 0.f;
#pragma unroll
  for (int j = 0; j < NC; ++j) acc += wdot4<W>(g[j], v[j], w, lane * 4 + 128 * j);
  const float dot = warp_sum(acc) / static_cast<float>(NC * 128);
  const float k = rstd * rstd * dot;
#pragma unroll
  for (int j = 0; j < NC; ++j) {
    const int c = lane * 4 + 128 * j;
    float4 o = norm_grad4<W>(g[j], v[j], w, c, rstd, k);
    if (addend != nullptr) o = add4(__ldg(reinterpret_cast<const float4*>(addend + off + c)), o);
    *reinterpret_cast<float4*>(dx + off + c) = o;
  }
}

template <typename W, typename D, typename Y, int NC>
__global__ void __launch_bounds__(256)
add_rmsnorm_fwd_reg_kernel(const float* __restrict__ residual, const D* __restrict__ delta, const W* __restrict__ w,
                           float* __restrict__ h, Y* __restrict__ y, float* __restrict__ rstd_out, int64_t n_rows,
                           float eps) {
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= n_rows) return;
  const int64_t off = row * (NC * 128);
  float4 v[NC];
#pragma unroll
  for (int j = 0; j < NC; ++j) {
    const int c = lane * 4 + 128 * j;
    v[j] = add4(__ldg(reinterpret_cast<const float4*>(residual + off + c)), dload4<D>(delta + off + c));
  }
  float acc = 0.f;
#pragma unroll
  for (int j = 0; j < NC; ++j) {
    *reinterpret_cast<float4*>(h + off + lane * 4 + 128 * j) = v[j];
    acc += sumsq4(v[j]);
  }
  const float rstd = norm::row_rstd(acc, NC * 128, eps);
#pragma unroll
  for (int j = 0; j < NC; ++j)
    dstore4<Y>(y + off + lane * 4 + 128 * j, norm_out4<W>(v[j], w, lane * 4 + 128 * j, rstd));
  if (rstd_out != nullptr && lane == 0) rstd_out[row] = rstd;
}

template <typename W, typename D, typename G, int NC>
__global__ void __launch_bounds__(256, 2)
add_rmsnorm_bwd_reg_kernel(const G* __restrict__ dy, const float* __restrict__ grad_h,
                           const float* __restrict__ residual, const D* __restrict__ delta, const W* __restrict__ w,
                           const float* __restrict__ rstd_in, float* __restrict__ dx, D* __restrict__ dx16,
                           int64_t n_rows) {
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= n_rows) return;
  const int64_t off = row * (NC * 128);
  const float rstd = rstd_in[row];
  float4 g[NC], v[NC];
#pragma unroll
  for (int j = 0; j < NC; ++j) {
    const int c = lane * 4 + 128 * j;
    v[j] = add4(__ldg(reinterpret_cast<const float4*>(residual + off + c)), dload4<D>(delta + off + c));
    g[j] = dload4<G>(dy + off + c);
  }
  float acc = 0.f;
#pragma unroll
  for (int j = 0; j < NC; ++j) acc += wdot4<W>(g[j], v[j], w, lane * 4 + 128 * j);
  const float dot = warp_sum(acc) / static_cast<float>(NC * 128);
  const float k = rstd * rstd * dot;
#pragma unroll
  for (int j = 0; j < NC; ++j) {
    const int c = lane * 4 + 128 * j;
    float4 o = norm_grad4<W>(g[j], v[j], w, c, rstd, k);
    if (grad_h != nullptr) o = add4(__ldg(reinterpret_cast<const float4*>(grad_h + off + c)), o);
    *reinterpret_cast<float4*>(dx + off + c) = o;
    if (dx16 != nullptr) dstore4<D>(dx16 + off + c, o);
  }
}

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
  const cudaStream_t st = as_stream(stream);
  if (w_dtype != DECIK_F32 && w_dtype != DECIK_F16)
    return set_error(DECIK_ERR_INVALID, "rmsnorm_fwd: w_dtype must be F32 or F16");
  const bool wf = w_dtype == DECIK_F32;
  if (n_cols == 12 * 128) {  // the 1.5B hidden size: the row stays in registers
    if (wf) rmsnorm_fwd_reg_kernel<float, 12><<<grid, 256, 0, st>>>(x, static_cast<const float*>(w), y, rstd, n_rows, stride_x, stride_y, eps);
    else rmsnorm_fwd_reg_kernel<__half, 12><<<grid, 256, 0, st>>>(x, static_cast<const __half*>(w), y, rstd, n_rows, stride_x, stride_y, eps);
  } else if (wf) {
    rmsnorm_fwd_kernel<float><<<grid, 256, 0, st>>>(x, static_cast<const float*>(w), y, rstd, n_rows, n_cols, stride_x, stride_y, eps);
  } else {
    rmsnorm_fwd_kernel<__half><<<grid, 256, 0, st>>>(x, static_cast<const __half*>(w), y, rstd, n_rows, n_cols, stride_x, stride_y, eps);
  }
  return check_launch("rmsnorm_fwd");
}

namespace decik {
namespace {

int rmsnorm_bwd_impl(const float* dy, const float* x, const void* w, int w_dtype, const float* rstd,
                     const float* addend, float* dx, int64_t n_rows, int n_cols, void* stream, const char* what) {
  if (n_rows == 0) return DECIK_OK;
  if (n_rows < 0 || n_cols <= 0 || n_cols % 4 != 0 || n_cols > kMaxCols)
    return set_error(DECIK_ERR_INVALID, "%s: n_cols %d", what, n_cols);
  if (!dy || !x || !w || !rstd || !dx) return set_error(DECIK_ERR_INVALID, "%s: null pointer", what);
  if (!aligned16(dy) || !aligned16(x) || !aligned16(dx) || (addend && !aligned16(addend)))
    return set_error(DECIK_ERR_INVALID, "%s: dy, x, addend, dx must be 16-byte aligned", what);
  const int grid = static_cast<int>((n_rows + 7) / 8);
  const cudaStream_t st = as_stream(stream);
  if (w_dtype != DECIK_F32 && w_dtype != DECIK_F16)
    return set_error(DECIK_ERR_INVALID, "%s: w_dtype must be F32 or F16", what);
  const bool wf = w_dtype == DECIK_F32;
  if (n_cols == 12 * 128) {
    if (wf) rmsnorm_bwd_reg_kernel<float, 12><<<grid, 256, 0, st>>>(dy, x, static_cast<const float*>(w), rstd, addend, dx, n_rows);
    else rmsnorm_bwd_reg_kernel<__half, 12><<<grid, 256, 0, st>>>(dy, x, static_cast<const __half*>(w), rstd, addend, dx, n_rows);
  } else if (wf) {
    rmsnorm_bwd_kernel<float><<<grid, 256, 0, st>>>(dy, x, static_cast<const float*>(w), rstd, addend, dx, n_rows, n_cols);
  } else {
    rmsnorm_bwd_kernel<__half><<<grid, 256, 0, st>>>(dy, x, static_cast<const __half*>(w), rstd, addend, dx, n_rows, n_cols);
  }
  return check_launch(what);
}

}  // namespace
}  // namespace decik

extern "C" int decik_rmsnorm_bwd(const float* dy, const float* x, const void* w, int w_dtype,
                                 const float* rstd, float* dx, int64_t n_rows, int n_cols,
                                 void* stream) {
  return decik::rmsnorm_bwd_impl(dy, x, w, w_dtype, rstd, nullptr, dx, n_rows, n_cols, stream, "rmsnorm_bwd");
}

extern "C" int decik_rmsnorm_bwd_add(const float* dy, const float* x, const void* w, int w_dtype, const float* rstd,
                                     const float* addend, float* dx, int64_t n_rows, int n_cols, void* stream) {
  return decik::rmsnorm_bwd_impl(dy, x, w, w_dtype, rstd, addend, dx, n_rows, n_cols, stream, "rmsnorm_bwd_add");
}

namespace decik {
namespace {

int add_rmsnorm_check(int64_t n_rows, int n_cols, const void* delta, int d_dtype, int w_dtype, const char* what) {
  using namespace decik;
  if (n_rows < 0 || n_cols <= 0 || n_cols % 4 != 0 || n_cols > kMaxCols)
    return set_error(DECIK_ERR_INVALID, "%s: n_cols %d (multiple of 4, <= 8192)", what, n_cols);
  if (w_dtype != DECIK_F32 && w_dtype != DECIK_F16)
    return set_error(DECIK_ERR_INVALID, "%s: w_dtype must be F32 or F16", what);
  if (d_dtype != DECIK_F32 && d_dtype != DECIK_F16 && d_dtype != DECIK_BF16)
    return set_error(DECIK_ERR_INVALID, "%s: delta dtype must be F32, F16 or BF16", what);
  const uintptr_t align = d_dtype == DECIK_F32 ? 15u : 7u;
  if (reinterpret_cast<uintptr_t>(delta) & align)
    return set_error(DECIK_ERR_INVALID, "%s: delta must be %d-byte aligned", what, static_cast<int>(align + 1));
  return DECIK_OK;
}

// Y / G: the type of y / dy, fp32 or (the 16-bit entry points) delta's type D
template <typename W, typename D, bool Y16>
void launch_add_fwd(const float* residual, const void* delta, const void* w, float* h, void* y, float* rstd,
                    int64_t n_rows, int n_cols, float eps, cudaStream_t st) {
  using Y = typename std::conditional<Y16, D, float>::type;
  if (n_cols == 12 * 128)
    add_rmsnorm_fwd_reg_kernel<W, D, Y, 12><<<static_cast<int>((n_rows + 7) / 8), 256, 0, st>>>(
        residual, static_cast<const D*>(delta), static_cast<const W*>(w), h, static_cast<Y*>(y), rstd, n_rows, eps);
  else
    add_rmsnorm_fwd_kernel<W, D, Y><<<static_cast<int>((n_rows + 7) / 8), 256, 0, st>>>(
        residual, static_cast<const D*>(delta), static_cast<const W*>(w), h, static_cast<Y*>(y), rstd, n_rows, n_cols,
        eps);
}
template <typename W, typename D, bool G16>
void launch_add_bwd(const void* dy, const float* grad_h, const float* residual, const void* delta, const void* w,
                    const float* rstd, float* dx, void* dx16, int64_t n_rows, int n_cols, cudaStream_t st) {
  using G = typename std::conditional<G16, D, float>::type;
  if (n_cols == 12 * 128)
    add_rmsnorm_bwd_reg_kernel<W, D, G, 12><<<static_cast<int>((n_rows + 7) / 8), 256, 0, st>>>(
        static_cast<const G*>(dy), grad_h, residual, static_cast<const D*>(delta), static_cast<const W*>(w), rstd, dx,
        static_cast<D*>(dx16), n_rows);
  else
    add_rmsnorm_bwd_kernel<W, D, G><<<static_cast<int>((n_rows + 7) / 8), 256, 0, st>>>(
        static_cast<const G*>(dy), grad_h, residual, static_cast<const D*>(delta), static_cast<const W*>(w), rstd, dx,
        static_cast<D*>(dx16), n_rows, n_cols);
}

}  // namespace
}  // namespace decik

namespace decik {
namespace {

template <bool Y16>
int add_rmsnorm_fwd_impl(const float* residual, const void* delta, int delta_dtype, const void* w, int w_dtype,
                         float* h, void* y, float* rstd, int64_t n_rows, int n_cols, float eps, void* stream,
                         const char* what) {
  if (n_rows == 0) return DECIK_OK;
  if (!residual || !delta || !w || !h || !y) return set_error(DECIK_ERR_INVALID, "%s: null pointer", what);
  if (int rc = add_rmsnorm_check(n_rows, n_cols, delta, delta_dtype, w_dtype, what)) return rc;
  if (Y16 && delta_dtype == DECIK_F32) return set_error(DECIK_ERR_INVALID, "%s: delta must be F16 or BF16", what);
  if (!aligned16(residual) || !aligned16(h) || (Y16 ? (reinterpret_cast<uintptr_t>(y) & 7u) != 0 : !aligned16(y)))
    return set_error(DECIK_ERR_INVALID, "%s: residual, h (16 bytes) or y (16 / 8 bytes) misaligned", what);
  const cudaStream_t st = as_stream(stream);
  const bool wf = w_dtype == DECIK_F32;
  if (delta_dtype == DECIK_F32) {
    (wf ? launch_add_fwd<float, float, false> : launch_add_fwd<__half, float, false>)(residual, delta, w, h, y, rstd,
                                                                                   n_rows, n_cols, eps, st);
  } else if (delta_dtype == DECIK_F16) {
    (wf ? launch_add_fwd<float, __half, Y16> : launch_add_fwd<__half, __half, Y16>)(residual, delta, w, h, y, rstd,
                                                                                  n_rows, n_cols, eps, st);
  } else {
    (wf ? launch_add_fwd<float, __nv_bfloat16, Y16> : launch_add_fwd<__half, __nv_bfloat16, Y16>)(
        residual, delta, w, h, y, rstd, n_rows, n_cols, eps, st);
  }
  return check_launch(what);
}

template <bool G16>
int add_rmsnorm_bwd_impl(const void* dy, const float* grad_h, const float* residual, const void* delta,
                         int delta_dtype, const void* w, int w_dtype, const float* rstd, float* dx, void* dx16,
                         int64_t n_rows, int n_cols, void* stream, const char* what) {
  if (n_rows == 0) return DECIK_OK;
  if (!dy || !residual || !delta || !w || !rstd || !dx) return set_error(DECIK_ERR_INVALID, "%s: null pointer", what);
  if (int rc = add_rmsnorm_check(n_rows, n_cols, delta, delta_dtype, w_dtype, what)) return rc;
  if (G16 && delta_dtype == DECIK_F32) return set_error(DECIK_ERR_INVALID, "%s: delta must be F16 or BF16", what);
  if ((G16 ? (reinterpret_cast<uintptr_t>(dy) & 7u) != 0 : !aligned16(dy)) || !aligned16(residual) || !aligned16(dx) ||
      (grad_h && !aligned16(grad_h)))
    return set_error(DECIK_ERR_INVALID, "%s: dy, grad_h, residual or dx misaligned", what);
  if (dx16 && (reinterpret_cast<uintptr_t>(dx16) & (delta_dtype == DECIK_F32 ? 15u : 7u)))
    return set_error(DECIK_ERR_INVALID, "%s: dx16 misaligned", what);
  const cudaStream_t st = as_stream(stream);
  const bool wf = w_dtype == DECIK_F32;
  if (delta_dtype == DECIK_F32) {
    (wf ? launch_add_bwd<float, float, false> : launch_add_bwd<__half, float, false>)(dy, grad_h, residual, delta, w,
                                                                                   rstd, dx, dx16, n_rows, n_cols, st);
  } else if (delta_dtype == DECIK_F16) {
    (wf ? launch_add_bwd<float, __half, G16> : launch_add_bwd<__half, __half, G16>)(dy, grad_h, residual, delta, w,
                                                                                  rstd, dx, dx16, n_rows, n_cols, st);
  } else {
    (wf ? launch_add_bwd<float, __nv_bfloat16, G16> : launch_add_bwd<__half, __nv_bfloat16, G16>)(
        dy, grad_h, residual, delta, w, rstd, dx, dx16, n_rows, n_cols, st);
  }
  return check_launch(what);
}

}  // namespace
}  // namespace decik

extern "C" int decik_add_rmsnorm_fwd(const float* residual, const void* delta, int delta_dtype, const void* w,
                                     int w_dtype, float* h, float* y, float* rstd, int64_t n_rows, int n_cols,
                                     float eps, void* stream) {
  return decik::add_rmsnorm_fwd_impl<false>(residual, delta, delta_dtype, w, w_dtype, h, y, rstd, n_rows, n_cols, eps,
                                            stream, "add_rmsnorm_fwd");
}

extern "C" int decik_add_rmsnorm_fwd16(const float* residual, const void* delta, int delta_dtype, const void* w,
                                       int w_dtype, float* h, void* y16, float* rstd, int64_t n_rows, int n_cols,
                                       float eps, void* stream) {
  return decik::add_rmsnorm_fwd_impl<true>(residual, delta, delta_dtype, w, w_dtype, h, y16, rstd, n_rows, n_cols, eps,
                                           stream, "add_rmsnorm_fwd16");
}

extern "C" int decik_add_rmsnorm_bwd(const float* dy, const float* grad_h, const float* residual, const void* delta,
                                     int delta_dtype, const void* w, int w_dtype, const float* rstd, float* dx,
                                     void* dx16, int64_t n_rows, int n_cols, void* stream) {
  return decik::add_rmsnorm_bwd_impl<false>(dy, grad_h, residual, delta, delta_dtype, w, w_dtype, rstd, dx, dx16, n_rows,
                                            n_cols, stream, "add_rmsnorm_bwd");
}

extern "C" int decik_add_rmsnorm_bwd16(const void* dy16, const float* grad_h, const float* residual,
                                       const void* delta, int delta_dtype, const void* w, int w_dtype,
                                       const float* rstd, float* dx, void* dx16, int64_t n_rows, int n_cols,
                                       void* stream) {
  return decik::add_rmsnorm_bwd_impl<true>(dy16, grad_h, residual, delta, delta_dtype, w, w_dtype, rstd, dx, dx16,
                                           n_rows, n_cols, stream, "add_rmsnorm_bwd16");
}
