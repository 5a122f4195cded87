// SwiGLU of the Qwen2 MLP, silu(gate) * up, forward and backward, for the fused MLP node that
// replaces the reference's RecomputedMLP (solution/mlp.py:62-110) and its SwiGLU kernels
// (solution/swiglu.py:15-37). gate and up are the two halves of one projection output
// gu = x16 . [W_gate; W_up]^T ([T, 2 * inter], row stride ld), in the compute dtype; the
// arithmetic is fp32, rounded once to the compute dtype:
//   forward   s = sigmoid(g), out = g * s * u
//   backward  dup = grad * g * s, dgate = grad * u * s * (1 + g * (1 - s))
// (the same expressions and order as the reference). dgate and dup are written into one
// [T, 2 * inter] buffer laid out like gu, the operand of one dX = dgu . [W_gate; W_up] GEMM.
// HBM-bound: 8 elements (16 bytes) per load, grid-stride over rows x 8-column groups (the forward
// takes two groups per step so that four loads are in flight per thread).
#include "common.cuh"
#include "swiglu_math.cuh"

namespace decik {
namespace {

template <typename T>
__device__ __forceinline__ void load8(const T* p, float (&f)[8]) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = Dt<T>::lo_f(w[i]);
    f[2 * i + 1] = Dt<T>::hi_f(w[i]);
  }
}
template <typename T>
__device__ __forceinline__ void store8(T* p, const float (&f)[8]) {
  *reinterpret_cast<uint4*>(p) = make_uint4(Dt<T>::pack2(f[0], f[1]), Dt<T>::pack2(f[2], f[3]),
                                            Dt<T>::pack2(f[4], f[5]), Dt<T>::pack2(f[6], f[7]));
}
using swiglu::sigmoid;

template <typename T>
__global__ void __launch_bounds__(256) swiglu_fwd_kernel(const T* __restrict__ gu, int64_t ld, T* __restrict__ out,
                                                          int64_t ldo, int64_t n_rows, int inter) {
  const int groups = inter / 8;
  const int64_t total = n_rows * groups;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  // two 8-column groups per step, their four loads issued before any arithmetic
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total; i += 2 * stride) {
    const int64_t j = i + stride;
    const bool two = j < total;
    const int64_t row0 = i / groups, row1 = two ? j / groups : row0;
    const int c0 = static_cast<int>(i - row0 * groups) * 8;
    const int c1 = two ? static_cast<int>(j - row1 * groups) * 8 : c0;
    float g0[8], u0[8], g1[8], u1[8], o[8];
    load8<T>(gu + row0 * ld + c0, g0);
    load8<T>(gu + row0 * ld + inter + c0, u0);
    load8<T>(gu + row1 * ld + c1, g1);
    load8<T>(gu + row1 * ld + inter + c1, u1);
#pragma unroll
    for (int e = 0; e < 8; ++e) o[e] = g0[e] * sigmoid(g0[e]) * u0[e];
    store8<T>(out + row0 * ldo + c0, o);
    if (two) {
#pragma unroll
      for (int e = 0; e < 8; ++e) o[e] = g1[e] * sigmoid(g1[e]) * u1[e];
      store8<T>(out + row1 * ldo + c1, o);
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(256) swiglu_bwd_kernel(const T* __restrict__ grad, int64_t ldg,
                                                          const T* __restrict__ gu, int64_t ld, T* __restrict__ dgu,
                                                          int64_t ldd, int64_t n_rows, int inter) {
  const int groups = inter / 8;
  const int64_t total = n_rows * groups;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t row = i / groups;
    const int c = static_cast<int>(i - row * groups) * 8;
    float gr[8], g[8], u[8], dg[8], du[8];
    load8<T>(grad + row * ldg + c, gr);
    load8<T>(gu + row * ld + c, g);
    load8<T>(gu + row * ld + inter + c, u);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float s = sigmoid(g[e]);
      du[e] = gr[e] * g[e] * s;
      dg[e] = gr[e] * u[e] * s * (1.0f + g[e] * (1.0f - s));
    }
    store8<T>(dgu + row * ldd + c, dg);
    store8<T>(dgu + row * ldd + inter + c, du);
  }
}

int grid_for(int64_t work) {
  const int64_t blocks = (work + 255) / 256;
  const int64_t cap = static_cast<int64_t>(sm_count()) * 8;  // 8 resident 256-thread CTAs per SM
  return static_cast<int>(blocks < cap ? (blocks > 0 ? blocks : 1) : cap);
}

bool aligned_rows(const void* p, int64_t ld) { return aligned16(p) && (ld % 8) == 0; }

}  // namespace
}  // namespace decik

extern "C" int decik_swiglu_fwd(const void* gu, int64_t ld, void* out, int64_t ldo, int64_t n_rows, int inter,
                                int dtype, void* stream) {
  using namespace decik;
  if (n_rows == 0) return DECIK_OK;
  if (n_rows < 0 || inter <= 0 || inter % 8 != 0 || ld < 2 * static_cast<int64_t>(inter) || ldo < inter)
    return set_error(DECIK_ERR_INVALID, "swiglu_fwd: inter %d (multiple of 8), ld %lld >= 2 inter, ldo %lld >= inter",
                     inter, (long long)ld, (long long)ldo);
  if (!gu || !out) return set_error(DECIK_ERR_INVALID, "swiglu_fwd: null pointer");
  if (!aligned_rows(gu, ld) || !aligned_rows(out, ldo))
    return set_error(DECIK_ERR_INVALID, "swiglu_fwd: rows must start 16-byte aligned");
  const int grid = grid_for(n_rows * (inter / 8));
  return DECIK_DISPATCH_16(dtype, [&] {
    swiglu_fwd_kernel<T><<<grid, 256, 0, as_stream(stream)>>>(static_cast<const T*>(gu), ld, static_cast<T*>(out),
                                                               ldo, n_rows, inter);
    return check_launch("swiglu_fwd");
  });
}

extern "C" int decik_swiglu_bwd(const void* grad, int64_t ldg, const void* gu, int64_t ld, void* dgu, int64_t ldd,
                                int64_t n_rows, int inter, int dtype, void* stream) {
  using namespace decik;
  if (n_rows == 0) return DECIK_OK;
  if (n_rows < 0 || inter <= 0 || inter % 8 != 0 || ld < 2 * static_cast<int64_t>(inter) ||
      ldd < 2 * static_cast<int64_t>(inter) || ldg < inter)
    return set_error(DECIK_ERR_INVALID, "swiglu_bwd: inter %d (multiple of 8), ld / ldd >= 2 inter, ldg >= inter", inter);
  if (!grad || !gu || !dgu) return set_error(DECIK_ERR_INVALID, "swiglu_bwd: null pointer");
  if (!aligned_rows(grad, ldg) || !aligned_rows(gu, ld) || !aligned_rows(dgu, ldd))
    return set_error(DECIK_ERR_INVALID, "swiglu_bwd: rows must start 16-byte aligned");
  const int grid = grid_for(n_rows * (inter / 8));
  return DECIK_DISPATCH_16(dtype, [&] {
    swiglu_bwd_kernel<T><<<grid, 256, 0, as_stream(stream)>>>(static_cast<const T*>(grad), ldg,
                                                               static_cast<const T*>(gu), ld, static_cast<T*>(dgu),
                                                               ldd, n_rows, inter);
    return check_launch("swiglu_bwd");
  });
}
