// LoRA add + RoPE + cast to head-major (forward) and its transpose (backward), bit-exact with the
// reference's skc_rope_fwd_kernel / skc_rope_bwd_kernel (solution/attn.py:28-90).
//
// HBM-bound. One thread owns 8 dims d in [8c, 8c+8) of one (token, head) together with their
// rotation partners d + D/2, so every input is read once with 16-byte loads (q_base, q_lora, k,
// and the fp32 cos/sin rows) and every output written once with 16-byte stores. All products and
// sums are rounded one at a time (__fmul_rn / __fadd_rn), as the reference kernels run with
// enable_fp_fusion=False.
#include "common.cuh"

namespace decik {
namespace {

__device__ __forceinline__ void load8f(const float* p, float (&f)[8]) {
  const float4 a = __ldg(reinterpret_cast<const float4*>(p));
  const float4 b = __ldg(reinterpret_cast<const float4*>(p) + 1);
  f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w;
  f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
}

// Work item w -> (token, head, chunk) over q heads then k heads.
template <typename T>
__global__ void __launch_bounds__(256)
rope_fwd_kernel(const T* __restrict__ qb, const T* __restrict__ ql, const T* __restrict__ kin,
                const float* __restrict__ cosp, const float* __restrict__ sinp, T* __restrict__ qo,
                T* __restrict__ ko, int64_t n_tok, int hq, int hk, int D) {
  const int half = D >> 1;
  const int chunks = half >> 3;
  const int heads = hq + hk;
  const int64_t total = n_tok * heads * chunks;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t w = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; w < total; w += stride) {
    const int c = static_cast<int>(w % chunks);
    const int64_t th = w / chunks;
    const int h = static_cast<int>(th % heads);
    const int64_t t = th / heads;
    const int d_lo = c * 8;
    const int d_hi = half + c * 8;
    float x_lo[8], x_hi[8];
    const bool is_q = h < hq;
    if (is_q) {
      const int64_t base = t * (static_cast<int64_t>(hq) * D) + static_cast<int64_t>(h) * D;
      unpack8<T>(ldg16(qb + base + d_lo), x_lo);
      unpack8<T>(ldg16(qb + base + d_hi), x_hi);
      if (ql != nullptr) {
        float l_lo[8], l_hi[8];
        unpack8<T>(ldg16(ql + base + d_lo), l_lo);
        unpack8<T>(ldg16(ql + base + d_hi), l_hi);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          x_lo[i] = __fadd_rn(x_lo[i], l_lo[i]);
          x_hi[i] = __fadd_rn(x_hi[i], l_hi[i]);
        }
      }
    } else {
      const int hk_i = h - hq;
      const int64_t base = t * (static_cast<int64_t>(hk) * D) + static_cast<int64_t>(hk_i) * D;
      unpack8<T>(ldg16(kin + base + d_lo), x_lo);
      unpack8<T>(ldg16(kin + base + d_hi), x_hi);
    }
    float c_lo[8], c_hi[8], s_lo[8], s_hi[8];
    load8f(cosp + t * D + d_lo, c_lo);
    load8f(cosp + t * D + d_hi, c_hi);
    load8f(sinp + t * D + d_lo, s_lo);
    load8f(sinp + t * D + d_hi, s_hi);
    float o_lo[8], o_hi[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      // d < D/2: rot = -x[d + D/2];  d >= D/2: rot = x[d - D/2]   (solution/attn.py:45-46)
      o_lo[i] = __fadd_rn(__fmul_rn(x_lo[i], c_lo[i]), __fmul_rn(-x_hi[i], s_lo[i]));
      o_hi[i] = __fadd_rn(__fmul_rn(x_hi[i], c_hi[i]), __fmul_rn(x_lo[i], s_hi[i]));
    }
    T* dst = is_q ? qo + (static_cast<int64_t>(h) * n_tok + t) * D
                  : ko + (static_cast<int64_t>(h - hq) * n_tok + t) * D;
    stg16(dst + d_lo, pack8<T>(o_lo));
    stg16(dst + d_hi, pack8<T>(o_hi));
  }
}

template <typename T>
__global__ void __launch_bounds__(256)
rope_bwd_kernel(const T* __restrict__ gq, const T* __restrict__ gk, const float* __restrict__ cosp,
                const float* __restrict__ sinp, T* __restrict__ dq, T* __restrict__ dk,
                int64_t n_tok, int hq, int hk, int D) {
  const int half = D >> 1;
  const int chunks = half >> 3;
  const int heads = hq + hk;
  const int64_t total = n_tok * heads * chunks;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t w = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; w < total; w += stride) {
    const int c = static_cast<int>(w % chunks);
    const int64_t th = w / chunks;
    const int h = static_cast<int>(th % heads);
    const int64_t t = th / heads;
    const int d_lo = c * 8;
    const int d_hi = half + c * 8;
    const bool is_q = h < hq;
    const T* src = is_q ? gq + (static_cast<int64_t>(h) * n_tok + t) * D
                        : gk + (static_cast<int64_t>(h - hq) * n_tok + t) * D;
    float g_lo[8], g_hi[8];
    unpack8<T>(ldg16(src + d_lo), g_lo);
    unpack8<T>(ldg16(src + d_hi), g_hi);
    float c_lo[8], c_hi[8], s_lo[8], s_hi[8];
    load8f(cosp + t * D + d_lo, c_lo);
    load8f(cosp + t * D + d_hi, c_hi);
    load8f(sinp + t * D + d_lo, s_lo);
    load8f(sinp + t * D + d_hi, s_hi);
    float o_lo[8], o_hi[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      // a = g[d] * cos[d];  b = g[dj] * sin[dj], dj = (d + D/2) % D;  a + (d < D/2 ? b : -b)
      o_lo[i] = __fadd_rn(__fmul_rn(g_lo[i], c_lo[i]), __fmul_rn(g_hi[i], s_hi[i]));
      o_hi[i] = __fadd_rn(__fmul_rn(g_hi[i], c_hi[i]), -__fmul_rn(g_lo[i], s_lo[i]));
    }
    T* dst = is_q ? dq + t * (static_cast<int64_t>(hq) * D) + static_cast<int64_t>(h) * D
                  : dk + t * (static_cast<int64_t>(hk) * D) + static_cast<int64_t>(h - hq) * D;
    stg16(dst + d_lo, pack8<T>(o_lo));
    stg16(dst + d_hi, pack8<T>(o_hi));
  }
}

int grid_for(int64_t items) {
  const int64_t want = (items + 255) / 256;
  const int64_t cap = static_cast<int64_t>(sm_count()) * 16;
  return static_cast<int>(want < 1 ? 1 : (want < cap ? want : cap));
}

}  // namespace
}  // namespace decik

extern "C" int decik_rope_fwd(const void* q_base, const void* q_lora, const void* k,
                              const float* cos, const float* sin, void* q_out, void* k_out,
                              int64_t n_tok, int n_heads, int n_kv, int head_dim, int dtype,
                              void* stream) {
  using namespace decik;
  if (n_tok == 0) return DECIK_OK;
  if (n_tok < 0 || n_heads <= 0 || n_kv < 0 || head_dim <= 0 || head_dim % 16 != 0)
    return set_error(DECIK_ERR_INVALID, "rope_fwd: bad sizes (T=%lld, H=%d, Hk=%d, D=%d)",
                     (long long)n_tok, n_heads, n_kv, head_dim);
  if (!q_base || !cos || !sin || !q_out || (n_kv > 0 && (!k || !k_out)))
    return set_error(DECIK_ERR_INVALID, "rope_fwd: null pointer");
  if (!aligned16(q_base) || (q_lora && !aligned16(q_lora)) || (k && !aligned16(k)) ||
      !aligned16(cos) || !aligned16(sin) || !aligned16(q_out) || (k_out && !aligned16(k_out)))
    return set_error(DECIK_ERR_INVALID, "rope_fwd: pointers must be 16-byte aligned");
  const int64_t items = n_tok * (n_heads + n_kv) * (head_dim / 16);
  return DECIK_DISPATCH_16(dtype, [&] {
    rope_fwd_kernel<T><<<grid_for(items), 256, 0, as_stream(stream)>>>(
        static_cast<const T*>(q_base), static_cast<const T*>(q_lora), static_cast<const T*>(k), cos,
        sin, static_cast<T*>(q_out), static_cast<T*>(k_out), n_tok, n_heads, n_kv, head_dim);
    return check_launch("rope_fwd");
  });
}

extern "C" int decik_rope_bwd(const void* grad_q, const void* grad_k, const float* cos,
                              const float* sin, void* dq, void* dk, int64_t n_tok, int n_heads,
                              int n_kv, int head_dim, int dtype, void* stream) {
  using namespace decik;
  if (n_tok == 0) return DECIK_OK;
  if (n_tok < 0 || n_heads <= 0 || n_kv < 0 || head_dim <= 0 || head_dim % 16 != 0)
    return set_error(DECIK_ERR_INVALID, "rope_bwd: bad sizes");
  if (!grad_q || !cos || !sin || !dq || (n_kv > 0 && (!grad_k || !dk)))
    return set_error(DECIK_ERR_INVALID, "rope_bwd: null pointer");
  if (!aligned16(grad_q) || (grad_k && !aligned16(grad_k)) || !aligned16(cos) ||
      !aligned16(sin) || !aligned16(dq) || (dk && !aligned16(dk)))
    return set_error(DECIK_ERR_INVALID, "rope_bwd: pointers must be 16-byte aligned");
  const int64_t items = n_tok * (n_heads + n_kv) * (head_dim / 16);
  return DECIK_DISPATCH_16(dtype, [&] {
    rope_bwd_kernel<T><<<grid_for(items), 256, 0, as_stream(stream)>>>(
        static_cast<const T*>(grad_q), static_cast<const T*>(grad_k), cos, sin,
        static_cast<T*>(dq), static_cast<T*>(dk), n_tok, n_heads, n_kv, head_dim);
    return check_launch("rope_bwd");
  });
}
