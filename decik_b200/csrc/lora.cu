// LoRA dropout helpers, bit-exact with the reference's Triton kernels (solution/attn.py:130-180):
// keep-mask bit packing, the masked fp16/bf16 LoRA inputs, and the LoRA input gradient through
// both masks. All HBM-bound; each thread handles 8 consecutive columns (one mask byte).
#include "common.cuh"

namespace decik {
namespace {

__global__ void __launch_bounds__(256)
keep_pack_kernel(const uint8_t* __restrict__ kq, const uint8_t* __restrict__ kv,
                 uint8_t* __restrict__ bq, uint8_t* __restrict__ bv, int64_t n_bytes_out) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n_bytes_out; i += stride) {
    uint32_t aq = 0, av = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) {  // bit j of byte i = keep[8i + j] (solution/attn.py:139-141)
      aq |= (kq[8 * i + j] ? 1u : 0u) << j;
      av |= (kv[8 * i + j] ? 1u : 0u) << j;
    }
    bq[i] = static_cast<uint8_t>(aq);
    bv[i] = static_cast<uint8_t>(av);
  }
}

template <typename T>
__global__ void __launch_bounds__(256)
lora_inputs_kernel(const float* __restrict__ x, const uint8_t* __restrict__ bq,
                   const uint8_t* __restrict__ bv, const float* __restrict__ sq,
                   const float* __restrict__ sv, T* __restrict__ xq, T* __restrict__ xv,
                   int64_t n_groups) {
  const float scale_q = __ldg(sq), scale_v = __ldg(sv);
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t g = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; g < n_groups; g += stride) {
    const float4 a = __ldg(reinterpret_cast<const float4*>(x + 8 * g));
    const float4 b = __ldg(reinterpret_cast<const float4*>(x + 8 * g) + 1);
    const float xs[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
    const uint32_t mq = bq[g], mv = bv[g];
    float oq[8], ov[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {  // x * (keep * scale), each product rounded (:162-165)
      oq[j] = __fmul_rn(xs[j], __fmul_rn(static_cast<float>((mq >> j) & 1u), scale_q));
      ov[j] = __fmul_rn(xs[j], __fmul_rn(static_cast<float>((mv >> j) & 1u), scale_v));
    }
    stg16(xq + 8 * g, pack8<T>(oq));
    stg16(xv + 8 * g, pack8<T>(ov));
  }
}

template <typename T>
__global__ void __launch_bounds__(256)
lora_input_grad_kernel(const T* __restrict__ gq, const T* __restrict__ gv,
                       const uint8_t* __restrict__ bq, const uint8_t* __restrict__ bv,
                       float* __restrict__ out, float scale_q, float scale_v, int64_t n_groups) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t g = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; g < n_groups; g += stride) {
    float fq[8], fv[8];
    unpack8<T>(ldg16(gq + 8 * g), fq);
    unpack8<T>(ldg16(gv + 8 * g), fv);
    const uint32_t mq = bq[g], mv = bv[g];
    float o[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {  // (g_q * keep) * s_q + (g_v * keep) * s_v (:176-180)
      const float tq = __fmul_rn(__fmul_rn(fq[j], static_cast<float>((mq >> j) & 1u)), scale_q);
      const float tv = __fmul_rn(__fmul_rn(fv[j], static_cast<float>((mv >> j) & 1u)), scale_v);
      o[j] = __fadd_rn(tq, tv);
    }
    reinterpret_cast<float4*>(out + 8 * g)[0] = make_float4(o[0], o[1], o[2], o[3]);
    reinterpret_cast<float4*>(out + 8 * g)[1] = make_float4(o[4], o[5], o[6], o[7]);
  }
}

int grid_for(int64_t items) {
  const int64_t want = (items + 255) / 256;
  const int64_t cap = static_cast<int64_t>(sm_count()) * 16;
  return static_cast<int>(want < 1 ? 1 : (want < cap ? want : cap));
}

}  // namespace
}  // namespace decik

extern "C" int decik_keep_pack(const uint8_t* keep_q, const uint8_t* keep_v, uint8_t* bits_q,
                               uint8_t* bits_v, int64_t n_rows, int width, void* stream) {
  using namespace decik;
  if (n_rows == 0) return DECIK_OK;
  if (n_rows < 0 || width <= 0 || width % 8 != 0)
    return set_error(DECIK_ERR_INVALID, "keep_pack: width %d must be a positive multiple of 8", width);
  if (!keep_q || !keep_v || !bits_q || !bits_v) return set_error(DECIK_ERR_INVALID, "keep_pack: null pointer");
  const int64_t n = n_rows * (width / 8);
  keep_pack_kernel<<<grid_for(n), 256, 0, as_stream(stream)>>>(keep_q, keep_v, bits_q, bits_v, n);
  return check_launch("keep_pack");
}

extern "C" int decik_lora_inputs(const float* x, const uint8_t* bits_q, const uint8_t* bits_v,
                                 const float* scale_q, const float* scale_v, void* xq, void* xv,
                                 int64_t n_rows, int width, int out_dtype, void* stream) {
  using namespace decik;
  if (n_rows == 0) return DECIK_OK;
  if (n_rows < 0 || width <= 0 || width % 8 != 0)
    return set_error(DECIK_ERR_INVALID, "lora_inputs: width %d must be a positive multiple of 8", width);
  if (!x || !bits_q || !bits_v || !scale_q || !scale_v || !xq || !xv)
    return set_error(DECIK_ERR_INVALID, "lora_inputs: null pointer");
  if (!aligned16(x) || !aligned16(xq) || !aligned16(xv))
    return set_error(DECIK_ERR_INVALID, "lora_inputs: x, xq, xv must be 16-byte aligned");
  const int64_t n = n_rows * (width / 8);
  return DECIK_DISPATCH_16(out_dtype, [&] {
    lora_inputs_kernel<T><<<grid_for(n), 256, 0, as_stream(stream)>>>(
        x, bits_q, bits_v, scale_q, scale_v, static_cast<T*>(xq), static_cast<T*>(xv), n);
    return check_launch("lora_inputs");
  });
}

extern "C" int decik_lora_input_grad(const void* g_q, const void* g_v, const uint8_t* bits_q,
                                     const uint8_t* bits_v, float* out, int64_t n_rows, int width,
                                     float scale_q, float scale_v, int in_dtype, void* stream) {
  using namespace decik;
  if (n_rows == 0) return DECIK_OK;
  if (n_rows < 0 || width <= 0 || width % 8 != 0)
    return set_error(DECIK_ERR_INVALID, "lora_input_grad: width %d must be a positive multiple of 8", width);
  if (!g_q || !g_v || !bits_q || !bits_v || !out)
    return set_error(DECIK_ERR_INVALID, "lora_input_grad: null pointer");
  if (!aligned16(g_q) || !aligned16(g_v) || !aligned16(out))
    return set_error(DECIK_ERR_INVALID, "lora_input_grad: g_q, g_v, out must be 16-byte aligned");
  const int64_t n = n_rows * (width / 8);
  return DECIK_DISPATCH_16(in_dtype, [&] {
    lora_input_grad_kernel<T><<<grid_for(n), 256, 0, as_stream(stream)>>>(
        static_cast<const T*>(g_q), static_cast<const T*>(g_v), bits_q, bits_v, out, scale_q,
        scale_v, n);
    return check_launch("lora_input_grad");
  });
}
