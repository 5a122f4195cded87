// NF4 double-quant dequant, bit-exact with the reference's skc_nf4_dequant_kernel
// (solution/nf4.py:28-49) and so with bitsandbytes' dequantize_4bit.
//
// HBM-bound: per weight 0.5 B of nibbles + 1/blocksize B of absmax (+ fp32 absmax2 every
// blocksize*blocksize2 weights) are read and 2 B (fp16/bf16) written. Each thread takes 16
// packed bytes (one 16-byte load, 32 weights) per step of a grid-stride loop sized to the SM
// count, and writes 64 bytes with 16-byte stores. The 16 / 256-entry code tables sit in shared
// memory. Products and sums use __fmul_rn / __fadd_rn so that nothing is contracted to an FMA:
// scale = code2[q] * absmax2 then + offset (two roundings), w = code[nibble] * scale.
#include "common.cuh"

namespace decik {
namespace {

template <typename OutT>
struct Store32;  // writes 32 fp32 weights as OutT

template <>
struct Store32<float> {
  static __device__ __forceinline__ void run(float* out, const float (&w)[32]) {
#pragma unroll
    for (int i = 0; i < 8; ++i)
      reinterpret_cast<float4*>(out)[i] = make_float4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
  }
};

template <typename T>
struct Store32 {
  static __device__ __forceinline__ void run(T* out, const float (&w)[32]) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      uint4 v;
      v.x = Dt<T>::pack2(w[8 * i + 0], w[8 * i + 1]);
      v.y = Dt<T>::pack2(w[8 * i + 2], w[8 * i + 3]);
      v.z = Dt<T>::pack2(w[8 * i + 4], w[8 * i + 5]);
      v.w = Dt<T>::pack2(w[8 * i + 6], w[8 * i + 7]);
      reinterpret_cast<uint4*>(out)[i] = v;
    }
  }
};

template <typename OutT>
__device__ __forceinline__ OutT cvt_out(float x);
template <> __device__ __forceinline__ float cvt_out<float>(float x) { return x; }
template <> __device__ __forceinline__ __half cvt_out<__half>(float x) { return __float2half_rn(x); }
template <> __device__ __forceinline__ __nv_bfloat16 cvt_out<__nv_bfloat16>(float x) {
  return __float2bfloat16_rn(x);
}

struct Nf4Args {
  const uint8_t* packed;
  const void* absmax;
  const float* absmax2;
  const float* code2;
  const float* offset;
  const float* code;
  int64_t n_bytes;
  int blocksize;
  int blocksize2;
  int bs_shift;   // log2(blocksize) when both block sizes are powers of two (the POW2 kernels)
  int bs2_shift;  // log2(blocksize2)
};

// Up to kMaxJobs weights in one launch: grid y = job. All of a launch's jobs share the template
// flags (nested, vectorised) and the output type.
constexpr int kMaxJobs = 4;
struct Nf4Batch {
  Nf4Args a[kMaxJobs];
  void* out[kMaxJobs];
};

// Block indices: weight i is in absmax block i / blocksize and that block's absmax2 entry is
// block / blocksize2. 64-bit divisions by run-time values are long instruction sequences, so the
// POW2 kernels (both sizes powers of two, as bitsandbytes uses: 64 and 256) shift instead.
template <bool POW2>
__device__ __forceinline__ int64_t div_bs(const Nf4Args& a, int64_t i) { return POW2 ? (i >> a.bs_shift) : i / a.blocksize; }
template <bool POW2>
__device__ __forceinline__ int64_t div_bs2(const Nf4Args& a, int64_t b) { return POW2 ? (b >> a.bs2_shift) : b / a.blocksize2; }

template <bool NESTED, bool POW2>
__device__ __forceinline__ float block_scale(const Nf4Args& a, const float* s_code2, float offset,
                                             int64_t block) {
  if (NESTED) {
    const uint8_t q = __ldg(reinterpret_cast<const uint8_t*>(a.absmax) + block);
    const float s = __fmul_rn(s_code2[q], __ldg(a.absmax2 + div_bs2<POW2>(a, block)));
    return __fadd_rn(s, offset);
  }
  return __ldg(reinterpret_cast<const float*>(a.absmax) + block);
}

// VEC: 16 bytes per step (needs 16-byte aligned packed and out). Otherwise one byte per step.
template <typename OutT, bool NESTED, bool VEC, bool POW2>
__global__ void __launch_bounds__(256) nf4_dequant_kernel(const __grid_constant__ Nf4Batch bt) {
  const Nf4Args& a = bt.a[blockIdx.y];
  OutT* __restrict__ out = static_cast<OutT*>(bt.out[blockIdx.y]);
  __shared__ float s_code[16];
  __shared__ float s_code2[256];
  if (threadIdx.x < 16) s_code[threadIdx.x] = a.code[threadIdx.x];
  if (NESTED) s_code2[threadIdx.x] = a.code2[threadIdx.x];  // blockDim.x == 256
  __syncthreads();
  const float offset = NESTED ? __ldg(a.offset) : 0.f;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  const int64_t tid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (VEC) {
    const int64_t n_chunks = a.n_bytes >> 4;
    for (int64_t c = tid; c < n_chunks; c += stride) {
      const uint4 raw = ldg16(a.packed + (c << 4));
      const uint32_t words[4] = {raw.x, raw.y, raw.z, raw.w};
      float w[32];
      const int64_t first = div_bs<POW2>(a, c << 5);         // block of weight 32c
      const int64_t last = div_bs<POW2>(a, (c << 5) + 31);   // block of weight 32c + 31
      if (first == last) {  // the whole chunk in one absmax block (blocksize >= 32)
        const float scale = block_scale<NESTED, POW2>(a, s_code2, offset, first);
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const uint32_t b = (words[j >> 2] >> ((j & 3) * 8)) & 0xFFu;
          w[2 * j] = __fmul_rn(s_code[b >> 4], scale);
          w[2 * j + 1] = __fmul_rn(s_code[b & 15u], scale);
        }
      } else {
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int64_t block = div_bs<POW2>(a, ((c << 4) + j) * 2);
          const float scale = block_scale<NESTED, POW2>(a, s_code2, offset, block);
          const uint32_t b = (words[j >> 2] >> ((j & 3) * 8)) & 0xFFu;
          w[2 * j] = __fmul_rn(s_code[b >> 4], scale);
          w[2 * j + 1] = __fmul_rn(s_code[b & 15u], scale);
        }
      }
      Store32<OutT>::run(out + (c << 5), w);
    }
    // tail bytes (n_bytes % 16) by the first threads
    const int64_t tail0 = n_chunks << 4;
    for (int64_t i = tail0 + tid; i < a.n_bytes; i += stride) {
      const uint32_t b = a.packed[i];
      const float scale = block_scale<NESTED, POW2>(a, s_code2, offset, div_bs<POW2>(a, i * 2));
      out[2 * i] = cvt_out<OutT>(__fmul_rn(s_code[b >> 4], scale));
      out[2 * i + 1] = cvt_out<OutT>(__fmul_rn(s_code[b & 15u], scale));
    }
  } else {
    for (int64_t i = tid; i < a.n_bytes; i += stride) {
      const uint32_t b = a.packed[i];
      const float scale = block_scale<NESTED, POW2>(a, s_code2, offset, div_bs<POW2>(a, i * 2));
      out[2 * i] = cvt_out<OutT>(__fmul_rn(s_code[b >> 4], scale));
      out[2 * i + 1] = cvt_out<OutT>(__fmul_rn(s_code[b & 15u], scale));
    }
  }
}

template <typename OutT>
int launch(const Nf4Batch& bt, int n, bool nested, bool vec, cudaStream_t stream) {
  int64_t work = 0;
  for (int j = 0; j < n; ++j) work = std::max<int64_t>(work, vec ? (bt.a[j].n_bytes >> 4) + 1 : bt.a[j].n_bytes);
  const int64_t want = (work + 255) / 256;
  const int64_t cap = std::max<int64_t>(1, static_cast<int64_t>(sm_count()) * 8 / n);
  const dim3 grid(static_cast<unsigned>(want < cap ? (want > 0 ? want : 1) : cap), static_cast<unsigned>(n));
  bool pow2 = true;
  for (int j = 0; j < n; ++j) pow2 = pow2 && bt.a[j].bs_shift >= 0 && (!nested || bt.a[j].bs2_shift >= 0);
  if (nested) {
    if (vec) {
      if (pow2) nf4_dequant_kernel<OutT, true, true, true><<<grid, 256, 0, stream>>>(bt);
      else nf4_dequant_kernel<OutT, true, true, false><<<grid, 256, 0, stream>>>(bt);
    } else {
      if (pow2) nf4_dequant_kernel<OutT, true, false, true><<<grid, 256, 0, stream>>>(bt);
      else nf4_dequant_kernel<OutT, true, false, false><<<grid, 256, 0, stream>>>(bt);
    }
  } else {
    if (vec) {
      if (pow2) nf4_dequant_kernel<OutT, false, true, true><<<grid, 256, 0, stream>>>(bt);
      else nf4_dequant_kernel<OutT, false, true, false><<<grid, 256, 0, stream>>>(bt);
    } else {
      if (pow2) nf4_dequant_kernel<OutT, false, false, true><<<grid, 256, 0, stream>>>(bt);
      else nf4_dequant_kernel<OutT, false, false, false><<<grid, 256, 0, stream>>>(bt);
    }
  }
  return check_launch("nf4_dequant");
}

// log2(v) when v is a power of two, else -1
int log2_exact(int v) {
  if (v <= 0 || (v & (v - 1)) != 0) return -1;
  int k = 0;
  while ((1 << k) < v) ++k;
  return k;
}

int check_job(const decik_nf4_job& j) {
  if (j.n_bytes < 0) return set_error(DECIK_ERR_INVALID, "nf4_dequant: n_bytes < 0");
  if (j.n_bytes > 0 && (!j.packed || !j.absmax || !j.code || !j.out))
    return set_error(DECIK_ERR_INVALID, "nf4_dequant: null pointer");
  if (j.blocksize <= 0 || j.blocksize % 2 != 0)
    return set_error(DECIK_ERR_INVALID, "nf4_dequant: blocksize %d must be even and > 0", j.blocksize);
  if (j.nested && (!j.absmax2 || !j.code2 || !j.offset || j.blocksize2 <= 0))
    return set_error(DECIK_ERR_INVALID, "nf4_dequant: nested needs absmax2, code2, offset, blocksize2");
  return DECIK_OK;
}

// groups the jobs by (nested, vectorised) and launches each group in batches of kMaxJobs
int run_jobs(const decik_nf4_job* jobs, int n_jobs, int out_dtype, cudaStream_t s) {
  if (out_dtype != DECIK_F16 && out_dtype != DECIK_BF16 && out_dtype != DECIK_F32)
    return set_error(DECIK_ERR_INVALID, "nf4_dequant: out_dtype %d", out_dtype);
  for (int j = 0; j < n_jobs; ++j) {
    const int rc = check_job(jobs[j]);
    if (rc) return rc;
  }
  for (int kind = 0; kind < 4; ++kind) {
    const bool nested = kind & 1, vec = kind & 2;
    Nf4Batch bt;
    int n = 0;
    for (int j = 0; j < n_jobs; ++j) {
      const decik_nf4_job& jb = jobs[j];
      if (jb.n_bytes == 0 || (jb.nested != 0) != nested || (aligned16(jb.packed) && aligned16(jb.out)) != vec) continue;
      bt.a[n] = Nf4Args{jb.packed, jb.absmax, jb.absmax2, jb.code2, jb.offset, jb.code, jb.n_bytes, jb.blocksize,
                        jb.blocksize2, log2_exact(jb.blocksize), nested ? log2_exact(jb.blocksize2) : 0};
      bt.out[n] = jb.out;
      if (++n == kMaxJobs || j == n_jobs - 1) {
        int rc = DECIK_OK;
        if (n > 0) {
          switch (out_dtype) {
            case DECIK_F16: rc = launch<__half>(bt, n, nested, vec, s); break;
            case DECIK_BF16: rc = launch<__nv_bfloat16>(bt, n, nested, vec, s); break;
            default: rc = launch<float>(bt, n, nested, vec, s); break;
          }
        }
        if (rc) return rc;
        n = 0;
      }
    }
    if (n > 0) {  // the last job of the list was not of this kind
      int rc;
      switch (out_dtype) {
        case DECIK_F16: rc = launch<__half>(bt, n, nested, vec, s); break;
        case DECIK_BF16: rc = launch<__nv_bfloat16>(bt, n, nested, vec, s); break;
        default: rc = launch<float>(bt, n, nested, vec, s); break;
      }
      if (rc) return rc;
    }
  }
  return DECIK_OK;
}

}  // namespace
}  // namespace decik

extern "C" int decik_nf4_dequant(const uint8_t* packed, const void* absmax, const float* absmax2,
                                 const float* code2, const float* offset, const float* code,
                                 void* out, int64_t n_bytes, int nested, int blocksize,
                                 int blocksize2, int out_dtype, void* stream) {
  if (n_bytes < 0) return decik::set_error(DECIK_ERR_INVALID, "nf4_dequant: n_bytes < 0");
  if (n_bytes == 0) return DECIK_OK;
  const decik_nf4_job j{packed, absmax, absmax2, code2, offset, code, out, n_bytes, nested, blocksize, blocksize2};
  return decik::run_jobs(&j, 1, out_dtype, decik::as_stream(stream));
}

extern "C" int decik_nf4_dequant_batch(const decik_nf4_job* jobs, int n_jobs, int out_dtype, void* stream) {
  if (n_jobs < 0 || (n_jobs > 0 && jobs == nullptr))
    return decik::set_error(DECIK_ERR_INVALID, "nf4_dequant_batch: bad job list");
  return decik::run_jobs(jobs, n_jobs, out_dtype, decik::as_stream(stream));
}
