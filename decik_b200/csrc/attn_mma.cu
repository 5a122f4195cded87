// Packed varlen causal GQA attention, forward and backward, on the warp-level tensor path
// (mma.sync m16n8k16, fp32 accumulate). Replaces VarlenSDPA (solution/varlen.py:134-168): one
// launch each way over every row of the packed sequence (cu_seqlens), GQA without expanding K/V,
// fully-masked causal tiles never visited, logsumexp written by the forward so the backward does
// not recompute it.
//
// The forward runs on tcgen05 (attn_fwd_sm100.cu); this file holds the backward and the C entries.
// Backward: CTA = 64 keys of one row x one kv head, 4 warps x 16 keys; it loops over the query
// heads of its group and the query blocks at or below the diagonal, so dK/dV of the kv head are
// summed in registers (no GQA reduce pass). S^T and dP^T are computed key-major so P^T and dS^T
// feed dV += P^T dO and dK += dS^T Q straight from the accumulators; dS^T goes through shared
// memory for dQ = dS K, which is added to an fp32 accumulator with atomics and scaled/cast by a
// final pass.
#include "attn_common.cuh"

namespace decik {
namespace attn {
namespace {

using ptx::ldsm_x4;
using ptx::ldsm_x4_t;
using ptx::smem_u32;

template <typename T>
__device__ __forceinline__ uint32_t pack2(float lo, float hi) { return Dt<T>::pack2(lo, hi); }

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

constexpr int BBN = 64, BBM = 64, BTHREADS = 128;
// K, V (64 rows each), 2 stages x (Q, dO) (64 rows each), dS^T [64 x 64], lse/delta 2 x 2 x 64
constexpr int kBwdSmem = (2 + 4) * BBN * kRowBytes + BBN * BBM * 2 + 4 * BBM * 4;

struct BwdParams {
  Tensor3 q, k, v, dout;
  Tensor3Mut dk, dv;
  const float* lse;
  const float* delta;
  float* dq_acc;
  const int32_t* cu;
  int64_t n_tok;
  int n_heads, groups;
  float scale, scale_log2;
};

// element offset in the [64 x 64] 16-bit dS^T tile (8 chunks per row, swizzled)
__device__ __forceinline__ int swz64(int row, int chunk) { return row * 64 + ((chunk ^ (row & 7)) << 3); }

template <typename T>
__global__ void __launch_bounds__(BTHREADS, 2) attn_bwd_kernel(BwdParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int n_block = blockIdx.x;
  const int row = blockIdx.y, kvh = blockIdx.z;
  const int start = p.cu[row];
  const int L = p.cu[row + 1] - start;
  const int n0 = n_block * BBN;
  if (n0 >= L) return;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t4 = lane & 3;
  const int64_t tok_end = static_cast<int64_t>(start) + L;

  const uint32_t sK = smem_u32(smem);
  const uint32_t sV = sK + BBN * kRowBytes;
  const uint32_t sQD = sV + BBN * kRowBytes;  // stage s: Q at sQD + s*2*64 rows, dO after Q
  const uint32_t sDS = sQD + 4 * BBM * kRowBytes;
  float* s_stats = reinterpret_cast<float*>(smem + (2 + 4) * BBN * kRowBytes + BBN * BBM * 2);  // [2][lse 64, delta 64]

  load_tile<BBN, BTHREADS>(sK, p.k, start + n0, tok_end, kvh, tid);
  load_tile<BBN, BTHREADS>(sV, p.v, start + n0, tok_end, kvh, tid);

  const int m_first = n0 / BBM;  // first query block touching the diagonal
  const int n_mb = (L + BBM - 1) / BBM - m_first;
  const int n_iter = n_mb * p.groups;

  auto issue = [&](int it) {
    const int stage = it & 1;
    const int h = kvh * p.groups + it / n_mb;
    const int m0 = (m_first + it % n_mb) * BBM;
    const uint32_t sq = sQD + stage * (2 * BBM * kRowBytes);
    load_tile<BBM, BTHREADS>(sq, p.q, start + m0, tok_end, h, tid);
    load_tile<BBM, BTHREADS>(sq + BBM * kRowBytes, p.dout, start + m0, tok_end, h, tid);
    if (tid < BBM) {
      const int qi = m0 + tid;
      float* st = s_stats + stage * 2 * BBM;
      const int64_t idx = static_cast<int64_t>(h) * p.n_tok + start + qi;
      st[tid] = qi < L ? p.lse[idx] * kLog2e : INFINITY;  // exp2(s - inf) = 0 for padding rows
      st[BBM + tid] = qi < L ? p.delta[idx] : 0.f;
    }
  };
  issue(0);
  ptx::cp_async_commit();

  float dv[16][4], dk[16][4];
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    dv[i][0] = dv[i][1] = dv[i][2] = dv[i][3] = 0.f;
    dk[i][0] = dk[i][1] = dk[i][2] = dk[i][3] = 0.f;
  }
  const int kv_row0 = n0 + warp * 16 + g;  // key index in the row of accumulator rows g, g+8

  for (int it = 0; it < n_iter; ++it) {
    if (it + 1 < n_iter) {
      issue(it + 1);
      ptx::cp_async_commit();
      ptx::cp_async_wait<1>();
    } else {
      ptx::cp_async_wait<0>();
    }
    __syncthreads();
    const int stage = it & 1;
    const int h = kvh * p.groups + it / n_mb;
    const int m0 = (m_first + it % n_mb) * BBM;
    const uint32_t sQ = sQD + stage * (2 * BBM * kRowBytes);
    const uint32_t sDO = sQ + BBM * kRowBytes;
    const float* lse2 = s_stats + stage * 2 * BBM;
    const float* dlt = lse2 + BBM;

    // S^T = K Q^T and dP^T = V dO^T: [16 keys x 64 queries] per warp
    float s[8][4], dp[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      s[i][0] = s[i][1] = s[i][2] = s[i][3] = 0.f;
      dp[i][0] = dp[i][1] = dp[i][2] = dp[i][3] = 0.f;
    }
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      uint32_t ak[4], av[4];
      ldsm_x4(sK + 2 * swz(warp * 16 + (lane & 15), kk * 2 + (lane >> 4)), ak[0], ak[1], ak[2], ak[3]);
      ldsm_x4(sV + 2 * swz(warp * 16 + (lane & 15), kk * 2 + (lane >> 4)), av[0], av[1], av[2], av[3]);
#pragma unroll
      for (int np = 0; np < 4; ++np) {
        const int r = np * 16 + (lane & 7) + ((lane >> 4) << 3);
        const int c = kk * 2 + ((lane >> 3) & 1);
        uint32_t b0, b1, b2, b3;
        ldsm_x4(sQ + 2 * swz(r, c), b0, b1, b2, b3);
        ptx::mma16816<T>(s[2 * np], ak, b0, b1);
        ptx::mma16816<T>(s[2 * np + 1], ak, b2, b3);
        ldsm_x4(sDO + 2 * swz(r, c), b0, b1, b2, b3);
        ptx::mma16816<T>(dp[2 * np], av, b0, b1);
        ptx::mma16816<T>(dp[2 * np + 1], av, b2, b3);
      }
    }
    // P^T = exp2(S^T * scale*log2e - lse*log2e), masked; dS^T = P^T * (dP^T - delta)
    const bool need_mask = m0 < n0 + BBN || m0 + BBM > L || n0 + BBN > L;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int qc = j * 8 + 2 * t4 + (e & 1);  // query column in the block
        float pe = ptx::ex2(s[j][e] * p.scale_log2 - lse2[qc]);
        if (need_mask) {
          const int kv = kv_row0 + ((e >> 1) << 3);
          const int qi = m0 + qc;
          if (kv > qi || kv >= L || qi >= L) pe = 0.f;
        }
        s[j][e] = pe;
        dp[j][e] = pe * (dp[j][e] - dlt[qc]);
      }
    }
    // dV += P^T dO, dK += dS^T Q  (A from the accumulators, B = dO / Q via transposed ldmatrix)
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      const uint32_t ap[4] = {pack2<T>(s[2 * kk][0], s[2 * kk][1]), pack2<T>(s[2 * kk][2], s[2 * kk][3]),
                              pack2<T>(s[2 * kk + 1][0], s[2 * kk + 1][1]),
                              pack2<T>(s[2 * kk + 1][2], s[2 * kk + 1][3])};
      const uint32_t ad[4] = {pack2<T>(dp[2 * kk][0], dp[2 * kk][1]), pack2<T>(dp[2 * kk][2], dp[2 * kk][3]),
                              pack2<T>(dp[2 * kk + 1][0], dp[2 * kk + 1][1]),
                              pack2<T>(dp[2 * kk + 1][2], dp[2 * kk + 1][3])};
      if (kk == 0 || true) {
        // dS^T rows of this warp into shared memory for dQ (16 keys x 16 queries per kk)
        const int r = warp * 16 + g;
        const int col = kk * 16 + 2 * t4;
        uint8_t* sds = smem + (sDS - sK);
        *reinterpret_cast<uint32_t*>(sds + 2 * (swz64(r, col >> 3) + (col & 7))) = ad[0];
        *reinterpret_cast<uint32_t*>(sds + 2 * (swz64(r + 8, col >> 3) + (col & 7))) = ad[1];
        *reinterpret_cast<uint32_t*>(sds + 2 * (swz64(r, (col + 8) >> 3) + (col & 7))) = ad[2];
        *reinterpret_cast<uint32_t*>(sds + 2 * (swz64(r + 8, (col + 8) >> 3) + (col & 7))) = ad[3];
      }
#pragma unroll
      for (int dp2 = 0; dp2 < 8; ++dp2) {
        const int r = kk * 16 + (lane & 7) + (((lane >> 3) & 1) << 3);
        const int c = dp2 * 2 + (lane >> 4);
        uint32_t b0, b1, b2, b3;
        ldsm_x4_t(sDO + 2 * swz(r, c), b0, b1, b2, b3);
        ptx::mma16816<T>(dv[2 * dp2], ap, b0, b1);
        ptx::mma16816<T>(dv[2 * dp2 + 1], ap, b2, b3);
        ldsm_x4_t(sQ + 2 * swz(r, c), b0, b1, b2, b3);
        ptx::mma16816<T>(dk[2 * dp2], ad, b0, b1);
        ptx::mma16816<T>(dk[2 * dp2 + 1], ad, b2, b3);
      }
    }
    __syncthreads();  // dS^T complete
    // dQ[16 queries of this warp x 128] = dS K = (dS^T)^T K, then atomically added
    {
      float dq[16][4];
#pragma unroll
      for (int i = 0; i < 16; ++i) dq[i][0] = dq[i][1] = dq[i][2] = dq[i][3] = 0.f;
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {  // 16 keys per step
        uint32_t a[4];
        // A[m = query][k = key] read from dS^T[key][query] with a transposed ldmatrix
        const int mi = lane >> 3, r8 = lane & 7;
        const int krow = kk * 16 + r8 + ((mi >> 1) << 3);
        const int qcol = warp * 16 + ((mi & 1) << 3);
        ldsm_x4_t(sDS + 2 * swz64(krow, qcol >> 3), a[0], a[1], a[2], a[3]);
#pragma unroll
        for (int dp2 = 0; dp2 < 8; ++dp2) {
          const int r = kk * 16 + (lane & 7) + (((lane >> 3) & 1) << 3);
          const int c = dp2 * 2 + (lane >> 4);
          uint32_t b0, b1, b2, b3;
          ldsm_x4_t(sK + 2 * swz(r, c), b0, b1, b2, b3);
          ptx::mma16816<T>(dq[2 * dp2], a, b0, b1);
          ptx::mma16816<T>(dq[2 * dp2 + 1], a, b2, b3);
        }
      }
      const int q0 = m0 + warp * 16 + g;
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const int qi = q0 + i * 8;
        if (qi < L) {
          float* dst = p.dq_acc + ((static_cast<int64_t>(start) + qi) * p.n_heads + h) * D + 2 * t4;
#pragma unroll
          for (int dt = 0; dt < 16; ++dt) {
            atomicAdd(dst + dt * 8, dq[dt][2 * i]);
            atomicAdd(dst + dt * 8 + 1, dq[dt][2 * i + 1]);
          }
        }
      }
    }
    __syncthreads();  // stage and dS^T free for the next iteration
  }

  // dK *= scale; write dK, dV of the valid keys
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const int kv = kv_row0 + i * 8;
    if (kv < L) {
      const int64_t tok = static_cast<int64_t>(start) + kv;
      T* dkp = static_cast<T*>(p.dk.ptr) + tok * p.dk.tok + static_cast<int64_t>(kvh) * p.dk.head + 2 * t4;
      T* dvp = static_cast<T*>(p.dv.ptr) + tok * p.dv.tok + static_cast<int64_t>(kvh) * p.dv.head + 2 * t4;
#pragma unroll
      for (int dt = 0; dt < 16; ++dt) {
        *reinterpret_cast<uint32_t*>(dkp + dt * 8) = pack2<T>(dk[dt][2 * i] * p.scale, dk[dt][2 * i + 1] * p.scale);
        *reinterpret_cast<uint32_t*>(dvp + dt * 8) = pack2<T>(dv[dt][2 * i], dv[dt][2 * i + 1]);
      }
    }
  }
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
  if (n_rows < 0 || max_len < 0 || n_tok < 0 || n_heads <= 0 || n_kv <= 0 || n_heads % n_kv)
    return set_error(DECIK_ERR_INVALID, "varlen_attn_bwd: bad sizes");
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
    BwdParams p;
    p.q = {q.ptr, q.tok_stride, q.head_stride};
    p.k = {k.ptr, k.tok_stride, k.head_stride};
    p.v = {v.ptr, v.tok_stride, v.head_stride};
    p.dout = {dout.ptr, dout.tok_stride, dout.head_stride};
    p.dk = {dk.ptr, dk.tok_stride, dk.head_stride};
    p.dv = {dv.ptr, dv.tok_stride, dv.head_stride};
    p.lse = lse;
    p.delta = delta;
    p.dq_acc = dq_acc;
    p.cu = cu_seqlens;
    p.n_tok = n_tok;
    p.n_heads = n_heads;
    p.groups = n_heads / n_kv;
    p.scale = scale;
    p.scale_log2 = scale * kLog2e;
    static bool attr = false;
    if (!attr) {
      cudaFuncSetAttribute(attn_bwd_kernel<__half>, cudaFuncAttributeMaxDynamicSharedMemorySize, kBwdSmem);
      cudaFuncSetAttribute(attn_bwd_kernel<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize, kBwdSmem);
      attr = true;
    }
    dim3 grid((max_len + BBN - 1) / BBN, n_rows, n_kv);
    attn_bwd_kernel<T><<<grid, BTHREADS, kBwdSmem, s>>>(p);
    rc = check_launch("varlen_attn_bwd");
    if (rc) return rc;
    const int64_t n8 = n_tok * n_heads * (D / 8);
    attn_bwd_post_kernel<T><<<static_cast<unsigned>((n8 + 255) / 256), 256, 0, s>>>(
        dq_acc, Tensor3Mut{dq.ptr, dq.tok_stride, dq.head_stride}, n_tok, n_heads, scale);
    return check_launch("varlen_attn_bwd post");
  });
}
