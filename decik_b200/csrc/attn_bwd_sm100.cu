// Packed varlen causal GQA attention backward on tcgen05 / TMEM with TMA-fed operands. Replaces
// the backward of VarlenSDPA (solution/varlen.py:154-168): the forward's logsumexp is reused (no
// forward recompute), and dK / dV of each kv head are summed over its query heads inside the CTA
// (no GQA-expanded copies, no reduce pass).
//
// CTA = one 128-key block of one row x one kv head. It loops over the query heads of the group and
// the 64-query blocks at or below the diagonal. Per iteration (S^T etc. are key-major):
//   S^T  = K Q^T      [128 keys x 64 q]   SS, M=128 N=64  K=128
//   dP^T = V dO^T     [128 x 64]           SS
//   softmax WG: P^T = exp2(S^T*scale*log2e - lse*log2e), dS^T = P^T (dP^T - delta)  -> TMEM (16-bit)
//               and dS^T -> shared memory (the operand of dQ)
//   dV  += P^T dO     [128 keys x 128 d]   TS (A = P^T in TMEM), M=128 N=128 K=64
//   dK  += dS^T Q     [128 x 128]          TS
//   dQ^T = K^T dS^T   [128 d x 64 q]       SS, both operands MN-major
//   dQ WG: dQ^T (thread = one d) staged in shared memory; a TMA reduce-add adds the [64 x 128]
//          fp32 tile into the dq accumulator
// TMEM (512 cols): S^T [0,64) dP^T [64,128) dQ^T [128,192) P^T [192,224) dS^T [224,256)
//                  dV [256,384) dK [384,512).
// The softmax WG copies S^T / dP^T to registers and releases them at once, so the MMA warp issues
// the next iteration's S^T / dP^T while this iteration's softmax runs.
// 14 warps: 0-7 softmax in two column halves + dK/dV epilogue (thread = key row), 8-11 dQ (thread =
// d), 12 TMA, 13 MMA (event-driven issue: it polls the barriers of its three kinds of work).
// Every mbarrier wait is bounded (error word + wind-down).
#include <cudaTypedefs.h>

#include "attn_common.cuh"
#include "sm100.cuh"

namespace decik {
namespace attn {

int make_tile_map(CUtensorMap* map, const void* ptr, int64_t tok_stride, int64_t head_stride, int64_t n_tok,
                  int n_heads, int dtype, int* order, int box_rows);
int make_f32_rows_map(CUtensorMap* map, float* ptr, int64_t n_tok, int n_heads, int box_rows);
int* attn_error_word();

namespace {

using namespace sm100;

constexpr int BN = 128;  // keys per CTA
constexpr int BM = 64;   // queries per iteration
constexpr int KHALF = BN * 128;  // [128 rows x 64] 16-bit half: 16 KB
constexpr int KTILE = 2 * KHALF;
constexpr int QHALF = BM * 128;  // [64 rows x 64] half: 8 KB
constexpr int QTILE = 2 * QHALF;
constexpr int NTHREADS = 448;  // 14 warps
constexpr int NST = 3;  // Q / dO / stats stages in flight
// shared memory map (offsets from a 1024-aligned base)
constexpr int OFF_K = 0, OFF_V = KTILE, OFF_Q = 2 * KTILE;   // Q[s] at OFF_Q + s * 2 * QTILE, dO after it
constexpr int OFF_DS = OFF_Q + NST * 2 * QTILE;              // dS^T [128 keys x 64 q], 16 KB
constexpr int OFF_DQS = OFF_DS + KHALF;                      // dQ staging [64 q][128 d] fp32, 32 KB
constexpr int OFF_STAT = OFF_DQS + BM * 128 * 4;             // [NST][-lse*log2e 64 | -delta 64] fp32
constexpr int OFF_BAR = OFF_STAT + NST * 2 * BM * 4;
enum { B_KV = 0, B_QF = 1, B_QE = B_QF + NST, B_SF = B_QE + NST, B_SFREE, B_PR, B_PFREE, B_DQF, B_DQFREE, B_DONE,
       N_BAR };
constexpr int OFF_TMEM = OFF_BAR + N_BAR * 8;
constexpr int kSmem = OFF_TMEM + 16 + 1024;
constexpr uint32_t T_S = 0, T_DP = 64, T_DQ = 128, T_P = 192, T_DS = 224, T_DV = 256, T_DK = 384;

struct Params {
  CUtensorMap tq, tk, tv, tdo, tdq;
  void* dk;
  int64_t dk_tok, dk_head;
  void* dv;
  int64_t dv_tok, dv_head;
  const float* lse;
  const float* delta;
  float* dq_acc;
  const int32_t* cu;
  int64_t n_tok;
  int n_heads, groups;
  int order_q, order_k, order_v, order_do;
  float scale, scale_log2;
  int* err;
};

__device__ __forceinline__ void load_half(uint32_t dst, const CUtensorMap* map, uint32_t bar, int order, int c,
                                          int tok, int head) {
  if (order == 0) tma_load_3d(dst, map, bar, c, tok, head);
  else tma_load_3d(dst, map, bar, c, head, tok);
}

// Descriptors are built once; a k-step advances the 14-bit start-address field (bytes >> 4), which
// never carries out of the field for shared-memory addresses.
// S^T / dP^T: A [128 x 128] (K-major, 16 KB halves) times B [64 x 128]^T (K-major, 8 KB halves)
__device__ __forceinline__ void issue_nt(uint32_t d, uint64_t da, uint64_t db, uint32_t idesc) {
#pragma unroll
  for (int kk = 0; kk < 8; ++kk)
    umma_ss(d, da + (((kk >> 2) * KHALF + (kk & 3) * 32) >> 4), db + (((kk >> 2) * QHALF + (kk & 3) * 32) >> 4),
            idesc, kk > 0);
}
// dV / dK: D [128 x 128] (+)= A (TMEM, 16-bit, [128 x 64]) * B [64 q x 128 d] (MN-major, 8 KB halves)
__device__ __forceinline__ void issue_tn(uint32_t d, uint32_t a_tmem, uint64_t db, uint32_t idesc, bool acc) {
#pragma unroll
  for (int kk = 0; kk < 4; ++kk) umma_ts(d, a_tmem + kk * 8, db + kk * (2048 >> 4), idesc, (acc || kk > 0) ? 1u : 0u);
}
// dQ^T [128 d x 64 q] = K^T (MN-major view of the K tile) * dS^T (MN-major [128 keys x 64 q])
__device__ __forceinline__ void issue_dq(uint32_t d, uint64_t da, uint64_t db, uint32_t idesc) {
#pragma unroll
  for (int kk = 0; kk < 8; ++kk) umma_ss(d, da + kk * (2048 >> 4), db + kk * (2048 >> 4), idesc, kk > 0);
}

template <typename T>
__device__ __forceinline__ uint32_t pk2(float lo, float hi);
template <> __device__ __forceinline__ uint32_t pk2<__nv_bfloat16>(float lo, float hi) { return pack_bf16x2(lo, hi); }
template <> __device__ __forceinline__ uint32_t pk2<__half>(float lo, float hi) { return pack_f16x2(lo, hi); }

template <typename T>
__global__ void __launch_bounds__(NTHREADS, 1) attn_bwd_sm100_kernel(const __grid_constant__ Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sb = smem_u32(smem);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  const int n_block = blockIdx.x;
  const int row = blockIdx.y, kvh = blockIdx.z;
  const int start = p.cu[row];
  const int L = p.cu[row + 1] - start;
  const int n0 = n_block * BN;
  if (n0 >= L) return;
  const int m_first = n0 / BM;
  const int n_mb = (L + BM - 1) / BM - m_first;
  const int n_iter = n_mb * p.groups;
  auto bar = [&](int i) { return sb + OFF_BAR + 8 * i; };
  auto it_head = [&](int it) { return kvh * p.groups + it / n_mb; };
  auto it_m0 = [&](int it) { return (m_first + it % n_mb) * BM; };

  if (threadIdx.x == 0) {
    mbar_init(bar(B_KV), 1);
    for (int s = 0; s < NST; ++s) {
      mbar_init(bar(B_QF + s), 2);  // the TMA arrival (with its bytes) + the stats arrival
      mbar_init(bar(B_QE + s), 1);
    }
    mbar_init(bar(B_SF), 1);
    mbar_init(bar(B_SFREE), 256);
    mbar_init(bar(B_PR), 256);
    mbar_init(bar(B_PFREE), 1);
    mbar_init(bar(B_DQF), 1);
    mbar_init(bar(B_DQFREE), 128);
    mbar_init(bar(B_DONE), 1);
    fence_barrier_init();
  }
  if (warp == 13) {
    tmem_alloc(sb + OFF_TMEM, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(smem + OFF_TMEM);
  float* stat = reinterpret_cast<float*>(smem + OFF_STAT);

  if (warp == 12) {
    // ---------------------------------------------------------------- TMA producer
    int issued = 0;
    if (lane == 0) {
      prefetch_tmap(&p.tq);
      prefetch_tmap(&p.tk);
      prefetch_tmap(&p.tv);
      prefetch_tmap(&p.tdo);
      prefetch_tmap(&p.tdq);
      mbar_expect_tx(bar(B_KV), 2 * KTILE);
      for (int c = 0; c < 2; ++c) {
        load_half(sb + OFF_K + c * KHALF, &p.tk, bar(B_KV), p.order_k, 64 * c, start + n0, kvh);
        load_half(sb + OFF_V + c * KHALF, &p.tv, bar(B_KV), p.order_v, 64 * c, start + n0, kvh);
      }
    }
    bool ok = true;
    for (int it = 0; it < n_iter; ++it) {
      const int s = it % NST;
      if (it >= NST) ok = mbar_wait(bar(B_QE + s), ((it - NST) / NST) & 1, p.err, 401);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      const int h = it_head(it), m0 = it_m0(it);
      if (lane == 0) {  // Q and dO tiles first: their latency overlaps the stats loads below
        const uint32_t q = sb + OFF_Q + s * 2 * QTILE;
        mbar_expect_tx(bar(B_QF + s), 2 * QTILE);
        for (int c = 0; c < 2; ++c) {
          load_half(q + c * QHALF, &p.tq, bar(B_QF + s), p.order_q, 64 * c, start + m0, h);
          load_half(q + QTILE + c * QHALF, &p.tdo, bar(B_QF + s), p.order_do, 64 * c, start + m0, h);
        }
      }
      // -lse (log2 domain) and -delta of the 64 queries: plain loads by the warp, then the 2nd arrival
      float* st = stat + s * 2 * BM;
      for (int i = lane; i < BM; i += 32) {
        const int qi = m0 + i;
        const int64_t idx = static_cast<int64_t>(h) * p.n_tok + start + qi;
        st[i] = qi < L ? -p.lse[idx] * kLog2e : -INFINITY;
        st[BM + i] = qi < L ? -p.delta[idx] : 0.f;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(B_QF + s));
      issued = it + 1;
    }
    if (lane == 0) {
      for (int it = max(0, issued - NST); it < issued; ++it)
        mbar_wait(bar(B_QF + it % NST), (it / NST) & 1, p.err, 402);
      mbar_wait(bar(B_KV), 0, p.err, 403);
    }
  } else if (warp == 13) {
    // ---------------------------------------------------------------- MMA issue (one thread)
    // Event-driven: the thread polls the barriers its three kinds of work depend on and issues
    // whichever is ready, so no wait holds back work that could already run.
    if (lane == 0) {
      constexpr int ab = std::is_same<T, __nv_bfloat16>::value ? 1 : 0;
      const uint32_t id_nt = idesc_f16(ab, BN, BM, 0, 0);   // S^T, dP^T
      const uint32_t id_tn = idesc_f16(ab, BN, 128, 0, 1);  // dV, dK
      const uint32_t id_dq = idesc_f16(ab, 128, BM, 1, 1);  // dQ^T
      const uint64_t dK = smem_desc_sw128(sb + OFF_K, 16, 1024), dV = smem_desc_sw128(sb + OFF_V, 16, 1024);
      const uint64_t dKt = smem_desc_sw128(sb + OFF_K, KHALF, 1024), dDS = smem_desc_sw128(sb + OFF_DS, KHALF, 1024);
      const uint64_t dQk = smem_desc_sw128(sb + OFF_Q, 16, 1024);      // stage 0 Q, K-major
      const uint64_t dQm = smem_desc_sw128(sb + OFF_Q, QHALF, 1024);   // stage 0 Q, MN-major
      constexpr uint64_t kStage = (2 * QTILE) >> 4, kDO = QTILE >> 4;  // stage stride, Q -> dO offset
      bool ok = mbar_wait(bar(B_KV), 0, p.err, 501) && mbar_wait(bar(B_QF), 0, p.err, 502);
      if (ok) {
        tc_fence_after();
        issue_nt(tmem + T_S, dK, dQk, id_nt);
        issue_nt(tmem + T_DP, dV, dQk + kDO, id_nt);
        umma_commit(bar(B_SF));
      }
      int nS = 1, nV = 0, nQ = 0;  // next iteration whose S^T/dP^T, dV/dK, dQ^T is to be issued
      long long t_last = cycles();
      while (ok && nQ < n_iter) {
        bool progress = false;
        // S^T / dP^T of the next iteration: the softmax copied the previous one out, Q/dO landed
        if (nS < n_iter && mbar_test(bar(B_SFREE), (nS - 1) & 1) &&
            mbar_test(bar(B_QF + nS % NST), (nS / NST) & 1)) {
          tc_fence_after();
          issue_nt(tmem + T_S, dK, dQk + (nS % NST) * kStage, id_nt);
          issue_nt(tmem + T_DP, dV, dQk + (nS % NST) * kStage + kDO, id_nt);
          umma_commit(bar(B_SF));
          ++nS;
          progress = true;
        }
        // dV += P^T dO, dK += dS^T Q once the softmax wrote P^T / dS^T
        if (nV < nS && mbar_test(bar(B_PR), nV & 1)) {
          tc_fence_after();
          const int s = nV % NST;
          issue_tn(tmem + T_DV, tmem + T_P, dQm + s * kStage + kDO, id_tn, nV > 0);
          issue_tn(tmem + T_DK, tmem + T_DS, dQm + s * kStage, id_tn, nV > 0);
          umma_commit(bar(B_PFREE));
          umma_commit(bar(B_QE + s));
          ++nV;
          progress = true;
        }
        // dQ^T once dS^T is in shared memory and the dQ warps read the previous dQ^T out
        if (nQ < nV && (nQ == 0 || mbar_test(bar(B_DQFREE), (nQ - 1) & 1))) {
          tc_fence_after();
          issue_dq(tmem + T_DQ, dKt, dDS, id_dq);
          umma_commit(bar(B_DQF));
          ++nQ;
          progress = true;
        }
        if (progress) {
          t_last = cycles();
        } else if (cycles() - t_last > kWaitLimitCycles) {
          report(p.err, 503);
          ok = false;
        }
      }
      umma_commit(bar(B_DONE));
      mbar_wait(bar(B_DONE), 0, p.err, 507);
    }
  } else if (warp < 8) {
    // ---------------------------------------------------------------- softmax (thread = key row)
    // warpgroup `half` handles query columns [32 * half, 32 * half + 32) of every key row
    const int half = warp >> 2;
    const int r = (warp & 3) * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const int key = n0 + r;
    const int c0 = 32 * half;
    uint8_t* ds_row = smem + OFF_DS + r * 128;
    bool ok = true;
    for (int it = 0; it < n_iter; ++it) {
      const int s = it % NST;
      const int m0 = it_m0(it);
      ok = mbar_wait(bar(B_SF), it & 1, p.err, 601) && mbar_wait(bar(B_QF + s), (it / NST) & 1, p.err, 602);
      if (!ok) break;
      tc_fence_after();
      uint32_t sv[32], dp[32];
      tmem_ld32(tmem + lane_off + T_S + c0, sv);
      tmem_ld32(tmem + lane_off + T_DP + c0, dp);
      tmem_ld_wait();
      tc_fence_before();
      mbar_arrive(bar(B_SFREE));
      const float4* nl4 = reinterpret_cast<const float4*>(stat + s * 2 * BM + c0);       // -lse * log2e
      const float4* nd4 = reinterpret_cast<const float4*>(stat + s * 2 * BM + BM + c0);  // -delta
      // visible query columns of this key: qc >= key - m0 (causal) and qc < L - m0 (row end)
      const int qlo = key - m0 - c0;
      const int qhi = (key < L ? min(BM, L - m0) : 0) - c0;
      const bool masked = qlo > 0 || qhi < 32;
      const uint64_t sc2 = f2(p.scale_log2, p.scale_log2);
      uint32_t pp[16], dd[16];
#pragma unroll
      for (int c = 0; c < 8; ++c) {  // 4 query columns per step, as two packed pairs
        const float4 nl = nl4[c], nd = nd4[c];
        float e[4];
        f2split(ffma2(f2(__uint_as_float(sv[4 * c]), __uint_as_float(sv[4 * c + 1])), sc2, f2(nl.x, nl.y)), e[0], e[1]);
        f2split(ffma2(f2(__uint_as_float(sv[4 * c + 2]), __uint_as_float(sv[4 * c + 3])), sc2, f2(nl.z, nl.w)), e[2], e[3]);
#pragma unroll
        for (int i = 0; i < 4; ++i) e[i] = ptx::ex2(e[i]);
        if (masked) {
#pragma unroll
          for (int i = 0; i < 4; ++i)
            if (4 * c + i < qlo || 4 * c + i >= qhi) e[i] = 0.f;
        }
        const uint64_t p01 = f2(e[0], e[1]), p23 = f2(e[2], e[3]);
        const uint64_t g01 = fmul2(p01, fadd2(f2(__uint_as_float(dp[4 * c]), __uint_as_float(dp[4 * c + 1])), f2(nd.x, nd.y)));
        const uint64_t g23 = fmul2(p23, fadd2(f2(__uint_as_float(dp[4 * c + 2]), __uint_as_float(dp[4 * c + 3])), f2(nd.z, nd.w)));
        float g[4];
        f2split(g01, g[0], g[1]);
        f2split(g23, g[2], g[3]);
        pp[2 * c] = pk2<T>(e[0], e[1]);
        pp[2 * c + 1] = pk2<T>(e[2], e[3]);
        dd[2 * c] = pk2<T>(g[0], g[1]);
        dd[2 * c + 1] = pk2<T>(g[2], g[3]);
      }
      // P^T / dS^T TMEM slots are free once the previous dV / dK MMAs completed
      if (it > 0) ok = mbar_wait(bar(B_PFREE), (it - 1) & 1, p.err, 603);
      if (!ok) break;
      tc_fence_after();
      tmem_st16(tmem + lane_off + T_P + c0 / 2, pp);
      tmem_st16(tmem + lane_off + T_DS + c0 / 2, dd);
      // dS^T smem tile is free once the previous dQ^T MMA completed
      if (it > 0) ok = mbar_wait(bar(B_DQF), (it - 1) & 1, p.err, 604);
      if (!ok) break;
#pragma unroll
      for (int c = 0; c < 4; ++c) {  // 16-byte chunk (c0 / 8 + c) of this key's 64 queries, 128B-swizzled
        const int chunk = c0 / 8 + c;
        *reinterpret_cast<uint4*>(ds_row + ((chunk ^ (r & 7)) << 4)) =
            make_uint4(dd[4 * c], dd[4 * c + 1], dd[4 * c + 2], dd[4 * c + 3]);
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(bar(B_PR));
    }
    // epilogue: warpgroup 0 writes the dV rows, warpgroup 1 the dK rows (x scale)
    if (ok && mbar_wait(bar(B_DONE), 0, p.err, 605)) {
      tc_fence_after();
      const bool valid = key < L;
      const int64_t tok = static_cast<int64_t>(start) + key;
      const uint32_t base = tmem + lane_off + (half ? T_DK : T_DV);
      const float mul = half ? p.scale : 1.f;
      T* dst = half ? static_cast<T*>(p.dk) + tok * p.dk_tok + static_cast<int64_t>(kvh) * p.dk_head
                    : static_cast<T*>(p.dv) + tok * p.dv_tok + static_cast<int64_t>(kvh) * p.dv_head;
#pragma unroll
      for (int c4 = 0; c4 < 4; ++c4) {
        uint32_t o[32];
        tmem_ld32(base + 32 * c4, o);
        tmem_ld_wait();
        uint32_t w[16];
#pragma unroll
        for (int i = 0; i < 16; ++i)
          w[i] = pk2<T>(__uint_as_float(o[2 * i]) * mul, __uint_as_float(o[2 * i + 1]) * mul);
        if (valid) {
#pragma unroll
          for (int i = 0; i < 4; ++i)
            reinterpret_cast<uint4*>(dst + 32 * c4)[i] = make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
        }
      }
    }
  } else if (warp < 12) {
    // ---------------------------------------------------------------- dQ (thread = one of the 128 dims)
    const int d = (warp & 3) * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>((warp & 3) * 32) << 16;
    for (int it = 0; it < n_iter; ++it) {
      const bool got = mbar_wait(bar(B_DQF), it & 1, p.err, 701);
      if (!named_bar_and(1, 128, got)) break;  // the 4 warps leave together (they share named barriers)
      tc_fence_after();
      uint32_t v[64];
      tmem_ld32(tmem + lane_off + T_DQ, *reinterpret_cast<uint32_t(*)[32]>(&v[0]));
      tmem_ld32(tmem + lane_off + T_DQ + 32, *reinterpret_cast<uint32_t(*)[32]>(&v[32]));
      tmem_ld_wait();
      tc_fence_before();
      mbar_arrive(bar(B_DQFREE));
      // stage dQ^T as [64 q][128 d] fp32 and let the TMA engine add the tile into the fp32
      // accumulator: no per-thread global reductions compete with the softmax warps' traffic
      const int h = it_head(it), m0 = it_m0(it);
      if (d == 0 && it > 0) bulk_wait_read0();  // the previous tile has been read out of the staging buffer
      named_bar(1, 128);
      float* stg = reinterpret_cast<float*>(smem + OFF_DQS);
#pragma unroll
      for (int c = 0; c < BM; ++c) stg[c * 128 + d] = __uint_as_float(v[c]);
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      named_bar(1, 128);
      if (d == 0) {
        tma_reduce_add_3d(&p.tdq, sb + OFF_DQS, 0, h, start + m0);
        bulk_commit();
      }
    }
    if (d == 0) bulk_wait0();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 13) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace

int bwd_sm100(const decik_tensor3& q, const decik_tensor3& k, const decik_tensor3& v, const decik_tensor3& dout,
              const decik_tensor3_mut& dk, const decik_tensor3_mut& dv, const float* lse, const float* delta,
              float* dq_acc, const int32_t* cu, int n_rows, int max_len, int64_t n_tok, int n_heads, int n_kv,
              float scale, int dtype, cudaStream_t stream) {
  Params p;
  int rc = make_tile_map(&p.tq, q.ptr, q.tok_stride, q.head_stride, n_tok, n_heads, dtype, &p.order_q, BM);
  if (!rc) rc = make_tile_map(&p.tdo, dout.ptr, dout.tok_stride, dout.head_stride, n_tok, n_heads, dtype, &p.order_do, BM);
  if (!rc) rc = make_tile_map(&p.tk, k.ptr, k.tok_stride, k.head_stride, n_tok, n_kv, dtype, &p.order_k, BN);
  if (!rc) rc = make_tile_map(&p.tv, v.ptr, v.tok_stride, v.head_stride, n_tok, n_kv, dtype, &p.order_v, BN);
  if (!rc) rc = make_f32_rows_map(&p.tdq, dq_acc, n_tok, n_heads, BM);
  if (rc) return rc;
  p.dk = dk.ptr;
  p.dk_tok = dk.tok_stride;
  p.dk_head = dk.head_stride;
  p.dv = dv.ptr;
  p.dv_tok = dv.tok_stride;
  p.dv_head = dv.head_stride;
  p.lse = lse;
  p.delta = delta;
  p.dq_acc = dq_acc;
  p.cu = cu;
  p.n_tok = n_tok;
  p.n_heads = n_heads;
  p.groups = n_heads / n_kv;
  p.scale = scale;
  p.scale_log2 = scale * kLog2e;
  p.err = attn_error_word();
  dim3 grid((max_len + BN - 1) / BN, n_rows, n_kv);
  if (dtype == DECIK_BF16) {
    static bool set = false;
    if (!set) {
      cudaFuncSetAttribute(attn_bwd_sm100_kernel<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
      set = true;
    }
    attn_bwd_sm100_kernel<__nv_bfloat16><<<grid, NTHREADS, kSmem, stream>>>(p);
  } else {
    static bool set = false;
    if (!set) {
      cudaFuncSetAttribute(attn_bwd_sm100_kernel<__half>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
      set = true;
    }
    attn_bwd_sm100_kernel<__half><<<grid, NTHREADS, kSmem, stream>>>(p);
  }
  return check_launch("varlen_attn_bwd (sm100)");
}

}  // namespace attn
}  // namespace decik
