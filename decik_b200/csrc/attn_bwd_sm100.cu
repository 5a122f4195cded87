// Packed varlen causal GQA attention backward on tcgen05 / TMEM with TMA-fed operands. Replaces
// the backward of VarlenSDPA (solution/varlen.py:154-168): the forward's logsumexp is reused (no
// forward recompute), and dK / dV of each kv head are summed over its query heads on chip (no
// GQA-expanded copies).
//
// CTA = one 128-key block of one row x one kv head x one subset of the group's query heads. It
// loops over its query heads and the 128-query blocks at or below the diagonal. Per iteration
// (S^T etc. are key-major; every MMA is M=128 N=128, kind::f16):
//   S^T  = K Q^T      SS              -> TMEM S/P
//   dP^T = V dO^T     SS              -> TMEM dP/dQ
//   softmax warps, in two phases:
//     P phase:  P^T = exp2(S^T*scale*log2e - lse*log2e) -> TMEM (operand type, over S^T columns the
//               same warpgroup has read; an f16 copy stays in registers)
//     dS phase: dS^T = P^T (dP^T - delta) -> shared memory
//   dV  += P^T dO     TS (A = P^T in TMEM)
//   dK  += dS^T Q     SS (A = dS^T, K-major)
//   dQ   = dS K       SS (A = the same dS^T tile read MN-major)  -> TMEM dP/dQ
//   dQ warps: read dQ out of TMEM at once (freeing the columns for the next dP^T), then stream it as
//   16-column fp32 chunks through two staging buffers (64-byte swizzle) into the fp32 dq
//   accumulator by TMA bulk reduce-add, concurrently with the next softmax.
// TMEM (512 columns): dK [0,128) dV [128,256) dP^T/dQ [256,384) S^T/P^T [384,512). The softmax
// warpgroups take interleaved 32-query blocks (w and w + 2), so each writes P^T only over S^T
// columns it has itself read. Issue order per iteration i: dV(i) and S(i+1) once P^T(i) is written
// (S(i+1) overwrites P^T(i) after dV(i) in issue order: tcgen05 MMAs of one thread execute in
// order; both run under the dS phase of i), dQ(i) and dK(i) once dS^T(i) is written, dP(i+1) once
// the dQ warps read dQ(i) out. The P phase of i+1 needs only S(i+1), so it runs while dQ(i) is
// computed and read out and dP(i+1) is computed. What then sets the period is the dQ warps'
// stream of fp32 reduce-adds (64 KB per iteration), not the softmax.
// With more than one head subset per key block, dK / dV go to fp32 accumulators by TMA reduce-add
// (the caller casts them); with one, they are written directly. Launch order: key block 0 of every
// row first (the longest CTAs), or, when the dq accumulator is far larger than L2, the key blocks
// of one (row, kv head) together (their dQ reduce-adds then stay in L2).
// 16 warps: 0-7 softmax and the dK/dV epilogue (warpgroup w: query columns [64w, 64w+64), thread =
// key row), 8-11 dQ (thread = query row), 12 TMA + lse/delta loads, 13 MMA issue (one thread).
// Every mbarrier wait is bounded (error word + wind-down).
#include <cudaTypedefs.h>

#include "attn_common.cuh"
#include "sm100.cuh"

namespace decik {
namespace attn {

int make_tile_map(CUtensorMap* map, const void* ptr, int64_t tok_stride, int64_t head_stride, int64_t n_tok,
                  int n_heads, int dtype, int* order, int box_rows);
int make_f32_chunk_map(CUtensorMap* map, float* ptr, int64_t n_tok, int n_heads, int box_rows);
int* attn_error_word();

namespace {

using namespace sm100;

constexpr int BN = 128;                   // keys per CTA
constexpr int BM = 128;                   // queries per iteration
constexpr int HALF = 128 * 128;           // [128 rows x 64] 16-bit half of a tile: 16 KB
constexpr int TILE = 2 * HALF;            // [128 rows x 128] 16-bit tile: 32 KB
constexpr int CHUNK = 128 * 16 * 4;       // [128 rows x 16] fp32 staging chunk: 8 KB
constexpr int NTHREADS = 512;             // 16 warps = 4 warpgroups
// shared memory map (offsets from a 1024-aligned base)
constexpr int OFF_K = 0, OFF_V = TILE, OFF_Q = 2 * TILE;  // Q stage s at OFF_Q + s * TILE
constexpr int OFF_DO = 4 * TILE, OFF_DS = 5 * TILE;       // dO (one stage), dS^T
constexpr int OFF_STG = 6 * TILE;                          // dQ staging: two chunk buffers
constexpr int OFF_STAT = OFF_STG + 2 * CHUNK;              // [2][-lse*log2e 128 | -delta 128] fp32
constexpr int OFF_BAR = OFF_STAT + 2 * 2 * BM * 4;
enum { B_KV = 0, B_QF, B_QF1, B_QE, B_QE1, B_DOF, B_DOE, B_SF, B_DPF, B_PF, B_DSF, B_DSFREE, B_DQF,
       B_DQFREE, B_DONE, N_BAR };
constexpr int OFF_TMEM = OFF_BAR + N_BAR * 8;
constexpr int kSmem = OFF_TMEM + 16 + 1024;
constexpr uint32_t T_DK = 0, T_DV = 128, T_DPQ = 256, T_SP = 384;
// registers per thread: 128 at launch (512 threads), then per warpgroup: the softmax warpgroups need
// 112, the dQ warpgroup (a 128-value row per thread) 152, the issue warpgroup (TMA producer and the
// MMA thread, which keeps its descriptors and unrolls its k-steps so the tensor pipe never waits on
// issue) 136. The sum must not exceed the 65,536 the block was launched with, or setmaxnreg.inc
// would wait forever.
constexpr int kRegsLaunch = 128, kRegsSoftmax = 112, kRegsDq = 152, kRegsIssue = 136;
static_assert(2 * 128 * kRegsSoftmax + 128 * kRegsDq + 128 * kRegsIssue <= NTHREADS * kRegsLaunch, "register split");
static_assert(NTHREADS * kRegsLaunch == 65536, "launch register count");
static_assert(kSmem <= 227 * 1024, "shared memory");
// at the end, dV and dK are staged as 8 chunks each over the Q stages and over dO + dS^T
static_assert(OFF_Q + 8 * CHUNK <= OFF_DO && OFF_DO + 8 * CHUNK <= OFF_STG, "epilogue staging");

struct Params {
  CUtensorMap tq, tk, tv, tdo, tdq, tdk, tdv;
  void* dk;
  int64_t dk_tok, dk_head;
  void* dv;
  int64_t dv_tok, dv_head;
  const float* lse;
  const float* delta;
  const int32_t* cu;
  int64_t n_tok;
  int n_heads, groups, n_kv, n_split, heads_per_split;
  int rows_outer;  // grid x = key block, y = (row, kv head, subset); else x and y swapped
  int order_q, order_k, order_v, order_do;
  float scale, scale_log2;
  int* err;
};

__device__ __forceinline__ void load_half(uint32_t dst, const CUtensorMap* map, uint32_t bar, int order, int c,
                                          int tok, int head) {
  if (order == 0) tma_load_3d(dst, map, bar, c, tok, head);
  else tma_load_3d(dst, map, bar, c, head, tok);
}
__device__ __forceinline__ void load_tile(uint32_t dst, const CUtensorMap* map, uint32_t bar, int order, int tok,
                                          int head) {
  load_half(dst, map, bar, order, 0, tok, head);
  load_half(dst + HALF, map, bar, order, 64, tok, head);
}
// a [128 x 128] tile into L2 ahead of its load
__device__ __forceinline__ void prefetch_tile(const CUtensorMap* map, int order, int tok, int head) {
#pragma unroll
  for (int c = 0; c < 128; c += 64) {
    if (order == 0) tma_prefetch_3d(map, c, tok, head);
    else tma_prefetch_3d(map, c, head, tok);
  }
}

// Descriptors are built once; a k-step advances the 14-bit start-address field (bytes >> 4), which
// never carries out of the field for shared-memory addresses.
// K-major A and B, K = 128 over two 64-element halves: k-step kk at half kk/4, 32 bytes * (kk % 4)
__device__ __forceinline__ uint64_t kstep_k(uint64_t d, int kk) {
  return d + ((((kk >> 2) * HALF) + (kk & 3) * 32) >> 4);
}
// MN-major operand (MN = 128 over two halves, LBO = HALF): a k-step is 16 rows of 128 bytes
__device__ __forceinline__ uint64_t kstep_mn(uint64_t d, int kk) { return d + kk * (2048 >> 4); }

__device__ __forceinline__ void issue_ss_kk(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, bool acc) {
#pragma unroll
  for (int kk = 0; kk < 8; ++kk) umma_ss(d, kstep_k(a, kk), kstep_k(b, kk), idesc, (acc || kk > 0) ? 1u : 0u);
}
__device__ __forceinline__ void issue_ss_km(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, bool acc) {
#pragma unroll
  for (int kk = 0; kk < 8; ++kk) umma_ss(d, kstep_k(a, kk), kstep_mn(b, kk), idesc, (acc || kk > 0) ? 1u : 0u);
}
__device__ __forceinline__ void issue_ss_mm(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, bool acc) {
#pragma unroll
  for (int kk = 0; kk < 8; ++kk) umma_ss(d, kstep_mn(a, kk), kstep_mn(b, kk), idesc, (acc || kk > 0) ? 1u : 0u);
}
// TMEM column (16-bit pairs) of P^T for the 32-query block b, within the dP^T/P^T columns: the
// softmax warpgroup that owns block b writes it over dP^T columns it has already read
__host__ __device__ constexpr int p_col(int b) { return 16 * (b >> 1) + 32 * (b & 1); }
// dV += P^T dO: k-step kk covers queries [16 kk, 16 kk + 16), i.e. block kk / 2
__device__ __forceinline__ void issue_pv(uint32_t d, uint32_t p_tmem, uint64_t b, uint32_t idesc, bool acc) {
#pragma unroll
  for (int kk = 0; kk < 8; ++kk)
    umma_ts(d, p_tmem + p_col(kk >> 1) + (kk & 1) * 8, kstep_mn(b, kk), idesc, (acc || kk > 0) ? 1u : 0u);
}

template <typename T>
__device__ __forceinline__ uint32_t pk2(float lo, float hi);
template <> __device__ __forceinline__ uint32_t pk2<__nv_bfloat16>(float lo, float hi) { return pack_bf16x2(lo, hi); }
template <> __device__ __forceinline__ uint32_t pk2<__half>(float lo, float hi) { return pack_f16x2(lo, hi); }
// the two values of an f16 pair as fp32 (exact)
__device__ __forceinline__ void unpk2(uint32_t v, float& lo, float& hi) {
  const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&v));
  lo = f.x;
  hi = f.y;
}

// Row `r` (64 bytes: 16 fp32) of a [128 x 16] staging chunk laid out with the TMA 64-byte swizzle:
// 16-byte unit j of row r sits at unit j ^ ((r >> 1) & 3).
__device__ __forceinline__ void stage_row16(uint8_t* chunk, int r, const uint32_t* v) {
#pragma unroll
  for (int j = 0; j < 4; ++j)
    *reinterpret_cast<uint4*>(chunk + r * 64 + ((j ^ ((r >> 1) & 3)) << 4)) =
        make_uint4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
}

template <typename T>
__global__ void __launch_bounds__(NTHREADS, 1) attn_bwd_sm100_kernel(const __grid_constant__ Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sb = smem_u32(smem);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  // one grid dimension walks the key blocks, the other (row, kv head, head subset); see bwd_sm100
  const int n_block = p.rows_outer ? blockIdx.x : blockIdx.y;
  const int rkv = p.rows_outer ? blockIdx.y : blockIdx.x;
  const int split = rkv % p.n_split;
  const int kvh = (rkv / p.n_split) % p.n_kv;
  const int row = rkv / (p.n_split * p.n_kv);
  const int start = p.cu[row];
  const int L = p.cu[row + 1] - start;
  const int n0 = n_block * BN;
  const int h_first = split * p.heads_per_split;
  const int n_heads_here = min(p.heads_per_split, p.groups - h_first);
  if (n0 >= L || n_heads_here <= 0) return;
  const int m_first = n0 / BM;
  const int n_mb = (L + BM - 1) / BM - m_first;
  const int n_iter = n_mb * n_heads_here;
  const bool direct = p.n_split == 1;  // dK / dV written directly, else reduced into fp32
  auto bar = [&](int i) { return sb + OFF_BAR + 8 * i; };
  auto it_head = [&](int it) { return kvh * p.groups + h_first + it / n_mb; };
  auto it_m0 = [&](int it) { return (m_first + it % n_mb) * BM; };

  if (threadIdx.x == 0) {
    mbar_init(bar(B_KV), 1);
    mbar_init(bar(B_QF), 2);  // the TMA arrival (with its bytes) + the lse/delta arrival
    mbar_init(bar(B_QF1), 2);
    mbar_init(bar(B_QE), 1);
    mbar_init(bar(B_QE1), 1);
    mbar_init(bar(B_DOF), 1);
    mbar_init(bar(B_DOE), 1);
    mbar_init(bar(B_SF), 1);
    mbar_init(bar(B_DPF), 1);
    mbar_init(bar(B_PF), 256);
    mbar_init(bar(B_DSF), 256);
    mbar_init(bar(B_DSFREE), 1);
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

  if (warp >= 12) {
    // warpgroup 3 (TMA producer, MMA issuer, two idle warps): 128 -> kRegsIssue registers
    reg_set<kRegsLaunch, kRegsIssue>();
  }
  if (warp == 12) {
    // ---------------------------------------------------------------- TMA producer + lse / delta
    int issued_q = 0, issued_do = 0;
    if (lane == 0) {
      prefetch_tmap(&p.tq);
      prefetch_tmap(&p.tk);
      prefetch_tmap(&p.tv);
      prefetch_tmap(&p.tdo);
      mbar_expect_tx(bar(B_KV), 2 * TILE);
      load_tile(sb + OFF_K, &p.tk, bar(B_KV), p.order_k, start + n0, kvh);
      load_tile(sb + OFF_V, &p.tv, bar(B_KV), p.order_v, start + n0, kvh);
    }
    // -lse * log2e and -delta of iteration j's 128 queries, 4 + 4 per lane, loaded one iteration
    // ahead so that their latency hides behind the waits below
    float nl[4], nd[4];
    auto fetch_stats = [&](int j) {
      const int hj = it_head(j), mj = it_m0(j);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int qi = mj + lane + 32 * k;
        const int64_t idx = static_cast<int64_t>(hj) * p.n_tok + start + qi;
        nl[k] = qi < L ? -__ldg(p.lse + idx) * kLog2e : -INFINITY;
        nd[k] = qi < L ? -__ldg(p.delta + idx) : 0.f;
      }
    };
    fetch_stats(0);
    bool ok = true;
    for (int it = 0; it < n_iter && ok; ++it) {
      const int s = it & 1;
      const int h = it_head(it), m0 = it_m0(it);
      // Q stage s is free once dK of iteration it - 2 completed
      if (it >= 2) ok = mbar_wait(bar(B_QE + s), ((it - 2) >> 1) & 1, p.err, 401);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      if (lane == 0) {
        mbar_expect_tx(bar(B_QF + s), TILE);
        load_tile(sb + OFF_Q + s * TILE, &p.tq, bar(B_QF + s), p.order_q, start + m0, h);
      }
      float* st = stat + s * 2 * BM;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        st[lane + 32 * k] = nl[k];
        st[BM + lane + 32 * k] = nd[k];
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(B_QF + s));
      if (it + 1 < n_iter) fetch_stats(it + 1);
      issued_q = it + 1;
      // the single dO stage is free once dV of iteration it - 1 completed
      if (it >= 1) ok = mbar_wait(bar(B_DOE), (it - 1) & 1, p.err, 402);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      if (lane == 0) {
        mbar_expect_tx(bar(B_DOF), TILE);
        load_tile(sb + OFF_DO, &p.tdo, bar(B_DOF), p.order_do, start + m0, h);
        // dO(it + 1) is loaded only once dV(it) has read this stage, right before dP(it + 1) needs
        // it: bring it (and Q two iterations ahead) into L2 now, an iteration early
        if (it + 1 < n_iter) prefetch_tile(&p.tdo, p.order_do, start + it_m0(it + 1), it_head(it + 1));
        if (it + 2 < n_iter) prefetch_tile(&p.tq, p.order_q, start + it_m0(it + 2), it_head(it + 2));
      }
      issued_do = it + 1;
    }
    if (lane == 0) {  // no TMA write may still be in flight when the CTA ends
      for (int it = max(0, issued_q - 2); it < issued_q; ++it)
        mbar_wait(bar(B_QF + (it & 1)), (it >> 1) & 1, p.err, 403);
      if (issued_do > 0) mbar_wait(bar(B_DOF), (issued_do - 1) & 1, p.err, 404);
      mbar_wait(bar(B_KV), 0, p.err, 405);
    }
  } else if (warp == 13) {
    // ---------------------------------------------------------------- MMA issue (one thread)
    // Per iteration: dV(it) and S(it+1) once P^T(it) is in TMEM (they run under the dS phase of
    // it), then dQ(it) and dK(it) once dS^T(it) is in shared memory, then dP(it+1) once the dQ warps
    // read dQ(it) out (it runs under the P phase of it+1).
    if (lane == 0) {
      constexpr int ab = std::is_same<T, __nv_bfloat16>::value ? 1 : 0;
      const uint32_t id_kk = idesc_f16(ab, 128, 128, 0, 0);  // S^T, dP^T
      const uint32_t id_km = idesc_f16(ab, 128, 128, 0, 1);  // dV (A in TMEM), dK
      const uint32_t id_mm = idesc_f16(ab, 128, 128, 1, 1);  // dQ
      const uint64_t dKk = smem_desc_sw128(sb + OFF_K, 16, 1024), dVk = smem_desc_sw128(sb + OFF_V, 16, 1024);
      const uint64_t dKm = smem_desc_sw128(sb + OFF_K, HALF, 1024);
      const uint64_t dQk0 = smem_desc_sw128(sb + OFF_Q, 16, 1024), dQm0 = smem_desc_sw128(sb + OFF_Q, HALF, 1024);
      const uint64_t dOk = smem_desc_sw128(sb + OFF_DO, 16, 1024), dOm = smem_desc_sw128(sb + OFF_DO, HALF, 1024);
      const uint64_t dSk = smem_desc_sw128(sb + OFF_DS, 16, 1024), dSm = smem_desc_sw128(sb + OFF_DS, HALF, 1024);
      constexpr uint64_t kStage = TILE >> 4;
      bool ok = mbar_wait(bar(B_KV), 0, p.err, 501) && mbar_wait(bar(B_QF), 0, p.err, 502);
      if (ok) {
        tc_fence_after();
        issue_ss_kk(tmem + T_SP, dKk, dQk0, id_kk, false);  // S^T(0)
        umma_commit(bar(B_SF));
        ok = mbar_wait(bar(B_DOF), 0, p.err, 503);
      }
      if (ok) {
        tc_fence_after();
        issue_ss_kk(tmem + T_DPQ, dVk, dOk, id_kk, false);  // dP^T(0)
        umma_commit(bar(B_DPF));
      }
      for (int it = 0; it < n_iter && ok; ++it) {
        const int s = it & 1;
        // dV += P^T dO once the softmax wrote P^T(it) (over the S^T columns); frees dO
        ok = mbar_wait(bar(B_PF), it & 1, p.err, 504);
        if (!ok) break;
        tc_fence_after();
        issue_pv(tmem + T_DV, tmem + T_SP, dOm, id_km, it > 0);
        umma_commit(bar(B_DOE));
        if (it + 1 < n_iter) {
          // S^T(it+1) over P^T(it): after dV(it) in issue order (tcgen05 MMAs of one thread execute
          // in order)
          ok = mbar_wait(bar(B_QF + (s ^ 1)), ((it + 1) >> 1) & 1, p.err, 506);
          if (!ok) break;
          tc_fence_after();
          issue_ss_kk(tmem + T_SP, dKk, dQk0 + (s ^ 1) * kStage, id_kk, false);
          umma_commit(bar(B_SF));
        }
        // dQ(it) = dS K over the dP^T columns, which the softmax read before it wrote dS
        ok = mbar_wait(bar(B_DSF), it & 1, p.err, 505);
        if (!ok) break;
        tc_fence_after();
        issue_ss_mm(tmem + T_DPQ, dSm, dKm, id_mm, false);
        umma_commit(bar(B_DQF));
        // dK += dS^T Q(it), while the dQ warps read dQ(it) out; frees dS^T and the Q stage
        issue_ss_km(tmem + T_DK, dSk, dQm0 + s * kStage, id_km, it > 0);
        umma_commit(bar(B_DSFREE));
        umma_commit(bar(B_QE + s));
        if (it + 1 < n_iter) {
          // dP^T(it+1) once dO(it+1) landed and the dQ warps read dQ(it) out
          ok = mbar_wait(bar(B_DOF), (it + 1) & 1, p.err, 507) && mbar_wait(bar(B_DQFREE), it & 1, p.err, 508);
          if (!ok) break;
          tc_fence_after();
          issue_ss_kk(tmem + T_DPQ, dVk, dOk, id_kk, false);
          umma_commit(bar(B_DPF));
        }
      }
      umma_commit(bar(B_DONE));
      mbar_wait(bar(B_DONE), 0, p.err, 509);
    }
  } else if (warp >= 8 && warp < 12) {
    // ---------------------------------------------------------------- dQ (thread = query row)
    reg_set<kRegsLaunch, kRegsDq>();
    const int r = (warp & 3) * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const bool leader = warp == 8 && lane == 0;
    bool ok = true;
    int staged = 0;  // chunks handed to the TMA engine
    for (int j = 0; j < n_iter; ++j) {
      // every dQ thread takes part in the barrier-AND, also after a failed wait: the outcome is
      // the same for all of them, so the named barriers below always see 128 threads
      ok = named_bar_and(3, 128, ok && mbar_wait(bar(B_DQF), j & 1, p.err, 701));
      if (!ok) continue;
      tc_fence_after();
      uint32_t v[128];
#pragma unroll
      for (int q = 0; q < 4; ++q) tmem_ld32(tmem + lane_off + T_DPQ + 32 * q, *reinterpret_cast<uint32_t(*)[32]>(&v[32 * q]));
      tmem_ld_wait();
      tc_fence_before();
      mbar_arrive(bar(B_DQFREE));
      const int h = it_head(j), m0 = it_m0(j);
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        // buffer (staged & 1) was last read by the chunk two back: wait for that read only
        if (leader && staged >= 2) bulk_wait_read1();
        named_bar(3, 128);
        uint8_t* buf = smem + OFF_STG + (staged & 1) * CHUNK;
        stage_row16(buf, r, &v[16 * c]);
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        named_bar(3, 128);
        if (leader) {
          tma_reduce_add_3d(&p.tdq, smem_u32(buf), 16 * c, h, start + m0);
          bulk_commit();
        }
        ++staged;
      }
    }
    if (leader) bulk_wait0();
  } else if (warp < 8) {
    // ---------------------------------------------------------------- softmax, dK/dV epilogue
    reg_set<kRegsLaunch, kRegsSoftmax>();
    const int wg = warp >> 2;                      // query columns [64 wg, 64 wg + 64)
    const int r = (warp & 3) * 32 + lane;          // key row
    const uint32_t lane_off = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const int key = n0 + r;
    const int bar_id = 1 + wg;                     // named barrier of this warpgroup
    const bool leader = (warp & 3) == 0 && lane == 0;
    uint8_t* ds_row = smem + OFF_DS + r * 128;
    bool ok = true;
    // a bounded wait, made uniform across the warp (the TMEM accesses below are warp-collective)
    auto wait_w = [&](int b, int parity, int code) -> bool {
      return __all_sync(0xffffffffu, mbar_wait(bar(b), parity, p.err, code));
    };

    const float sc = p.scale_log2;
    for (int it = 0; it < n_iter; ++it) {
      const int s = it & 1;
      const int m0 = it_m0(it);
      if (!ok) continue;
      const float* st = stat + s * 2 * BM;
      // P phase: P^T = exp2(S^T * scale * log2e - lse * log2e), written in the operand type over
      // S^T columns this warpgroup has read (dV(it) reads it from there, then S^T(it+1) overwrites
      // it). P stays in registers for the dS phase as f16 pairs: P <= 1, and f16's 11-bit
      // significand keeps dS as accurate as with fp32 P (bf16 pairs raised dQ's error by a fifth)
      ok = wait_w(B_SF, it & 1, 602) && wait_w(B_QF + s, (it >> 1) & 1, 604);
      if (!ok) continue;
      tc_fence_after();
      uint32_t pp[2][16];
#pragma unroll
      for (int h2 = 0; h2 < 2; ++h2) {
        const int blk = 2 * h2 + wg;       // 32-query block of this pass: warpgroup w takes w, w + 2
        const int c0 = 32 * blk;           // its first query column
        uint32_t sv[32];
        tmem_ld32(tmem + lane_off + T_SP + c0, sv);
        tmem_ld_wait();
        const float4* nl4 = reinterpret_cast<const float4*>(st + c0);  // -lse * log2e
        // visible query columns of this key: q >= key (causal) and q < L (row end)
        const int qlo = key - m0 - c0;
        const int qhi = (key < L ? min(BM, L - m0) : 0) - c0;
        const bool masked = qlo > 0 || qhi < 32;
        const uint32_t p_tm = tmem + lane_off + T_SP + p_col(blk);
#pragma unroll
        for (int c = 0; c < 8; ++c) {  // 4 query columns per step
          const float4 nl = nl4[c];
          const float nls[4] = {nl.x, nl.y, nl.z, nl.w};
          float e[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) e[i] = ptx::ex2(fmaf(__uint_as_float(sv[4 * c + i]), sc, nls[i]));
          if (masked) {
#pragma unroll
            for (int i = 0; i < 4; ++i)
              if (4 * c + i < qlo || 4 * c + i >= qhi) e[i] = 0.f;
          }
          pp[h2][2 * c] = pack_f16x2(e[0], e[1]);
          pp[h2][2 * c + 1] = pack_f16x2(e[2], e[3]);
          // the operand copy two columns at a time (a 16-column store would need 16 more live
          // registers and spills at this warpgroup's register budget)
          if constexpr (!std::is_same<T, __half>::value)
            tmem_st2(p_tm + 2 * c, pk2<T>(e[0], e[1]), pk2<T>(e[2], e[3]));
        }
        if constexpr (std::is_same<T, __half>::value) tmem_st16(p_tm, pp[h2]);
      }
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(bar(B_PF));
      // dS phase: dS^T = P^T (dP^T - delta) into shared memory, once dQ(it - 1) / dK(it - 1) have
      // read the previous dS^T
      ok = wait_w(B_DPF, it & 1, 603) && (it == 0 || wait_w(B_DSFREE, (it - 1) & 1, 605));
      if (!ok) continue;
      tc_fence_after();
#pragma unroll
      for (int h2 = 0; h2 < 2; ++h2) {
        const int blk = 2 * h2 + wg;
        const int c0 = 32 * blk;
        uint32_t dp[32];
        tmem_ld32(tmem + lane_off + T_DPQ + c0, dp);
        tmem_ld_wait();
        const float4* nd4 = reinterpret_cast<const float4*>(st + BM + c0);  // -delta
        uint32_t dd[16];
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          const float4 nd = nd4[c];
          const float nds[4] = {nd.x, nd.y, nd.z, nd.w};
          float e[4], g[4];
          unpk2(pp[h2][2 * c], e[0], e[1]);
          unpk2(pp[h2][2 * c + 1], e[2], e[3]);
#pragma unroll
          for (int i = 0; i < 4; ++i) g[i] = e[i] * (__uint_as_float(dp[4 * c + i]) + nds[i]);
          dd[2 * c] = pk2<T>(g[0], g[1]);
          dd[2 * c + 1] = pk2<T>(g[2], g[3]);
        }
#pragma unroll
        for (int c = 0; c < 4; ++c) {  // 16-byte unit of this key's row in its 64-query half, 128B-swizzled
          const int unit = 4 * (blk & 1) + c;
          *reinterpret_cast<uint4*>(ds_row + (blk >> 1) * HALF + ((unit ^ (r & 7)) << 4)) =
              make_uint4(dd[4 * c], dd[4 * c + 1], dd[4 * c + 2], dd[4 * c + 3]);
        }
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      tc_fence_before();
      mbar_arrive(bar(B_DSF));
    }
    // epilogue: warpgroup 0 takes the dV rows, warpgroup 1 the dK rows (x scale); every thread of
    // the warpgroup reaches this barrier-AND, so the named barrier below sees all 128
    ok = named_bar_and(bar_id, 128, ok && mbar_wait(bar(B_DONE), 0, p.err, 606));
    if (ok) {
      tc_fence_after();
      const uint32_t base = tmem + lane_off + (wg ? T_DK : T_DV);
      const float mul = wg ? p.scale : 1.f;
      if (direct) {
        const bool valid = key < L;
        const int64_t tok = static_cast<int64_t>(start) + key;
        T* dst = wg ? static_cast<T*>(p.dk) + tok * p.dk_tok + static_cast<int64_t>(kvh) * p.dk_head
                    : static_cast<T*>(p.dv) + tok * p.dv_tok + static_cast<int64_t>(kvh) * p.dv_head;
#pragma unroll 1
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
      } else {
        // fp32 partial sums (unscaled: the cast pass applies the scale to dK, as to dQ): 8 chunks
        // [128 keys x 16 d] staged over the free Q stages (dV) and over dO + dS^T (dK), then added
        // into the accumulator by the TMA engine
        uint8_t* area = smem + (wg ? OFF_DO : OFF_Q);
#pragma unroll 1
        for (int c = 0; c < 8; ++c) {
          uint32_t o[16];
          tmem_ld16(base + 16 * c, o);
          tmem_ld_wait();
          stage_row16(area + c * CHUNK, r, o);
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        named_bar(bar_id, 128);
        if (leader) {
          const CUtensorMap* map = wg ? &p.tdk : &p.tdv;
          for (int c = 0; c < 8; ++c) tma_reduce_add_3d(map, smem_u32(area + c * CHUNK), 16 * c, kvh, start + n0);
          bulk_commit();
        }
      }
    }
    if (leader) bulk_wait0();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 13) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace

// Number of head subsets per (key block, kv head): enough CTAs to fill the GPU about three times,
// never more than the group size. One subset keeps dK / dV on chip (no fp32 accumulators).
constexpr int kSplitWaves = 3;
int bwd_sm100_splits(int64_t n_tok, int n_rows, int n_heads, int n_kv) {
  const int groups = n_heads / n_kv;
  const int64_t base = ((n_tok + BN - 1) / BN + n_rows) * static_cast<int64_t>(n_kv);
  const int64_t want = std::min<int64_t>(
      std::max<int64_t>((kSplitWaves * static_cast<int64_t>(sm_count()) + base - 1) / std::max<int64_t>(base, 1), 1),
      groups);
  const int per = static_cast<int>((groups + want - 1) / want);  // heads per subset
  return (groups + per - 1) / per;                                // no empty subset
}

int bwd_sm100(const decik_tensor3& q, const decik_tensor3& k, const decik_tensor3& v, const decik_tensor3& dout,
              const decik_tensor3_mut& dk, const decik_tensor3_mut& dv, const float* lse, const float* delta,
              float* dq_acc, float* dk_acc, float* dv_acc, int n_split, const int32_t* cu, int n_rows,
              int max_len, int64_t n_tok, int n_heads, int n_kv, float scale, int dtype, cudaStream_t stream) {
  Params p;
  int rc = make_tile_map(&p.tq, q.ptr, q.tok_stride, q.head_stride, n_tok, n_heads, dtype, &p.order_q, BM);
  if (!rc) rc = make_tile_map(&p.tdo, dout.ptr, dout.tok_stride, dout.head_stride, n_tok, n_heads, dtype, &p.order_do, BM);
  if (!rc) rc = make_tile_map(&p.tk, k.ptr, k.tok_stride, k.head_stride, n_tok, n_kv, dtype, &p.order_k, BN);
  if (!rc) rc = make_tile_map(&p.tv, v.ptr, v.tok_stride, v.head_stride, n_tok, n_kv, dtype, &p.order_v, BN);
  if (!rc) rc = make_f32_chunk_map(&p.tdq, dq_acc, n_tok, n_heads, BM);
  if (!rc && n_split > 1) rc = make_f32_chunk_map(&p.tdk, dk_acc, n_tok, n_kv, BN);
  if (!rc && n_split > 1) rc = make_f32_chunk_map(&p.tdv, dv_acc, n_tok, n_kv, BN);
  if (rc) return rc;
  if (n_split == 1) {
    p.tdk = p.tdq;  // unused
    p.tdv = p.tdq;
  }
  p.dk = dk.ptr;
  p.dk_tok = dk.tok_stride;
  p.dk_head = dk.head_stride;
  p.dv = dv.ptr;
  p.dv_tok = dv.tok_stride;
  p.dv_head = dv.head_stride;
  p.lse = lse;
  p.delta = delta;
  p.cu = cu;
  p.n_tok = n_tok;
  p.n_heads = n_heads;
  p.groups = n_heads / n_kv;
  p.n_kv = n_kv;
  p.n_split = n_split;
  p.heads_per_split = (p.groups + n_split - 1) / n_split;
  p.scale = scale;
  p.scale_log2 = scale * kLog2e;
  p.err = attn_error_word();
  // Launch order. Blocks start in grid order, x fastest. While the fp32 dq accumulator stays near
  // L2 size, key block 0 of every row goes first (the heaviest CTAs: they see every query of
  // their row), which keeps the tail short. Beyond twice the L2, that order has every row's
  // accumulator live at once and the dQ reduce-adds go to HBM; then the key blocks of one
  // (row, kv head) launch together, so the CTAs resident at a time add into a few heads' worth of
  // accumulator that stays in L2 (the 7B block at 131,072 tokens: 98.9 -> 65.7 ms).
  const int64_t rkv = static_cast<int64_t>(n_rows) * n_kv * n_split;
  const int64_t n_kb = (max_len + BN - 1) / BN;
  p.rows_outer = n_tok * n_heads * D * 4 > 2 * l2_bytes() && rkv <= 65535;
  if (!p.rows_outer && (rkv > INT32_MAX || n_kb > 65535))
    return set_error(DECIK_ERR_UNSUPPORTED, "varlen_attn_bwd: grid too large (rows x kv heads x subsets %lld, key blocks %lld)",
                     (long long)rkv, (long long)n_kb);
  const dim3 grid = p.rows_outer ? dim3(static_cast<unsigned>(n_kb), static_cast<unsigned>(rkv), 1)
                                 : dim3(static_cast<unsigned>(rkv), static_cast<unsigned>(n_kb), 1);
  if (dtype == DECIK_BF16) {
    static std::atomic<unsigned long long> set{0};
    if (int rc = ensure_dyn_smem(attn_bwd_sm100_kernel<__nv_bfloat16>, kSmem, set, "attn_bwd_sm100")) return rc;
    attn_bwd_sm100_kernel<__nv_bfloat16><<<grid, NTHREADS, kSmem, stream>>>(p);
  } else {
    static std::atomic<unsigned long long> set{0};
    if (int rc = ensure_dyn_smem(attn_bwd_sm100_kernel<__half>, kSmem, set, "attn_bwd_sm100")) return rc;
    attn_bwd_sm100_kernel<__half><<<grid, NTHREADS, kSmem, stream>>>(p);
  }
  return check_launch("attn_bwd_sm100");
}

}  // namespace attn
}  // namespace decik
