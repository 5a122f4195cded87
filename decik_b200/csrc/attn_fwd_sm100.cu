// Packed varlen causal GQA attention forward on the 5th-generation tensor cores (tcgen05 + TMEM,
// operands staged by TMA). Replaces the forward of VarlenSDPA (solution/varlen.py:144-151): one
// launch over every row of the packed sequence, GQA without expanding K/V, fully-masked causal
// tiles never visited, logsumexp written for the backward.
//
// Work tile = one 128-query block of one row x two query heads of the same kv head (so each K/V
// tile loaded by TMA feeds two 128x128x128 QK^T and two PV products). In the longest-first tile
// order the kernel is persistent: one CTA per SM takes tiles from a ticket counter until none are
// left, so TMEM allocation and barrier setup happen once per SM, and the next tile's first QK^T
// runs while the softmax warps write the previous tile's output; in the row-major order (see
// fwd_sm100) each CTA takes one tile. 10 warps:
//   warps 0-3  softmax of query tile 0 (thread = one query row = one TMEM lane) and its output
//   warps 4-7  the same for query tile 1
//   warp 8     tile tickets and the TMA producer: Q0, Q1 per tile, K_j / V_j through a 2-stage ring
//              that runs on across tiles
//   warp 9     TMEM allocation and the single-thread tcgen05.mma issue
//   warps 10-11 idle (they complete the third warpgroup for the register split)
// TMEM (512 columns): S0 [0,128), S1 [128,256), O0 [256,384), O1 [384,512); P (16-bit) overwrites
// the first 64 columns of its S. The MMA thread ping-pongs the two tiles so the tensor core runs
// one tile's QK^T / PV while the other tile's softmax runs:
//   S0(0) S1(0) | PV0(j) S0(j+1) PV1(j) S1(j+1) | ...
// and issues each PV in two halves of 64 keys, the first once the softmax has written that half of
// P (it then computes the other half's exponentials while the first half runs).
// Online softmax in the exp2 domain; O is rescaled in TMEM only when a row max grows by more than
// 2^8 (the final O / l is exact for any reference max). Every mbarrier wait is bounded: a wait that
// gives up records a code in the error word and the CTA winds down (waiting for its own MMAs and
// TMA loads, then freeing TMEM).
#include <cudaTypedefs.h>

#include <atomic>
#include <type_traits>

#include "attn_common.cuh"
#include "sm100.cuh"

namespace decik {
namespace attn {

int make_tile_map(CUtensorMap* map, const void* ptr, int64_t tok_stride, int64_t head_stride, int64_t n_tok,
                  int n_heads, int dtype, int* order, int box_rows);
int* attn_error_word();

namespace {

using namespace sm100;

constexpr int BM = 128, BN = 128;
constexpr int HALF = BM * 64 * 2;       // one [128 rows x 64] 16-bit swizzled half tile: 16 KB
constexpr int TILE = 2 * HALF;          // 32 KB
constexpr int NTHREADS = 384;  // 12 warps = 3 warpgroups (warps 10-11 only complete warpgroup 2)
// registers per thread: 168 at launch (the most 384 threads can have), then per warpgroup: the
// softmax warpgroups 184 (their loop plus the persistent tile state), warpgroup 2 (producer and
// MMA issue) 128. The sum must not exceed what the block was launched with, or setmaxnreg.inc
// would wait forever.
constexpr int kRegsLaunch = 168, kRegsSoftmax = 184, kRegsIssue = 128;
static_assert(2 * 128 * kRegsSoftmax + 128 * kRegsIssue <= NTHREADS * kRegsLaunch, "register split");
static_assert(NTHREADS * kRegsLaunch <= 65536, "launch register count");
constexpr int OFF_Q0 = 0, OFF_Q1 = TILE, OFF_K = 2 * TILE, OFF_V = 4 * TILE;
constexpr int STAGE = 32 * 64;                                 // per softmax warp: 32 rows x 32 columns
constexpr int OFF_STAGE = 6 * TILE;                            // 8 warps x STAGE: output staging
constexpr int OFF_RING = OFF_STAGE + 8 * STAGE;                // int32 [2] tile tickets
constexpr int OFF_BAR = OFF_RING + 16;
enum {
  B_Q = 0, B_QE, B_KF, B_KE = B_KF + 2, B_VF = B_KE + 2, B_VE = B_VF + 2, B_SF = B_VE + 2, B_PR = B_SF + 2,
  B_OF = B_PR + 2, B_OE = B_OF + 2, B_TF = B_OE + 2, B_TE = B_TF + 2, B_DONE = B_TE + 2, B_PH = B_DONE + 1,
  N_BAR = B_PH + 2
};
constexpr int OFF_TMEM = OFF_BAR + N_BAR * 8;
constexpr int kSmem = OFF_TMEM + 16 + 1024;  // + slack for the 1024-byte alignment
static_assert(kSmem <= 227 * 1024, "shared memory");

// Ticket counters, one per launch that may be in flight at the same time (a launch takes the next
// slot round-robin). The last CTA of a launch to finish puts its slot back to zero.
constexpr int kSlots = 64;
__device__ unsigned int g_ticket[kSlots];
__device__ unsigned int g_exit[kSlots];

struct Params {
  CUtensorMap tq, tk, tv;
  void* o;
  int64_t o_tok, o_head;
  float* lse;
  const int32_t* cu;
  int64_t n_tok;
  int n_heads, groups, pairs, n_mblocks, n_rows, zs;
  unsigned n_tickets;
  int heavy_first;  // ticket order: see fwd_sm100
  int persistent;   // tickets from the counter; else CTA b takes ticket b and nothing else
  int slot;
  int order_q, order_k, order_v;  // 0: coordinates (d, tok, head); 1: (d, head, tok)
  float scale_log2;
  int* err;
};

struct WorkTile {
  int start, L, m0, n_kv, kvh, h0;
  bool has1;
};

// Ticket t -> work tile; false for a query block past its row's end. heavy_first: tickets walk the
// query blocks from the last (the most key blocks) for every row at once; else one row's query
// blocks from its last, row after row.
__device__ __forceinline__ bool decode_tile(const Params& p, const int* cu, unsigned t, WorkTile& w) {
  int mb, rz;
  if (p.heavy_first) {
    const unsigned per = static_cast<unsigned>(p.n_rows) * p.zs;
    mb = p.n_mblocks - 1 - static_cast<int>(t / per);
    rz = static_cast<int>(t % per);
  } else {
    mb = p.n_mblocks - 1 - static_cast<int>(t % p.n_mblocks);
    rz = static_cast<int>(t / p.n_mblocks);
  }
  const int row = rz % p.n_rows, z = rz / p.n_rows;
  w.start = __ldg(cu + row);
  w.L = __ldg(cu + row + 1) - w.start;
  w.m0 = mb * BM;
  if (w.m0 >= w.L) return false;
  w.n_kv = (min(w.m0 + BM, w.L) + BN - 1) / BN;
  w.kvh = z / p.pairs;
  const int pair = z % p.pairs;
  w.h0 = w.kvh * p.groups + 2 * pair;
  w.has1 = 2 * pair + 1 < p.groups;
  return true;
}

__device__ __forceinline__ void load_half(uint32_t dst, const CUtensorMap* map, uint32_t bar, int order,
                                          int c, int tok, int head) {
  if (order == 0) tma_load_3d(dst, map, bar, c, tok, head);
  else tma_load_3d(dst, map, bar, c, head, tok);
}

// S = Q K^T: 8 steps of K = 16 over head_dim; both operands K-major, 128B-swizzled halves.
__device__ __forceinline__ void issue_qk(uint32_t d, uint32_t q, uint32_t k, uint32_t idesc) {
#pragma unroll
  for (int kk = 0; kk < 8; ++kk) {
    const uint32_t off = (kk >> 2) * HALF + (kk & 3) * 32;
    umma_ss(d, smem_desc_sw128(q + off, 16, 1024), smem_desc_sw128(k + off, 16, 1024), idesc, kk > 0);
  }
}
// O (+)= P V: P [128 x 128] 16-bit in TMEM (8 columns per K = 16 step), V MN-major in shared memory.
// O += P V over keys [64 half, 64 half + 64) (k-steps 4 half .. 4 half + 3): P's columns
// [32 half, 32 half + 32)
__device__ __forceinline__ void issue_pv_half(uint32_t d, uint32_t p, uint32_t v, uint32_t idesc, bool acc, int half) {
#pragma unroll
  for (int k4 = 0; k4 < 4; ++k4) {
    const int kk = 4 * half + k4;
    umma_ts(d, p + kk * 8, smem_desc_sw128(v + kk * 2048, HALF, 1024), idesc, (acc || kk > 0) ? 1u : 0u);
  }
}

template <typename T>
__device__ __forceinline__ uint32_t pk2(float lo, float hi);
template <> __device__ __forceinline__ uint32_t pk2<__nv_bfloat16>(float lo, float hi) { return pack_bf16x2(lo, hi); }
template <> __device__ __forceinline__ uint32_t pk2<__half>(float lo, float hi) { return pack_f16x2(lo, hi); }

template <typename T>
__global__ void __launch_bounds__(NTHREADS, 1) attn_fwd_sm100_kernel(const __grid_constant__ Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sb = smem_u32(smem);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  auto bar = [&](int i) { return sb + OFF_BAR + 8 * i; };
  volatile int* ring = reinterpret_cast<volatile int*>(smem + OFF_RING);

  const int* cu = p.cu;
  if (!p.persistent) {  // one ticket per CTA: a query block past its row's end leaves at once
    WorkTile w0;
    if (!decode_tile(p, cu, blockIdx.x, w0)) return;  // uniform: before any barrier or TMEM use
  }

  if (threadIdx.x == 0) {
    mbar_init(bar(B_Q), 1);
    mbar_init(bar(B_QE), 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(bar(B_KF + s), 1);
      mbar_init(bar(B_KE + s), 1);
      mbar_init(bar(B_VF + s), 1);
      mbar_init(bar(B_VE + s), 1);
      mbar_init(bar(B_SF + s), 1);
      mbar_init(bar(B_PR + s), 128);
      mbar_init(bar(B_PH + s), 128);
      mbar_init(bar(B_OF + s), 1);
      mbar_init(bar(B_OE + s), 128);
      mbar_init(bar(B_TF + s), 1);
      mbar_init(bar(B_TE + s), 1 + 256);  // the MMA thread and every softmax thread
    }
    mbar_init(bar(B_DONE), 1);
    fence_barrier_init();
  }
  if (warp == 9) {
    tmem_alloc(sb + OFF_TMEM, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(smem + OFF_TMEM);

  if (warp >= 8) {
    reg_set<kRegsLaunch, kRegsIssue>();
    if (warp == 8) {
      // ---------------------------------------------------------------- tickets + TMA producer
      if (lane == 0) {
        prefetch_tmap(&p.tq);
        prefetch_tmap(&p.tk);
        prefetch_tmap(&p.tv);
        unsigned* ticket = &g_ticket[p.slot];
        int k = 0;          // tiles published
        int q_loaded = 0;   // tiles whose Q load was issued
        uint32_t g = 0;     // K/V loads issued (ring position, across tiles)
        bool ok = true;
        while (ok) {
          WorkTile w;
          unsigned t;
          if (p.persistent) {
            do {
              t = atomicAdd(ticket, 1u);
            } while (t < p.n_tickets && !decode_tile(p, cu, t, w));
          } else {
            t = k == 0 && decode_tile(p, cu, blockIdx.x, w) ? blockIdx.x : p.n_tickets;
          }
          const bool end = t >= p.n_tickets;
          // ring slot k & 1 was last used by tile k - 2: wait until everyone read it
          if (k >= 2) ok = mbar_wait(bar(B_TE + (k & 1)), ((k - 2) >> 1) & 1, p.err, 106);
          if (!ok) break;
          ring[k & 1] = end ? -1 : static_cast<int>(t);
          mbar_arrive(bar(B_TF + (k & 1)));
          ++k;
          if (end) break;
          // Q of this tile once the previous tile's QK^T products are done with the Q buffers
          if (q_loaded >= 1) ok = mbar_wait(bar(B_QE), (q_loaded - 1) & 1, p.err, 107);
          if (!ok) break;
          mbar_expect_tx(bar(B_Q), w.has1 ? 2 * TILE : TILE);
          for (int hh = 0; hh < (w.has1 ? 2 : 1); ++hh)
            for (int c = 0; c < 2; ++c)
              load_half(sb + (hh ? OFF_Q1 : OFF_Q0) + c * HALF, &p.tq, bar(B_Q), p.order_q, 64 * c, w.start + w.m0,
                        w.h0 + hh);
          ++q_loaded;
          for (int j = 0; j < w.n_kv && ok; ++j, ++g) {
            const int s = g & 1;
            if (g >= 2) ok = mbar_wait(bar(B_KE + s), ((g - 2) >> 1) & 1, p.err, 101);
            if (!ok) break;
            mbar_expect_tx(bar(B_KF + s), TILE);
            for (int c = 0; c < 2; ++c)
              load_half(sb + OFF_K + s * TILE + c * HALF, &p.tk, bar(B_KF + s), p.order_k, 64 * c, w.start + j * BN, w.kvh);
            if (g >= 2) ok = mbar_wait(bar(B_VE + s), ((g - 2) >> 1) & 1, p.err, 102);
            if (!ok) {
              ++g;  // its K load is in flight
              break;
            }
            mbar_expect_tx(bar(B_VF + s), TILE);
            for (int c = 0; c < 2; ++c)
              load_half(sb + OFF_V + s * TILE + c * HALF, &p.tv, bar(B_VF + s), p.order_v, 64 * c, w.start + j * BN, w.kvh);
          }
        }
        // wind down: the last loads must have landed before the CTA exits
        for (uint32_t j = g >= 2 ? g - 2 : 0; j < g; ++j) {
          mbar_wait(bar(B_KF + (j & 1)), (j >> 1) & 1, p.err, 103);
          mbar_wait(bar(B_VF + (j & 1)), (j >> 1) & 1, p.err, 104);
        }
        if (q_loaded > 0) mbar_wait(bar(B_Q), (q_loaded - 1) & 1, p.err, 105);
      }
    } else if (warp == 9) {
      // ---------------------------------------------------------------- MMA issue (one thread)
      if (lane == 0) {
        constexpr int ab = std::is_same<T, __nv_bfloat16>::value ? 1 : 0;
        const uint32_t id_qk = idesc_f16(ab, BM, BN, 0, 0);
        const uint32_t id_pv = idesc_f16(ab, BM, D, 0, 1);
        const uint32_t tS0 = tmem, tS1 = tmem + 128, tO0 = tmem + 256, tO1 = tmem + 384;
        const uint32_t q0 = sb + OFF_Q0, q1 = sb + OFF_Q1;
        int k = 0, k1 = 0;                  // tiles taken; of them with a second query head
        uint32_t g = 0, g0 = 0, g1 = 0;     // K/V uses; softmax iterations of query tile 0 / 1
        bool ok = true;
        while (ok) {
          ok = mbar_wait(bar(B_TF + (k & 1)), (k >> 1) & 1, p.err, 208);
          if (!ok) break;
          const int t = ring[k & 1];
          mbar_arrive(bar(B_TE + (k & 1)));
          if (t < 0) break;
          WorkTile w;
          decode_tile(p, cu, static_cast<unsigned>(t), w);
          ok = mbar_wait(bar(B_Q), k & 1, p.err, 201) && mbar_wait(bar(B_KF + (g & 1)), (g >> 1) & 1, p.err, 202);
          if (!ok) break;
          // S0(0), S1(0): S0 / S1 were last read by the previous tile's PV products, issued before
          tc_fence_after();
          issue_qk(tS0, q0, sb + OFF_K + (g & 1) * TILE, id_qk);
          umma_commit(bar(B_SF + 0));
          if (w.has1) {
            issue_qk(tS1, q1, sb + OFF_K + (g & 1) * TILE, id_qk);
            umma_commit(bar(B_SF + 1));
          }
          umma_commit(bar(B_KE + (g & 1)));
          // O0 / O1 are overwritten by the tile's first PV: the previous tile's output must be read out
          if (k >= 1) ok = mbar_wait(bar(B_OE + 0), (k - 1) & 1, p.err, 209);
          if (ok && w.has1 && k1 >= 1) ok = mbar_wait(bar(B_OE + 1), (k1 - 1) & 1, p.err, 210);
          // one key block: PV0(j), [S0(j+1)], PV1(j), [S1(j+1)]; the last block (no next) is peeled
          // off so that the steady loop carries no per-block branches
          auto block = [&](auto has_next, int j) -> bool {
            constexpr bool next = decltype(has_next)::value;
            const int s = g & 1;
            const uint32_t v = sb + OFF_V + s * TILE;
            const uint32_t kn = sb + OFF_K + ((g + 1) & 1) * TILE;
            // each PV in two halves: keys 0-63 once the softmax has written their P, while it
            // computes the rest
            if (!mbar_wait(bar(B_VF + s), (g >> 1) & 1, p.err, 203) || !mbar_wait(bar(B_PH + 0), g0 & 1, p.err, 211))
              return false;
            tc_fence_after();
            issue_pv_half(tO0, tS0, v, id_pv, j > 0, 0);
            if (!mbar_wait(bar(B_PR + 0), g0 & 1, p.err, 204)) return false;
            tc_fence_after();
            issue_pv_half(tO0, tS0, v, id_pv, true, 1);
            ++g0;
            if (next) {
              if (!mbar_wait(bar(B_KF + ((g + 1) & 1)), ((g + 1) >> 1) & 1, p.err, 205)) return false;
              tc_fence_after();
              issue_qk(tS0, q0, kn, id_qk);
              umma_commit(bar(B_SF + 0));
            }
            if (w.has1) {
              if (!mbar_wait(bar(B_PH + 1), g1 & 1, p.err, 212)) return false;
              tc_fence_after();
              issue_pv_half(tO1, tS1, v, id_pv, j > 0, 0);
              if (!mbar_wait(bar(B_PR + 1), g1 & 1, p.err, 206)) return false;
              tc_fence_after();
              issue_pv_half(tO1, tS1, v, id_pv, true, 1);
              ++g1;
            }
            umma_commit(bar(B_VE + s));
            if (next) {
              if (w.has1) {
                issue_qk(tS1, q1, kn, id_qk);
                umma_commit(bar(B_SF + 1));
              }
              umma_commit(bar(B_KE + ((g + 1) & 1)));
            }
            ++g;
            return true;
          };
          for (int j = 0; ok && j + 1 < w.n_kv; ++j) ok = block(std::true_type{}, j);
          umma_commit(bar(B_QE));  // every QK^T of the tile is issued: Q is free once they are done
          if (ok) ok = block(std::false_type{}, w.n_kv - 1);
          if (!ok) break;
          umma_commit(bar(B_OF + 0));
          if (w.has1) umma_commit(bar(B_OF + 1));
          ++k;
          if (w.has1) ++k1;
        }
        umma_commit(bar(B_DONE));
        mbar_wait(bar(B_DONE), 0, p.err, 207);  // nothing in flight before TMEM is freed
      }
    }
  } else {
    reg_set<kRegsLaunch, kRegsSoftmax>();
    // ---------------------------------------------------------------- softmax of one query tile
    const int tile = warp >> 2;
    const int r = (warp & 3) * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const uint32_t tS = tmem + tile * 128 + lane_off;
    const uint32_t tO = tmem + 256 + tile * 128 + lane_off;
    int k = 0, kt = 0;     // tiles taken; of them with this query tile
    uint32_t gi = 0;       // softmax iterations of this query tile
    bool ok = true;
    // a bounded wait, made uniform across the warp (the TMEM accesses below are warp-collective)
    auto wait_w = [&](int b, int parity, int code) -> bool {
      return __all_sync(0xffffffffu, mbar_wait(bar(b), parity, p.err, code));
    };
    while (ok) {
      ok = wait_w(B_TF + (k & 1), (k >> 1) & 1, 305);
      if (!ok) break;
      const int t = ring[k & 1];
      mbar_arrive(bar(B_TE + (k & 1)));
      ++k;
      if (t < 0) break;
      WorkTile w;
      decode_tile(p, cu, static_cast<unsigned>(t), w);
      if (tile == 1 && !w.has1) continue;
      const int qi = w.m0 + r;
      float m_run = -INFINITY, l = 0.f;
      for (int j = 0; j < w.n_kv; ++j, ++gi) {
        ok = wait_w(B_SF + tile, gi & 1, 301 + tile);
        if (!ok) break;
        tc_fence_after();
        // keys past min(query, row end) are masked; only the diagonal / last block has any
        const int lim = min(qi, w.L - 1) - j * BN;  // last visible column of this row in this block
        const bool masked = lim < BN - 1;
        // pass 1: row max of the raw scores (scale > 0 commutes with max); keys past min(query, row
        // end) count as -inf. The second 64 columns stay in registers for pass 2.
        float mx = -INFINITY;
        uint32_t s1v[64];
        {
          uint32_t sv[64];
          tmem_ld32(tS, *reinterpret_cast<uint32_t(*)[32]>(&sv[0]));
          tmem_ld32(tS + 32, *reinterpret_cast<uint32_t(*)[32]>(&sv[32]));
          tmem_ld32(tS + 64, *reinterpret_cast<uint32_t(*)[32]>(&s1v[0]));
          tmem_ld32(tS + 96, *reinterpret_cast<uint32_t(*)[32]>(&s1v[32]));
          tmem_ld_wait();
          if (masked) {
#pragma unroll
            for (int c = 0; c < 64; ++c) {
              if (c > lim) sv[c] = __float_as_uint(-INFINITY);
              if (64 + c > lim) s1v[c] = __float_as_uint(-INFINITY);
            }
          }
          // four independent max chains (16 steps each instead of one of 64); max is exact, so the
          // result equals the single chain's
          float mq[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
          for (int c = 0; c < 64; c += 2) {
            const int a2 = (c >> 1) & 1;
            mq[a2] = fmax3(mq[a2], __uint_as_float(sv[c]), __uint_as_float(sv[c + 1]));
            mq[2 + a2] = fmax3(mq[2 + a2], __uint_as_float(s1v[c]), __uint_as_float(s1v[c + 1]));
          }
          mx = fmaxf(fmaxf(mq[0], mq[1]), fmaxf(mq[2], mq[3]));
        }
        const float m_new = fmaxf(m_run, mx * p.scale_log2);
        const bool resc = m_new > m_run + 8.f;
        float alpha = 1.f;
        if (resc) {
          alpha = ptx::ex2(m_run - m_new);
          m_run = m_new;
          l *= alpha;
        }
        if (j > 0 && __any_sync(0xffffffffu, resc)) {  // rescale this warp's O rows in TMEM
#pragma unroll
          for (int c4 = 0; c4 < 4; ++c4) {
            uint32_t o[32];
            tmem_ld32(tO + 32 * c4, o);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
            tmem_st32(tO + 32 * c4, o);
          }
          tmem_st_wait();
        }
        // pass 2: P = exp2(s * scale*log2e - m_run), packed FMA for the arguments and packed adds for
        // the sum; P (16-bit pairs) overwrites the first 64 columns of S: the first half's P over
        // columns 0-31 (re-read just before), then the second half's over 32-63
        const uint64_t sc2 = f2(p.scale_log2, p.scale_log2);
        const uint64_t nm2 = f2(-m_run, -m_run);
        uint64_t acc[4] = {0, 0, 0, 0};
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          uint32_t sv[64], pk[32];
          if (h == 0) {
            tmem_ld32(tS, *reinterpret_cast<uint32_t(*)[32]>(&sv[0]));
            tmem_ld32(tS + 32, *reinterpret_cast<uint32_t(*)[32]>(&sv[32]));
            tmem_ld_wait();
            if (masked) {
#pragma unroll
              for (int c = 0; c < 64; ++c)
                if (c > lim) sv[c] = __float_as_uint(-INFINITY);
            }
          }
#pragma unroll
          for (int c = 0; c < 32; ++c) {
            const uint32_t a0 = h ? s1v[2 * c] : sv[2 * c], a1 = h ? s1v[2 * c + 1] : sv[2 * c + 1];
            float x0, x1;
            f2split(ffma2(f2(__uint_as_float(a0), __uint_as_float(a1)), sc2, nm2), x0, x1);
            const float e0 = ptx::ex2(x0), e1 = ptx::ex2(x1);
            acc[c & 3] = fadd2(acc[c & 3], f2(e0, e1));
            pk[c] = pk2<T>(e0, e1);
          }
          tmem_st32(tS + 32 * h, pk);
          if (h == 0) {  // keys 0-63 of P are in TMEM: the first half of PV may start
            tmem_st_wait();
            tc_fence_before();
            mbar_arrive(bar(B_PH + tile));
          }
        }
        float s0, s1, s2, s3, s4, s5, s6, s7;
        f2split(acc[0], s0, s1);
        f2split(acc[1], s2, s3);
        f2split(acc[2], s4, s5);
        f2split(acc[3], s6, s7);
        l += ((s0 + s1) + (s2 + s3)) + ((s4 + s5) + (s6 + s7));
        tmem_st_wait();
        tc_fence_before();
        mbar_arrive(bar(B_PR + tile));
      }
      if (!ok) break;
      // output: O / l -> 16-bit row, logsumexp; then O is free for the next tile's first PV
      ok = wait_w(B_OF + tile, kt & 1, 311 + tile);
      if (!ok) break;
      tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      const int h = w.h0 + tile;
      // 32 columns at a time through this warp's staging rows (16-byte unit u of row x at unit
      // u ^ ((x >> 1) & 3): conflict-free both ways), then stored as 8 rows x 64 contiguous bytes
      // per instruction instead of 32 rows x 16 bytes; O is read in two halves (register budget)
      uint8_t* stg = smem + OFF_STAGE + warp * STAGE;
      const int rr = lane >> 2, uu = lane & 3;  // store lane map: row 8 i + rr, unit uu
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        uint32_t o[2][32];
        tmem_ld32(tO + 64 * half, o[0]);
        tmem_ld32(tO + 64 * half + 32, o[1]);
        tmem_ld_wait();
        if (half == 1) {  // O is free for the next tile's first PV
          tc_fence_before();
          mbar_arrive(bar(B_OE + tile));
          ++kt;
        }
#pragma unroll
        for (int c2 = 0; c2 < 2; ++c2) {
          const int c4 = 2 * half + c2;
          uint32_t wv[16];
#pragma unroll
          for (int i = 0; i < 16; ++i)
            wv[i] = pk2<T>(__uint_as_float(o[c2][2 * i]) * inv, __uint_as_float(o[c2][2 * i + 1]) * inv);
#pragma unroll
          for (int u = 0; u < 4; ++u)
            *reinterpret_cast<uint4*>(stg + lane * 64 + ((u ^ ((lane >> 1) & 3)) << 4)) =
                make_uint4(wv[4 * u], wv[4 * u + 1], wv[4 * u + 2], wv[4 * u + 3]);
          __syncwarp();
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int x = 8 * i + rr;             // row within the warp
            const int q = w.m0 + (warp & 3) * 32 + x;
            const uint4 val = *reinterpret_cast<const uint4*>(stg + x * 64 + ((uu ^ ((x >> 1) & 3)) << 4));
            if (q < w.L)
              *reinterpret_cast<uint4*>(static_cast<T*>(p.o) + (static_cast<int64_t>(w.start) + q) * p.o_tok +
                                        static_cast<int64_t>(h) * p.o_head + 32 * c4 + 8 * uu) = val;
          }
          __syncwarp();
        }
      }
      if (qi < w.L) p.lse[static_cast<int64_t>(h) * p.n_tok + w.start + qi] = (m_run + __log2f(l)) * kLn2;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (p.persistent && threadIdx.x == 0) {
    // every CTA has drawn its last ticket once it is here: the last one resets the slot
    __threadfence();
    if (atomicAdd(&g_exit[p.slot], 1u) == gridDim.x - 1) {
      atomicExch(&g_ticket[p.slot], 0u);
      atomicExch(&g_exit[p.slot], 0u);
    }
  }
  if (warp == 9) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

std::atomic<unsigned> g_next_slot{0};

}  // namespace

int fwd_sm100(const decik_tensor3& q, const decik_tensor3& k, const decik_tensor3& v, const decik_tensor3_mut& out,
              float* lse, const int32_t* cu, int n_rows, int max_len, int64_t n_tok, int n_heads, int n_kv,
              float scale, int dtype, cudaStream_t stream) {
  Params p;
  int rc = make_tile_map(&p.tq, q.ptr, q.tok_stride, q.head_stride, n_tok, n_heads, dtype, &p.order_q, BM);
  if (!rc) rc = make_tile_map(&p.tk, k.ptr, k.tok_stride, k.head_stride, n_tok, n_kv, dtype, &p.order_k, BN);
  if (!rc) rc = make_tile_map(&p.tv, v.ptr, v.tok_stride, v.head_stride, n_tok, n_kv, dtype, &p.order_v, BN);
  if (rc) return rc;
  p.o = out.ptr;
  p.o_tok = out.tok_stride;
  p.o_head = out.head_stride;
  p.lse = lse;
  p.cu = cu;
  p.n_tok = n_tok;
  p.n_heads = n_heads;
  p.groups = n_heads / n_kv;
  p.pairs = (p.groups + 1) / 2;
  p.n_mblocks = (max_len + BM - 1) / BM;
  p.n_rows = n_rows;
  p.zs = n_kv * p.pairs;
  p.scale_log2 = scale * kLog2e;
  p.err = attn_error_word();
  const uint64_t tickets = static_cast<uint64_t>(p.n_mblocks) * n_rows * p.zs;
  if (tickets >= (1ull << 31))
    return set_error(DECIK_ERR_UNSUPPORTED, "varlen_attn_fwd: too many tiles (%llu)", (unsigned long long)tickets);
  p.n_tickets = static_cast<unsigned>(tickets);
  // Ticket order. A tile's work grows with its query block, so taking the last query blocks of
  // every row first is the longest-first order that keeps the tail short. It spreads the CTAs
  // working at a time over all rows, each reading its own row's K / V: fine while K and V fit well
  // inside L2. Beyond that, one row's query blocks go together so that they share its K / V tiles
  // through L2 (the 7B block at 131,072 tokens).
  const int64_t kv_bytes = n_tok * n_kv * D * 2 * 2;
  p.heavy_first = kv_bytes <= l2_bytes() / 2;
  // Persistent CTAs pay off where tiles are short (their setup and output then weigh) and the
  // longest-first order puts few past-the-row-end tickets among them. The row-major order has a
  // run of such tickets per row and long tiles: there every CTA takes one ticket, its own index.
  p.persistent = p.heavy_first;
  p.slot = static_cast<int>(g_next_slot.fetch_add(1u) % kSlots);
  const dim3 grid(static_cast<unsigned>(p.persistent ? std::min<uint64_t>(sm_count(), tickets) : tickets));
  if (dtype == DECIK_BF16) {
    static std::atomic<unsigned long long> set{0};
    if (int rc = ensure_dyn_smem(attn_fwd_sm100_kernel<__nv_bfloat16>, kSmem, set, "attn_fwd_sm100")) return rc;
    attn_fwd_sm100_kernel<__nv_bfloat16><<<grid, NTHREADS, kSmem, stream>>>(p);
  } else {
    static std::atomic<unsigned long long> set{0};
    if (int rc = ensure_dyn_smem(attn_fwd_sm100_kernel<__half>, kSmem, set, "attn_fwd_sm100")) return rc;
    attn_fwd_sm100_kernel<__half><<<grid, NTHREADS, kSmem, stream>>>(p);
  }
  return check_launch("varlen_attn_fwd (sm100)");
}

}  // namespace attn
}  // namespace decik
