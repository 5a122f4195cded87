// Packed varlen causal GQA attention forward on the 5th-generation tensor cores (tcgen05 + TMEM,
// operands staged by TMA). Replaces the forward of VarlenSDPA (solution/varlen.py:144-151): one
// launch over every row of the packed sequence, GQA without expanding K/V, fully-masked causal
// tiles never visited, logsumexp written for the backward.
//
// CTA = one 128-query block of one row x two query heads of the same kv head (so each K/V tile
// loaded by TMA feeds two 128x128x128 QK^T and two PV products). 10 warps:
//   warps 0-3  softmax of query tile 0 (thread = one query row = one TMEM lane)
//   warps 4-7  softmax of query tile 1
//   warp 8     TMA producer: Q0, Q1 once, then K_j / V_j into a 2-stage ring
//   warp 9     TMEM allocation and the single-thread tcgen05.mma issue
// TMEM (512 columns): S0 [0,128), S1 [128,256), O0 [256,384), O1 [384,512); P (16-bit) overwrites
// the first 64 columns of its S. The MMA thread ping-pongs the two tiles so the tensor core runs
// one tile's QK^T / PV while the other tile's softmax runs:
//   S0(0) S1(0) | PV0(j) S0(j+1) PV1(j) S1(j+1) | ...
// Online softmax in the exp2 domain; O is rescaled in TMEM only when a row max grows by more than
// 2^8 (the final O / l is exact for any reference max). Every mbarrier wait is bounded: a wait that
// gives up records a code in the error word and the CTA winds down (waiting for its own MMAs and
// TMA loads, then freeing TMEM).
#include <cudaTypedefs.h>

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
constexpr int NTHREADS = 320;
constexpr int OFF_Q0 = 0, OFF_Q1 = TILE, OFF_K = 2 * TILE, OFF_V = 4 * TILE, OFF_BAR = 6 * TILE;
enum { B_Q = 0, B_KF = 1, B_KE = 3, B_VF = 5, B_VE = 7, B_SF = 9, B_PR = 11, B_OF = 13, B_DONE = 15, N_BAR = 16 };
constexpr int OFF_TMEM = OFF_BAR + N_BAR * 8;
constexpr int kSmem = OFF_TMEM + 16 + 1024;  // + slack for the 1024-byte alignment

struct Params {
  CUtensorMap tq, tk, tv;
  void* o;
  int64_t o_tok, o_head;
  float* lse;
  const int32_t* cu;
  int64_t n_tok;
  int n_heads, groups, pairs, n_mblocks, n_rows;
  int heavy_first;  // grid x = (row, kv head, pair), y = query block from the last; else see below
  int order_q, order_k, order_v;  // 0: coordinates (d, tok, head); 1: (d, head, tok)
  float scale_log2;
  int* err;
};

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
__device__ __forceinline__ void issue_pv(uint32_t d, uint32_t p, uint32_t v, uint32_t idesc, bool acc) {
#pragma unroll
  for (int kk = 0; kk < 8; ++kk)
    umma_ts(d, p + kk * 8, smem_desc_sw128(v + kk * 2048, HALF, 1024), idesc, (acc || kk > 0) ? 1u : 0u);
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

  // heavy_first: y walks the query blocks from the last (the most key blocks) for every row at once;
  // else x walks one row's query blocks from its last, y the rows, z the (kv head, pair)
  const int m_block = p.n_mblocks - 1 - static_cast<int>(p.heavy_first ? blockIdx.y : blockIdx.x);
  const int row = p.heavy_first ? static_cast<int>(blockIdx.x % p.n_rows) : static_cast<int>(blockIdx.y);
  const int z = p.heavy_first ? static_cast<int>(blockIdx.x / p.n_rows) : static_cast<int>(blockIdx.z);
  const int kvh = z / p.pairs;
  const int pair = z % p.pairs;
  const int h0 = kvh * p.groups + 2 * pair;
  const bool has1 = 2 * pair + 1 < p.groups;
  const int start = p.cu[row];
  const int L = p.cu[row + 1] - start;
  const int m0 = m_block * BM;
  if (m0 >= L) return;  // uniform: before any barrier or TMEM use
  const int n_kv = (min(m0 + BM, L) + BN - 1) / BN;
  auto bar = [&](int i) { return sb + OFF_BAR + 8 * i; };

  if (threadIdx.x == 0) {
    mbar_init(bar(B_Q), 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(bar(B_KF + s), 1);
      mbar_init(bar(B_KE + s), 1);
      mbar_init(bar(B_VF + s), 1);
      mbar_init(bar(B_VE + s), 1);
      mbar_init(bar(B_SF + s), 1);
      mbar_init(bar(B_PR + s), 128);
      mbar_init(bar(B_OF + s), 1);
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

  if (warp == 8) {
    // ---------------------------------------------------------------- TMA producer
    if (lane == 0) {
      prefetch_tmap(&p.tq);
      prefetch_tmap(&p.tk);
      prefetch_tmap(&p.tv);
      mbar_expect_tx(bar(B_Q), has1 ? 2 * TILE : TILE);
      for (int hh = 0; hh < (has1 ? 2 : 1); ++hh)
        for (int c = 0; c < 2; ++c)
          load_half(sb + (hh ? OFF_Q1 : OFF_Q0) + c * HALF, &p.tq, bar(B_Q), p.order_q, 64 * c, start + m0, h0 + hh);
      int issued = 0;
      bool ok = true;
      for (int j = 0; j < n_kv && ok; ++j) {
        const int s = j & 1;
        if (j >= 2) ok = mbar_wait(bar(B_KE + s), ((j - 2) >> 1) & 1, p.err, 101);
        if (!ok) break;
        mbar_expect_tx(bar(B_KF + s), TILE);
        for (int c = 0; c < 2; ++c)
          load_half(sb + OFF_K + s * TILE + c * HALF, &p.tk, bar(B_KF + s), p.order_k, 64 * c, start + j * BN, kvh);
        if (j >= 2) ok = mbar_wait(bar(B_VE + s), ((j - 2) >> 1) & 1, p.err, 102);
        if (!ok) break;
        mbar_expect_tx(bar(B_VF + s), TILE);
        for (int c = 0; c < 2; ++c)
          load_half(sb + OFF_V + s * TILE + c * HALF, &p.tv, bar(B_VF + s), p.order_v, 64 * c, start + j * BN, kvh);
        issued = j + 1;
      }
      // wind down: the loads of the last two uses must have landed before the CTA exits
      for (int j = max(0, issued - 2); j < issued; ++j) {
        mbar_wait(bar(B_KF + (j & 1)), (j >> 1) & 1, p.err, 103);
        mbar_wait(bar(B_VF + (j & 1)), (j >> 1) & 1, p.err, 104);
      }
      mbar_wait(bar(B_Q), 0, p.err, 105);
    }
  } else if (warp == 9) {
    // ---------------------------------------------------------------- MMA issue (one thread)
    if (lane == 0) {
      constexpr int ab = std::is_same<T, __nv_bfloat16>::value ? 1 : 0;
      const uint32_t id_qk = idesc_f16(ab, BM, BN, 0, 0);
      const uint32_t id_pv = idesc_f16(ab, BM, D, 0, 1);
      const uint32_t tS0 = tmem, tS1 = tmem + 128, tO0 = tmem + 256, tO1 = tmem + 384;
      const uint32_t q0 = sb + OFF_Q0, q1 = sb + OFF_Q1;
      bool ok = mbar_wait(bar(B_Q), 0, p.err, 201) && mbar_wait(bar(B_KF), 0, p.err, 202);
      if (ok) {
        tc_fence_after();
        issue_qk(tS0, q0, sb + OFF_K, id_qk);
        umma_commit(bar(B_SF + 0));
        if (has1) {
          issue_qk(tS1, q1, sb + OFF_K, id_qk);
          umma_commit(bar(B_SF + 1));
        }
        umma_commit(bar(B_KE + 0));
      }
      for (int j = 0; j < n_kv && ok; ++j) {
        const int s = j & 1;
        const uint32_t v = sb + OFF_V + s * TILE;
        const bool next = j + 1 < n_kv;
        const uint32_t kn = sb + OFF_K + ((j + 1) & 1) * TILE;
        ok = mbar_wait(bar(B_VF + s), (j >> 1) & 1, p.err, 203) && mbar_wait(bar(B_PR + 0), j & 1, p.err, 204);
        if (!ok) break;
        tc_fence_after();
        issue_pv(tO0, tS0, v, id_pv, j > 0);
        if (next) {
          ok = mbar_wait(bar(B_KF + ((j + 1) & 1)), ((j + 1) >> 1) & 1, p.err, 205);
          if (!ok) break;
          tc_fence_after();
          issue_qk(tS0, q0, kn, id_qk);
          umma_commit(bar(B_SF + 0));
        }
        if (has1) {
          ok = mbar_wait(bar(B_PR + 1), j & 1, p.err, 206);
          if (!ok) break;
          tc_fence_after();
          issue_pv(tO1, tS1, v, id_pv, j > 0);
        }
        umma_commit(bar(B_VE + s));
        if (next) {
          if (has1) {
            issue_qk(tS1, q1, kn, id_qk);
            umma_commit(bar(B_SF + 1));
          }
          umma_commit(bar(B_KE + ((j + 1) & 1)));
        }
      }
      umma_commit(bar(B_OF + 0));
      umma_commit(bar(B_OF + 1));
      umma_commit(bar(B_DONE));
      mbar_wait(bar(B_DONE), 0, p.err, 207);  // nothing in flight before TMEM is freed
    }
  } else if (warp < 8 && (warp < 4 || has1)) {
    // ---------------------------------------------------------------- softmax of one query tile
    const int tile = warp >> 2;
    const int r = (warp & 3) * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const uint32_t tS = tmem + tile * 128 + lane_off;
    const uint32_t tO = tmem + 256 + tile * 128 + lane_off;
    const int qi = m0 + r;
    float m_run = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < n_kv; ++j) {
      ok = mbar_wait(bar(B_SF + tile), j & 1, p.err, 301 + tile);
      if (!ok) break;
      tc_fence_after();
      // keys past min(query, row end) are masked; only the diagonal / last block has any
      const int lim = min(qi, L - 1) - j * BN;  // last visible column of this row in this block
      const bool masked = lim < BN - 1;
      // pass 1: row max of the raw scores (scale > 0 commutes with max), 64 columns at a time
      float mx = -INFINITY;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        uint32_t sv[64];
        tmem_ld32(tS + 64 * h, *reinterpret_cast<uint32_t(*)[32]>(&sv[0]));
        tmem_ld32(tS + 64 * h + 32, *reinterpret_cast<uint32_t(*)[32]>(&sv[32]));
        tmem_ld_wait();
        if (masked) {
#pragma unroll
          for (int c = 0; c < 64; ++c)
            if (64 * h + c > lim) sv[c] = __float_as_uint(-INFINITY);
        }
#pragma unroll
        for (int c = 0; c < 64; c += 2) mx = fmax3(mx, __uint_as_float(sv[c]), __uint_as_float(sv[c + 1]));
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
      // the sum; P (16-bit pairs) overwrites the first 64 columns of S
      const uint64_t sc2 = f2(p.scale_log2, p.scale_log2);
      const uint64_t nm2 = f2(-m_run, -m_run);
      uint64_t acc[4] = {0, 0, 0, 0};
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        uint32_t sv[64], pk[32];
        tmem_ld32(tS + 64 * h, *reinterpret_cast<uint32_t(*)[32]>(&sv[0]));
        tmem_ld32(tS + 64 * h + 32, *reinterpret_cast<uint32_t(*)[32]>(&sv[32]));
        tmem_ld_wait();
        if (masked) {
#pragma unroll
          for (int c = 0; c < 64; ++c)
            if (64 * h + c > lim) sv[c] = __float_as_uint(-INFINITY);
        }
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          float x0, x1;
          f2split(ffma2(f2(__uint_as_float(sv[2 * c]), __uint_as_float(sv[2 * c + 1])), sc2, nm2), x0, x1);
          const float e0 = ptx::ex2(x0), e1 = ptx::ex2(x1);
          acc[c & 3] = fadd2(acc[c & 3], f2(e0, e1));
          pk[c] = pk2<T>(e0, e1);
        }
        tmem_st32(tS + 32 * h, pk);
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
    // epilogue: O / l -> 16-bit row, logsumexp
    if (ok && mbar_wait(bar(B_OF + tile), 0, p.err, 311 + tile)) {
      tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      const int h = h0 + tile;
      T* dst = static_cast<T*>(p.o) + (static_cast<int64_t>(start) + qi) * p.o_tok + static_cast<int64_t>(h) * p.o_head;
#pragma unroll
      for (int c4 = 0; c4 < 4; ++c4) {
        uint32_t o[32];
        tmem_ld32(tO + 32 * c4, o);
        tmem_ld_wait();
        uint32_t w[16];
#pragma unroll
        for (int i = 0; i < 16; ++i)
          w[i] = pk2<T>(__uint_as_float(o[2 * i]) * inv, __uint_as_float(o[2 * i + 1]) * inv);
        if (qi < L) {
#pragma unroll
          for (int i = 0; i < 4; ++i)
            reinterpret_cast<uint4*>(dst + 32 * c4)[i] = make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
        }
      }
      if (qi < L) p.lse[static_cast<int64_t>(h) * p.n_tok + start + qi] = (m_run + __log2f(l)) * kLn2;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

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
  p.scale_log2 = scale * kLog2e;
  p.err = attn_error_word();
  p.n_rows = n_rows;
  // Launch order (blocks start in grid order, x fastest). A CTA's work grows with its query block,
  // so starting the last query blocks of every row first is the longest-first order that keeps the
  // tail short. It spreads the resident CTAs over all rows, each reading its own row's K / V: fine
  // while K and V fit well inside L2. Beyond that, one row's query blocks launch together so that
  // they share its K / V tiles through L2.
  const int64_t kv_bytes = n_tok * n_kv * D * 2 * 2;
  const int64_t zs = static_cast<int64_t>(n_kv) * p.pairs;
  p.heavy_first = kv_bytes <= l2_bytes() / 2 && n_rows * zs <= INT32_MAX && p.n_mblocks <= 65535;
  if (!p.heavy_first && (n_rows > 65535 || zs > 65535))
    return set_error(DECIK_ERR_UNSUPPORTED, "varlen_attn_fwd: grid too large (%d rows)", n_rows);
  const dim3 grid = p.heavy_first ? dim3(static_cast<unsigned>(n_rows * zs), static_cast<unsigned>(p.n_mblocks), 1)
                                  : dim3(static_cast<unsigned>(p.n_mblocks), static_cast<unsigned>(n_rows),
                                         static_cast<unsigned>(zs));
  if (dtype == DECIK_BF16) {
    static bool set = false;
    if (!set) {
      cudaFuncSetAttribute(attn_fwd_sm100_kernel<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
      set = true;
    }
    attn_fwd_sm100_kernel<__nv_bfloat16><<<grid, NTHREADS, kSmem, stream>>>(p);
  } else {
    static bool set = false;
    if (!set) {
      cudaFuncSetAttribute(attn_fwd_sm100_kernel<__half>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
      set = true;
    }
    attn_fwd_sm100_kernel<__half><<<grid, NTHREADS, kSmem, stream>>>(p);
  }
  return check_launch("varlen_attn_fwd (sm100)");
}

}  // namespace attn
}  // namespace decik
