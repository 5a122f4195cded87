// The projection GEMMs of the attention block on the 5th-generation tensor cores (tcgen05 + TMEM,
// operands staged by TMA), with the work around them fused in. They replace the cuBLAS calls of
// the block: the forward's q|k|v|LoRA-down F.linear and the backward's dX / dA / dB products
// (the three NF4Linear GEMMs of the reference, solution/nf4.py:93-104, and the LoRA branch's
// matmuls, solution/attn.py:217-273).
//
// Forward, two kernels:
// 1. x_cast_lora_down_kernel: x fp32 [T, H] -> x16 = dt(x) [T, H] and u = [dt(x16 [A_q; A_v]^T) | 1 | 0]
//    [T, 64] (the reference's lora_A products, solution/attn.py:225-227, and a column of ones) in
//    one pass over x: the cast has to read x anyway, and the rank-32 product rides along on mma.sync.
// 2. proj_gemm_kernel<EPI_QKV>: y = x16 [W_q; W_k; W_v]^T + u b_ext^T on tcgen05 CTA pairs, tile
//    256 tokens x 256 outputs (two heads), K-major A and B from TMA, fp32 accumulators in TMEM (two
//    buffers, so a tile's epilogue overlaps the next tile's MMAs). The last K block multiplies u by
//    b_ext = [scaling B_q | scaling B_v | bias | 0]: the LoRA-up of q and v and the bias land in the
//    accumulator. The epilogue is RoPE with separate roundings and no FMA (solution/attn.py:39-60)
//    on q and k, and the head-major q / k and token-major v tiles leave through shared memory by
//    TMA stores. y never reaches HBM.
// Backward:
// 3. proj_gemm_kernel<EPI_F32>: dx = dy W_cat on CTA pairs, tile 256 x 192 (dy [T, 2080] and the
//    transposed weight W_cat^T [H, 2080], both K-major), fp32 out by TMA stores: the three
//    NF4Linear input gradients and both LoRA input gradients summed in one product (K = 2080, the
//    tail zero-filled by TMA).
// 4. lora_grad_kernel: dA = du^T x16 [32, H] and dB = scaling g^T u [(Hq + Hk) 128, 16] as
//    token-chunked mma.sync products reduced into fp32 outputs (red.global.add).
// The MLP node uses the same kernel for gate | up with SwiGLU in the epilogue (EPI_SWIGLU) and for
// grad_hidden = grad W_down with the SwiGLU backward in the epilogue (EPI_DSWIGLU).
//
// GEMM kernel roles (12 warps, one CTA per SM, persistent over tiles in n-fastest order so the
// CTAs running together share their A row tiles in L2): warp 0 TMA producer (one thread), warp 1
// TMEM allocation and the single-thread tcgen05.mma issue (the pair's leader CTA issues for both),
// warps 2-3 idle, warps 4-11 the epilogue (warp w reads TMEM lanes 32 (w % 4) .. + 31; warps 4-7
// and 8-11 split the tile's columns). No TMA load uses cluster multicast: each CTA of a pair loads
// its own A rows and its own half of B. Every mbarrier wait is bounded (sm100::mbar_wait): one that
// gives up records a code in the error word and the CTA winds down.
#include <cudaTypedefs.h>

#include <atomic>
#include <type_traits>

#include "common.cuh"
#include "norm_math.cuh"
#include "ptx.cuh"
#include "sm100.cuh"
#include "swiglu_math.cuh"

namespace decik {
namespace attn {
int* attn_error_word();
int make_tile_map_ex(CUtensorMap* map, const void* ptr, int64_t tok_stride, int64_t head_stride, int64_t n_tok,
                     int n_heads, int dtype, int* order, int box_rows, int box_inner, int swizzle_bytes);
int make_map_2d(CUtensorMap* map, const void* ptr, int dtype, uint64_t inner, uint64_t outer, uint64_t row_bytes,
                uint32_t box_inner, uint32_t box_outer, int swizzle_bytes = 128);
}  // namespace attn

namespace proj {
namespace {

using namespace sm100;

constexpr int BM = 128, BK = 64, NTHREADS = 384, kEpiWarps = 8, kD = 128, kR = 16;
// epilogues: EPI_QKV the attention projections (RoPE, head-major q / k, v); EPI_F32 fp32 out;
// EPI_STORE16 / EPI_STORE16_MN 16-bit out (B K-major / MN-major); EPI_SWIGLU the MLP's gate | up
// with SwiGLU (writes gu and silu(gate) * up); EPI_DSWIGLU grad_hidden . with the SwiGLU backward
// (writes [dgate | dup])
enum { EPI_QKV = 0, EPI_F32 = 1, EPI_STORE16 = 2, EPI_STORE16_MN = 3, EPI_SWIGLU = 4, EPI_DSWIGLU = 5 };

template <int EPI> struct Cfg;
template <> struct Cfg<EPI_QKV> {  // two heads per tile; a CTA pair holds one head each of B
  static constexpr int BN = 256, STAGES = 4;
  static constexpr bool B_MN = false;
};
// EPI_F32 / EPI_STORE16 produce outputs of hidden = 1536 columns (dX, the down projection):
// 256 x 192 pair tiles give 1536 / 192 = 8 column tiles, 512 tiles at 16,384 rows = 6.9 rounds of
// 74 pairs, where 256 x 256 tiles leave the sixth round 19 % full (the block's dX: 126 us with
// 256 x 256 tiles, 92-96 us with 256 x 192). B is K-major (the caller passes the transposed weight
// for dX).
template <> struct Cfg<EPI_F32> {
  static constexpr int BN = 192, STAGES = 5;
  static constexpr bool B_MN = false;
};
template <> struct Cfg<EPI_STORE16> {
  static constexpr int BN = 192, STAGES = 5;
  static constexpr bool B_MN = false;
};
template <> struct Cfg<EPI_STORE16_MN> {
  static constexpr int BN = 256, STAGES = 4;
  static constexpr bool B_MN = true;
};
template <> struct Cfg<EPI_SWIGLU> {  // a pair's tile: 128 gate columns (CTA 0's B) | the same 128 up (CTA 1's)
  static constexpr int BN = 256, STAGES = 4;
  static constexpr bool B_MN = false;
};
template <> struct Cfg<EPI_DSWIGLU> {
  static constexpr int BN = 256, STAGES = 4;
  static constexpr bool B_MN = true;
};

// PAIR: the tile is computed by a cluster of two CTAs with cta_group::2 MMAs (M = 256: each CTA
// its own 128 rows of A; B split by its N columns, BN / 2 rows in each CTA's shared memory)
template <int EPI, bool PAIR>
struct Layout {
  static constexpr int BN = Cfg<EPI>::BN;
  static constexpr int S = PAIR ? Cfg<EPI>::STAGES : (EPI == EPI_QKV ? 3 : Cfg<EPI>::STAGES);
  static constexpr int A_BYTES = BM * BK * 2;  // 128 rows x 128 B, 128-byte swizzle
  static constexpr int B_BYTES = (PAIR ? BN / 2 : BN) * BK * 2;
  static constexpr int OFF_A = 0;
  static constexpr int OFF_B = S * A_BYTES;
  // per epilogue warp: EPI_F32 two 4 KB staging tiles (double buffer); EPI_QKV one 4 KB staging
  // tile (the tile's two heads x [32 rows x 32 columns], 64-byte swizzle) and its RoPE tables (cos,
  // sin: 32 rows x 16 fp32, the 16-byte pieces of a row XOR-swizzled by (row / 2) % 4 so that both
  // the coalesced fills and each thread's row reads are conflict-free)
  static constexpr int OFF_STG = OFF_B + S * B_BYTES;
  static constexpr int STG_WARP = EPI == EPI_QKV ? 4096 : (EPI == EPI_SWIGLU ? 12288 : 8192);
  static constexpr int OFF_TAB = OFF_STG + kEpiWarps * STG_WARP;
  // per warp: EPI_QKV the RoPE tables, EPI_DSWIGLU the gate / up values of 32 rows x 32 columns
  static constexpr int TAB_WARP = (EPI == EPI_QKV || EPI == EPI_DSWIGLU) ? 2 * 32 * 64 : 0;
  static constexpr int OFF_BAR = OFF_TAB + kEpiWarps * TAB_WARP;
  static constexpr int N_BAR = 2 * S + 5;  // full[S], empty[S], acc_full[2], acc_empty[2], done
  static constexpr int OFF_TMEM = OFF_BAR + 8 * N_BAR;
  static constexpr int SMEM = OFF_TMEM + 16 + 1024;  // + slack for the 1024-byte alignment
  static_assert(SMEM <= 227 * 1024, "shared memory");
  static_assert(OFF_STG % 1024 == 0, "staging tiles need the swizzle atom's alignment");
};

struct Params {
  CUtensorMap ta, tb;     // A [M, K] K-major; B [N, K] K-major or [K, N] (MN-major)
  CUtensorMap ta2, tb2;   // EPI_QKV with LoRA: one more K block, A = u [M, 64], B = [N, 64] scaled lora_B
  CUtensorMap to[3];      // EPI_QKV: q, k, v tile maps; EPI_F32: the fp32 output
  int order[3];           // tile-map coordinate order of q, k, v (0: d, tok, head; 1: d, head, tok)
  int64_t M;
  int N, K, n_tiles_n, n_tiles;
  int lora;               // EPI_QKV: the extra K block (u x [scaled lora_B | bias]) joins the K loop
  int b_tile_step;        // PAIR, B K-major: rows of B per column tile; the CTA of rank r loads
  int b_rank_off;         //   rows tile * b_tile_step + r * b_rank_off (MN-major B: its columns)
  const void* gu;         // EPI_DSWIGLU: the forward's [gate | up] 16-bit [M, 2 inter]
  int64_t ld_gu;
  int inter;              // EPI_SWIGLU / EPI_DSWIGLU
  float scaling;
  const float* cosp;
  const float* sinp;
  int hq, hk;
  int* err;
};

// Tile t -> (row block, column block). Tiles go in groups of kGroupRows row blocks, row block
// fastest within a group: the tiles resident at a time share a few row blocks of A and a few column
// blocks of B, so both stay in L2 while the output streams through it (column block fastest over
// all rows re-read B from HBM once the output had pushed it out of L2).
constexpr int kGroupRows = 16;
__device__ __forceinline__ void tile_coords(int tile, int n_tiles_n, int m_tiles, int& mt, int& nt) {
  const int per_group = kGroupRows * n_tiles_n;
  const int g = tile / per_group, r = tile % per_group;
  const int rows = min(kGroupRows, m_tiles - g * kGroupRows);
  mt = g * kGroupRows + r % rows;
  nt = r / rows;
}

template <typename T>
__device__ __forceinline__ float rnd(float x) {
  return Dt<T>::to_f(Dt<T>::from_f(x));
}

// the separate SwiGLU kernels' sigmoid (swiglu.cu)
using swiglu::sigmoid;

// one row (this lane's) of 32 fp32 values (bit patterns in v) rounded to T into a [32 rows x 32]
// 16-bit staging tile with the 64-byte swizzle (16-byte piece p of row r at p ^ ((r / 2) % 4))
template <typename T>
__device__ __forceinline__ void store_row32(uint8_t* tile, int lane, const uint32_t (&v)[32]) {
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    float f[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) f[e] = __uint_as_float(v[8 * j + e]);
    *reinterpret_cast<uint4*>(tile + lane * 64 + ((j ^ ((lane >> 1) & 3)) << 4)) = pack8<T>(f);
  }
}

template <typename T, int EPI, bool PAIR>
__global__ void __launch_bounds__(NTHREADS, 1) proj_gemm_kernel(const __grid_constant__ Params p) {
  using L = Layout<EPI, PAIR>;
  constexpr int BN = L::BN, S = L::S;
  constexpr bool BMN = Cfg<EPI>::B_MN;
  // PAIR: rank 0 is the leader: its mbarriers count both CTAs' loads and epilogues, its thread
  // issues the MMAs; pairs walk tiles of 256 rows
  const uint32_t rank = PAIR ? cluster_rank() : 0u;
  const int unit = PAIR ? static_cast<int>(blockIdx.x >> 1) : static_cast<int>(blockIdx.x);
  const int n_units = PAIR ? static_cast<int>(gridDim.x >> 1) : static_cast<int>(gridDim.x);
  constexpr int TM = PAIR ? 2 * BM : BM;  // rows per tile
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sb = smem_u32(smem);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const auto full = [&](int s) { return sb + L::OFF_BAR + 8 * s; };
  const auto empty = [&](int s) { return sb + L::OFF_BAR + 8 * (S + s); };
  const auto acc_full = [&](int b) { return sb + L::OFF_BAR + 8 * (2 * S + b); };
  const auto acc_empty = [&](int b) { return sb + L::OFF_BAR + 8 * (2 * S + 2 + b); };
  const uint32_t done = sb + L::OFF_BAR + 8 * (2 * S + 4);

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(full(s), 1);
      mbar_init(empty(s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(acc_full(b), 1);
      mbar_init(acc_empty(b), PAIR ? 2 * kEpiWarps : kEpiWarps);
    }
    mbar_init(done, 1);
    fence_barrier_init();
  }
  if (warp == 1) {
    if constexpr (PAIR) {
      tmem_alloc_pair(sb + L::OFF_TMEM, 512);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(sb + L::OFF_TMEM, 512);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  __syncthreads();
  if constexpr (PAIR) cluster_sync();  // the leader's barriers exist before the peer signals them
  tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(smem + L::OFF_TMEM);
  const int nk = (p.K + BK - 1) / BK;
  const int nkt = nk + (EPI == EPI_QKV && p.lora ? 1 : 0);  // K blocks per tile, the LoRA one last

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      prefetch_tmap(&p.ta);
      prefetch_tmap(&p.tb);
      uint32_t it = 0;
      bool ok = true;
      for (int tile = unit; tile < p.n_tiles && ok; tile += n_units) {
        // this CTA's A rows and B rows (columns of an MN-major B) of the tile
        int mt, nt;
        tile_coords(tile, p.n_tiles_n, p.n_tiles / p.n_tiles_n, mt, nt);
        const int m0 = mt * TM + static_cast<int>(rank) * BM;
        const int n0 = PAIR ? nt * p.b_tile_step + static_cast<int>(rank) * p.b_rank_off : nt * BN;
        for (int kb = 0; kb < nkt; ++kb, ++it) {
          const int s = static_cast<int>(it % S);
          if (it >= static_cast<uint32_t>(S) && !(ok = mbar_wait(empty(s), ((it / S) - 1) & 1, p.err, 301))) break;
          if constexpr (PAIR) {
            // both CTAs' bytes complete on the leader's full barrier
            const uint32_t fb = map_to_rank(full(s), 0);
            if (rank == 0) mbar_expect_tx(full(s), 2 * (L::A_BYTES + L::B_BYTES));
            if (kb == nk) {
              tma_load_2d_pair(sb + L::OFF_A + s * L::A_BYTES, &p.ta2, fb, 0, m0);
              tma_load_2d_pair(sb + L::OFF_B + s * L::B_BYTES, &p.tb2, fb, 0, n0);
            } else {
              tma_load_2d_pair(sb + L::OFF_A + s * L::A_BYTES, &p.ta, fb, kb * BK, m0);
              if constexpr (!BMN) {
                tma_load_2d_pair(sb + L::OFF_B + s * L::B_BYTES, &p.tb, fb, kb * BK, n0);
              } else {  // this CTA's BN / 2 columns of B as 64-column blocks (MN-major)
#pragma unroll
                for (int j = 0; j < BN / 2 / 64; ++j)
                  tma_load_2d_pair(sb + L::OFF_B + s * L::B_BYTES + j * (64 * BK * 2), &p.tb, fb, n0 + 64 * j, kb * BK);
              }
            }
            continue;
          }
          mbar_expect_tx(full(s), L::A_BYTES + L::B_BYTES);
          if (kb == nk) {  // the LoRA K block: u [tokens, 64] against the scaled lora_B columns
            tma_load_2d(sb + L::OFF_A + s * L::A_BYTES, &p.ta2, full(s), 0, m0);
            tma_load_2d(sb + L::OFF_B + s * L::B_BYTES, &p.tb2, full(s), 0, n0);
            continue;
          }
          tma_load_2d(sb + L::OFF_A + s * L::A_BYTES, &p.ta, full(s), kb * BK, m0);
          if constexpr (!BMN) {
            tma_load_2d(sb + L::OFF_B + s * L::B_BYTES, &p.tb, full(s), kb * BK, n0);
          } else {
#pragma unroll
            for (int j = 0; j < BN / 64; ++j)
              tma_load_2d(sb + L::OFF_B + s * L::B_BYTES + j * (64 * BK * 2), &p.tb, full(s), n0 + 64 * j, kb * BK);
          }
        }
      }
      // wind down: the loads in flight land before the CTA leaves (a pair's loads all complete on
      // the leader's barriers; the peer stays until the leader has waited, at the closing cluster sync)
      if (rank == 0)
        for (uint32_t j = it > static_cast<uint32_t>(S) ? it - S : 0; j < it; ++j)
          mbar_wait(full(static_cast<int>(j % S)), (j / S) & 1, p.err, 302);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issue (one thread)
    if (lane == 0 && rank == 0) {
      constexpr int ab = std::is_same<T, __nv_bfloat16>::value ? 1 : 0;
      const uint32_t idesc = idesc_f16(ab, TM, BN, 0, BMN ? 1 : 0);
      uint32_t it = 0;
      int i = 0;
      bool ok = true;
      for (int tile = unit; tile < p.n_tiles && ok; tile += n_units, ++i) {
        const int b = i & 1;
        if (i >= 2 && !(ok = mbar_wait(acc_empty(b), ((i >> 1) - 1) & 1, p.err, 311))) break;
        tc_fence_after();
        const uint32_t d = tmem + b * 256;
        for (int kb = 0; kb < nkt; ++kb, ++it) {
          const int s = static_cast<int>(it % S);
          if (!(ok = mbar_wait(full(s), (it / S) & 1, p.err, 312))) break;
          tc_fence_after();
          const uint32_t a = sb + L::OFF_A + s * L::A_BYTES, bb = sb + L::OFF_B + s * L::B_BYTES;
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            const uint64_t ad = smem_desc_sw128(a + kk * 32, 16, 1024);
            const uint64_t bd = BMN ? smem_desc_sw128(bb + kk * 2048, 64 * BK * 2, 1024)
                                    : smem_desc_sw128(bb + kk * 32, 16, 1024);
            if constexpr (PAIR) umma_ss_pair(d, ad, bd, idesc, (kb | kk) != 0 ? 1u : 0u);
            else umma_ss(d, ad, bd, idesc, (kb | kk) != 0 ? 1u : 0u);
          }
          if constexpr (PAIR) umma_commit_pair_mc(empty(s), 0x3);  // both CTAs' stage s is free
          else umma_commit(empty(s));
        }
        if (!ok) break;
        if constexpr (PAIR) umma_commit_pair_mc(acc_full(b), 0x3);
        else umma_commit(acc_full(b));
      }
      // every MMA this thread issued has completed before TMEM is freed
      if constexpr (PAIR) umma_commit_pair_mc(done, 0x1);
      else umma_commit(done);
      mbar_wait(done, 0, p.err, 313);
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------------------ epilogue
    const int ew = warp - 4, wg = ew >> 2, q4 = warp & 3;
    uint8_t* stg = smem + L::OFF_STG + ew * L::STG_WARP;
    const uint32_t stg_s = sb + L::OFF_STG + ew * L::STG_WARP;
    const uint32_t lane_base = static_cast<uint32_t>(32 * q4) << 16;
    uint32_t n_chunks = 0;  // EPI_F32: staging tiles used so far (double buffer)
    int i = 0;
    // PAIR: this CTA's accumulator rows are its own 128 rows of the tile, all BN columns; the
    // buffer is released on the leader's barrier
    const uint32_t acc_empty_leader0 = PAIR ? map_to_rank(acc_empty(0), 0) : acc_empty(0);
    const uint32_t acc_empty_leader1 = PAIR ? map_to_rank(acc_empty(1), 0) : acc_empty(1);
    // EPI_DSWIGLU: the forward's gate and up of the warp's 32 rows x 32 columns j.. come in by
    // coalesced cp.async into a swizzled table ([gate | up][32 rows][64 B]); a chunk's table is
    // issued one step ahead (the first chunk of a tile before its accumulator is ready) so the HBM
    // latency overlaps the previous chunk's work
    uint8_t* gu_tab = smem + L::OFF_TAB + ew * L::TAB_WARP;
    const auto load_gu = [&](int64_t row_base, int j) {
      const T* gu = static_cast<const T*>(p.gu);
#pragma unroll
      for (int i2 = 0; i2 < 8; ++i2) {
        const int piece = lane + 32 * i2;
        const int which = piece >> 7, row = (piece >> 2) & 31, c4 = piece & 3;
        const int64_t rr = row_base + row < p.M ? row_base + row : p.M - 1;
        const T* src = gu + rr * p.ld_gu + (which ? p.inter : 0) + j + 8 * c4;
        ptx::cp_async16(ptx::smem_u32(gu_tab + which * 2048 + row * 64 + ((c4 ^ ((row >> 1) & 3)) << 4)), src, true);
      }
      ptx::cp_async_commit();
    };
    for (int tile = unit; tile < p.n_tiles; tile += n_units, ++i) {
      int mt, nt;
      tile_coords(tile, p.n_tiles_n, p.n_tiles / p.n_tiles_n, mt, nt);
      const int m0 = mt * TM + static_cast<int>(rank) * BM, n0 = nt * BN;
      const int b = i & 1;
      const int64_t row0 = m0 + 32 * q4;
      if constexpr (EPI == EPI_DSWIGLU) load_gu(row0, n0 + wg * (BN / 2));
      bool ok = mbar_wait(acc_full(b), (i >> 1) & 1, p.err, 321);
      // EPI_QKV: the eight epilogue warps leave together (they meet at named barriers below)
      if constexpr (EPI == EPI_QKV) ok = named_bar_and(1, 256, ok);
      if (!ok) {
        if constexpr (EPI == EPI_DSWIGLU) ptx::cp_async_wait<0>();  // no copy may land after the CTA leaves
        break;
      }
      tc_fence_after();
      const uint32_t tacc = tmem + lane_base + b * 256;
      if constexpr (EPI == EPI_F32) {
#pragma unroll 1
        for (int c = 0; c < BN / 2; c += 32, ++n_chunks) {
          const int col = wg * (BN / 2) + c;
          uint32_t v[32];
          tmem_ld32(tacc + col, v);
          tmem_ld_wait();
          if (lane == 0) bulk_wait_read1();  // the store that last used this buffer has read it
          __syncwarp();
          uint8_t* row = stg + (n_chunks & 1) * 4096 + lane * 128;
#pragma unroll
          for (int j = 0; j < 8; ++j)
            *reinterpret_cast<uint4*>(row + ((j ^ (lane & 7)) << 4)) =
                make_uint4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
          fence_proxy_async();
          __syncwarp();
          if (lane == 0) {
            if (row0 < p.M && n0 + col < p.N)
              tma_store_2d(&p.to[0], stg_s + (n_chunks & 1) * 4096, n0 + col, static_cast<int>(row0));
            bulk_commit();  // one group per chunk, stored or not: the wait above counts groups
          }
        }
      } else if constexpr (EPI == EPI_STORE16 || EPI == EPI_STORE16_MN) {
        // warpgroup wg: columns [128 wg, 128 wg + 128) in chunks of 32 through a ring of four 2 KB
        // staging tiles ([32 rows x 32 columns] 16-bit, 64-byte swizzle)
#pragma unroll 1
        for (int c = 0; c < BN / 2; c += 32, ++n_chunks) {
          const int col = wg * (BN / 2) + c;
          uint32_t v[32];
          tmem_ld32(tacc + col, v);
          tmem_ld_wait();
          if (lane == 0) bulk_wait_read<3>();  // the store that last used this slot has read it
          __syncwarp();
          const int slot = static_cast<int>(n_chunks & 3) * 2048;
          store_row32<T>(stg + slot, lane, v);
          fence_proxy_async();
          __syncwarp();
          if (lane == 0) {
            if (row0 < p.M && n0 + col < p.N)
              tma_store_2d(&p.to[0], stg_s + slot, n0 + col, static_cast<int>(row0));
            bulk_commit();  // one group per chunk, stored or not: the wait above counts groups
          }
        }
      } else if constexpr (EPI == EPI_SWIGLU) {
        // accumulator columns [0, 128): gate of j0 .. j0 + 127, [128, 256): up of the same j;
        // warpgroup wg takes j in [64 wg, 64 wg + 64) in chunks of 32: gate and up rounded to T (the
        // values the separate SwiGLU kernel reads back), h = silu(gate) * up from them; gate, up
        // and h leave through three 2 KB staging tiles (double-buffered: 2 x 6 KB per warp)
        const int j0 = nt * (BN / 2);
#pragma unroll 1
        for (int c = 0; c < BN / 4; c += 32, ++n_chunks) {
          const int jl = wg * (BN / 4) + c;
          uint32_t g[32], u[32];
          tmem_ld32(tacc + jl, g);
          tmem_ld32(tacc + BN / 2 + jl, u);
          tmem_ld_wait();
          if (lane == 0) bulk_wait_read1();
          __syncwarp();
          const int base = static_cast<int>(n_chunks & 1) * 6144;
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            const float gf = rnd<T>(__uint_as_float(g[e])), uf = rnd<T>(__uint_as_float(u[e]));
            g[e] = __float_as_uint(gf);
            u[e] = __float_as_uint(uf);
          }
          store_row32<T>(stg + base, lane, g);
          store_row32<T>(stg + base + 2048, lane, u);
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            const float gf = __uint_as_float(g[e]), uf = __uint_as_float(u[e]);
            g[e] = __float_as_uint(gf * sigmoid(gf) * uf);
          }
          store_row32<T>(stg + base + 4096, lane, g);
          fence_proxy_async();
          __syncwarp();
          if (lane == 0) {
            if (row0 < p.M) {
              const int t = static_cast<int>(row0);
              tma_store_2d(&p.to[0], stg_s + base, j0 + jl, t);                 // gate
              tma_store_2d(&p.to[0], stg_s + base + 2048, p.inter + j0 + jl, t);  // up
              tma_store_2d(&p.to[1], stg_s + base + 4096, j0 + jl, t);          // h
            }
            bulk_commit();
          }
        }
      } else if constexpr (EPI == EPI_DSWIGLU) {
        // accumulator = grad_hidden for j in [n0, n0 + 256); warpgroup wg takes [128 wg, 128 wg + 128)
        // in chunks of 32 (the gate / up table of the first one was issued before the accumulator
        // was ready); dgate and dup leave through two 2 KB tiles (double-buffered)
        uint8_t* tab = gu_tab;
#pragma unroll 1
        for (int c = 0; c < BN / 2; c += 32, ++n_chunks) {
          const int jl = wg * (BN / 2) + c;
          uint32_t gr[32];
          tmem_ld32(tacc + jl, gr);
          tmem_ld_wait();
          float gv[32], uv[32];
          ptx::cp_async_wait<0>();
          __syncwarp();
#pragma unroll
          for (int j4 = 0; j4 < 4; ++j4) {
            const int off = lane * 64 + ((j4 ^ ((lane >> 1) & 3)) << 4);
            unpack8<T>(*reinterpret_cast<const uint4*>(tab + off), *reinterpret_cast<float(*)[8]>(&gv[8 * j4]));
            unpack8<T>(*reinterpret_cast<const uint4*>(tab + 2048 + off), *reinterpret_cast<float(*)[8]>(&uv[8 * j4]));
          }
          __syncwarp();  // the table is in registers: the next chunk's may come in
          if (c + 32 < BN / 2) load_gu(row0, n0 + jl + 32);
          uint32_t dg[32], du[32];
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            const float grf = rnd<T>(__uint_as_float(gr[e]));  // grad_hidden as the 16-bit GEMM output
            const float sg = sigmoid(gv[e]);
            du[e] = __float_as_uint(grf * gv[e] * sg);
            dg[e] = __float_as_uint(grf * uv[e] * sg * (1.0f + gv[e] * (1.0f - sg)));
          }
          if (lane == 0) bulk_wait_read1();
          __syncwarp();
          const int base = static_cast<int>(n_chunks & 1) * 4096;
          store_row32<T>(stg + base, lane, dg);
          store_row32<T>(stg + base + 2048, lane, du);
          fence_proxy_async();
          __syncwarp();
          if (lane == 0) {
            if (row0 < p.M) {
              const int t = static_cast<int>(row0);
              tma_store_2d(&p.to[0], stg_s + base, n0 + jl, t);                 // dgate
              tma_store_2d(&p.to[0], stg_s + base + 2048, p.inter + n0 + jl, t);  // dup
            }
            bulk_commit();
          }
        }
      } else {
        // Warpgroup wg takes head_dim columns [32 wg, 32 wg + 32) and their RoPE partners + 64 of
        // both heads of the tile, so each RoPE table piece is loaded once for two heads.
        const int h0 = n0 / kD;  // the tile's first head: q heads, then k, then v
        const auto kind_of = [&](int hh) { return hh < p.hq ? 0 : (hh < p.hq + p.hk ? 1 : 2); };
        const int kind2[2] = {kind_of(h0), kind_of(h0 + 1)};
        const bool any_rope = kind2[0] != 2 || kind2[1] != 2;
        uint8_t* tab = smem + L::OFF_TAB + ew * L::TAB_WARP;  // [cos | sin][32 rows][64 B]
        // the warp's 32 table rows of columns [d0, d0 + 16): 2 tables x 32 rows x 4 pieces of 16 B,
        // eight coalesced cp.async per lane (rows past the end read the last row; not stored)
        const auto load_tab = [&](int d0) {
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const int piece = lane + 32 * i;
            const int which = piece >> 7, row = (piece >> 2) & 31, c4 = piece & 3;
            const int64_t rr = row0 + row < p.M ? row0 + row : p.M - 1;
            const float* src = (which ? p.sinp : p.cosp) + rr * kD + d0 + 4 * c4;
            ptx::cp_async16_ca(ptx::smem_u32(tab + which * 2048 + row * 64 + ((c4 ^ ((row >> 1) & 3)) << 4)), src);
          }
          ptx::cp_async_commit();
        };
        // two passes: outputs d in [0, 64) (x[d] cos[d] - x[d + 64] sin[d]), then d in [64, 128)
        // (x[d] cos[d] + x[d - 64] sin[d]); each fills the staging tile and leaves by two TMA stores
#pragma unroll 1
        for (int pass = 0; pass < 2; ++pass) {
          const int lo0 = 32 * wg;  // this warpgroup's columns in [0, 64)
          if (lane == 0) bulk_wait_read0();  // the previous stores have read the staging tile
          __syncwarp();
          if (any_rope) load_tab(pass * kD / 2 + lo0);
#pragma unroll 1
          for (int c = 0; c < 32; c += 16) {
            float cs[16], sn[16];
            if (any_rope) {
              ptx::cp_async_wait<0>();
              __syncwarp();
#pragma unroll
              for (int j4 = 0; j4 < 4; ++j4) {
                const int off = lane * 64 + ((j4 ^ ((lane >> 1) & 3)) << 4);
                const float4 a = *reinterpret_cast<const float4*>(tab + off);
                const float4 b2 = *reinterpret_cast<const float4*>(tab + 2048 + off);
                cs[4 * j4] = a.x; cs[4 * j4 + 1] = a.y; cs[4 * j4 + 2] = a.z; cs[4 * j4 + 3] = a.w;
                sn[4 * j4] = b2.x; sn[4 * j4 + 1] = b2.y; sn[4 * j4 + 2] = b2.z; sn[4 * j4 + 3] = b2.w;
              }
              __syncwarp();
              if (c == 0) load_tab(pass * kD / 2 + lo0 + 16);  // the next columns, during the math
            }
#pragma unroll
            for (int hd = 0; hd < 2; ++hd) {
              const int kind = kind2[hd];
              const bool rope = kind != 2;
              uint32_t alo[16], ahi[16];
              const int lo = lo0 + c;  // x[lo] pairs with x[lo + 64]
              tmem_ld16(tacc + hd * kD + lo, alo);
              tmem_ld16(tacc + hd * kD + lo + kD / 2, ahi);
              tmem_ld_wait();
              float o[16];
#pragma unroll
              for (int e = 0; e < 16; ++e) {
                // the accumulator holds x16 W^T + u (scaled lora_B)^T + 1 . bias in fp32
                const float xl = __uint_as_float(alo[e]);
                const float xh = __uint_as_float(ahi[e]);
                if (!rope) o[e] = pass ? xh : xl;
                else if (pass == 0) o[e] = __fadd_rn(__fmul_rn(xl, cs[e]), __fmul_rn(-xh, sn[e]));
                else o[e] = __fadd_rn(__fmul_rn(xh, cs[e]), __fmul_rn(xl, sn[e]));
              }
              // [32 rows x 32 columns] per head, 64-byte rows, 16-byte pieces swizzled by (row / 2) % 4
#pragma unroll
              for (int j = 0; j < 2; ++j) {
                const int piece = c / 8 + j;
                *reinterpret_cast<uint4*>(stg + hd * 2048 + lane * 64 + ((piece ^ ((lane >> 1) & 3)) << 4)) =
                    pack8<T>(*reinterpret_cast<const float(*)[8]>(&o[8 * j]));
              }
            }
          }
          fence_proxy_async();
          __syncwarp();
          if (lane == 0) {
            if (row0 < p.M) {
              const int t = static_cast<int>(row0);
              const int d = pass * kD / 2 + lo0;
#pragma unroll
              for (int hd = 0; hd < 2; ++hd) {
                const int hh = h0 + hd, kind = kind2[hd];
                const int head = kind == 0 ? hh : (kind == 1 ? hh - p.hq : hh - p.hq - p.hk);
                if (p.order[kind] == 0) tma_store_3d(&p.to[kind], stg_s + hd * 2048, d, t, head);
                else tma_store_3d(&p.to[kind], stg_s + hd * 2048, d, head, t);
              }
            }
            bulk_commit();
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if constexpr (PAIR) mbar_arrive_remote(b ? acc_empty_leader1 : acc_empty_leader0);
        else mbar_arrive(acc_empty(b));
      }
    }
    if (lane == 0) bulk_wait0();  // the stores have finished before the CTA leaves
  }
  tc_fence_before();
  __syncthreads();
  if constexpr (PAIR) cluster_sync();  // neither CTA frees TMEM or leaves while its peer still works
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    if constexpr (PAIR) tmem_dealloc_pair(tmem, 512);
    else tmem_dealloc(tmem, 512);
  }
}

// ------------------------------------------------------------------------------------------------
// x fp32 -> x16, u = dt(x16 [A_q; A_v]^T); with NORM, x = RMSNorm(h) first
// ------------------------------------------------------------------------------------------------
constexpr int kCastTok = 64, kCastThreads = 256, kCastK = 128, kCastLd = kCastK + 8;  // padded rows (16-bit)

// One CTA = 64 tokens; the K loop walks 128-column chunks of x. Each thread loads 8 float4 of a
// chunk (warp w: rows w, w + 8, ..., 512 contiguous bytes per row) with the next chunk's loads in
// flight during the current chunk's work; the 16-bit chunk goes to x16 and to shared memory, where
// mma.sync multiplies it by the matching 32 x 128 slice of [A_q; A_v].
// NORM: x holds the decoder layer's input h, and the pass first computes each row's rstd (a warp
// owns 8 whole rows; each lane sums its 16-byte pieces in column order, then the warp_sum tree:
// the plain norm kernel's reduction) and writes it to rstd_out; the chunk loop then casts
// x = w * (h * rstd) (the norm kernel's output, bit for bit) instead of h. The second read of the
// CTA's rows (393 KB) comes from L2.
template <typename T, typename W, bool NORM>
__global__ void __launch_bounds__(kCastThreads) x_cast_lora_down_kernel(const float* __restrict__ x, int64_t ldx,
                                                                        const T* __restrict__ a16, int64_t lda,
                                                                        T* __restrict__ x16, int64_t ldx16,
                                                                        T* __restrict__ u, int64_t n_tok, int hidden,
                                                                        const W* __restrict__ norm_w, float eps,
                                                                        float* __restrict__ rstd_out) {
  // u rows are 64 wide (the GEMM's LoRA K block): columns 32..63 are zero
  constexpr int kULd = 4 * kR;
  __shared__ __align__(16) T xs[kCastTok * kCastLd];
  __shared__ __align__(16) T as[2 * kR * kCastLd];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t t0 = static_cast<int64_t>(blockIdx.x) * kCastTok;
  const bool lora = a16 != nullptr;
  const int cc = 4 * lane;  // this thread's 4 columns of a chunk; rows warp + 8 i
  float4 cur[8], nxt[8];
  auto load = [&](int k0, float4 (&dst)[8]) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int64_t t = t0 + warp + 8 * i;
      dst[i] = t < n_tok ? __ldg(reinterpret_cast<const float4*>(x + t * ldx + k0 + cc)) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
  };
  float rs[8];
  if constexpr (NORM) {
    float ss[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) ss[i] = 0.f;
#pragma unroll 2
    for (int k0 = 0; k0 < hidden; k0 += kCastK) {
      load(k0, cur);
#pragma unroll
      for (int i = 0; i < 8; ++i) ss[i] += norm::sumsq4(cur[i]);
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      rs[i] = norm::row_rstd(ss[i], hidden, eps);
      const int64_t t = t0 + warp + 8 * i;
      if (rstd_out != nullptr && lane == 0 && t < n_tok) rstd_out[t] = rs[i];
    }
  }
  float acc[2][4];
#pragma unroll
  for (int n = 0; n < 2; ++n)
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[n][e] = 0.f;
  load(0, cur);
  for (int k0 = 0; k0 < hidden; k0 += kCastK) {
    if (k0 + kCastK < hidden) load(k0 + kCastK, nxt);
    if (lora) {  // A rows of this chunk: 32 rows x 128 columns, two 16-byte pieces per thread
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const int piece = tid + kCastThreads * i;
        const int ar = piece >> 4, ac = 8 * (piece & 15);
        ptx::cp_async16(ptx::smem_u32(as + ar * kCastLd + ac), a16 + ar * lda + k0 + ac, true);
      }
      ptx::cp_async_commit();
    }
    if constexpr (NORM) {
      const float4 wv = norm::wload4<W>(norm_w, k0 + cc);
#pragma unroll
      for (int i = 0; i < 8; ++i) cur[i] = norm::norm_out4w(cur[i], wv, rs[i]);
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int64_t t = t0 + warp + 8 * i;
      const uint2 v = make_uint2(Dt<T>::pack2(cur[i].x, cur[i].y), Dt<T>::pack2(cur[i].z, cur[i].w));
      if (t < n_tok) *reinterpret_cast<uint2*>(x16 + t * ldx16 + k0 + cc) = v;
      if (lora) *reinterpret_cast<uint2*>(xs + (warp + 8 * i) * kCastLd + cc) = v;
    }
    if (lora) {
      ptx::cp_async_wait<0>();
      __syncthreads();
      // warp w: tokens 16 (w & 3) .. + 15, u columns 16 (w >> 2) .. + 15 (two n8 tiles)
      const int mt = warp & 3, nh = warp >> 2;
#pragma unroll
      for (int kk = 0; kk < kCastK; kk += 16) {
        uint32_t a[4], b0, b1, b2, b3;
        const T* ap = xs + (16 * mt + (lane & 15)) * kCastLd + kk + 8 * (lane >> 4);
        ptx::ldsm_x4(ptx::smem_u32(ap), a[0], a[1], a[2], a[3]);
        // B (n x k, k contiguous): matrices (n 0-7, k 0-7), (n 0-7, k 8-15), (n 8-15, k 0-7), (n 8-15, k 8-15)
        const T* bp = as + (16 * nh + (lane & 7) + 8 * (lane >> 4)) * kCastLd + kk + 8 * ((lane >> 3) & 1);
        ptx::ldsm_x4(ptx::smem_u32(bp), b0, b1, b2, b3);
        ptx::mma16816<T>(acc[0], a, b0, b1);
        ptx::mma16816<T>(acc[1], a, b2, b3);
      }
      __syncthreads();  // xs / as are rewritten by the next chunk
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) cur[i] = nxt[i];
  }
  if (lora) {
    const int mt = warp & 3, nh = warp >> 2;
    const int g = lane >> 2, tq = lane & 3;
#pragma unroll
    for (int n = 0; n < 2; ++n) {
      const int col = 16 * nh + 8 * n + 2 * tq;
      const int64_t ta = t0 + 16 * mt + g, tb = ta + 8;
      if (ta < n_tok) *reinterpret_cast<uint32_t*>(u + ta * kULd + col) = Dt<T>::pack2(acc[n][0], acc[n][1]);
      if (tb < n_tok) *reinterpret_cast<uint32_t*>(u + tb * kULd + col) = Dt<T>::pack2(acc[n][2], acc[n][3]);
    }
  }
  // the second half of u's row: a 1 in column 32 (it multiplies the bias row of the extra K block),
  // zeros after it; without LoRA the first half is zero too. 64 tokens x 8 pieces of 16 bytes
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const int piece = tid + kCastThreads * i;
    const int64_t tz = t0 + (piece >> 3);
    const int pc = piece & 7;
    if (tz >= n_tok || (lora && pc < 4)) continue;
    uint4 z = make_uint4(0u, 0u, 0u, 0u);
    if (pc == 4) z.x = Dt<T>::pack2(1.f, 0.f);
    *reinterpret_cast<uint4*>(u + tz * kULd + 8 * pc) = z;
  }
}

// ------------------------------------------------------------------------------------------------
// dA = du^T x16, dB = scaling g^T u: reductions over the tokens on mma.sync
// ------------------------------------------------------------------------------------------------
// Output row block v (blockIdx.y): v < hidden / 128 -> dA^T rows (hidden columns 128 v ..): P = x16,
// Q = du (32 columns); else dB rows of lora_B head v - hidden / 128 (q heads, then v heads): P = the
// head's g columns of dy, Q = u_q or u_v (16 columns). out[m][n] += sum_t P[t][m] Q[t][n] over the
// block's token chunk (blockIdx.x), added into fp32 outputs zeroed by the caller.
constexpr int kGradTok = 512, kGradStep = 64, kGradThreads = 256, kPLd = 128 + 8, kQLd = 32 + 8;

template <typename T>
__global__ void __launch_bounds__(kGradThreads) lora_grad_kernel(const T* __restrict__ dy, int64_t ld_dy,
                                                                 const T* __restrict__ x16, int64_t ldx,
                                                                 const T* __restrict__ u, int64_t ldu, float* __restrict__ da,
                                                                 float* __restrict__ db, float scaling,
                                                                 int64_t n_tok, int hidden, int hq, int hk) {
  __shared__ __align__(16) T ps[2][kGradStep * kPLd];
  __shared__ __align__(16) T qs[2][kGradStep * kQLd];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int vb = blockIdx.y, n_da = hidden / kD;
  const bool is_a = vb < n_da;
  const int head = vb - n_da;  // dB: lora_B head slot (q heads, then v heads)
  const int nq = is_a ? 2 * kR : kR;  // Q columns
  const T* P;
  int64_t ldp;
  const T* Q;
  int64_t ldq;
  const int n_proj = (hq + 2 * hk) * kD;
  if (is_a) {
    P = x16 + vb * kD;
    ldp = ldx;
    Q = dy + n_proj;  // du_q | du_v
    ldq = ld_dy;
  } else {
    const int col = head < hq ? head * kD : (hq + hk + (head - hq)) * kD;
    P = dy + col;
    ldp = ld_dy;
    Q = u + (head < hq ? 0 : kR);
    ldq = ldu;
  }
  const int64_t tb0 = static_cast<int64_t>(blockIdx.x) * kGradTok;
  auto stage = [&](int buf, int64_t t0) {
    // P: 64 tokens x 128 columns = 1024 pieces of 16 bytes, 4 per thread
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int piece = tid + kGradThreads * i;
      const int row = piece >> 4, c = 8 * (piece & 15);
      const int64_t t = t0 + row;
      const bool ok = t < n_tok;
      ptx::cp_async16(ptx::smem_u32(&ps[buf][row * kPLd + c]), ok ? P + t * ldp + c : P, ok);
    }
    // Q: 64 tokens x nq columns (nq / 8 pieces per row)
    const int per_row = nq / 8;
    if (tid < kGradStep * per_row) {
      const int row = tid / per_row, c = 8 * (tid % per_row);
      const int64_t t = t0 + row;
      const bool ok = t < n_tok;
      ptx::cp_async16(ptx::smem_u32(&qs[buf][row * kQLd + c]), ok ? Q + t * ldq + c : Q, ok);
    }
    ptx::cp_async_commit();
  };
  float acc[4][4];
#pragma unroll
  for (int n = 0; n < 4; ++n)
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[n][e] = 0.f;
  const int n_steps = kGradTok / kGradStep;
  stage(0, tb0);
  for (int st = 0; st < n_steps; ++st) {
    const int buf = st & 1;
    if (st + 1 < n_steps) {
      stage(buf ^ 1, tb0 + (st + 1) * kGradStep);
      ptx::cp_async_wait<1>();
    } else {
      ptx::cp_async_wait<0>();
    }
    __syncthreads();
#pragma unroll
    for (int k0 = 0; k0 < kGradStep; k0 += 16) {
      // A (m = P column, k = token) from P[token][column] by transposed loads
      uint32_t a[4];
      const int tok = k0 + (lane & 7) + 8 * (lane >> 4);
      const int m = 16 * warp + 8 * ((lane >> 3) & 1);
      ptx::ldsm_x4_t(ptx::smem_u32(&ps[buf][tok * kPLd + m]), a[0], a[1], a[2], a[3]);
#pragma unroll
      for (int n2 = 0; n2 < 2; ++n2) {
        if (16 * n2 >= nq) break;
        uint32_t b0, b1, b2, b3;
        const int tq = k0 + (lane & 7) + 8 * ((lane >> 3) & 1);
        const int nn = 16 * n2 + 8 * (lane >> 4);
        ptx::ldsm_x4_t(ptx::smem_u32(&qs[buf][tq * kQLd + nn]), b0, b1, b2, b3);
        ptx::mma16816<T>(acc[2 * n2], a, b0, b1);
        ptx::mma16816<T>(acc[2 * n2 + 1], a, b2, b3);
      }
    }
    __syncthreads();
  }
  // C fragment: rows (m) g / g + 8 of the warp's 16, columns (n) 8 nt + 2 tq .. + 1
  const int g = lane >> 2, tq = lane & 3;
  const float mul = is_a ? 1.f : scaling;
#pragma unroll
  for (int nt = 0; nt < 4; ++nt) {
    if (8 * nt >= nq) break;
    const int n = 8 * nt + 2 * tq;
    const int m = 16 * warp + g;
    if (is_a) {  // dA [32, hidden]: element (n, hidden column 128 vb + m)
      float* base = da + vb * kD + m;
      atomicAdd(base + static_cast<int64_t>(n) * hidden, acc[nt][0]);
      atomicAdd(base + static_cast<int64_t>(n + 1) * hidden, acc[nt][1]);
      atomicAdd(base + static_cast<int64_t>(n) * hidden + 8, acc[nt][2]);
      atomicAdd(base + static_cast<int64_t>(n + 1) * hidden + 8, acc[nt][3]);
    } else {     // dB [(hq + hk) * 128, 16]: element (128 head + m, n)
      float* base = db + (static_cast<int64_t>(head) * kD + m) * kR + n;
      atomicAdd(base, mul * acc[nt][0]);
      atomicAdd(base + 1, mul * acc[nt][1]);
      atomicAdd(base + 8 * kR, mul * acc[nt][2]);
      atomicAdd(base + 8 * kR + 1, mul * acc[nt][3]);
    }
  }
}

// The extra K block's B operand [n_proj, 64]: row c of a q head holds scaling B_q[c] in columns
// 0..15 (against u_q), row c of a v head scaling B_v[c] in columns 16..31 (against u_v); every row
// holds its bias in column 32 (against the 1 in u's column 32); other entries 0; rounded to T (the
// bias is already T). bq / bv may be NULL (no LoRA).
template <typename T>
__global__ void lora_b_ext_kernel(const float* __restrict__ bq, const float* __restrict__ bv, float scaling,
                                  const T* __restrict__ bias, T* __restrict__ out, int hq, int hk) {
  const int n_proj = (hq + 2 * hk) * kD;
  const int i = blockIdx.x * blockDim.x + threadIdx.x;  // one 8-element piece of a row
  if (i >= n_proj * 8) return;
  const int row = i >> 3, piece = i & 7;
  float v[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  const float* src = nullptr;
  if (bq != nullptr && row < hq * kD && piece < 2) src = bq + row * kR + 8 * piece;
  else if (bv != nullptr && row >= (hq + hk) * kD && piece >= 2 && piece < 4)
    src = bv + (row - (hq + hk) * kD) * kR + 8 * (piece - 2);
  if (src != nullptr) {
#pragma unroll
    for (int e = 0; e < 8; ++e) v[e] = scaling * src[e];
  }
  if (piece == 4) v[0] = Dt<T>::to_f(bias[row]);
  *reinterpret_cast<uint4*>(out + static_cast<int64_t>(row) * 4 * kR + 8 * piece) = pack8<T>(v);
}

template <typename T, int EPI, bool PAIR>
int launch_gemm(const Params& p, cudaStream_t s, const char* what) {
  static std::atomic<unsigned long long> set{0};
  constexpr int smem = Layout<EPI, PAIR>::SMEM;
  if (int rc = ensure_dyn_smem(proj_gemm_kernel<T, EPI, PAIR>, smem, set, what)) return rc;
  if constexpr (!PAIR) {
    const int grid = p.n_tiles < sm_count() ? p.n_tiles : sm_count();
    proj_gemm_kernel<T, EPI, PAIR><<<grid, NTHREADS, smem, s>>>(p);
    return check_launch(what);
  } else {
    const int pairs = p.n_tiles < sm_count() / 2 ? p.n_tiles : sm_count() / 2;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * pairs, 1, 1);
    cfg.blockDim = dim3(NTHREADS, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, proj_gemm_kernel<T, EPI, PAIR>, p);
    if (e != cudaSuccess) return set_error(DECIK_ERR_CUDA, "%s: cluster launch: %s", what, cudaGetErrorString(e));
    return check_launch(what);
  }
}

}  // namespace
}  // namespace proj
}  // namespace decik

using decik::set_error;

extern "C" int decik_lora_b_ext(const float* b_q, const float* b_v, float scaling, const void* bias, void* out,
                                int n_heads, int n_kv, int dtype, void* stream) {
  using namespace decik;
  using namespace decik::proj;
  if (n_heads <= 0 || n_kv <= 0 || (b_q == nullptr) != (b_v == nullptr) || !bias || !out || !aligned16(out))
    return set_error(DECIK_ERR_INVALID, "lora_b_ext: heads %d/%d, b_q / b_v (both or neither), bias, or an unaligned out",
                     n_heads, n_kv);
  const int n = (n_heads + 2 * n_kv) * kD * 8;
  cudaStream_t s = as_stream(stream);
  if (dtype == DECIK_BF16) {
    using T = __nv_bfloat16;
    lora_b_ext_kernel<T><<<(n + 255) / 256, 256, 0, s>>>(b_q, b_v, scaling, static_cast<const T*>(bias),
                                                         static_cast<T*>(out), n_heads, n_kv);
  } else if (dtype == DECIK_F16) {
    using T = __half;
    lora_b_ext_kernel<T><<<(n + 255) / 256, 256, 0, s>>>(b_q, b_v, scaling, static_cast<const T*>(bias),
                                                         static_cast<T*>(out), n_heads, n_kv);
  } else {
    return set_error(DECIK_ERR_INVALID, "lora_b_ext: dtype %d", dtype);
  }
  return check_launch("lora_b_ext");
}

namespace decik {
namespace proj {
namespace {

// the first kernel of the forward projection: the cast + LoRA-down pass, with the input norm when
// norm_w is given
template <typename T>
int launch_cast(const float* x, int64_t ldx, const T* a16, int64_t lda, T* x16, int64_t ldx16, T* u, int64_t n_tok,
                int hidden, const void* norm_w, int norm_dtype, float eps, float* rstd, cudaStream_t s) {
  const int grid = static_cast<int>((n_tok + kCastTok - 1) / kCastTok);
  if (norm_w == nullptr)
    x_cast_lora_down_kernel<T, float, false><<<grid, kCastThreads, 0, s>>>(x, ldx, a16, lda, x16, ldx16, u, n_tok,
                                                                           hidden, nullptr, 0.f, nullptr);
  else if (norm_dtype == DECIK_F32)
    x_cast_lora_down_kernel<T, float, true><<<grid, kCastThreads, 0, s>>>(
        x, ldx, a16, lda, x16, ldx16, u, n_tok, hidden, static_cast<const float*>(norm_w), eps, rstd);
  else
    x_cast_lora_down_kernel<T, __half, true><<<grid, kCastThreads, 0, s>>>(
        x, ldx, a16, lda, x16, ldx16, u, n_tok, hidden, static_cast<const __half*>(norm_w), eps, rstd);
  return check_launch(norm_w == nullptr ? "x_cast_lora_down" : "rmsnorm_cast_lora_down");
}

int qkv_proj_fwd_impl(const float* x, int64_t ldx, const void* norm_w, int norm_dtype, float eps, float* rstd,
                      const void* w_cat, int64_t ldw, const void* ext_b, int lora, const float* cosp,
                      const float* sinp, decik_tensor3_mut q, decik_tensor3_mut k, decik_tensor3_mut v, void* x16,
                      int64_t ldx16, void* u, int64_t n_tok, int hidden, int n_heads, int n_kv, int head_dim,
                      int dtype, void* stream) {
  if (n_tok == 0) return DECIK_OK;
  if (n_tok < 0 || n_tok > (int64_t(1) << 31) - 1 || head_dim != kD || n_heads <= 0 || n_kv <= 0 ||
      hidden <= 0 || hidden % 128 != 0 || (n_heads + 2 * n_kv) % 2 != 0)
    return set_error(DECIK_ERR_INVALID, "qkv_proj_fwd: T=%lld hidden %d heads %d/%d head_dim %d (needs head_dim 128, "
                     "hidden %% 128 == 0, an even head count)", (long long)n_tok, hidden, n_heads, n_kv, head_dim);
  if (!x || !w_cat || !ext_b || !cosp || !sinp || !q.ptr || !k.ptr || !v.ptr || !x16 || !u)
    return set_error(DECIK_ERR_INVALID, "qkv_proj_fwd: NULL pointer");
  if (ldx < hidden || ldw < hidden || ldx16 < hidden)
    return set_error(DECIK_ERR_INVALID, "qkv_proj_fwd: row strides shorter than hidden");
  if (ldx % 4 || ldw % 8 || ldx16 % 8 || !aligned16(x) || !aligned16(w_cat) || !aligned16(x16) || !aligned16(u) ||
      !aligned16(ext_b) || !aligned16(cosp) || !aligned16(sinp))
    return set_error(DECIK_ERR_INVALID, "qkv_proj_fwd: rows and pointers need 16-byte alignment");
  if (dtype != DECIK_BF16 && dtype != DECIK_F16) return set_error(DECIK_ERR_INVALID, "qkv_proj_fwd: dtype %d", dtype);
  if (norm_w != nullptr && ((norm_dtype != DECIK_F32 && norm_dtype != DECIK_F16) || !(eps >= 0.f) ||
                            (norm_dtype == DECIK_F32 && !aligned16(norm_w))))
    return set_error(DECIK_ERR_INVALID, "qkv_proj_norm_fwd: norm weight dtype %d (F32 16-byte aligned, or F16), eps %g",
                     norm_dtype, static_cast<double>(eps));
  cudaStream_t s = as_stream(stream);
  const int n_proj = (n_heads + 2 * n_kv) * kD;
  constexpr int BN = Cfg<EPI_QKV>::BN;
  Params p{};
  int ord = 0;
  if (int rc = attn::make_map_2d(&p.ta, x16, dtype, hidden, n_tok, ldx16 * 2, 64, BM)) return rc;
  if (int rc = attn::make_map_2d(&p.tb, w_cat, dtype, hidden, n_proj, ldw * 2, 64, BN / 2)) return rc;
  p.lora = 1;  // the extra K block always runs: it carries the bias
  if (int rc = attn::make_map_2d(&p.ta2, u, dtype, 4 * kR, n_tok, 4 * kR * 2, 64, BM)) return rc;
  if (int rc = attn::make_map_2d(&p.tb2, ext_b, dtype, 4 * kR, n_proj, 4 * kR * 2, 64, BN / 2)) return rc;
  const decik_tensor3_mut outs[3] = {q, k, v};
  const int heads[3] = {n_heads, n_kv, n_kv};
  for (int j = 0; j < 3; ++j) {
    if (int rc = attn::make_tile_map_ex(&p.to[j], outs[j].ptr, outs[j].tok_stride, outs[j].head_stride, n_tok,
                                        heads[j], dtype, &ord, 32, 32, 64))
      return rc;
    p.order[j] = ord;
  }
  p.M = n_tok;
  p.N = n_proj;
  p.K = hidden;
  p.b_tile_step = BN;
  p.b_rank_off = BN / 2;
  p.n_tiles_n = n_proj / BN + (n_proj % BN ? 1 : 0);
  const int64_t m_tiles = (n_tok + 2 * BM - 1) / (2 * BM);  // CTA pairs: 256 rows per tile
  p.n_tiles = static_cast<int>(m_tiles * p.n_tiles_n);
  p.cosp = cosp;
  p.sinp = sinp;
  p.hq = n_heads;
  p.hk = n_kv;
  p.err = attn::attn_error_word();
  // x16 and u first (the GEMM's A operands), then the GEMM + epilogue
  const int64_t a_off = static_cast<int64_t>(n_proj) * ldw;
  if (dtype == DECIK_BF16) {
    using T = __nv_bfloat16;
    if (int rc = launch_cast<T>(x, ldx, lora ? static_cast<const T*>(w_cat) + a_off : nullptr, ldw,
                                static_cast<T*>(x16), ldx16, static_cast<T*>(u), n_tok, hidden, norm_w, norm_dtype,
                                eps, rstd, s))
      return rc;
    return launch_gemm<T, EPI_QKV, true>(p, s, "qkv_proj_gemm");
  }
  using T = __half;
  if (int rc = launch_cast<T>(x, ldx, lora ? static_cast<const T*>(w_cat) + a_off : nullptr, ldw,
                              static_cast<T*>(x16), ldx16, static_cast<T*>(u), n_tok, hidden, norm_w, norm_dtype, eps,
                              rstd, s))
    return rc;
  return launch_gemm<T, EPI_QKV, true>(p, s, "qkv_proj_gemm");
}

}  // namespace
}  // namespace proj
}  // namespace decik

extern "C" int decik_qkv_proj_fwd(const float* x, int64_t ldx, const void* w_cat, int64_t ldw, const void* ext_b,
                                  int lora, const float* cosp, const float* sinp, decik_tensor3_mut q,
                                  decik_tensor3_mut k, decik_tensor3_mut v, void* x16, int64_t ldx16, void* u,
                                  int64_t n_tok, int hidden, int n_heads, int n_kv, int head_dim, int dtype,
                                  void* stream) {
  return decik::proj::qkv_proj_fwd_impl(x, ldx, nullptr, 0, 0.f, nullptr, w_cat, ldw, ext_b, lora, cosp, sinp, q, k,
                                        v, x16, ldx16, u, n_tok, hidden, n_heads, n_kv, head_dim, dtype, stream);
}

extern "C" int decik_qkv_proj_norm_fwd(const float* h, int64_t ldh, const void* norm_w, int norm_dtype, float eps,
                                       float* rstd, const void* w_cat, int64_t ldw, const void* ext_b, int lora,
                                       const float* cosp, const float* sinp, decik_tensor3_mut q, decik_tensor3_mut k,
                                       decik_tensor3_mut v, void* x16, int64_t ldx16, void* u, int64_t n_tok,
                                       int hidden, int n_heads, int n_kv, int head_dim, int dtype, void* stream) {
  if (n_tok != 0 && (norm_w == nullptr || rstd == nullptr))
    return decik::set_error(DECIK_ERR_INVALID, "qkv_proj_norm_fwd: NULL norm weight or rstd");
  return decik::proj::qkv_proj_fwd_impl(h, ldh, norm_w, norm_dtype, eps, rstd, w_cat, ldw, ext_b, lora, cosp, sinp, q,
                                        k, v, x16, ldx16, u, n_tok, hidden, n_heads, n_kv, head_dim, dtype, stream);
}

extern "C" int decik_proj_dx(const void* dy, int64_t ld_dy, int k_cols, const void* w_t, int64_t ldw, float* dx,
                             int64_t ld_dx, int64_t n_tok, int hidden, int dtype, void* stream) {
  using namespace decik;
  using namespace decik::proj;
  if (n_tok == 0) return DECIK_OK;
  if (n_tok < 0 || n_tok > (int64_t(1) << 31) - 1 || hidden <= 0 || hidden % 8 != 0 || k_cols <= 0 || k_cols % 8 != 0)
    return set_error(DECIK_ERR_INVALID, "proj_dx: T=%lld hidden %d K %d (multiples of 8)", (long long)n_tok, hidden,
                     k_cols);
  if (!dy || !w_t || !dx) return set_error(DECIK_ERR_INVALID, "proj_dx: NULL pointer");
  if (ld_dy < k_cols || ldw < k_cols || ld_dx < hidden)
    return set_error(DECIK_ERR_INVALID, "proj_dx: row strides shorter than the rows");
  if (ld_dy % 8 || ldw % 8 || ld_dx % 4 || !aligned16(dy) || !aligned16(w_t) || !aligned16(dx))
    return set_error(DECIK_ERR_INVALID, "proj_dx: rows and pointers need 16-byte alignment");
  if (dtype != DECIK_BF16 && dtype != DECIK_F16) return set_error(DECIK_ERR_INVALID, "proj_dx: dtype %d", dtype);
  constexpr int BN = Cfg<EPI_F32>::BN;
  Params p{};
  if (int rc = attn::make_map_2d(&p.ta, dy, dtype, k_cols, n_tok, ld_dy * 2, 64, BM)) return rc;
  if (int rc = attn::make_map_2d(&p.tb, w_t, dtype, k_cols, hidden, ldw * 2, 64, BN / 2)) return rc;
  if (int rc = attn::make_map_2d(&p.to[0], dx, DECIK_F32, hidden, n_tok, ld_dx * 4, 32, 32)) return rc;
  p.M = n_tok;
  p.N = hidden;
  p.K = k_cols;
  p.b_tile_step = BN;
  p.b_rank_off = BN / 2;
  p.n_tiles_n = (hidden + BN - 1) / BN;
  p.n_tiles = static_cast<int>(((n_tok + 2 * BM - 1) / (2 * BM)) * p.n_tiles_n);  // CTA pairs: 256 rows
  p.err = attn::attn_error_word();
  cudaStream_t s = as_stream(stream);
  if (dtype == DECIK_BF16) return launch_gemm<__nv_bfloat16, EPI_F32, true>(p, s, "proj_dx_gemm");
  return launch_gemm<__half, EPI_F32, true>(p, s, "proj_dx_gemm");
}

extern "C" int decik_lora_grads(const void* dy, int64_t ld_dy, const void* x16, int64_t ldx, const void* u,
                                int64_t ldu, float* da, float* db, float scaling, int64_t n_tok, int hidden,
                                int n_heads, int n_kv, int dtype, void* stream) {
  using namespace decik;
  using namespace decik::proj;
  if (n_tok < 0 || hidden <= 0 || hidden % kD != 0 || n_heads <= 0 || n_kv <= 0)
    return set_error(DECIK_ERR_INVALID, "lora_grads: T=%lld hidden %d heads %d/%d", (long long)n_tok, hidden, n_heads, n_kv);
  if (!dy || !x16 || !u || !da || !db) return set_error(DECIK_ERR_INVALID, "lora_grads: NULL pointer");
  if (ld_dy < static_cast<int64_t>(n_heads + 2 * n_kv) * kD + 2 * kR || ldx < hidden)
    return set_error(DECIK_ERR_INVALID, "lora_grads: dy rows need (heads + 2 kv heads) x 128 + 32 columns, x16 rows hidden");
  if (ld_dy % 8 || ldx % 8 || ldu % 8 || ldu < 2 * kR || !aligned16(dy) || !aligned16(x16) || !aligned16(u))
    return set_error(DECIK_ERR_INVALID, "lora_grads: rows and pointers need 16-byte alignment (u rows >= 32)");
  cudaStream_t s = as_stream(stream);
  cudaError_t e = cudaMemsetAsync(da, 0, sizeof(float) * 2 * kR * hidden, s);
  if (e == cudaSuccess) e = cudaMemsetAsync(db, 0, sizeof(float) * (n_heads + n_kv) * kD * kR, s);
  if (e != cudaSuccess) return set_error(DECIK_ERR_CUDA, "lora_grads: memset: %s", cudaGetErrorString(e));
  if (n_tok == 0) return DECIK_OK;
  const dim3 grid(static_cast<unsigned>((n_tok + kGradTok - 1) / kGradTok), hidden / kD + n_heads + n_kv);
  if (dtype == DECIK_BF16) {
    using T = __nv_bfloat16;
    lora_grad_kernel<T><<<grid, kGradThreads, 0, s>>>(static_cast<const T*>(dy), ld_dy, static_cast<const T*>(x16),
                                                      ldx, static_cast<const T*>(u), ldu, da, db, scaling, n_tok, hidden,
                                                      n_heads, n_kv);
  } else if (dtype == DECIK_F16) {
    using T = __half;
    lora_grad_kernel<T><<<grid, kGradThreads, 0, s>>>(static_cast<const T*>(dy), ld_dy, static_cast<const T*>(x16),
                                                      ldx, static_cast<const T*>(u), ldu, da, db, scaling, n_tok, hidden,
                                                      n_heads, n_kv);
  } else {
    return set_error(DECIK_ERR_INVALID, "lora_grads: dtype %d", dtype);
  }
  return check_launch("lora_grads");
}

namespace decik {
namespace proj {
namespace {

template <int EPI>
int launch_typed(const Params& p, int dtype, cudaStream_t s, const char* what) {
  if (dtype == DECIK_BF16) return launch_gemm<__nv_bfloat16, EPI, true>(p, s, what);
  if (dtype == DECIK_F16) return launch_gemm<__half, EPI, true>(p, s, what);
  return set_error(DECIK_ERR_INVALID, "%s: dtype %d", what, dtype);
}

bool rows16(const void* ptr, int64_t ld) { return aligned16(ptr) && ld % 8 == 0; }

}  // namespace
}  // namespace proj
}  // namespace decik

extern "C" int decik_gemm16(const void* a, int64_t lda, const void* b, int64_t ldb, int b_mn, void* out, int64_t ldo,
                            int64_t m, int n, int k, int dtype, void* stream) {
  using namespace decik;
  using namespace decik::proj;
  if (m == 0 || n == 0) return DECIK_OK;
  if (m < 0 || m > (int64_t(1) << 31) - 1 || n < 0 || k <= 0 || n % 8 != 0 || k % 8 != 0)
    return set_error(DECIK_ERR_INVALID, "gemm16: M=%lld N=%d K=%d (N, K multiples of 8)", (long long)m, n, k);
  if (!a || !b || !out) return set_error(DECIK_ERR_INVALID, "gemm16: NULL pointer");
  if (!rows16(a, lda) || !rows16(b, ldb) || !rows16(out, ldo) || lda < k || ldb < (b_mn ? n : k) || ldo < n)
    return set_error(DECIK_ERR_INVALID, "gemm16: rows and pointers need 16-byte alignment and full-width strides");
  const int BN = b_mn ? Cfg<EPI_STORE16_MN>::BN : Cfg<EPI_STORE16>::BN;
  Params p{};
  if (int rc = attn::make_map_2d(&p.ta, a, dtype, k, m, lda * 2, 64, BM)) return rc;
  if (b_mn) {
    if (int rc = attn::make_map_2d(&p.tb, b, dtype, n, k, ldb * 2, 64, 64)) return rc;
  } else {
    if (int rc = attn::make_map_2d(&p.tb, b, dtype, k, n, ldb * 2, 64, BN / 2)) return rc;
  }
  if (int rc = attn::make_map_2d(&p.to[0], out, dtype, n, m, ldo * 2, 32, 32, 64)) return rc;
  p.M = m;
  p.N = n;
  p.K = k;
  p.b_tile_step = BN;
  p.b_rank_off = BN / 2;
  p.n_tiles_n = (n + BN - 1) / BN;
  p.n_tiles = static_cast<int>(((m + 2 * BM - 1) / (2 * BM)) * p.n_tiles_n);
  p.err = attn::attn_error_word();
  cudaStream_t s = as_stream(stream);
  return b_mn ? launch_typed<EPI_STORE16_MN>(p, dtype, s, "gemm16") : launch_typed<EPI_STORE16>(p, dtype, s, "gemm16");
}

extern "C" int decik_mlp_gate_up(const void* x16, int64_t ldx, const void* w_gu, int64_t ldw, void* gu, int64_t ldgu,
                                 void* h, int64_t ldh, int64_t m, int hidden, int inter, int dtype, void* stream) {
  using namespace decik;
  using namespace decik::proj;
  if (m == 0) return DECIK_OK;
  if (m < 0 || m > (int64_t(1) << 31) - 1 || hidden <= 0 || hidden % 8 != 0 || inter <= 0 || inter % 128 != 0)
    return set_error(DECIK_ERR_INVALID, "mlp_gate_up: M=%lld hidden %d inter %d (inter %% 128 == 0)", (long long)m,
                     hidden, inter);
  if (!x16 || !w_gu || !gu || !h) return set_error(DECIK_ERR_INVALID, "mlp_gate_up: NULL pointer");
  if (!rows16(x16, ldx) || !rows16(w_gu, ldw) || !rows16(gu, ldgu) || !rows16(h, ldh) || ldx < hidden ||
      ldw < hidden || ldgu < 2 * static_cast<int64_t>(inter) || ldh < inter)
    return set_error(DECIK_ERR_INVALID, "mlp_gate_up: rows and pointers need 16-byte alignment and full-width strides");
  Params p{};
  if (int rc = attn::make_map_2d(&p.ta, x16, dtype, hidden, m, ldx * 2, 64, BM)) return rc;
  if (int rc = attn::make_map_2d(&p.tb, w_gu, dtype, hidden, 2 * static_cast<int64_t>(inter), ldw * 2, 64, BM))
    return rc;
  if (int rc = attn::make_map_2d(&p.to[0], gu, dtype, 2 * static_cast<int64_t>(inter), m, ldgu * 2, 32, 32, 64))
    return rc;
  if (int rc = attn::make_map_2d(&p.to[1], h, dtype, inter, m, ldh * 2, 32, 32, 64)) return rc;
  p.M = m;
  p.N = 2 * inter;
  p.K = hidden;
  p.inter = inter;
  p.b_tile_step = BM;    // gate rows j0 .. j0 + 127 in CTA 0, up rows inter + j0 .. in CTA 1
  p.b_rank_off = inter;
  p.n_tiles_n = inter / 128;
  p.n_tiles = static_cast<int>(((m + 2 * BM - 1) / (2 * BM)) * p.n_tiles_n);
  p.err = attn::attn_error_word();
  return launch_typed<EPI_SWIGLU>(p, dtype, as_stream(stream), "mlp_gate_up");
}

extern "C" int decik_mlp_down_grad(const void* grad, int64_t ldg, const void* w_down, int64_t ldw, const void* gu,
                                   int64_t ldgu, void* dgu, int64_t lddgu, int64_t m, int hidden, int inter, int dtype,
                                   void* stream) {
  using namespace decik;
  using namespace decik::proj;
  if (m == 0) return DECIK_OK;
  if (m < 0 || m > (int64_t(1) << 31) - 1 || hidden <= 0 || hidden % 8 != 0 || inter <= 0 || inter % 256 != 0)
    return set_error(DECIK_ERR_INVALID, "mlp_down_grad: M=%lld hidden %d inter %d (inter %% 256 == 0)", (long long)m,
                     hidden, inter);
  if (!grad || !w_down || !gu || !dgu) return set_error(DECIK_ERR_INVALID, "mlp_down_grad: NULL pointer");
  if (!rows16(grad, ldg) || !rows16(w_down, ldw) || !rows16(gu, ldgu) || !rows16(dgu, lddgu) || ldg < hidden ||
      ldw < inter || ldgu < 2 * static_cast<int64_t>(inter) || lddgu < 2 * static_cast<int64_t>(inter))
    return set_error(DECIK_ERR_INVALID, "mlp_down_grad: rows and pointers need 16-byte alignment and full-width strides");
  constexpr int BN = Cfg<EPI_DSWIGLU>::BN;
  Params p{};
  if (int rc = attn::make_map_2d(&p.ta, grad, dtype, hidden, m, ldg * 2, 64, BM)) return rc;
  if (int rc = attn::make_map_2d(&p.tb, w_down, dtype, inter, hidden, ldw * 2, 64, 64)) return rc;
  if (int rc = attn::make_map_2d(&p.to[0], dgu, dtype, 2 * static_cast<int64_t>(inter), m, lddgu * 2, 32, 32, 64))
    return rc;
  p.M = m;
  p.N = inter;
  p.K = hidden;
  p.inter = inter;
  p.gu = gu;
  p.ld_gu = ldgu;
  p.b_tile_step = BN;
  p.b_rank_off = BN / 2;
  p.n_tiles_n = inter / BN;
  p.n_tiles = static_cast<int>(((m + 2 * BM - 1) / (2 * BM)) * p.n_tiles_n);
  p.err = attn::attn_error_word();
  return launch_typed<EPI_DSWIGLU>(p, dtype, as_stream(stream), "mlp_down_grad");
}

namespace decik {
namespace proj {
namespace {

// dst [cols, rows] = src [rows, cols]^T for 16-bit values: 64 x 64 tiles through shared memory
// (rows padded by one 32-bit word: conflict-free column reads), 16-byte global loads and stores.
__global__ void __launch_bounds__(256) transpose16_kernel(const uint16_t* __restrict__ src, int64_t lds,
                                                          uint16_t* __restrict__ dst, int64_t ldd, int64_t rows,
                                                          int64_t cols) {
  __shared__ uint16_t tile[64][64 + 2];
  const int64_t r0 = static_cast<int64_t>(blockIdx.y) * 64, c0 = static_cast<int64_t>(blockIdx.x) * 64;
  const int tid = threadIdx.x;
#pragma unroll
  for (int i = 0; i < 2; ++i) {  // 64 rows x 8 pieces of 8 values
    const int piece = tid + 256 * i;
    const int r = piece >> 3, c = 8 * (piece & 7);
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (r0 + r < rows && c0 + c < cols) v = *reinterpret_cast<const uint4*>(src + (r0 + r) * lds + c0 + c);
    const uint16_t* e = reinterpret_cast<const uint16_t*>(&v);
#pragma unroll
    for (int k = 0; k < 8; ++k) tile[r][c + k] = e[k];
  }
  __syncthreads();
#pragma unroll
  for (int i = 0; i < 2; ++i) {  // output rows = source columns
    const int piece = tid + 256 * i;
    const int c = piece >> 3, r = 8 * (piece & 7);
    if (c0 + c >= cols || r0 + r >= rows) continue;
    uint4 v;
    uint16_t* e = reinterpret_cast<uint16_t*>(&v);
#pragma unroll
    for (int k = 0; k < 8; ++k) e[k] = tile[r + k][c];
    *reinterpret_cast<uint4*>(dst + (c0 + c) * ldd + r0 + r) = v;
  }
}

}  // namespace
}  // namespace proj
}  // namespace decik

extern "C" int decik_transpose16(const void* src, int64_t lds, void* dst, int64_t ldd, int64_t rows, int64_t cols,
                                 void* stream) {
  using namespace decik;
  if (rows == 0 || cols == 0) return DECIK_OK;
  if (rows < 0 || cols < 0 || rows % 8 || cols % 8 || lds < cols || ldd < rows || lds % 8 || ldd % 8 ||
      !aligned16(src) || !aligned16(dst))
    return set_error(DECIK_ERR_INVALID, "transpose16: %lld x %lld (multiples of 8), strides, 16-byte alignment",
                     (long long)rows, (long long)cols);
  const dim3 grid(static_cast<unsigned>((cols + 63) / 64), static_cast<unsigned>((rows + 63) / 64));
  proj::transpose16_kernel<<<grid, 256, 0, as_stream(stream)>>>(static_cast<const uint16_t*>(src), lds,
                                                                static_cast<uint16_t*>(dst), ldd, rows, cols);
  return check_launch("transpose16");
}
