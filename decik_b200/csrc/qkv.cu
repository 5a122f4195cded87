// The projection epilogues of the attention block: everything between the one q|k|v|LoRA-down GEMM
// and the attention kernels, and back.
//
// Forward. The caller runs one GEMM y = x16 . [W_q; W_k; W_v; A_q; A_v]^T + [b_q; b_k; b_v; 0]
// (the three NF4Linear calls and both lora_A products of the reference, solution/nf4.py:93-97 and
// solution/attn.py:225-227, share their input x16, so they are one GEMM). This kernel then does,
// per token, what the reference's patched Qwen2Attention.forward builds from those outputs
// (solution/attn.py:395-411, LoRAPairFromNorm.forward :217-228, skc_rope_fwd_kernel :28-61):
//   q_lora = dt(dt(u_q . B16_q^T) * scaling)          v_lora likewise from u_v, B_v
//   q_out  = rope(f32(q_base) + f32(q_lora))  head-major     k_out = rope(k) head-major
//   v_out  = dt(f32(v_base) + f32(v_lora))
// RoPE rounds each product and the sum separately (no FMA), as the reference kernels run with
// enable_fp_fusion=False, so for equal inputs q_out/k_out match skc_rope_fwd_kernel bit for bit.
//
// Backward. The caller places dv (from the attention backward) in the v columns of dy; this kernel
// writes the rest of dy = [rope^T(dq) | rope^T(dk) | dv | du_q | du_v], the operand of one
// dX = dy . [W_q; W_k; W_v; A_q; A_v] GEMM (the three NF4Linear backward GEMMs and both LoRA input
// gradients of LoRAPairFromNorm.backward, :235-273, summed in fp32 inside the GEMM):
//   rope^T as skc_rope_bwd_kernel (solution/attn.py:64-90), rounded to dt
//   du_q = dt(g_q . B16_q), g_q = dt(rope^T(dq) * scaling)      du_v likewise from dv, B_v.
//
// Work split. One warp per (16-token tile, head): the forward CTA takes 4 heads of a tile (small
// enough for 4 CTAs per SM), the backward CTA all heads of a tile (it sums du over them). The tile's
// cos/sin rows and each warp's 16 x 128 input tile are copied into shared memory with cp.async, so
// a warp has its whole tile in flight at once and the cos/sin rows are read once per CTA. The rank-16 LoRA products run on mma.sync m16n8k16 (2 x 16 x 1792
// MACs per token: far too small for tcgen05 tiles, too many for plain FMAs) with lora_B fragments
// prepared once per step by decik_lora_pack; their results pass through the padded shared tile.
// The element-wise work uses a row-contiguous lane map: 16 lanes x 4 columns cover one 64-column
// half of a row, and each lane also holds the RoPE partners 64 columns away. HBM-bound.
#include "common.cuh"
#include "ptx.cuh"

namespace decik {
namespace {

constexpr int kD = 128;     // head_dim
constexpr int kR = 16;      // LoRA rank
// backward: warps per CTA; warp w takes heads w, w + 16, ...: at the 1.5B shape (16 heads of q,
// k, v) every head's tile load is in flight at once (8 warps, two heads each in turn: 52 us at
// 16,384 tokens)
constexpr int kWarps = 16;
constexpr int kFwdWarps = 4;  // forward: warps per CTA = heads per CTA (grid.y covers the heads)
constexpr int kLd = kD + 8; // shared tile row, elements (272 bytes: conflict-free for both maps)
constexpr int kTile = 16 * kLd;               // one warp's 16 x 128 tile, elements
constexpr int kFragWords = 16 * 32 * 2;       // one head's lora_B fragments, 32-bit words (4 KB)
constexpr int kCsBytes = 2 * 16 * kD * 4;     // cos + sin rows of the tile

struct QkvFwdParams {
  const void* y;
  int64_t ldy;
  const void* u;
  int64_t ldu;
  const uint32_t* frag;  // forward-layout lora_B fragments, q heads then v heads (NULL: no LoRA)
  float scaling;
  const float* cosp;
  const float* sinp;
  void* q;
  int64_t q_tok, q_head;
  void* k;
  int64_t k_tok, k_head;
  void* v;
  int64_t v_tok, v_head;
  void* u_out;  // optional compact [T, 2R] copy of u
  int64_t n_tok;
  int hq, hk;
};

struct QkvBwdParams {
  const void* gq;
  int64_t gq_tok, gq_head;
  const void* gk;
  int64_t gk_tok, gk_head;
  const float* cosp;
  const float* sinp;
  const uint32_t* frag;  // backward-layout lora_B fragments (NULL: no LoRA)
  float scaling;
  void* dy;
  int64_t ldy;
  int64_t n_tok;
  int hq, hk;
  // fp32 accumulators of the attention backward, token-major [tok][heads][128], read instead of
  // the 16-bit gradients when set: q_acc (x q_mul) replaces gq, k_acc (x k_mul) gk, and v_acc is
  // rounded into dy's v columns (else the caller placed dv there)
  const float* q_acc;
  const float* k_acc;
  const float* v_acc;
  float q_mul, k_mul;
};

__device__ __forceinline__ uint32_t ld_u32(const void* p) {
  return __ldg(reinterpret_cast<const unsigned int*>(p));
}
__device__ __forceinline__ void st_u32(void* p, uint32_t v) { *reinterpret_cast<uint32_t*>(p) = v; }
__device__ __forceinline__ void st_u64(void* p, uint2 v) { *reinterpret_cast<uint2*>(p) = v; }

template <typename T>
__device__ __forceinline__ float rnd(float x) {  // round to the 16-bit type and back
  return Dt<T>::to_f(Dt<T>::from_f(x));
}
template <typename T>
__device__ __forceinline__ void unpack4(uint2 w, float (&f)[4]) {
  f[0] = Dt<T>::lo_f(w.x); f[1] = Dt<T>::hi_f(w.x); f[2] = Dt<T>::lo_f(w.y); f[3] = Dt<T>::hi_f(w.y);
}
template <typename T>
__device__ __forceinline__ uint2 pack4(const float (&f)[4]) {
  return make_uint2(Dt<T>::pack2(f[0], f[1]), Dt<T>::pack2(f[2], f[3]));
}
__device__ __forceinline__ void ld4s(const float* p, float (&f)[4]) {
  const float4 v = *reinterpret_cast<const float4*>(p);
  f[0] = v.x; f[1] = v.y; f[2] = v.z; f[3] = v.w;
}

// The tile's cos and sin rows into shared memory (rows past the end zero-filled).
__device__ __forceinline__ void stage_cos_sin(float* cs, const float* cosp, const float* sinp, int64_t t0,
                                              int nrows) {
  for (int i = threadIdx.x; i < 2 * 16 * (kD / 4); i += blockDim.x) {
    const int which = i >> 9;
    const int row = (i >> 5) & 15;
    const int c = (i & 31) * 4;
    const bool ok = row < nrows;
    const float* src = (which ? sinp : cosp) + (ok ? (t0 + row) * kD + c : 0);
    ptx::cp_async16(ptx::smem_u32(cs + (which * 16 + row) * kD + c), src, ok);
  }
}

// 16 rows x 128 16-bit values (row stride `tok` elements) into a warp's padded shared tile.
template <typename T>
__device__ __forceinline__ void stage_tile(T* tile, const T* src, int64_t tok, int nrows, int lane) {
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int row = 2 * i + (lane >> 4);
    const int chunk = (lane & 15) * 8;
    const bool ok = row < nrows;
    ptx::cp_async16(ptx::smem_u32(tile + row * kLd + chunk), ok ? src + row * tok + chunk : src, ok);
  }
}

// The same [16 x 128] tile from an fp32 accumulator with row stride `tok` (floats), each value
// scaled by `mul` and rounded to T: what the attention backward's cast pass would have stored.
template <typename T>
__device__ __forceinline__ void stage_tile_acc(T* tile, const float* src, int64_t tok, int nrows, int lane, float mul) {
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int row = 2 * i + (lane >> 4);
    const int chunk = (lane & 15) * 8;
    float f[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if (row < nrows) {
      const float4 a = __ldg(reinterpret_cast<const float4*>(src + row * tok + chunk));
      const float4 b = __ldg(reinterpret_cast<const float4*>(src + row * tok + chunk + 4));
      f[0] = a.x * mul; f[1] = a.y * mul; f[2] = a.z * mul; f[3] = a.w * mul;
      f[4] = b.x * mul; f[5] = b.y * mul; f[6] = b.z * mul; f[7] = b.w * mul;
    }
    *reinterpret_cast<uint4*>(tile + row * kLd + chunk) = pack8<T>(f);
  }
}

template <typename T>
__global__ void lora_pack_kernel(const float* __restrict__ aq, const float* __restrict__ av, T* __restrict__ a_out,
                                 int64_t lda, int hidden, const float* __restrict__ bq,
                                 const float* __restrict__ bv, uint32_t* __restrict__ frag, int hq, int hk) {
  const int64_t n_a = a_out != nullptr ? 2LL * kR * hidden : 0;
  const int64_t n_f = static_cast<int64_t>(hq + hk) * kFragWords;
  const int64_t total = n_a + 2 * n_f;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total; i += stride) {
    if (i < n_a) {  // A_q then A_v, as rows of the projection weight
      const int64_t r = i / hidden, c = i % hidden;
      const float x = r < kR ? aq[r * hidden + c] : av[(r - kR) * hidden + c];
      a_out[r * lda + c] = Dt<T>::from_f(x);
      continue;
    }
    const bool bwd = i >= n_a + n_f;
    const int64_t w = i - n_a - (bwd ? n_f : 0);
    const int half = static_cast<int>(w & 1);
    const int lane = static_cast<int>((w >> 1) & 31);
    const int head = static_cast<int>(w >> 10);
    const int g = lane >> 2, tq = lane & 3;
    const float* B = head < hq ? bq + static_cast<int64_t>(head) * kD * kR
                               : bv + static_cast<int64_t>(head - hq) * kD * kR;
    uint32_t val;
    if (!bwd) {
      // forward (u . B^T): n-tile n, b[half] = B[8n + g][2tq + 8 half .. + 1]
      const int n = static_cast<int>((w >> 6) & 15);
      const float* b = B + (8 * n + g) * kR + 2 * tq + 8 * half;
      val = Dt<T>::pack2(b[0], b[1]);
    } else {
      // backward (g . B): k-step s, n-tile i2, b[half] = B[16s + 2tq + 8 half .. + 1][8 i2 + g]
      const int i2 = static_cast<int>((w >> 6) & 1);
      const int s = static_cast<int>((w >> 7) & 7);
      const int col = 16 * s + 2 * tq + 8 * half;
      val = Dt<T>::pack2(B[col * kR + 8 * i2 + g], B[(col + 1) * kR + 8 * i2 + g]);
    }
    frag[(bwd ? n_f : 0) + w] = val;
  }
}

template <typename T>
__global__ void __launch_bounds__(kFwdWarps * 32)
qkv_fwd_kernel(const QkvFwdParams p) {
  extern __shared__ __align__(16) unsigned char smem[];
  float* cs = reinterpret_cast<float*>(smem);   // [cos 16 x 128 | sin 16 x 128]
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int g = lane >> 2;
  const int tq = lane & 3;
  const int64_t t0 = static_cast<int64_t>(blockIdx.x) * 16;
  const int nrows = static_cast<int>(p.n_tok - t0 < 16 ? p.n_tok - t0 : 16);
  T* ys = reinterpret_cast<T*>(smem + kCsBytes) + warp * 2 * kTile;  // input tile
  T* ls = ys + kTile;                                                 // LoRA tile
  const T* y = static_cast<const T*>(p.y);
  const int n_heads = p.hq + 2 * p.hk;
  const bool lora = p.frag != nullptr;

  stage_cos_sin(cs, p.cosp, p.sinp, t0, nrows);
  int h = blockIdx.y * kFwdWarps + warp;  // one head per warp
  if (h < n_heads) stage_tile<T>(ys, y + t0 * p.ldy + static_cast<int64_t>(h) * kD, p.ldy, nrows, lane);
  ptx::cp_async_commit();

  // u as m16n8k16 A fragments: a0 (row g, 2tq..+1), a1 (g + 8, ..), a2 (g, 2tq+8..), a3 (g + 8, ..)
  uint32_t aq[4] = {0u, 0u, 0u, 0u};
  uint32_t av[4] = {0u, 0u, 0u, 0u};
  if (lora) {
    const T* u = static_cast<const T*>(p.u) + t0 * p.ldu;
    const int c = 2 * tq;
    if (g < nrows) {
      aq[0] = ld_u32(u + g * p.ldu + c);
      aq[2] = ld_u32(u + g * p.ldu + c + 8);
      av[0] = ld_u32(u + g * p.ldu + kR + c);
      av[2] = ld_u32(u + g * p.ldu + kR + c + 8);
    }
    if (g + 8 < nrows) {
      aq[1] = ld_u32(u + (g + 8) * p.ldu + c);
      aq[3] = ld_u32(u + (g + 8) * p.ldu + c + 8);
      av[1] = ld_u32(u + (g + 8) * p.ldu + kR + c);
      av[3] = ld_u32(u + (g + 8) * p.ldu + kR + c + 8);
    }
    if (p.u_out != nullptr && warp == 0 && blockIdx.y == 0) {
      T* uo = static_cast<T*>(p.u_out) + t0 * 2 * kR;
      if (g < nrows) {
        st_u32(uo + g * 2 * kR + c, aq[0]);
        st_u32(uo + g * 2 * kR + c + 8, aq[2]);
        st_u32(uo + g * 2 * kR + kR + c, av[0]);
        st_u32(uo + g * 2 * kR + kR + c + 8, av[2]);
      }
      if (g + 8 < nrows) {
        st_u32(uo + (g + 8) * 2 * kR + c, aq[1]);
        st_u32(uo + (g + 8) * 2 * kR + c + 8, aq[3]);
        st_u32(uo + (g + 8) * 2 * kR + kR + c, av[1]);
        st_u32(uo + (g + 8) * 2 * kR + kR + c + 8, av[3]);
      }
    }
  }

  // lora = dt(dt(u . B16^T) * scaling) of head h into the LoRA tile (C fragment of n-tile n:
  // rows g / g + 8, columns 8n + 2tq .. + 1)
  auto lora_tile = [&](int hh) {
    const bool is_v = hh >= p.hq + p.hk;
    const int slot = is_v ? p.hq + (hh - p.hq - p.hk) : hh;
    const uint2* bf = reinterpret_cast<const uint2*>(p.frag + static_cast<int64_t>(slot) * kFragWords) + lane;
    uint2 b[16];
#pragma unroll
    for (int n = 0; n < 16; ++n) b[n] = __ldg(bf + n * 32);
    uint32_t a[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) a[i] = is_v ? av[i] : aq[i];
#pragma unroll
    for (int n = 0; n < 16; ++n) {
      float c[4] = {0.f, 0.f, 0.f, 0.f};
      ptx::mma16816<T>(c, a, b[n].x, b[n].y);
      const int col = 8 * n + 2 * tq;
      st_u32(ls + g * kLd + col, Dt<T>::pack2(__fmul_rn(rnd<T>(c[0]), p.scaling), __fmul_rn(rnd<T>(c[1]), p.scaling)));
      st_u32(ls + (g + 8) * kLd + col,
             Dt<T>::pack2(__fmul_rn(rnd<T>(c[2]), p.scaling), __fmul_rn(rnd<T>(c[3]), p.scaling)));
    }
  };
  const auto has_lora = [&](int hh) { return lora && (hh < p.hq || hh >= p.hq + p.hk); };

  if (h < n_heads && has_lora(h)) lora_tile(h);
  ptx::cp_async_wait<0>();
  __syncthreads();  // cos/sin rows come from every warp's copies

  const int c4 = (lane & 15) * 4;
  const int er = lane >> 4;
  if (h < n_heads) {
    const int kind = h < p.hq ? 0 : (h < p.hq + p.hk ? 1 : 2);  // q, k, v
    T* out;
    int64_t otok;
    if (kind == 0) {
      out = static_cast<T*>(p.q) + static_cast<int64_t>(h) * p.q_head;
      otok = p.q_tok;
    } else if (kind == 1) {
      out = static_cast<T*>(p.k) + static_cast<int64_t>(h - p.hq) * p.k_head;
      otok = p.k_tok;
    } else {
      out = static_cast<T*>(p.v) + static_cast<int64_t>(h - p.hq - p.hk) * p.v_head;
      otok = p.v_tok;
    }
    const bool with_lora = has_lora(h);
#pragma unroll 4
    for (int i = 0; i < 8; ++i) {
      const int row = 2 * i + er;
      if (row < nrows) {
        float lo[4], hi[4];
        unpack4<T>(*reinterpret_cast<const uint2*>(ys + row * kLd + c4), lo);
        unpack4<T>(*reinterpret_cast<const uint2*>(ys + row * kLd + c4 + kD / 2), hi);
        if (with_lora) {
          float ll[4], lh[4];
          unpack4<T>(*reinterpret_cast<const uint2*>(ls + row * kLd + c4), ll);
          unpack4<T>(*reinterpret_cast<const uint2*>(ls + row * kLd + c4 + kD / 2), lh);
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            lo[e] = __fadd_rn(lo[e], ll[e]);
            hi[e] = __fadd_rn(hi[e], lh[e]);
          }
        }
        T* dst = out + (t0 + row) * otok + c4;
        if (kind != 2) {
          float cl[4], ch[4], sl[4], sh[4];
          ld4s(cs + row * kD + c4, cl);
          ld4s(cs + row * kD + c4 + kD / 2, ch);
          ld4s(cs + (16 + row) * kD + c4, sl);
          ld4s(cs + (16 + row) * kD + c4 + kD / 2, sh);
          float ol[4], oh[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            // d < D/2: x[d] cos[d] + (-x[d + D/2]) sin[d];  d + D/2: x[d + D/2] cos + x[d] sin
            ol[e] = __fadd_rn(__fmul_rn(lo[e], cl[e]), __fmul_rn(-hi[e], sl[e]));
            oh[e] = __fadd_rn(__fmul_rn(hi[e], ch[e]), __fmul_rn(lo[e], sh[e]));
          }
          st_u64(dst, pack4<T>(ol));
          st_u64(dst + kD / 2, pack4<T>(oh));
        } else {
          st_u64(dst, pack4<T>(lo));
          st_u64(dst + kD / 2, pack4<T>(hi));
        }
      }
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(kWarps * 32, 2)
qkv_bwd_kernel(const QkvBwdParams p) {
  extern __shared__ __align__(16) unsigned char smem[];
  float* cs = reinterpret_cast<float*>(smem);
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int64_t t0 = static_cast<int64_t>(blockIdx.x) * 16;
  const int nrows = static_cast<int>(p.n_tok - t0 < 16 ? p.n_tok - t0 : 16);
  T* ts = reinterpret_cast<T*>(smem + kCsBytes) + warp * kTile;
  T* dy = static_cast<T*>(p.dy);
  const int n_heads = p.hq + 2 * p.hk;
  const bool lora = p.frag != nullptr;
  // v heads feed the LoRA gradient, and are rounded into dy when they come as an accumulator
  const int n_work = lora || p.v_acc != nullptr ? n_heads : p.hq + p.hk;
  const auto src_of = [&](int hh, int64_t& tok) -> const T* {
    if (hh < p.hq) {
      tok = p.gq_tok;
      return static_cast<const T*>(p.gq) + static_cast<int64_t>(hh) * p.gq_head + t0 * p.gq_tok;
    }
    if (hh < p.hq + p.hk) {
      tok = p.gk_tok;
      return static_cast<const T*>(p.gk) + static_cast<int64_t>(hh - p.hq) * p.gk_head + t0 * p.gk_tok;
    }
    tok = p.ldy;
    return dy + t0 * p.ldy + static_cast<int64_t>(hh) * kD;  // dv, placed by the caller
  };
  // stages head hh's tile: from an fp32 accumulator when there is one, else by cp.async
  const auto stage = [&](int hh) {
    const float* acc = nullptr;
    int64_t rs = 0;
    float mul = 1.f;
    if (hh < p.hq) {
      acc = p.q_acc ? p.q_acc + (t0 * p.hq + hh) * kD : nullptr;
      rs = static_cast<int64_t>(p.hq) * kD;
      mul = p.q_mul;
    } else if (hh < p.hq + p.hk) {
      acc = p.k_acc ? p.k_acc + (t0 * p.hk + (hh - p.hq)) * kD : nullptr;
      rs = static_cast<int64_t>(p.hk) * kD;
      mul = p.k_mul;
    } else {
      acc = p.v_acc ? p.v_acc + (t0 * p.hk + (hh - p.hq - p.hk)) * kD : nullptr;
      rs = static_cast<int64_t>(p.hk) * kD;
    }
    if (acc != nullptr) {
      stage_tile_acc<T>(ts, acc, rs, nrows, lane, mul);
    } else {
      int64_t tok;
      const T* src = src_of(hh, tok);
      stage_tile<T>(ts, src, tok, nrows, lane);
    }
  };

  stage_cos_sin(cs, p.cosp, p.sinp, t0, nrows);
  int h = warp;
  if (h < n_work) stage(h);
  ptx::cp_async_commit();
  ptx::cp_async_wait<0>();
  __syncthreads();

  const int c4 = (lane & 15) * 4;
  const int er = lane >> 4;
  float cq[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
  float cv[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
  const uint32_t ts_frag = ptx::smem_u32(ts + (lane & 15) * kLd + (lane >> 4) * 8);
  while (h < n_work) {
    const bool is_v = h >= p.hq + p.hk;
    const bool is_q = h < p.hq;
    const bool to_g = lora && (is_q || is_v);
    const bool v_store = is_v && p.v_acc != nullptr;  // dv rounded from its accumulator into dy
    const int64_t ycol = static_cast<int64_t>(h) * kD;
#pragma unroll 4
    for (int i = 0; i < 8; ++i) {
      const int row = 2 * i + er;
      T* tp = ts + row * kLd + c4;
      float lo[4], hi[4];
      unpack4<T>(*reinterpret_cast<const uint2*>(tp), lo);
      unpack4<T>(*reinterpret_cast<const uint2*>(tp + kD / 2), hi);
      if (!is_v) {
        float cl[4], ch[4], sl[4], sh[4];
        ld4s(cs + row * kD + c4, cl);
        ld4s(cs + row * kD + c4 + kD / 2, ch);
        ld4s(cs + (16 + row) * kD + c4, sl);
        ld4s(cs + (16 + row) * kD + c4 + kD / 2, sh);
        float ol[4], oh[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          // d < D/2: g[d] cos[d] + g[d + D/2] sin[d + D/2];  d + D/2: g[d + D/2] cos - g[d] sin[d]
          ol[e] = __fadd_rn(__fmul_rn(lo[e], cl[e]), __fmul_rn(hi[e], sh[e]));
          oh[e] = __fadd_rn(__fmul_rn(hi[e], ch[e]), -__fmul_rn(lo[e], sl[e]));
        }
        const uint2 wl = pack4<T>(ol), wh = pack4<T>(oh);
        if (row < nrows) {
          st_u64(dy + (t0 + row) * p.ldy + ycol + c4, wl);
          st_u64(dy + (t0 + row) * p.ldy + ycol + c4 + kD / 2, wh);
        }
        unpack4<T>(wl, lo);  // the rounded values are what the LoRA branch scales
        unpack4<T>(wh, hi);
      } else if (v_store && row < nrows) {
        st_u64(dy + (t0 + row) * p.ldy + ycol + c4, pack4<T>(lo));
        st_u64(dy + (t0 + row) * p.ldy + ycol + c4 + kD / 2, pack4<T>(hi));
      }
      if (to_g) {
        // g = dt(x * scaling) (solution/attn.py:250), in place: the A operand of du = g . B16
        float sl4[4], sh4[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          sl4[e] = __fmul_rn(lo[e], p.scaling);
          sh4[e] = __fmul_rn(hi[e], p.scaling);
        }
        *reinterpret_cast<uint2*>(tp) = pack4<T>(sl4);
        *reinterpret_cast<uint2*>(tp + kD / 2) = pack4<T>(sh4);
      }
    }
    if (to_g) {
      __syncwarp();
      const int slot = is_v ? p.hq + (h - p.hq - p.hk) : h;
      const uint2* bf = reinterpret_cast<const uint2*>(p.frag + static_cast<int64_t>(slot) * kFragWords) + lane;
#pragma unroll
      for (int s = 0; s < 8; ++s) {
        uint32_t a[4];
        ptx::ldsm_x4(ts_frag + s * 32, a[0], a[1], a[2], a[3]);
        const uint2 b0 = __ldg(bf + (2 * s) * 32), b1 = __ldg(bf + (2 * s + 1) * 32);
        if (is_v) {
          ptx::mma16816<T>(cv[0], a, b0.x, b0.y);
          ptx::mma16816<T>(cv[1], a, b1.x, b1.y);
        } else {
          ptx::mma16816<T>(cq[0], a, b0.x, b0.y);
          ptx::mma16816<T>(cq[1], a, b1.x, b1.y);
        }
      }
    }
    h += kWarps;
    if (h >= n_work) break;
    __syncwarp();
    stage(h);
    ptx::cp_async_commit();
    ptx::cp_async_wait<0>();
    __syncwarp();
  }
  if (!lora) return;
  // du: per-warp partials (C fragment of n-tile i: rank 8i + 2tq + e at rows g, g + 8) summed
  // over the warps in shared memory, reusing the tiles' space
  __syncthreads();
  float* red = reinterpret_cast<float*>(smem + kCsBytes);  // [warps][2][16][16]
  {
    const int g = lane >> 2, tq = lane & 3;
    float* rw = red + warp * 2 * 256;
#pragma unroll
    for (int i = 0; i < 2; ++i) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int r = 8 * i + 2 * tq + e;
        rw[g * 16 + r] = cq[i][e];
        rw[(g + 8) * 16 + r] = cq[i][2 + e];
        rw[256 + g * 16 + r] = cv[i][e];
        rw[256 + (g + 8) * 16 + r] = cv[i][2 + e];
      }
    }
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < 512; idx += blockDim.x) {  // [q | v] x 16 rows x 16 ranks
    const int which = idx >> 8, row = (idx >> 4) & 15, r = idx & 15;
    float sum = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) sum += red[w * 512 + which * 256 + row * 16 + r];
    if (row < nrows)
      dy[(t0 + row) * p.ldy + static_cast<int64_t>(n_heads) * kD + which * kR + r] = Dt<T>::from_f(sum);
  }
}

bool al4(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 3u) == 0; }
bool al8(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 7u) == 0; }
bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace
}  // namespace decik

using namespace decik;

extern "C" int64_t decik_lora_frag_bytes(int n_heads, int n_kv) {
  if (n_heads <= 0 || n_kv <= 0) return 0;
  return 2LL * (n_heads + n_kv) * kFragWords * 4;
}

extern "C" int decik_lora_pack(const float* a_q, const float* a_v, void* a_out, int64_t lda, int hidden,
                               const float* b_q, const float* b_v, void* frag, int n_heads, int n_kv,
                               int head_dim, int rank, int dtype, void* stream) {
  if (n_heads <= 0 || n_kv <= 0 || hidden < 0) return set_error(DECIK_ERR_INVALID, "lora_pack: bad sizes");
  if (head_dim != kD || rank != kR)
    return set_error(DECIK_ERR_UNSUPPORTED, "lora_pack: head_dim must be 128 and rank 16");
  if (dtype != DECIK_F16 && dtype != DECIK_BF16)
    return set_error(DECIK_ERR_INVALID, "lora_pack: dtype must be F16 or BF16");
  if (b_q == nullptr || b_v == nullptr || frag == nullptr || !al4(frag) ||
      (a_out != nullptr && (a_q == nullptr || a_v == nullptr || lda < hidden)))
    return set_error(DECIK_ERR_INVALID, "lora_pack: null pointer or bad leading dimension");
  const int64_t total = (a_out != nullptr ? 2LL * kR * hidden : 0) + 2LL * (n_heads + n_kv) * kFragWords;
  const int blocks = static_cast<int>(std::min<int64_t>((total + 255) / 256, 4 * sm_count()));
  if (dtype == DECIK_BF16)
    lora_pack_kernel<__nv_bfloat16><<<blocks, 256, 0, as_stream(stream)>>>(
        a_q, a_v, static_cast<__nv_bfloat16*>(a_out), lda, hidden, b_q, b_v, static_cast<uint32_t*>(frag), n_heads, n_kv);
  else
    lora_pack_kernel<__half><<<blocks, 256, 0, as_stream(stream)>>>(
        a_q, a_v, static_cast<__half*>(a_out), lda, hidden, b_q, b_v, static_cast<uint32_t*>(frag), n_heads, n_kv);
  return check_launch("lora_pack");
}

extern "C" int decik_qkv_epilogue_fwd(const void* y, int64_t ldy, const void* u, int64_t ldu,
                                      const void* frag, float scaling, const float* cos,
                                      const float* sin, decik_tensor3_mut q, decik_tensor3_mut k,
                                      decik_tensor3_mut v, void* u_out, int64_t n_tok, int n_heads,
                                      int n_kv, int head_dim, int dtype, void* stream) {
  if (n_tok < 0 || n_heads <= 0 || n_kv <= 0)
    return set_error(DECIK_ERR_INVALID, "qkv_epilogue_fwd: bad sizes");
  if (head_dim != kD) return set_error(DECIK_ERR_UNSUPPORTED, "qkv_epilogue_fwd: head_dim must be 128");
  if (dtype != DECIK_F16 && dtype != DECIK_BF16)
    return set_error(DECIK_ERR_INVALID, "qkv_epilogue_fwd: dtype must be F16 or BF16");
  const bool lora = frag != nullptr;
  if (lora && u == nullptr) return set_error(DECIK_ERR_INVALID, "qkv_epilogue_fwd: LoRA needs u");
  if (n_tok == 0) return DECIK_OK;
  const int64_t width = static_cast<int64_t>(n_heads + 2 * n_kv) * kD;
  if (y == nullptr || cos == nullptr || sin == nullptr || q.ptr == nullptr || k.ptr == nullptr ||
      v.ptr == nullptr)
    return set_error(DECIK_ERR_INVALID, "qkv_epilogue_fwd: null pointer");
  if (ldy < width || (ldy % 8) || !al16(y) || !al16(cos) || !al16(sin) ||
      (lora && (ldu < 2 * kR || (ldu & 1) || !al4(u) || !al16(frag))) || (u_out != nullptr && !al4(u_out)))
    return set_error(DECIK_ERR_INVALID, "qkv_epilogue_fwd: misaligned pointer or leading dimension");
  for (const decik_tensor3_mut* t : {&q, &k, &v})
    if (!al8(t->ptr) || (t->tok_stride % 4) || (t->head_stride % 4))
      return set_error(DECIK_ERR_INVALID, "qkv_epilogue_fwd: outputs need 8-byte alignment and strides % 4 == 0");
  QkvFwdParams p{y, ldy, u, ldu, static_cast<const uint32_t*>(frag), scaling, cos, sin,
                 q.ptr, q.tok_stride, q.head_stride, k.ptr, k.tok_stride, k.head_stride,
                 v.ptr, v.tok_stride, v.head_stride, lora ? u_out : nullptr, n_tok, n_heads, n_kv};
  const dim3 grid(static_cast<unsigned>((n_tok + 15) / 16),
                  static_cast<unsigned>((n_heads + 2 * n_kv + kFwdWarps - 1) / kFwdWarps));
  const int smem = kCsBytes + kFwdWarps * 2 * kTile * 2;
  if (dtype == DECIK_BF16) {
    static std::atomic<unsigned long long> set{0};
    if (int rc = ensure_dyn_smem(qkv_fwd_kernel<__nv_bfloat16>, smem, set, "qkv_epilogue_fwd")) return rc;
    qkv_fwd_kernel<__nv_bfloat16><<<grid, kFwdWarps * 32, smem, as_stream(stream)>>>(p);
  } else {
    static std::atomic<unsigned long long> set{0};
    if (int rc = ensure_dyn_smem(qkv_fwd_kernel<__half>, smem, set, "qkv_epilogue_fwd")) return rc;
    qkv_fwd_kernel<__half><<<grid, kFwdWarps * 32, smem, as_stream(stream)>>>(p);
  }
  return check_launch("qkv_epilogue_fwd");
}

namespace decik {
int qkv_bwd_launch(const QkvBwdParams& p, int dtype, cudaStream_t stream) {
  const unsigned grid = static_cast<unsigned>((p.n_tok + 15) / 16);
  const int smem = kCsBytes + kWarps * kTile * 2;  // >= the du partials [warps][2][16][16] fp32
  static_assert(kWarps * kTile * 2 >= kWarps * 2 * 256 * 4, "du partials must fit in the tiles' space");
  if (dtype == DECIK_BF16) {
    static std::atomic<unsigned long long> set{0};
    if (int rc = ensure_dyn_smem(qkv_bwd_kernel<__nv_bfloat16>, smem, set, "qkv_epilogue_bwd")) return rc;
    qkv_bwd_kernel<__nv_bfloat16><<<grid, kWarps * 32, smem, stream>>>(p);
  } else {
    static std::atomic<unsigned long long> set{0};
    if (int rc = ensure_dyn_smem(qkv_bwd_kernel<__half>, smem, set, "qkv_epilogue_bwd")) return rc;
    qkv_bwd_kernel<__half><<<grid, kWarps * 32, smem, stream>>>(p);
  }
  return check_launch("qkv_epilogue_bwd");
}

// The projection epilogue's backward reading the attention backward's fp32 accumulators (token-major
// [n_tok][heads][128]): dq = q_mul * q_acc always; dk = k_mul * k_acc when k_acc is set, else the
// 16-bit grad_k; dv = v_acc rounded into dy's v columns when v_acc is set, else already there.
// Called by decik_attn_qkv_bwd with validated, aligned buffers.
int qkv_epilogue_bwd_acc(const float* q_acc, float q_mul, const decik_tensor3& grad_k, const float* k_acc,
                         float k_mul, const float* v_acc, const float* cos, const float* sin, const void* frag,
                         float scaling, void* dy, int64_t ldy, int64_t n_tok, int n_heads, int n_kv, int dtype,
                         cudaStream_t stream) {
  if (n_tok == 0) return DECIK_OK;
  const bool lora = frag != nullptr;
  const int64_t width = static_cast<int64_t>(n_heads + 2 * n_kv) * kD + (lora ? 2 * kR : 0);
  if (ldy < width || (ldy % 8) || !al16(dy) || !al16(cos) || !al16(sin) || (lora && !al16(frag)) ||
      !al16(q_acc) || (k_acc && !al16(k_acc)) || (v_acc && !al16(v_acc)) ||
      (!k_acc && (!al16(grad_k.ptr) || (grad_k.tok_stride % 8) || (grad_k.head_stride % 8))))
    return set_error(DECIK_ERR_INVALID, "qkv_epilogue_bwd: misaligned pointer or leading dimension");
  const uint32_t* bfrag =
      lora ? static_cast<const uint32_t*>(frag) + static_cast<int64_t>(n_heads + n_kv) * kFragWords : nullptr;
  QkvBwdParams p{nullptr, 0, 0, grad_k.ptr, grad_k.tok_stride, grad_k.head_stride, cos, sin, bfrag, scaling,
                 dy, ldy, n_tok, n_heads, n_kv, q_acc, k_acc, v_acc, q_mul, k_mul};
  return qkv_bwd_launch(p, dtype, stream);
}
}  // namespace decik

extern "C" int decik_qkv_epilogue_bwd(decik_tensor3 grad_q, decik_tensor3 grad_k, const float* cos,
                                      const float* sin, const void* frag, float scaling, void* dy,
                                      int64_t ldy, int64_t n_tok, int n_heads, int n_kv, int head_dim,
                                      int dtype, void* stream) {
  if (n_tok < 0 || n_heads <= 0 || n_kv <= 0)
    return set_error(DECIK_ERR_INVALID, "qkv_epilogue_bwd: bad sizes");
  if (head_dim != kD) return set_error(DECIK_ERR_UNSUPPORTED, "qkv_epilogue_bwd: head_dim must be 128");
  if (dtype != DECIK_F16 && dtype != DECIK_BF16)
    return set_error(DECIK_ERR_INVALID, "qkv_epilogue_bwd: dtype must be F16 or BF16");
  const bool lora = frag != nullptr;
  if (n_tok == 0) return DECIK_OK;
  const int64_t width = static_cast<int64_t>(n_heads + 2 * n_kv) * kD + (lora ? 2 * kR : 0);
  if (grad_q.ptr == nullptr || grad_k.ptr == nullptr || cos == nullptr || sin == nullptr || dy == nullptr)
    return set_error(DECIK_ERR_INVALID, "qkv_epilogue_bwd: null pointer");
  if (ldy < width || (ldy % 8) || !al16(dy) || !al16(cos) || !al16(sin) || (lora && !al16(frag)))
    return set_error(DECIK_ERR_INVALID, "qkv_epilogue_bwd: misaligned pointer or leading dimension");
  for (const decik_tensor3* t : {&grad_q, &grad_k})
    if (!al16(t->ptr) || (t->tok_stride % 8) || (t->head_stride % 8))
      return set_error(DECIK_ERR_INVALID, "qkv_epilogue_bwd: gradients need 16-byte alignment and strides % 8 == 0");
  // the backward-layout fragments follow the forward ones in the buffer decik_lora_pack wrote
  const uint32_t* bfrag =
      lora ? static_cast<const uint32_t*>(frag) + static_cast<int64_t>(n_heads + n_kv) * kFragWords : nullptr;
  QkvBwdParams p{grad_q.ptr, grad_q.tok_stride, grad_q.head_stride, grad_k.ptr, grad_k.tok_stride,
                 grad_k.head_stride, cos, sin, bfrag, scaling, dy, ldy, n_tok, n_heads, n_kv,
                 nullptr, nullptr, nullptr, 1.f, 1.f};
  return decik::qkv_bwd_launch(p, dtype, as_stream(stream));
}
