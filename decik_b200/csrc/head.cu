// Row statistics of one chunk of LM-head logits, and the cross-entropy gradient written over
// them. Replaces skc_head_stats_kernel (solution/head.py:39-85) of the reference's FusedHeadLoss.
//
// One CTA per row of logits (16-bit, [rows, n_vocab], row stride ld). Pass 1 reads the row
// once and keeps, per thread, a running max m, sum of exp(z - m), sum of z * exp(z - m) and the
// first index of its maximum, 8 values (16 bytes) per step. The block then combines them:
// lse = m + log(s), entropy = lse - w / s, argmax = the smallest index holding the row maximum
// (torch.argmax's tie rule), token loss = lse - z[target] for a labelled row (0 <= target <
// n_vocab), 0 for an ignored one (target < 0), NaN for a target past the vocabulary; hit =
// labelled and argmax == target. Pass 2, for labelled rows only, writes
// softmax - onehot = exp(z - lse) - [col == target] over the logits in place, rounded to the
// logits' type: the operand of the gradient matmul dX = G . W. The arithmetic is fp32; the
// per-logit exponentials of both passes are exp(z - c) = 2^(z log2 e - c log2 e), one FMA and the
// hardware's ex2.approx (a relative error of a few 1e-7 for the logit ranges of a head; expf took
// most of the kernel's issue slots). HBM-bound: a labelled row moves 3 x n_vocab x 2 bytes (read,
// read, write).
#include <cfloat>

#include "common.cuh"
#include "ptx.cuh"

namespace decik {
namespace {

constexpr int kHeadThreads = 512;
constexpr float kLog2eHead = 1.4426950408889634f;

struct Stat {
  float m, s, w;  // max, sum exp(z - m), sum z exp(z - m)
  int idx;        // first index of the max
};

__device__ __forceinline__ Stat combine(Stat a, Stat b) {
  if (b.m > a.m || (b.m == a.m && b.idx < a.idx)) {
    const Stat t = a;
    a = b;
    b = t;
  }
  // a holds the larger max (the smaller index on a tie)
  if (b.m == -INFINITY) return a;
  const float f = expf(b.m - a.m);
  a.s += b.s * f;
  a.w += b.w * f;
  return a;
}

template <typename T>
__global__ void __launch_bounds__(kHeadThreads)
head_stats_kernel(T* __restrict__ logits, int64_t ld, const int64_t* __restrict__ target, float* __restrict__ lse_out,
                  float* __restrict__ entropy_out, float* __restrict__ loss_out, int* __restrict__ hit_out,
                  int n_vocab) {
  __shared__ Stat red[kHeadThreads / 32];
  __shared__ float s_lse;
  const int64_t row = blockIdx.x;
  T* z = logits + row * ld;
  const int64_t tgt = target[row];
  const bool labelled = tgt >= 0 && tgt < n_vocab;
  const bool invalid = tgt >= n_vocab;  // a target outside the vocabulary: NaN loss, no gradient
  Stat st{-INFINITY, 0.f, 0.f, n_vocab};
  for (int c = threadIdx.x * 8; c < n_vocab; c += kHeadThreads * 8) {
    const uint4 u = *reinterpret_cast<const uint4*>(z + c);
    const uint32_t wd[4] = {u.x, u.y, u.z, u.w};
    float v[8];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      v[2 * i] = Dt<T>::lo_f(wd[i]);
      v[2 * i + 1] = Dt<T>::hi_f(wd[i]);
    }
    float mx = v[0];
    int at = 0;
#pragma unroll
    for (int i = 1; i < 8; ++i)
      if (v[i] > mx) { mx = v[i]; at = i; }
    if (mx > st.m) {  // strictly larger: earlier columns keep the index on ties
      const float f = st.m == -INFINITY ? 0.f : ptx::ex2((st.m - mx) * kLog2eHead);
      st.s *= f;
      st.w *= f;
      st.m = mx;
      st.idx = c + at;
    }
    const float nm = -st.m * kLog2eHead;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float e = ptx::ex2(fmaf(v[i], kLog2eHead, nm));
      st.s += e;
      st.w += v[i] * e;
    }
  }
  // warp, then block combination
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    Stat other;
    other.m = __shfl_xor_sync(0xffffffffu, st.m, o);
    other.s = __shfl_xor_sync(0xffffffffu, st.s, o);
    other.w = __shfl_xor_sync(0xffffffffu, st.w, o);
    other.idx = __shfl_xor_sync(0xffffffffu, st.idx, o);
    st = combine(st, other);
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = st;
  __syncthreads();
  if (warp == 0) {
    st = lane < kHeadThreads / 32 ? red[lane] : Stat{-INFINITY, 0.f, 0.f, n_vocab};
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) {
      Stat other;
      other.m = __shfl_xor_sync(0xffffffffu, st.m, o);
      other.s = __shfl_xor_sync(0xffffffffu, st.s, o);
      other.w = __shfl_xor_sync(0xffffffffu, st.w, o);
      other.idx = __shfl_xor_sync(0xffffffffu, st.idx, o);
      st = combine(st, other);
    }
    if (lane == 0) {
      const float lse = st.m + logf(st.s);
      lse_out[row] = lse;
      entropy_out[row] = lse - st.w / st.s;
      const float zt = labelled ? Dt<T>::to_f(z[tgt]) : 0.f;
      loss_out[row] = labelled ? lse - zt : (invalid ? __int_as_float(0x7fc00000) : 0.f);
      hit_out[row] = labelled && st.idx == tgt ? 1 : 0;
      s_lse = lse;
    }
  }
  __syncthreads();
  if (!labelled) return;
  const float nl = -s_lse * kLog2eHead;
  for (int c = threadIdx.x * 8; c < n_vocab; c += kHeadThreads * 8) {
    const uint4 u = *reinterpret_cast<const uint4*>(z + c);
    const uint32_t wd[4] = {u.x, u.y, u.z, u.w};
    uint32_t o[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float a = ptx::ex2(fmaf(Dt<T>::lo_f(wd[i]), kLog2eHead, nl));
      float b = ptx::ex2(fmaf(Dt<T>::hi_f(wd[i]), kLog2eHead, nl));
      if (c + 2 * i == tgt) a -= 1.f;
      if (c + 2 * i + 1 == tgt) b -= 1.f;
      o[i] = Dt<T>::pack2(a, b);
    }
    *reinterpret_cast<uint4*>(z + c) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

}  // namespace
}  // namespace decik

extern "C" int decik_head_stats(void* logits, int64_t ld, const int64_t* target, float* lse, float* entropy,
                                float* token_loss, int* hit, int64_t n_rows, int n_vocab, int dtype, void* stream) {
  using namespace decik;
  if (n_rows == 0) return DECIK_OK;
  if (n_rows < 0 || n_rows > INT32_MAX || n_vocab <= 0 || n_vocab % 8 != 0 || ld < n_vocab || ld % 8 != 0)
    return set_error(DECIK_ERR_INVALID, "head_stats: n_vocab %d (multiple of 8), ld %lld (>= n_vocab, multiple of 8)",
                     n_vocab, (long long)ld);
  if (!logits || !target || !lse || !entropy || !token_loss || !hit)
    return set_error(DECIK_ERR_INVALID, "head_stats: null pointer");
  if (!aligned16(logits)) return set_error(DECIK_ERR_INVALID, "head_stats: logits must be 16-byte aligned");
  return DECIK_DISPATCH_16(dtype, [&] {
    head_stats_kernel<T><<<static_cast<unsigned>(n_rows), kHeadThreads, 0, as_stream(stream)>>>(
        static_cast<T*>(logits), ld, target, lse, entropy, token_loss, hit, n_vocab);
    return check_launch("head_stats");
  });
}
