// The padding-free packing of a right-padded [B, S] batch, built on the device.
//
// The reference builds it on the host side of the step (solution/varlen.py:191-226): mask.sum,
// a torch.equal check that the mask is right-padded, lengths.tolist() and mask.nonzero(), three
// device-to-host synchronisations. Here one kernel reads the mask once and writes everything the
// packed decoder needs on the device:
//   row lengths, cu_seqlens int32 [B + 1] (solution/varlen.py:35-40),
//   index int64 [T]: the flat position b * S + s of each real token, in row-major order,
//   positions int64 [T]: s, each token's position in its row (solution/varlen.py:221),
//   optionally the packed token ids (input_ids gathered at index),
// and a small summary [T, max_len, right-padded flag, min_len, lengths...] that the caller copies
// to pinned host memory: the one read the host needs (the sizes of the packed tensors).
//
// One CTA of 1024 threads. Phase 1: warp w scans rows w, w + 32, ... with coalesced loads; a row is
// right-padded iff its last 1 comes before its first 0, and then its length is the index of its
// first 0. Phase 2: a block-wide exclusive scan of the lengths gives cu_seqlens. Phase 3: each warp
// writes its rows' index / positions / ids, contiguous per row. The mask is HBM-read once
// (B * S elements); the outputs are written once (3 x 8 B per real token).
#include "common.cuh"

namespace decik {
namespace {

constexpr int kThreads = 1024;
constexpr int kWarps = kThreads / 32;
constexpr int64_t kMaxRows = 8192;  // lengths kept in shared memory (32 KB)

template <typename M>
__device__ __forceinline__ bool is_set(const M* mask, int64_t i) {
  return mask[i] != M(0);
}

template <typename M>
__global__ void __launch_bounds__(kThreads) pack_rows_kernel(const M* __restrict__ mask, const int64_t* __restrict__ ids,
                                                             int64_t batch, int64_t seq, int32_t* __restrict__ cu,
                                                             int64_t* __restrict__ index, int64_t* __restrict__ positions,
                                                             int64_t* __restrict__ ids_out, int32_t* __restrict__ summary) {
  extern __shared__ int32_t len_s[];  // [batch]
  __shared__ int32_t warp_part[kWarps];
  __shared__ int32_t red_max[kWarps], red_min[kWarps], red_bad[kWarps];
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;

  // phase 1: per-row length and right-padding check
  int bad_any = 0;
  for (int64_t b = warp; b < batch; b += kWarps) {
    const M* row = mask + b * seq;
    int64_t first_zero = seq, last_one = -1;
    for (int64_t s0 = 0; s0 < seq; s0 += 32) {
      const int64_t s = s0 + lane;
      const bool in = s < seq;
      const bool one = in && is_set(row, s);
      const unsigned ones = __ballot_sync(0xffffffffu, one);
      const unsigned zeros = __ballot_sync(0xffffffffu, in && !one);
      if (zeros != 0u && first_zero == seq) first_zero = s0 + __ffs(zeros) - 1;
      if (ones != 0u) last_one = s0 + 31 - __clz(ones);
    }
    const bool ok = last_one < first_zero;
    if (lane == 0) len_s[b] = ok ? static_cast<int32_t>(first_zero) : 0;
    bad_any |= ok ? 0 : 1;
  }
  __syncthreads();

  // phase 2: exclusive scan of the lengths (thread t sums a contiguous chunk of rows), max / min
  const int64_t per = (batch + kThreads - 1) / kThreads;
  const int64_t r0 = threadIdx.x * per;
  const int64_t r1 = r0 + per < batch ? r0 + per : batch;
  int32_t local = 0, mx = 0, mn = 0x7fffffff;
  for (int64_t r = r0; r < r1; ++r) {
    local += len_s[r];
    mx = max(mx, len_s[r]);
    mn = min(mn, len_s[r]);
  }
  int32_t incl = local;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int32_t v = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += v;
  }
  const int wmax = __reduce_max_sync(0xffffffffu, mx);
  const int wmin = __reduce_min_sync(0xffffffffu, mn);
  const int wbad = __reduce_or_sync(0xffffffffu, bad_any);
  if (lane == 31) warp_part[warp] = incl;
  if (lane == 0) {
    red_max[warp] = wmax;
    red_min[warp] = wmin;
    red_bad[warp] = wbad;
  }
  __syncthreads();
  if (warp == 0) {
    const int32_t v = warp_part[lane];
    int32_t w_incl = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int32_t t = __shfl_up_sync(0xffffffffu, w_incl, o);
      if (lane >= o) w_incl += t;
    }
    warp_part[lane] = w_incl - v;  // exclusive prefix of the warp totals
    const int gmax = __reduce_max_sync(0xffffffffu, red_max[lane]);
    const int gmin = __reduce_min_sync(0xffffffffu, red_min[lane]);
    const int gbad = __reduce_or_sync(0xffffffffu, red_bad[lane]);
    if (lane == 31) {
      summary[0] = w_incl;  // T
      summary[1] = gmax;
      summary[2] = gbad ? 0 : 1;
      summary[3] = batch > 0 ? gmin : 0;
      cu[batch] = w_incl;
    }
  }
  __syncthreads();
  int32_t run = warp_part[warp] + incl - local;  // exclusive prefix of this thread's first row
  for (int64_t r = r0; r < r1; ++r) {
    cu[r] = run;
    summary[4 + r] = len_s[r];
    run += len_s[r];
  }
  __syncthreads();
  // the starts are in cu (global, this CTA's own writes): make them visible to the whole CTA
  __threadfence_block();

  // phase 3: scatter, one warp per row, contiguous stores
  for (int64_t b = warp; b < batch; b += kWarps) {
    const int32_t start = cu[b];
    const int32_t n = len_s[b];
    const int64_t base = b * seq;
    for (int32_t s = lane; s < n; s += 32) {
      index[start + s] = base + s;
      positions[start + s] = s;
      if (ids_out != nullptr) ids_out[start + s] = ids[base + s];
    }
  }
}

}  // namespace
}  // namespace decik

extern "C" int decik_pack_rows(const void* mask, int mask_dtype, const int64_t* input_ids, int64_t batch, int64_t seq,
                               int32_t* cu_seqlens, int64_t* index, int64_t* positions, int64_t* ids_out,
                               int32_t* summary, void* stream) {
  using namespace decik;
  if (batch < 0 || seq < 0 || batch > kMaxRows || seq > (int64_t(1) << 30) || batch * seq > (int64_t(1) << 31) - 1)
    return set_error(DECIK_ERR_INVALID, "pack_rows: batch %lld x seq %lld outside [0, %lld] x [0, 2^30] (or B*S >= 2^31)",
                     (long long)batch, (long long)seq, (long long)kMaxRows);
  if (cu_seqlens == nullptr || summary == nullptr || (batch * seq > 0 && (mask == nullptr || index == nullptr || positions == nullptr)))
    return set_error(DECIK_ERR_INVALID, "pack_rows: NULL pointer");
  if ((ids_out == nullptr) != (input_ids == nullptr))
    return set_error(DECIK_ERR_INVALID, "pack_rows: input_ids and ids_out go together");
  const size_t smem = static_cast<size_t>(batch > 0 ? batch : 1) * sizeof(int32_t);
  static std::atomic<unsigned long long> set64{0}, set32{0}, set8{0};
  cudaStream_t s = as_stream(stream);
  switch (mask_dtype) {
    case 0: {  // int64 (transformers' attention_mask)
      if (int rc = ensure_dyn_smem(pack_rows_kernel<int64_t>, static_cast<int>(kMaxRows * 4), set64, "pack_rows")) return rc;
      pack_rows_kernel<int64_t><<<1, kThreads, smem, s>>>(static_cast<const int64_t*>(mask), input_ids, batch, seq,
                                                          cu_seqlens, index, positions, ids_out, summary);
      break;
    }
    case 1: {  // int32
      if (int rc = ensure_dyn_smem(pack_rows_kernel<int32_t>, static_cast<int>(kMaxRows * 4), set32, "pack_rows")) return rc;
      pack_rows_kernel<int32_t><<<1, kThreads, smem, s>>>(static_cast<const int32_t*>(mask), input_ids, batch, seq,
                                                          cu_seqlens, index, positions, ids_out, summary);
      break;
    }
    case 2: {  // bool / uint8
      if (int rc = ensure_dyn_smem(pack_rows_kernel<uint8_t>, static_cast<int>(kMaxRows * 4), set8, "pack_rows")) return rc;
      pack_rows_kernel<uint8_t><<<1, kThreads, smem, s>>>(static_cast<const uint8_t*>(mask), input_ids, batch, seq,
                                                          cu_seqlens, index, positions, ids_out, summary);
      break;
    }
    default:
      return set_error(DECIK_ERR_INVALID, "pack_rows: mask dtype code %d (0 int64, 1 int32, 2 uint8/bool)", mask_dtype);
  }
  return check_launch("pack_rows");
}
