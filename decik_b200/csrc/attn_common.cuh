// Parameters and tile helpers shared by the varlen attention kernels.
#pragma once

#include "common.cuh"
#include "ptx.cuh"

namespace decik {
namespace attn {

constexpr int D = 128;            // head_dim
constexpr int kRowBytes = D * 2;  // one 16-bit row of a tile
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

struct Tensor3 {
  const void* ptr;
  int64_t tok;
  int64_t head;
};
struct Tensor3Mut {
  void* ptr;
  int64_t tok;
  int64_t head;
};

// Element offset of 16-byte chunk `chunk` (0..15) of row `row` in a [rows x 128] 16-bit tile,
// XOR-swizzled so that the 8 rows an ldmatrix reads fall in 8 different bank groups.
__device__ __forceinline__ int swz(int row, int chunk) { return row * D + ((chunk ^ (row & 7)) << 3); }

// Copies rows [0, R) of a [R x 128] tile whose row r is token (tok0 + r) of head `head`;
// tokens >= tok_end are zero-filled. Spread over NT threads.
template <int R, int NT>
__device__ __forceinline__ void load_tile(uint32_t s_base, const Tensor3& t, int64_t tok0,
                                          int64_t tok_end, int head, int tid) {
  const char* g = static_cast<const char*>(t.ptr);
  constexpr int kChunks = R * 16;
#pragma unroll
  for (int i = tid; i < kChunks; i += NT) {
    const int r = i >> 4;
    const int c = i & 15;
    const int64_t tok = tok0 + r;
    const bool ok = tok < tok_end;
    const char* src = ok ? g + 2 * (tok * t.tok + static_cast<int64_t>(head) * t.head + c * 8) : g;
    ptx::cp_async16(s_base + 2 * swz(r, c), src, ok);
  }
}

}  // namespace attn
}  // namespace decik
