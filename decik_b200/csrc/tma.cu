// Host side of the sm_100a kernels: TMA tensor maps for [T, H, 128] 16-bit views, and the device
// error word that bounded waits write when they give up.
#include <cudaTypedefs.h>

#include <mutex>

#include "attn_common.cuh"

namespace decik {

// Set by kernels whose bounded waits gave up (first code wins); read and cleared by
// decik_kernel_error().
static __device__ int g_kernel_error = 0;

namespace attn {

// The device address of g_kernel_error on the current device, looked up once per device behind a
// mutex (host threads may drive different devices concurrently).
int* attn_error_word() {
  constexpr int kMaxDevices = 64;
  static std::mutex mu;
  static int* cached[kMaxDevices] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  std::lock_guard<std::mutex> lock(mu);
  if (cached[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_kernel_error) != cudaSuccess) return nullptr;
    cached[dev] = static_cast<int*>(p);
  }
  return cached[dev];
}

// cuTensorMapEncodeTiled from the driver (process-wide; the function-local static is initialised
// once, thread-safely).
static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static const PFN_cuTensorMapEncodeTiled_v12000 fn = []() -> PFN_cuTensorMapEncodeTiled_v12000 {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    return nullptr;
  }();
  return fn;
}

// A 3-D tiled map over a [T, H, 128] 16-bit view (head_dim contiguous) whose box is one
// box_rows x 64-element half tile with the 128-byte swizzle (the UMMA K-major / MN-major canonical layout).
// The two outer dimensions are ordered by increasing stride: order 0 = (d, token, head),
// order 1 = (d, head, token); the kernel passes its coordinates in that order.
// cuTensorMapEncodeTiled on a host thread that has not yet made a CUDA runtime call (an autograd
// worker, say) has no current context and returns CUDA_ERROR_INVALID_CONTEXT: bind the current
// device's primary context and encode again.
template <typename Encode>
static CUresult encode_with_context(Encode&& encode) {
  CUresult r = encode();
  if (r == CUDA_ERROR_INVALID_CONTEXT) {
    int dev = 0;
    if (cudaGetDevice(&dev) == cudaSuccess && cudaSetDevice(dev) == cudaSuccess) r = encode();
  }
  return r;
}

int make_tile_map_ex(CUtensorMap* map, const void* ptr, int64_t tok_stride, int64_t head_stride, int64_t n_tok,
                     int n_heads, int dtype, int* order, int box_rows, int box_inner, int swizzle_bytes);

int make_tile_map(CUtensorMap* map, const void* ptr, int64_t tok_stride, int64_t head_stride, int64_t n_tok,
                  int n_heads, int dtype, int* order, int box_rows) {
  return make_tile_map_ex(map, ptr, tok_stride, head_stride, n_tok, n_heads, dtype, order, box_rows, 64, 128);
}

// The same map with a box of box_inner elements of head_dim and the given swizzle (128 or 64 bytes;
// box_inner x 2 bytes must equal it).
int make_tile_map_ex(CUtensorMap* map, const void* ptr, int64_t tok_stride, int64_t head_stride, int64_t n_tok,
                     int n_heads, int dtype, int* order, int box_rows, int box_inner, int swizzle_bytes) {
  if (box_inner * 2 != swizzle_bytes || (swizzle_bytes != 128 && swizzle_bytes != 64))
    return set_error(DECIK_ERR_INVALID, "make_tile_map: box of %d elements with a %d-byte swizzle", box_inner,
                     swizzle_bytes);
  auto fn = encode_fn();
  if (fn == nullptr) return set_error(DECIK_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  const bool tok_inner = tok_stride <= head_stride || n_heads == 1;
  *order = tok_inner ? 0 : 1;
  cuuint64_t dims[3], strides[2];
  cuuint32_t box[3], estr[3] = {1, 1, 1};
  dims[0] = 128;
  if (tok_inner) {
    dims[1] = static_cast<cuuint64_t>(n_tok);
    dims[2] = static_cast<cuuint64_t>(n_heads);
    strides[0] = static_cast<cuuint64_t>(tok_stride) * 2;
    strides[1] = static_cast<cuuint64_t>(n_heads == 1 ? tok_stride * n_tok : head_stride) * 2;
    box[0] = static_cast<cuuint32_t>(box_inner); box[1] = static_cast<cuuint32_t>(box_rows); box[2] = 1;
  } else {
    dims[1] = static_cast<cuuint64_t>(n_heads);
    dims[2] = static_cast<cuuint64_t>(n_tok);
    strides[0] = static_cast<cuuint64_t>(head_stride) * 2;
    strides[1] = static_cast<cuuint64_t>(tok_stride) * 2;
    box[0] = static_cast<cuuint32_t>(box_inner); box[1] = 1; box[2] = static_cast<cuuint32_t>(box_rows);
  }
  const CUtensorMapDataType dt = dtype == DECIK_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUresult r = encode_with_context([&] {
    return fn(map, dt, 3, const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
              swizzle_bytes == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  });
  if (r != CUDA_SUCCESS)
    return set_error(DECIK_ERR_INVALID, "cuTensorMapEncodeTiled failed (%d): tok_stride %lld head_stride %lld",
                     static_cast<int>(r), (long long)tok_stride, (long long)head_stride);
  return DECIK_OK;
}

// A 2-D tiled map with the 128- or 64-byte swizzle over a row-major matrix of `outer` rows x
// `inner` elements (row stride row_bytes), box box_outer rows x box_inner elements (box_inner x the
// element size must equal the swizzle: one swizzle row). dtype: DECIK_F16 / DECIK_BF16 / DECIK_F32.
int make_map_2d(CUtensorMap* map, const void* ptr, int dtype, uint64_t inner, uint64_t outer, uint64_t row_bytes,
                uint32_t box_inner, uint32_t box_outer, int swizzle_bytes) {
  auto fn = encode_fn();
  if (fn == nullptr) return set_error(DECIK_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  const CUtensorMapDataType dt = dtype == DECIK_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                 : dtype == DECIK_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                      : CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
  const uint32_t esize = dtype == DECIK_F32 ? 4 : 2;
  if ((swizzle_bytes != 128 && swizzle_bytes != 64) || box_inner * esize != static_cast<uint32_t>(swizzle_bytes))
    return set_error(DECIK_ERR_INVALID, "make_map_2d: box inner %u x %u bytes is not one %d-byte swizzle row",
                     box_inner, esize, swizzle_bytes);
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_bytes};
  cuuint32_t box[2] = {box_inner, box_outer}, estr[2] = {1, 1};
  CUresult r = encode_with_context([&] {
    return fn(map, dt, 2, const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
              swizzle_bytes == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  });
  if (r != CUDA_SUCCESS)
    return set_error(DECIK_ERR_INVALID, "cuTensorMapEncodeTiled (2-D) failed (%d): %llu x %llu, row %llu bytes",
                     static_cast<int>(r), (unsigned long long)outer, (unsigned long long)inner,
                     (unsigned long long)row_bytes);
  return DECIK_OK;
}

// A 3-D map over an fp32 [T, H, 128] tensor (dims ordered d, head, token; head stride 512 B) whose
// box is box_rows tokens x one head x 128 dims, no swizzle: the target of the dq tile reductions.
// fp32 [n_tok, n_heads, 128] accumulator (dq, dk, dv) for TMA reduce-add of [box_rows x 16] chunks
// staged with the 64-byte swizzle (16 fp32 = 64 bytes per row).
int make_f32_chunk_map(CUtensorMap* map, float* ptr, int64_t n_tok, int n_heads, int box_rows) {
  auto fn = encode_fn();
  if (fn == nullptr) return set_error(DECIK_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[3] = {128, static_cast<cuuint64_t>(n_heads), static_cast<cuuint64_t>(n_tok)};
  cuuint64_t strides[2] = {128 * 4, static_cast<cuuint64_t>(n_heads) * 128 * 4};
  cuuint32_t box[3] = {16, 1, static_cast<cuuint32_t>(box_rows)}, estr[3] = {1, 1, 1};
  CUresult r = encode_with_context([&] {
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, ptr, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
              CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  });
  if (r != CUDA_SUCCESS) return set_error(DECIK_ERR_INVALID, "cuTensorMapEncodeTiled (fp32 chunks) failed (%d)", static_cast<int>(r));
  return DECIK_OK;
}

}  // namespace attn
}  // namespace decik

extern "C" int decik_kernel_error(int reset) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, decik::g_kernel_error, sizeof(int)) != cudaSuccess) return -1;
  if (reset && v != 0) {
    const int zero = 0;
    cudaMemcpyToSymbol(decik::g_kernel_error, &zero, sizeof(int));
  }
  return v;
}
