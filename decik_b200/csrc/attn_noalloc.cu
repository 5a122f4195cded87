// Attention backward for callers that must not allocate device memory.
//
// decik_varlen_attn_bwd needs a caller-provided workspace (the fp32 dq accumulator and the
// per-query rowsum(dO * O)). Some callers cannot provide one: code that runs inside a host
// framework whose device memory is entirely owned by its own pool and that forbids raw
// cudaMalloc after start-up, plugins loaded into such hosts, and code paths that run where an
// allocation could stall or fail (for instance while the caller already holds its allocator's
// lock). This entry point takes the same tensors but no workspace: its scratch is one static
// device array in this file, sized for at most kNoAllocTokenHeads (tokens x query heads).
//
// Properties a caller must know:
// - The array exists on every GPU that loads this library and stays allocated until the process
//   exits (about 8.5 MB per GPU).
// - The first call on a device looks the array's address up (cudaGetSymbolAddress, with that
//   device current) and caches it. The library is built as separate device modules and CUDA loads
//   modules lazily by default, so that first lookup is also when the driver loads this file's
//   module and reserves the 8.5 MB on the device: make the first call at start-up, before the
//   caller's pool claims the device memory and before any stream capture. A call with zero tokens
//   does only this set-up (no kernel runs), so it serves as the start-up call.
// - All calls share the one array. The kernels zero the dq accumulator and rewrite the delta
//   values at the start of every call, so stale contents from an earlier call do not matter, but
//   two calls whose kernels overlap on the GPU (different streams, no ordering) race on the array.
// - No cudaMalloc, cudaFree or allocating library routine is called.
#include <mutex>

#include "attn_common.cuh"

namespace decik {
namespace {

constexpr int64_t kNoAllocTokenHeads = 16384;
constexpr int64_t kNoAllocScratchBytes =
    ((kNoAllocTokenHeads * attn::D * 4 + 255) / 256) * 256 + ((kNoAllocTokenHeads * 4 + 255) / 256) * 256;
}  // namespace
namespace attn {
int64_t bwd_workspace_bytes(int64_t n_tok, int n_heads, bool kv_acc);
int varlen_attn_bwd_impl(const decik_tensor3& dout, const decik_tensor3& q, const decik_tensor3& k,
                         const decik_tensor3& v, const decik_tensor3& out, const float* lse,
                         const decik_tensor3_mut& dq, const decik_tensor3_mut& dk, const decik_tensor3_mut& dv,
                         const int32_t* cu_seqlens, int n_rows, int max_len, int64_t n_tok, int n_heads,
                         int n_kv, int head_dim, float scale, int dtype, void* workspace, bool allow_split,
                         cudaStream_t s);
}  // namespace attn
namespace {

static __device__ __align__(256) unsigned char g_bwd_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;

// The device address of g_bwd_scratch on the current device (looked up once per device).
int scratch_address(void** out) {
  static std::mutex mu;
  static void* cached[kMaxDevices] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_error(DECIK_ERR_CUDA, "varlen_attn_bwd_noalloc: cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices) return set_error(DECIK_ERR_UNSUPPORTED, "varlen_attn_bwd_noalloc: device %d", dev);
  std::lock_guard<std::mutex> lock(mu);
  if (cached[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_bwd_scratch);
    if (e != cudaSuccess || p == nullptr)
      return set_error(DECIK_ERR_CUDA, "varlen_attn_bwd_noalloc: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
    cached[dev] = p;
  }
  *out = cached[dev];
  return DECIK_OK;
}

}  // namespace
}  // namespace decik

extern "C" int decik_varlen_attn_bwd_noalloc(decik_tensor3 dout, decik_tensor3 q, decik_tensor3 k,
                                             decik_tensor3 v, decik_tensor3 out, const float* lse,
                                             decik_tensor3_mut dq, decik_tensor3_mut dk,
                                             decik_tensor3_mut dv, const int32_t* cu_seqlens, int n_rows,
                                             int max_len, int64_t n_tok, int n_heads, int n_kv, int head_dim,
                                             float scale, int dtype, void* stream) {
  using namespace decik;
  if (n_tok < 0 || n_heads <= 0)
    return set_error(DECIK_ERR_INVALID, "varlen_attn_bwd_noalloc: bad sizes (T=%lld, heads %d)", (long long)n_tok, n_heads);
  if (n_tok * n_heads > kNoAllocTokenHeads)
    return set_error(DECIK_ERR_INVALID,
                     "varlen_attn_bwd_noalloc: %lld tokens x %d heads exceeds the static scratch "
                     "(%lld token-heads); use decik_varlen_attn_bwd with a workspace",
                     (long long)n_tok, n_heads, (long long)kNoAllocTokenHeads);
  if (attn::bwd_workspace_bytes(n_tok, n_heads, false) > kNoAllocScratchBytes)
    return set_error(DECIK_ERR_INVALID, "varlen_attn_bwd_noalloc: workspace larger than the static scratch");
  void* scratch = nullptr;
  const int rc = scratch_address(&scratch);
  if (rc) return rc;
  if (n_rows == 0 || n_tok == 0 || max_len == 0) return DECIK_OK;  // set-up only
  // one head subset per key block: dK / dV stay on chip, so the scratch holds only dq and delta
  return attn::varlen_attn_bwd_impl(dout, q, k, v, out, lse, dq, dk, dv, cu_seqlens, n_rows, max_len, n_tok, n_heads,
                                    n_kv, head_dim, scale, dtype, scratch, false, as_stream(stream));
}
