// Shared helpers of the decik_b200 kernels: status reporting, dtype traits, vector packing.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <cstdarg>
#include <cstdio>

#include "decik_b200.h"

namespace decik {

// Records the calling thread's last error message; defined in capi.cu.
int set_error(int code, const char* fmt, ...);

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

// Returns DECIK_ERR_CUDA with the launch error, or DECIK_OK.
inline int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(DECIK_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  return DECIK_OK;
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Raises a kernel's dynamic shared-memory limit to `bytes` on the current device, once per device:
// the setting belongs to each device's context. `done` is the call site's bitmask of devices
// already set (devices 0-63); host threads driving different devices may call concurrently (a
// device set twice by two racing threads is harmless: the attribute call is idempotent).
template <typename Kernel>
inline int ensure_dyn_smem(Kernel kernel, int bytes, std::atomic<unsigned long long>& done, const char* what) {
  int dev = 0;
  cudaGetDevice(&dev);
  const unsigned long long bit = 1ull << (dev & 63);
  if (done.load(std::memory_order_acquire) & bit) return DECIK_OK;
  const cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e != cudaSuccess) return set_error(DECIK_ERR_CUDA, "%s: dynamic shared memory %d bytes: %s", what, bytes,
                                         cudaGetErrorString(e));
  done.fetch_or(bit, std::memory_order_acq_rel);
  return DECIK_OK;
}

inline int sm_count() {
  static int n = 0;
  if (n == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
  }
  return n;
}
inline int64_t l2_bytes() {
  static int n = 0;
  if (n == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrL2CacheSize, dev);
    if (n <= 0) n = 126 << 20;
  }
  return n;
}

// ---- dtype traits: 16-bit storage types and fp32 conversions (round to nearest even) ----
template <typename T> struct Dt;
template <> struct Dt<__half> {
  static __device__ __forceinline__ float to_f(__half x) { return __half2float(x); }
  static __device__ __forceinline__ __half from_f(float x) { return __float2half_rn(x); }
  static __device__ __forceinline__ uint32_t pack2(float lo, float hi) {
    __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  static __device__ __forceinline__ float lo_f(uint32_t v) {
    return __half2float(__ushort_as_half(static_cast<unsigned short>(v & 0xFFFFu)));
  }
  static __device__ __forceinline__ float hi_f(uint32_t v) {
    return __half2float(__ushort_as_half(static_cast<unsigned short>(v >> 16)));
  }
};
template <> struct Dt<__nv_bfloat16> {
  static __device__ __forceinline__ float to_f(__nv_bfloat16 x) { return __bfloat162float(x); }
  static __device__ __forceinline__ __nv_bfloat16 from_f(float x) { return __float2bfloat16_rn(x); }
  static __device__ __forceinline__ uint32_t pack2(float lo, float hi) {
    __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  static __device__ __forceinline__ float lo_f(uint32_t v) { return __uint_as_float(v << 16); }
  static __device__ __forceinline__ float hi_f(uint32_t v) { return __uint_as_float(v & 0xFFFF0000u); }
};

// 8 x 16-bit values <-> uint4
template <typename T>
__device__ __forceinline__ void unpack8(const uint4& v, float (&f)[8]) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = Dt<T>::lo_f(w[i]);
    f[2 * i + 1] = Dt<T>::hi_f(w[i]);
  }
}

template <typename T>
__device__ __forceinline__ uint4 pack8(const float (&f)[8]) {
  uint4 v;
  v.x = Dt<T>::pack2(f[0], f[1]);
  v.y = Dt<T>::pack2(f[2], f[3]);
  v.z = Dt<T>::pack2(f[4], f[5]);
  v.w = Dt<T>::pack2(f[6], f[7]);
  return v;
}

__device__ __forceinline__ uint4 ldg16(const void* p) {
  return __ldg(reinterpret_cast<const uint4*>(p));
}
__device__ __forceinline__ void stg16(void* p, const uint4& v) {
  *reinterpret_cast<uint4*>(p) = v;
}

}  // namespace decik

// Dispatches a body templated on the 16-bit element type named T.
#define DECIK_DISPATCH_16(dtype, ...)                         \
  [&]() -> int {                                              \
    if ((dtype) == DECIK_F16) {                               \
      using T = __half;                                       \
      return __VA_ARGS__();                                   \
    } else if ((dtype) == DECIK_BF16) {                       \
      using T = __nv_bfloat16;                                \
      return __VA_ARGS__();                                   \
    }                                                         \
    return decik::set_error(DECIK_ERR_INVALID, "dtype %d is not F16/BF16", (int)(dtype)); \
  }()
