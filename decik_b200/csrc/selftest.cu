// Self-test of the kernels' failure path: a bounded mbarrier wait that runs out.
//
// Every tcgen05 kernel here waits on mbarriers with mbar_wait (sm100.cuh): after a cycle limit it
// records a code in the device error word and winds down (frees its TMEM and returns) instead of
// spinning forever. The production limit (8e9 cycles) is never reached in a working kernel, so this
// entry point exercises the same path on purpose and cheaply: one warp allocates TMEM, waits on a
// barrier that nothing arrives on with a caller-given limit, reports kWaitSelftestCode, frees the
// TMEM and returns. No fault, trap or endless loop is involved; the context stays usable.
#include "attn_common.cuh"
#include "sm100.cuh"

namespace decik {
namespace attn {
int* attn_error_word();
}
namespace {

constexpr int kWaitSelftestCode = 901;

__global__ void __launch_bounds__(32) wait_selftest_kernel(int* err, long long limit, int* done) {
  using namespace sm100;
  __shared__ __align__(8) uint64_t bar;
  __shared__ uint32_t tmem_base;
  const uint32_t b = smem_u32(&bar);
  if (threadIdx.x == 0) {
    mbar_init(b, 1);
    fence_barrier_init();
  }
  __syncwarp();
  tmem_alloc(smem_u32(&tmem_base), 32);  // held while waiting, as a real kernel holds its TMEM
  tmem_relinquish();
  tc_fence_before();
  __syncwarp();
  tc_fence_after();
  bool ok = true;
  if (threadIdx.x == 0) ok = mbar_wait_limit(b, 0, err, kWaitSelftestCode, limit);  // no one arrives
  ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
  tc_fence_before();
  __syncwarp();
  tc_fence_after();
  tmem_dealloc(tmem_base, 32);            // the wind-down: TMEM back before the kernel leaves
  if (threadIdx.x == 0) *done = ok ? 1 : 2;
}

}  // namespace
}  // namespace decik

extern "C" int decik_wait_limit_selftest(long long limit_cycles, int* done, void* stream) {
  using namespace decik;
  if (limit_cycles <= 0 || limit_cycles > 4000000000ll)
    return set_error(DECIK_ERR_INVALID, "wait_limit_selftest: limit %lld cycles outside (0, 4e9]", limit_cycles);
  if (done == nullptr) return set_error(DECIK_ERR_INVALID, "wait_limit_selftest: done is NULL");
  int* err = attn::attn_error_word();
  if (err == nullptr) return set_error(DECIK_ERR_CUDA, "wait_limit_selftest: error word unavailable");
  wait_selftest_kernel<<<1, 32, 0, as_stream(stream)>>>(err, limit_cycles, done);
  return check_launch("wait_limit_selftest");
}
