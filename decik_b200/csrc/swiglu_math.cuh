// The sigmoid of SwiGLU (solution/swiglu.py:15-37: silu(g) = g * sigmoid(g)), shared by the
// separate SwiGLU kernels (swiglu.cu) and the MLP GEMM epilogues (proj_sm100.cu) so that the fused
// and the separate paths give the same bits. sigmoid(x) = 1 / (1 + 2^(-x log2 e)) on the hardware's
// approximate exp2 and reciprocal (ex2.approx.ftz, rcp.approx.ftz): a few fp32 ulp, far below the
// 16-bit rounding of every output. x below about -88 gives 2^... = inf and a reciprocal of +0; x
// above about 88 gives 0 and 1. expf with an IEEE division instead took 5 K of the grad_hidden
// epilogue's 6.5 K cycles per 32-column chunk, and that epilogue then bounded its GEMM.
#pragma once

namespace decik {
namespace swiglu {

__device__ __forceinline__ float sigmoid(float x) {
  float e, r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e) : "f"(x * -1.4426950408889634f));
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(1.0f + e));
  return r;
}

}  // namespace swiglu
}  // namespace decik
