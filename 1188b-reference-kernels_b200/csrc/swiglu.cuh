// SwiGLU activation shared by the standalone kernel and the fused fc1 GEMM
// epilogue, so both produce the same bits: silu(g) * u = g / (1 + exp(-g)) * u,
// evaluated in fp32.
//
// exp(-g) comes from the identity exp(x) = 2^(x log2 e): log2 e is split into
// a float and its remainder (Cody & Waite), so t = -g log2 e is carried as
// hi + lo with the product's rounding error recovered by an FMA; 2^hi is the
// hardware base-2 exponential (ex2.approx) and lo is applied to first order,
// 2^t ~= 2^hi (1 + lo ln 2). The reciprocal of 1 + exp(-g) is rcp.approx
// refined by one Newton step. The error is a few fp32 ulp, far below the
// bf16 rounding of the result, at about a third of the instructions of
// expf and an IEEE division: the fused epilogue of the wide GEMM tiles runs
// between two halves of the tensor-core work and is issue-bound on it.
// -g is clamped to [-100, 87] so that every intermediate stays finite (a NaN
// g still gives NaN; below g = -87 the result is a tiny value instead of -0).
#pragma once

#include <cuda_runtime.h>

namespace moe {

__device__ __forceinline__ float swiglu_f32(float g, float u) {
  constexpr float kLog2eHi = 1.44269502162933349609375f;  // float nearest log2(e)
  constexpr float kLog2eLo = 1.925963033500011e-8f;       // log2(e) - kLog2eHi
  constexpr float kLn2 = 0.693147180559945309f;
  const float ng = fminf(fmaxf(-g, -100.0f), 87.0f);
  const float hi = ng * kLog2eHi;
  const float lo = fmaf(ng, kLog2eLo, fmaf(ng, kLog2eHi, -hi));
  float e;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e) : "f"(hi));
  e *= fmaf(lo, kLn2, 1.0f);
  const float d = 1.0f + e;
  float r;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(d));
  r = fmaf(r, fmaf(-d, r, 1.0f), r);
  return (g * r) * u;
}

}  // namespace moe
