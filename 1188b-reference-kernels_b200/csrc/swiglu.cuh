// SwiGLU activation shared by the standalone kernel and the fused fc1 GEMM
// epilogues, so both produce the same bits: silu(g) * u = g / (1 + exp(-g)) * u,
// evaluated in fp32, two (gate, up) pairs at a time.
//
// exp(-g) comes from the identity exp(x) = 2^(x log2 e): log2 e is split into
// a float and its remainder (Cody & Waite), so t = -g log2 e is carried as
// hi + lo with the product's rounding error recovered by an FMA; 2^hi is the
// hardware base-2 exponential (ex2.approx) and lo is applied to first order,
// 2^t ~= 2^hi (1 + lo ln 2), so 1 + exp(-g) = 1 + e (1 + lo ln 2) is one FMA.
// Its reciprocal is rcp.approx refined by one Newton step. The error is a few
// fp32 ulp, far below the bf16 rounding of the result.
//
// The arithmetic runs on the sm_100 two-lane fp32 instructions (fma and mul
// on a register pair, each lane rounded exactly as the scalar operation); the
// exp2 and the reciprocal stay one per lane. Every rounding step is explicit,
// so the compiler contracts nothing and the bits do not depend on the call
// site. Against expf and an IEEE division this is about a quarter of the
// instructions: the fused epilogue of the wide GEMM tiles runs between two
// halves of the tensor-core work and is issue-bound on it.
// -g is clamped to [-100, 87] so that every intermediate stays finite (a NaN
// g still gives NaN; below g = -87 the result is a tiny value instead of -0).
// -x is formed as x * -1, which is exact.
#pragma once

#include <cuda_runtime.h>

namespace moe {

__device__ __forceinline__ float2 swiglu2_f32(float2 g, float2 u) {
  constexpr float kLog2eHi = 1.44269502162933349609375f;  // float nearest log2(e)
  constexpr float kLog2eLo = 1.925963033500011e-8f;       // log2(e) - kLog2eHi
  constexpr float kLn2 = 0.693147180559945309f;
  const float2 one = make_float2(1.0f, 1.0f);
  const float2 ng = make_float2(fminf(fmaxf(-g.x, -100.0f), 87.0f),
                                fminf(fmaxf(-g.y, -100.0f), 87.0f));
  const float2 hi = __fmul2_rn(ng, make_float2(kLog2eHi, kLog2eHi));
  const float2 lo = __ffma2_rn(ng, make_float2(kLog2eLo, kLog2eLo),
                               __ffma2_rn(ng, make_float2(kLog2eHi, kLog2eHi),
                                          __fmul2_rn(ng, make_float2(-kLog2eHi, -kLog2eHi))));
  float2 e;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e.x) : "f"(hi.x));
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e.y) : "f"(hi.y));
  const float2 d = __ffma2_rn(e, __ffma2_rn(lo, make_float2(kLn2, kLn2), one), one);
  float2 r;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r.x) : "f"(d.x));
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r.y) : "f"(d.y));
  r = __ffma2_rn(r, __ffma2_rn(__fmul2_rn(d, make_float2(-1.0f, -1.0f)), r, one), r);
  return __fmul2_rn(__fmul2_rn(g, r), u);
}

}  // namespace moe
