// SwiGLU activation shared by the standalone kernel and the fused fc1 GEMM
// epilogue, so both produce the same bits: silu(g) * u = g / (1 + exp(-g)) * u,
// evaluated in fp32.
#pragma once

#include <cuda_runtime.h>

namespace moe {

__device__ __forceinline__ float swiglu_f32(float g, float u) {
  const float s = g / (1.0f + expf(-g));
  return s * u;
}

}  // namespace moe
