// Backward of the two elementwise stages of the expert layer, the parts of
// the layer backward that are not GEMMs or the permute backward:
//
//   combine:  out[t] = sum_e probs[t,e] * rows[map[t,e]]   (forward, fp32 sum)
//             grad_rows[map[t,e]] = bf16(probs[t,e] * grad_out[t])
//             grad_probs[t,e]     = <grad_out[t], rows[map[t,e]]>  (fp32), 0 where unrouted
//   SwiGLU:   h = silu(g) * u with y = [g | u]
//             dg = dh * u * silu'(g),  du = dh * silu(g),  silu'(g) = s (1 + g (1 - s))
//
// The weighted combine has no reference kernel (it is the build's restatement
// of the reference's unweighted unpermute with the router gates applied); its
// backward follows from the forward by the chain rule, as torch.autograd
// would form it. Layout as in the forward: one 128-thread CTA per token over
// the token-major [T,E] int64 map, rows moved as 16-byte vectors of bf16.
#include "moe_common.cuh"
#include "rowcopy.cuh"

namespace moe {
namespace {

using rowcopy::compact_window;
using rowcopy::kRowThreads;
using rowcopy::kRowWarps;
using rowcopy::VecTraits;

constexpr int kBwdMaxE = 1024;

template <typename V>
__global__ void __launch_bounds__(kRowThreads) combine_backward_kernel(
    const V* __restrict__ grad_out, const V* __restrict__ rows, const int64_t* __restrict__ map,
    const float* __restrict__ probs, V* __restrict__ grad_rows, float* __restrict__ grad_probs,
    int64_t T, int E, int nvec, int64_t num_rows) {
  constexpr int kE = VecTraits<V>::kElems;
  __shared__ int64_t s_src[kBwdMaxE];
  __shared__ int s_e[kBwdMaxE];
  __shared__ float s_w[kBwdMaxE];
  __shared__ int s_wcnt[kRowWarps];
  __shared__ float s_red[kRowWarps];
  __shared__ int s_n;
  const int64_t t = blockIdx.x;
  const int tid = threadIdx.x;
  if (tid == 0) s_n = 0;
  for (int e0 = 0; e0 < E; e0 += kRowThreads) {
    const int e = e0 + tid;
    int64_t s = -1;
    if (e < E) s = __ldg(map + t * E + e);
    const bool valid = s >= 0 && s < num_rows;
    if (e < E && !valid) grad_probs[t * E + e] = 0.f;
    int pos;
    const int total = compact_window(valid, s_wcnt, pos);  // contains a __syncthreads
    const int base = s_n;
    if (valid) {
      s_src[base + pos] = s;
      s_e[base + pos] = e;
      s_w[base + pos] = __ldg(probs + t * E + e);
    }
    __syncthreads();
    if (tid == 0) s_n = base + total;
  }
  __syncthreads();
  const int n = s_n;
  const V* g_row = grad_out + t * nvec;
  for (int j = 0; j < n; ++j) {
    const int64_t r = s_src[j];
    const float w = s_w[j];
    float part = 0.f;
    for (int i = tid; i < nvec; i += kRowThreads) {
      float g[kE], y[kE], o[kE];
      VecTraits<V>::unpack(__ldg(g_row + i), g);
      VecTraits<V>::unpack(__ldg(rows + r * nvec + i), y);
#pragma unroll
      for (int q = 0; q < kE; ++q) {
        o[q] = __fmul_rn(w, g[q]);
        part = __fmaf_rn(g[q], y[q], part);
      }
      grad_rows[r * nvec + i] = VecTraits<V>::pack(o);
    }
    // fixed-order block reduction: lanes by xor butterfly, then warps 0..3
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) part += __shfl_xor_sync(0xffffffffu, part, off);
    if (lane_id() == 0) s_red[warp_id()] = part;
    __syncthreads();
    if (tid == 0) {
      float d = 0.f;
#pragma unroll
      for (int w2 = 0; w2 < kRowWarps; ++w2) d += s_red[w2];
      grad_probs[t * E + s_e[j]] = d;
    }
    __syncthreads();
  }
}

// dy = [dg | du] from y = [g | u] and dh, 8 bf16 per thread.
__global__ void swiglu_backward_kernel(const uint4* __restrict__ y, const uint4* __restrict__ dh,
                                       uint4* __restrict__ dy, int64_t M, int fvec) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= M * fvec) return;
  const int64_t m = i / fvec;
  const int c = static_cast<int>(i - m * fvec);
  const uint4 gq = __ldg(y + m * 2 * fvec + c);
  const uint4 uq = __ldg(y + m * 2 * fvec + fvec + c);
  const uint4 hq = __ldg(dh + m * fvec + c);
  float g[8], u[8], d[8], og[8], ou[8];
  VecTraits<uint4>::unpack(gq, g);
  VecTraits<uint4>::unpack(uq, u);
  VecTraits<uint4>::unpack(hq, d);
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    const float den = 1.0f + expf(-g[q]);
    const float sig = 1.0f / den;
    const float silu = g[q] / den;  // the forward's silu, same expression
    const float dsilu = sig * (1.0f + g[q] * (1.0f - sig));
    og[q] = d[q] * u[q] * dsilu;
    ou[q] = d[q] * silu;
  }
  dy[m * 2 * fvec + c] = VecTraits<uint4>::pack(og);
  dy[m * 2 * fvec + fvec + c] = VecTraits<uint4>::pack(ou);
}

template <typename V>
int launch_combine_backward(const void* grad_out, const void* rows, const int64_t* map,
                            const float* probs, void* grad_rows, float* grad_probs, int64_t T,
                            int64_t H, int64_t E, int64_t num_rows, cudaStream_t s) {
  const int nvec = static_cast<int>(H / VecTraits<V>::kElems);
  combine_backward_kernel<V><<<static_cast<unsigned>(T), kRowThreads, 0, s>>>(
      static_cast<const V*>(grad_out), static_cast<const V*>(rows), map, probs,
      static_cast<V*>(grad_rows), grad_probs, T, static_cast<int>(E), nvec, num_rows);
  MOE_CUDA_CHECK_LAUNCH("combine_backward launch");
  return MOE_OK;
}

}  // namespace
}  // namespace moe

using namespace moe;

extern "C" int moe_combine_backward(const void* grad_out, const void* rows,
                                    const int64_t* row_id_map_te, const float* probs,
                                    void* grad_rows, float* grad_probs, int64_t T, int64_t H,
                                    int64_t E, int64_t num_rows, moe_stream_t stream) {
  MOE_REQUIRE(T >= 0 && H >= 1 && E >= 1 && num_rows >= 0,
              "combine_backward: bad shape T=%lld H=%lld E=%lld rows=%lld", (long long)T,
              (long long)H, (long long)E, (long long)num_rows);
  MOE_REQUIRE(E <= kBwdMaxE, "combine_backward: E=%lld above %d", (long long)E, kBwdMaxE);
  MOE_REQUIRE(T <= 0x7fffffff && H <= (1 << 20), "combine_backward: T or H too large");
  if (T == 0) return MOE_OK;
  MOE_REQUIRE(grad_out && row_id_map_te && probs && grad_probs, "combine_backward: null pointer");
  MOE_REQUIRE(num_rows == 0 || (rows && grad_rows), "combine_backward: null rows");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const uintptr_t m = reinterpret_cast<uintptr_t>(grad_out) | reinterpret_cast<uintptr_t>(rows) |
                      reinterpret_cast<uintptr_t>(grad_rows);
  if (H % 8 == 0 && (m & 15) == 0)
    return launch_combine_backward<uint4>(grad_out, rows, row_id_map_te, probs, grad_rows,
                                          grad_probs, T, H, E, num_rows, s);
  if (H % 2 == 0 && (m & 3) == 0)
    return launch_combine_backward<uint32_t>(grad_out, rows, row_id_map_te, probs, grad_rows,
                                             grad_probs, T, H, E, num_rows, s);
  MOE_REQUIRE((m & 1) == 0, "combine_backward: rows must be 2-byte aligned");
  return launch_combine_backward<uint16_t>(grad_out, rows, row_id_map_te, probs, grad_rows,
                                           grad_probs, T, H, E, num_rows, s);
}

extern "C" int moe_swiglu_backward(const void* y, const void* dh, void* dy, int64_t M, int64_t F,
                                   moe_stream_t stream) {
  MOE_REQUIRE(M >= 0 && F >= 8 && F % 8 == 0,
              "swiglu_backward: M=%lld F=%lld (F must be a positive multiple of 8)", (long long)M,
              (long long)F);
  if (M == 0) return MOE_OK;
  MOE_REQUIRE(y && dh && dy, "swiglu_backward: null pointer");
  MOE_REQUIRE(((reinterpret_cast<uintptr_t>(y) | reinterpret_cast<uintptr_t>(dh) |
                reinterpret_cast<uintptr_t>(dy)) & 15) == 0,
              "swiglu_backward: y, dh and dy must be 16-byte aligned");
  const int fvec = static_cast<int>(F / 8);
  const int64_t n = M * fvec;
  const int threads = 256;
  swiglu_backward_kernel<<<static_cast<unsigned>((n + threads - 1) / threads), threads, 0,
                           reinterpret_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint4*>(y), static_cast<const uint4*>(dh), static_cast<uint4*>(dy), M,
      fvec);
  MOE_CUDA_CHECK_LAUNCH("swiglu_backward launch");
  return MOE_OK;
}
