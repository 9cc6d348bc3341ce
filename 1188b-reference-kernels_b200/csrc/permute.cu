// Token permute / unpermute (dispatch / combine) for the MoE expert layer.
//
// Both directions are row copies of H bf16 values driven by a row-id map:
//   permute   out[row[t,e]] = x[t]                (+ permuted probs)
//   unpermute out[t] = bf16(sum_e w(t,e) * pin[row[e,t]])
// They are HBM-bound. One 128-thread CTA owns one token: the map entries of
// the token are read once, compacted in ascending expert order through a
// warp ballot, and the H-element row moves as 16-byte vectors held in
// registers (VPT vectors per thread), so every global access is a coalesced
// 16-byte access and each source row is read exactly once.
//
// Reference behaviour: kernel_cases/case17_moe_permute_with_mask_map.py:58-71,
// kernel_cases/case22_ref_moe_permute_mask_kernel_true.py:47-69,
// kernel_cases/case15_moe_unpermute_mask_fwd.py:58-64,
// kernel_cases/case24_ref_moe_unpermute_mask_kernel_false.py:45-68.
#include <stdlib.h>

#include <algorithm>
#include <mutex>

#include "moe_common.cuh"
#include "rowcopy.cuh"
#include "swiglu.cuh"

namespace moe {
namespace {

using namespace rowcopy;

// 32-byte row vector moved by one 256-bit global load / store (sm_100), for
// the MOE_PERMUTE_V32=1 path: half the store instructions per row.
struct __align__(32) Vec32 {
  uint4 lo, hi;
};
template <typename V>
MOE_DEVICE V ld_row(const V* p) { return __ldg(p); }
template <>
MOE_DEVICE Vec32 ld_row<Vec32>(const Vec32* p) {
  Vec32 v;
  asm volatile("ld.global.nc.v8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(v.lo.x), "=r"(v.lo.y), "=r"(v.lo.z), "=r"(v.lo.w), "=r"(v.hi.x),
                 "=r"(v.hi.y), "=r"(v.hi.z), "=r"(v.hi.w)
               : "l"(p));
  return v;
}
template <typename V>
MOE_DEVICE void st_row(V* p, const V& v) { *p = v; }
template <>
MOE_DEVICE void st_row<Vec32>(Vec32* p, const Vec32& v) {
  asm volatile("st.global.v8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"l"(p), "r"(v.lo.x),
               "r"(v.lo.y), "r"(v.lo.z), "r"(v.lo.w), "r"(v.hi.x), "r"(v.hi.y), "r"(v.hi.z),
               "r"(v.hi.w)
               : "memory");
}

template <int VPT, bool kTrans, typename IdxT, typename V>
__global__ void __launch_bounds__(kRowThreads) permute_kernel(
    const V* __restrict__ x, const IdxT* __restrict__ map, const float* __restrict__ probs,
    V* __restrict__ out, float* __restrict__ pp, int64_t T, int E, int nvec,
    int64_t num_out) {
  __shared__ int64_t s_dst[kRowThreads];
  __shared__ float s_p[kRowThreads];
  __shared__ int s_wcnt[kRowWarps];
  const int64_t t = blockIdx.x;
  const int tid = threadIdx.x;
  const V* src = x + t * nvec;

  V r[VPT > 0 ? VPT : 1];
  if constexpr (VPT > 0) {
#pragma unroll
    for (int v = 0; v < VPT; ++v) {
      const int i = tid + v * kRowThreads;
      if (i < nvec) r[v] = ld_row(src + i);
    }
  }

  for (int e0 = 0; e0 < E; e0 += kRowThreads) {
    const int e = e0 + tid;
    int64_t d = -1;
    if (e < E) d = load_map<IdxT, kTrans>(map, T, E, t, e);
    const bool valid = d >= 0 && d < num_out;
    int pos;
    const int total = compact_window(valid, s_wcnt, pos);
    if (valid) {
      s_dst[pos] = d;
      if (probs) s_p[pos] = __ldg(probs + t * E + e);
    }
    __syncthreads();
    for (int j = 0; j < total; ++j) {
      const int64_t dd = s_dst[j];
      V* o = out + dd * nvec;
      if constexpr (VPT > 0) {
#pragma unroll
        for (int v = 0; v < VPT; ++v) {
          const int i = tid + v * kRowThreads;
          if (i < nvec) st_row(o + i, r[v]);
        }
      } else {
        for (int i = tid; i < nvec; i += kRowThreads) st_row(o + i, ld_row(src + i));
      }
      if (pp != nullptr && tid == 0) pp[dd] = s_p[j];
    }
    __syncthreads();
  }
}

// Permute through the bulk-copy (TMA) engine. A one-warp CTA walks the tokens
// blockIdx.x, blockIdx.x + gridDim.x, ...: each token row reaches shared
// memory with one bulk load, issued kBulkBufs - 1 tokens ahead into a ring of
// kBulkBufs row buffers, and each destination row leaves with one bulk store,
// issued by the lane that read that map entry. The SM executes a handful of
// instructions per row instead of one 16-byte load or store per thread, and
// every byte still crosses HBM once. A buffer is reloaded only after the
// stores that read it (the previous token's) have finished reading shared
// memory. The row wait is bounded (2 s): on a timeout the kernel records 1 in
// g_rowcopy_err (read by moe_permute_check), waits a bounded time for its
// loads in flight and returns.
constexpr int kBulkBufs = 3;
constexpr uint32_t kBulkMaxRowBytes = 32768;
__device__ int32_t g_rowcopy_err;

template <bool kTrans, typename IdxT>
__global__ void __launch_bounds__(32) permute_bulk_kernel(
    const char* __restrict__ x, const IdxT* __restrict__ map, const float* __restrict__ probs,
    char* __restrict__ out, float* __restrict__ pp, int64_t T, int E, uint32_t row_bytes,
    int64_t num_out) {
  extern __shared__ __align__(128) uint8_t smem[];
  const uint32_t stride = (row_bytes + 127u) & ~127u;
  const uint32_t buf0 = smem_u32(smem);
  const uint32_t bar0 = buf0 + kBulkBufs * stride;
  const int lane = lane_id();
  if (static_cast<int64_t>(blockIdx.x) >= T) return;  // CTA-uniform
  const int64_t n_tok = (T - 1 - static_cast<int64_t>(blockIdx.x)) / gridDim.x + 1;
  if (lane == 0) {
    for (int b = 0; b < kBulkBufs; ++b) mbar_init(bar0 + 8u * b, 1);
    fence_mbar_init();
  }
  __syncwarp();
  auto token = [&](int64_t i) { return static_cast<int64_t>(blockIdx.x) + i * gridDim.x; };
  auto load = [&](int64_t i) {
    const uint32_t b = static_cast<uint32_t>(i % kBulkBufs);
    mbar_arrive_expect_tx(bar0 + 8u * b, row_bytes);
    bulk_load(buf0 + b * stride, x + token(i) * row_bytes, row_bytes, bar0 + 8u * b);
  };
  int64_t issued = n_tok < kBulkBufs - 1 ? n_tok : kBulkBufs - 1;  // loads issued: tokens [0, issued)
  if (lane == 0)
    for (int64_t i = 0; i < issued; ++i) load(i);
  int64_t i = 0;
  for (; i < n_tok; ++i) {
    if (issued < n_tok) {
      // Token i-1's buffer takes token i + kBulkBufs - 1 once its stores read it.
      bulk_wait_read<0>();
      __syncwarp();
      if (lane == 0) load(issued);
      ++issued;
    }
    const uint32_t b = static_cast<uint32_t>(i % kBulkBufs);
    const uint32_t parity = static_cast<uint32_t>((i / kBulkBufs) & 1);
    bool ok = mbar_try_wait(bar0 + 8u * b, parity);
    if (!ok) {
      const unsigned long long t0 = globaltimer_ns();
      while (!(ok = mbar_try_wait(bar0 + 8u * b, parity)))
        if (globaltimer_ns() - t0 > kWaitTimeoutNs) break;
    }
    if (!__all_sync(0xffffffffu, ok)) break;
    const int64_t t = token(i);
    const uint32_t src = buf0 + b * stride;
    for (int e0 = 0; e0 < E; e0 += 32) {
      const int e = e0 + lane;
      int64_t d = -1;
      if (e < E) d = load_map<IdxT, kTrans>(map, T, E, t, e);
      if (d >= 0 && d < num_out) {
        bulk_store(out + d * static_cast<int64_t>(row_bytes), src, row_bytes);
        if (pp != nullptr) pp[d] = __ldg(probs + t * E + e);
      }
    }
    bulk_commit();  // one (possibly empty) group per token and lane
  }
  bulk_wait_all();
  if (i < n_tok && lane == 0) {  // a row never arrived: report, drain, return
    atomicExch(&g_rowcopy_err, 1);
    for (int64_t j = i; j < issued; ++j) {
      const uint32_t b = static_cast<uint32_t>(j % kBulkBufs);
      const unsigned long long t0 = globaltimer_ns();
      while (!mbar_try_wait(bar0 + 8u * b, static_cast<uint32_t>((j / kBulkBufs) & 1)))
        if (globaltimer_ns() - t0 > kWaitTimeoutNs) break;
    }
  }
}

// Permute driven by the router's expert list: experts[t, j] (j < k) names the
// experts token t goes to, so thread j reads its destination row straight
// from map[t, experts[t, j]] -- k scattered 8-byte loads per token instead of
// the whole E-entry map row and its ballot compaction. The copy is the same
// as permute_kernel's (a destination row is the same whatever order the
// experts come in). Entries naming an expert outside [0, E) or a row outside
// [0, num_out) are skipped.
constexpr int kListMaxK = 32;

template <int VPT, typename V>
__global__ void __launch_bounds__(kRowThreads) permute_list_kernel(
    const V* __restrict__ x, const int64_t* __restrict__ map_te,
    const int64_t* __restrict__ experts, int k, const float* __restrict__ probs,
    V* __restrict__ out, float* __restrict__ pp, int64_t T, int E, int nvec, int64_t num_out) {
  __shared__ int64_t s_dst[kListMaxK];
  const int64_t t = blockIdx.x;
  const int tid = threadIdx.x;
  const V* src = x + t * nvec;
  V r[VPT];
#pragma unroll
  for (int v = 0; v < VPT; ++v) {
    const int i = tid + v * kRowThreads;
    if (i < nvec) r[v] = __ldg(src + i);
  }
  if (tid < k) {
    const int64_t e = __ldg(experts + t * k + tid);
    int64_t d = -1;
    if (e >= 0 && e < E) d = __ldg(map_te + t * E + e);
    if (d >= num_out) d = -1;
    s_dst[tid] = d;
    if (d >= 0 && pp != nullptr) pp[d] = __ldg(probs + t * E + e);
  }
  __syncthreads();
  for (int j = 0; j < k; ++j) {
    const int64_t dd = s_dst[j];
    if (dd < 0) continue;  // block-uniform
    V* o = out + dd * nvec;
#pragma unroll
    for (int v = 0; v < VPT; ++v) {
      const int i = tid + v * kRowThreads;
      if (i < nvec) o[i] = r[v];
    }
  }
}

// probs_mode: -1 unweighted, 0 probs[t*E+e], 1 probs[src row].
// gp_out (optional, [T,E] fp32): the permute backward's prob gradient,
// gp_out[t,e] = pgrad[src row] for a routed (t,e), else 0.
template <int VPT, typename IdxT, typename V>
__global__ void __launch_bounds__(kRowThreads) unpermute_kernel(
    const V* __restrict__ pin, const IdxT* __restrict__ map, const float* __restrict__ probs,
    int probs_mode, V* __restrict__ out, float* __restrict__ acc_out, int64_t T, int E,
    int nvec, int64_t num_rows, const float* __restrict__ pgrad, float* __restrict__ gp_out) {
  constexpr int kE = VecTraits<V>::kElems;
  __shared__ int64_t s_src[kRowThreads];
  __shared__ float s_w[kRowThreads];
  __shared__ int s_wcnt[kRowWarps];
  const int64_t t = blockIdx.x;
  const int tid = threadIdx.x;
  const bool weighted = probs_mode >= 0;

  float acc[VPT][kE];
#pragma unroll
  for (int v = 0; v < VPT; ++v)
#pragma unroll
    for (int i = 0; i < kE; ++i) acc[v][i] = 0.f;

  for (int e0 = 0; e0 < E; e0 += kRowThreads) {
    const int e = e0 + tid;
    int64_t s = -1;
    if (e < E) s = load_map<IdxT, true>(map, T, E, t, e);
    const bool valid = s >= 0 && s < num_rows;
    if (gp_out != nullptr && e < E) gp_out[t * E + e] = valid ? __ldg(pgrad + s) : 0.f;
    int pos;
    const int total = compact_window(valid, s_wcnt, pos);
    if (valid) {
      s_src[pos] = s;
      float w = 1.f;
      if (probs_mode == 0) w = __ldg(probs + t * E + e);
      else if (probs_mode == 1) w = __ldg(probs + s);
      s_w[pos] = w;
    }
    __syncthreads();
    int j = 0;
    // Two source rows in flight per step; accumulation order stays ascending.
    for (; j + 1 < total; j += 2) {
      const V* a = pin + s_src[j] * nvec;
      const V* b = pin + s_src[j + 1] * nvec;
      const float wa = s_w[j], wb = s_w[j + 1];
      V qa[VPT], qb[VPT];
#pragma unroll
      for (int v = 0; v < VPT; ++v) {
        const int i = tid + v * kRowThreads;
        if (i < nvec) {
          qa[v] = a[i];
          qb[v] = b[i];
        }
      }
#pragma unroll
      for (int v = 0; v < VPT; ++v) {
        const int i = tid + v * kRowThreads;
        if (i < nvec) {
          accum_vec<V>(acc[v], qa[v], wa, weighted);
          accum_vec<V>(acc[v], qb[v], wb, weighted);
        }
      }
    }
    if (j < total) {
      const V* a = pin + s_src[j] * nvec;
      const float wa = s_w[j];
#pragma unroll
      for (int v = 0; v < VPT; ++v) {
        const int i = tid + v * kRowThreads;
        if (i < nvec) accum_vec<V>(acc[v], a[i], wa, weighted);
      }
    }
    __syncthreads();
  }

#pragma unroll
  for (int v = 0; v < VPT; ++v) {
    const int i = tid + v * kRowThreads;
    if (i < nvec) {
      out[t * nvec + i] = VecTraits<V>::pack(acc[v]);
      if (acc_out) {
        float* ao = acc_out + (t * nvec + i) * kE;
#pragma unroll
        for (int q = 0; q < kE; ++q) ao[q] = acc[v][q];
      }
    }
  }
}

// Combine with the whole source list staged first (up to kCombineMaxE map
// entries per token), then one pass over the row's column vectors that keeps
// up to 8 source rows in flight per thread. Same arithmetic and the same
// ascending-expert order as unpermute_kernel, so the results are identical;
// it only hides memory latency better (few registers, many loads in flight).
// kTrans: map is [E,T] (reference layout); otherwise token-major [T,E].
constexpr int kCombineMaxE = 1024;

template <bool kTrans, typename IdxT, typename V>
__global__ void __launch_bounds__(kRowThreads) combine_kernel(
    const V* __restrict__ pin, const IdxT* __restrict__ map, const float* __restrict__ probs,
    int probs_mode, V* __restrict__ out, float* __restrict__ acc_out, int64_t T, int E,
    int nvec, int64_t num_rows, const float* __restrict__ pgrad, float* __restrict__ gp_out) {
  constexpr int kE = VecTraits<V>::kElems;
  __shared__ int64_t s_src[kCombineMaxE];
  __shared__ float s_w[kCombineMaxE];
  __shared__ int s_wcnt[kRowWarps];
  __shared__ int s_n;
  const int64_t t = blockIdx.x;
  const int tid = threadIdx.x;
  const bool weighted = probs_mode >= 0;
  if (tid == 0) s_n = 0;
  for (int e0 = 0; e0 < E; e0 += kRowThreads) {
    const int e = e0 + tid;
    int64_t s = -1;
    if (e < E) s = load_map<IdxT, kTrans>(map, T, E, t, e);
    const bool valid = s >= 0 && s < num_rows;
    if (gp_out != nullptr && e < E) gp_out[t * E + e] = valid ? __ldg(pgrad + s) : 0.f;
    int pos;
    const int total = compact_window(valid, s_wcnt, pos);  // contains a __syncthreads
    const int base = s_n;
    if (valid) {
      s_src[base + pos] = s;
      float w = 1.f;
      if (probs_mode == 0) w = __ldg(probs + t * E + e);
      else if (probs_mode == 1) w = __ldg(probs + s);
      s_w[base + pos] = w;
    }
    __syncthreads();
    if (tid == 0) s_n = base + total;
  }
  __syncthreads();
  const int n = s_n;
  for (int i = tid; i < nvec; i += kRowThreads) {
    float acc[kE];
#pragma unroll
    for (int q = 0; q < kE; ++q) acc[q] = 0.f;
    int j = 0;
    for (; j + 8 <= n; j += 8) {
      V v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) v[u] = pin[s_src[j + u] * nvec + i];
#pragma unroll
      for (int u = 0; u < 8; ++u) accum_vec<V>(acc, v[u], s_w[j + u], weighted);
    }
    if (j + 4 <= n) {
      V v[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) v[u] = pin[s_src[j + u] * nvec + i];
#pragma unroll
      for (int u = 0; u < 4; ++u) accum_vec<V>(acc, v[u], s_w[j + u], weighted);
      j += 4;
    }
    for (; j < n; ++j) accum_vec<V>(acc, pin[s_src[j] * nvec + i], s_w[j], weighted);
    out[t * nvec + i] = VecTraits<V>::pack(acc);
    if (acc_out) {
      float* ao = acc_out + (t * nvec + i) * kE;
#pragma unroll
      for (int q = 0; q < kE; ++q) ao[q] = acc[q];
    }
  }
}

__global__ void swiglu_kernel(const uint4* __restrict__ y, uint4* __restrict__ h, int64_t M,
                              int fvec) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= M * fvec) return;
  const int64_t m = i / fvec;
  const int c = static_cast<int>(i - m * fvec);
  const uint4 g = __ldg(y + m * 2 * fvec + c);
  const uint4 u = __ldg(y + m * 2 * fvec + fvec + c);
  const uint32_t gg[4] = {g.x, g.y, g.z, g.w}, uu[4] = {u.x, u.y, u.z, u.w};
  uint32_t o[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const float2 hh = swiglu2_f32(make_float2(bf16_lo(gg[k]), bf16_hi(gg[k])),
                                  make_float2(bf16_lo(uu[k]), bf16_hi(uu[k])));
    o[k] = pack_bf16x2(hh.x, hh.y);
  }
  h[i] = make_uint4(o[0], o[1], o[2], o[3]);
}

template <typename V>
constexpr int row_elems() {
  if constexpr (sizeof(V) == 32) return 16;
  else return VecTraits<V>::kElems;
}

template <bool kTrans, typename IdxT, typename V>
int launch_permute_v(const void* x, const IdxT* map, const float* probs, void* out, float* pp,
                     int64_t T, int64_t H, int64_t E, int64_t num_out, cudaStream_t s) {
  const int nvec = static_cast<int>(H / row_elems<V>());
  const int vpt = (nvec + kRowThreads - 1) / kRowThreads;
  const V* xv = static_cast<const V*>(x);
  V* ov = static_cast<V*>(out);
  const unsigned grid = static_cast<unsigned>(T);
#define MOE_PERMUTE_CASE(VP)                                                                 \
  permute_kernel<VP, kTrans, IdxT, V><<<grid, kRowThreads, 0, s>>>(xv, map, probs, ov, pp, T, \
                                                                   (int)E, nvec, num_out)
  if (vpt <= 1) MOE_PERMUTE_CASE(1);
  else if (vpt <= 2) MOE_PERMUTE_CASE(2);
  else if (vpt <= 4) MOE_PERMUTE_CASE(4);
  else if (vpt <= 8) MOE_PERMUTE_CASE(8);
  else MOE_PERMUTE_CASE(0);
#undef MOE_PERMUTE_CASE
  MOE_CUDA_CHECK_LAUNCH("permute launch");
  return MOE_OK;
}

template <typename IdxT, typename V>
int launch_unpermute_v(const void* pin, const IdxT* map, const float* probs, int probs_mode,
                       void* out, float* acc_out, int64_t T, int64_t H, int64_t E,
                       int64_t num_rows, cudaStream_t s, const float* pgrad, float* gp_out) {
  const int nvec = static_cast<int>(H / VecTraits<V>::kElems);
  const int vpt = (nvec + kRowThreads - 1) / kRowThreads;
  const V* pv = static_cast<const V*>(pin);
  V* ov = static_cast<V*>(out);
  const unsigned grid = static_cast<unsigned>(T);
#define MOE_UNPERMUTE_CASE(VP)                                                           \
  unpermute_kernel<VP, IdxT, V><<<grid, kRowThreads, 0, s>>>(pv, map, probs, probs_mode, ov, \
                                                             acc_out, T, (int)E, nvec, num_rows, \
                                                             pgrad, gp_out)
  if (vpt <= 1) MOE_UNPERMUTE_CASE(1);
  else if (vpt <= 2) MOE_UNPERMUTE_CASE(2);
  else if (vpt <= 4) MOE_UNPERMUTE_CASE(4);
  else if (vpt <= 8) MOE_UNPERMUTE_CASE(8);
  else if (vpt <= 16) MOE_UNPERMUTE_CASE(16);
  else {
    set_last_error("unpermute: H=%lld exceeds this build (H <= %d for this row alignment)",
                   (long long)H, 16 * kRowThreads * VecTraits<V>::kElems);
    return MOE_ERR_UNSUPPORTED;
  }
#undef MOE_UNPERMUTE_CASE
  MOE_CUDA_CHECK_LAUNCH("unpermute launch");
  return MOE_OK;
}

// MOE_PERMUTE_BULK=1 routes eligible rows through permute_bulk_kernel. Off by
// default: at the layer's 16384 x 7168 permute it measured 4.5 TB/s against
// 5.2 TB/s for the register-staged kernel on the same box (the copy engine's
// per-SM bulk-store rate, not HBM, bounds it).
bool permute_bulk_enabled() {
  static const int v = [] {
    const char* e = getenv("MOE_PERMUTE_BULK");
    return (e != nullptr && e[0] == '1') ? 1 : 0;
  }();
  return v == 1;
}

// MOE_PERMUTE_V32=1 moves rows as 32-byte vectors where they allow it. Off by
// default: at the layer's permute it measured 5.27 TB/s against 5.45 TB/s
// with 16-byte vectors on the same box (fewer store instructions did not
// shorten it, so it is not issue-bound there).
bool permute_v32_enabled() {
  static const int v = [] {
    const char* e = getenv("MOE_PERMUTE_V32");
    return (e != nullptr && e[0] == '1') ? 1 : 0;
  }();
  return v == 1;
}

template <bool kTrans, typename IdxT>
int launch_permute_bulk(const void* x, const IdxT* map, const float* probs, void* out, float* pp,
                        int64_t T, int64_t H, int64_t E, int64_t num_out, cudaStream_t s) {
  const uint32_t row_bytes = static_cast<uint32_t>(H * 2);
  const uint32_t stride = (row_bytes + 127u) & ~127u;
  const size_t smem = kBulkBufs * stride + 8 * kBulkBufs;
  int dev = 0;
  MOE_CUDA_CALL(cudaGetDevice(&dev), "cudaGetDevice");
  static std::mutex mu;
  static bool attr_done[64] = {};
  {
    std::lock_guard<std::mutex> lock(mu);
    if (dev < 64 && !attr_done[dev]) {
      MOE_CUDA_CALL(cudaFuncSetAttribute(permute_bulk_kernel<kTrans, IdxT>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(kBulkBufs * kBulkMaxRowBytes + 64)),
                    "cudaFuncSetAttribute(permute_bulk)");
      attr_done[dev] = true;
    }
  }
  // One-warp CTAs, as many per SM as shared memory allows (at most 16).
  const int per_sm = static_cast<int>(std::min<size_t>(16, (227u * 1024u) / (smem + 1024)));
  const unsigned grid =
      static_cast<unsigned>(std::min<int64_t>(T, static_cast<int64_t>(num_sms(dev)) * per_sm));
  permute_bulk_kernel<kTrans, IdxT><<<grid, 32, smem, s>>>(
      static_cast<const char*>(x), map, probs, static_cast<char*>(out), pp, T, static_cast<int>(E),
      row_bytes, num_out);
  MOE_CUDA_CHECK_LAUNCH("permute_bulk launch");
  return MOE_OK;
}

template <bool kTrans, typename IdxT>
int launch_permute(const void* x, const IdxT* map, const float* probs, void* out, float* pp,
                   int64_t T, int64_t H, int64_t E, int64_t num_out, cudaStream_t s) {
  // Bulk copies need 16-byte rows and addresses; rows up to 32 KB (H <= 16384).
  if (permute_bulk_enabled() && vec_bytes(x, out, H) == 16 &&
      static_cast<uint64_t>(H) * 2 <= kBulkMaxRowBytes)
    return launch_permute_bulk<kTrans, IdxT>(x, map, probs, out, pp, T, H, E, num_out, s);
  // 32-byte vectors (MOE_PERMUTE_V32=1) when rows and both pointers allow them.
  const bool v32 = permute_v32_enabled() && H % 16 == 0 &&
                   ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(out)) & 31) == 0;
  if (v32) return launch_permute_v<kTrans, IdxT, Vec32>(x, map, probs, out, pp, T, H, E, num_out, s);
  switch (vec_bytes(x, out, H)) {
    case 16: return launch_permute_v<kTrans, IdxT, uint4>(x, map, probs, out, pp, T, H, E, num_out, s);
    case 4: return launch_permute_v<kTrans, IdxT, uint32_t>(x, map, probs, out, pp, T, H, E, num_out, s);
    default: return launch_permute_v<kTrans, IdxT, uint16_t>(x, map, probs, out, pp, T, H, E, num_out, s);
  }
}

template <bool kTrans, typename IdxT, typename V>
int launch_combine_v(const void* pin, const IdxT* map, const float* probs, int probs_mode,
                     void* out, float* acc_out, int64_t T, int64_t H, int64_t E, int64_t num_rows,
                     cudaStream_t s, const float* pgrad, float* gp_out) {
  const int nvec = static_cast<int>(H / VecTraits<V>::kElems);
  combine_kernel<kTrans, IdxT, V><<<static_cast<unsigned>(T), kRowThreads, 0, s>>>(
      static_cast<const V*>(pin), map, probs, probs_mode, static_cast<V*>(out), acc_out, T,
      (int)E, nvec, num_rows, pgrad, gp_out);
  MOE_CUDA_CHECK_LAUNCH("combine launch");
  return MOE_OK;
}

template <bool kTrans, typename IdxT>
int launch_combine(const void* pin, const IdxT* map, const float* probs, int probs_mode,
                   void* out, float* acc_out, int64_t T, int64_t H, int64_t E, int64_t num_rows,
                   cudaStream_t s, const float* pgrad = nullptr, float* gp_out = nullptr) {
  switch (vec_bytes(pin, out, H)) {
    case 16:
      return launch_combine_v<kTrans, IdxT, uint4>(pin, map, probs, probs_mode, out, acc_out, T,
                                                   H, E, num_rows, s, pgrad, gp_out);
    case 4:
      return launch_combine_v<kTrans, IdxT, uint32_t>(pin, map, probs, probs_mode, out, acc_out,
                                                      T, H, E, num_rows, s, pgrad, gp_out);
    default:
      return launch_combine_v<kTrans, IdxT, uint16_t>(pin, map, probs, probs_mode, out, acc_out,
                                                      T, H, E, num_rows, s, pgrad, gp_out);
  }
}

template <typename IdxT>
int launch_unpermute(const void* pin, const IdxT* map, const float* probs, int probs_mode,
                     void* out, float* acc_out, int64_t T, int64_t H, int64_t E, int64_t num_rows,
                     cudaStream_t s, const float* pgrad = nullptr, float* gp_out = nullptr) {
  if (E <= kCombineMaxE)
    return launch_combine<true, IdxT>(pin, map, probs, probs_mode, out, acc_out, T, H, E,
                                      num_rows, s, pgrad, gp_out);
  switch (vec_bytes(pin, out, H)) {
    case 16:
      return launch_unpermute_v<IdxT, uint4>(pin, map, probs, probs_mode, out, acc_out, T, H, E,
                                             num_rows, s, pgrad, gp_out);
    case 4:
      return launch_unpermute_v<IdxT, uint32_t>(pin, map, probs, probs_mode, out, acc_out, T, H,
                                                E, num_rows, s, pgrad, gp_out);
    default:
      return launch_unpermute_v<IdxT, uint16_t>(pin, map, probs, probs_mode, out, acc_out, T, H,
                                                E, num_rows, s, pgrad, gp_out);
  }
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

int check_row_args(const char* op, const void* a, const void* b, int64_t T, int64_t H, int64_t E) {
  MOE_REQUIRE(T >= 0 && H >= 0 && E >= 1, "%s: bad shape T=%lld H=%lld E=%lld", op,
              (long long)T, (long long)H, (long long)E);
  MOE_REQUIRE(T <= 0x7fffffff && H <= 0x7fffffff && E <= 0x7fffffff, "%s: size too large", op);
  MOE_REQUIRE(((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b)) & 1) == 0,
              "%s: row pointers must be 2-byte aligned", op);
  return MOE_OK;
}

}  // namespace
}  // namespace moe

using namespace moe;

extern "C" int moe_permute_topk(const void* x, const int64_t* row_id_map_te,
                                const int64_t* topk_experts, int32_t k, const float* probs,
                                void* out, float* permuted_probs, int64_t T, int64_t H, int64_t E,
                                int64_t num_out, moe_stream_t stream) {
  int st = check_row_args("permute_topk", x, out, T, H, E);
  if (st) return st;
  MOE_REQUIRE(k >= 1 && k <= kListMaxK, "permute_topk: k=%d out of [1,%d]", k, kListMaxK);
  MOE_REQUIRE(num_out >= 0, "permute_topk: num_out=%lld < 0", (long long)num_out);
  if (T == 0 || H == 0 || num_out == 0) return MOE_OK;
  MOE_REQUIRE((probs == nullptr) == (permuted_probs == nullptr),
              "permute_topk: probs and permuted_probs must both be given or both be null");
  MOE_REQUIRE(x && out && row_id_map_te && topk_experts, "permute_topk: null pointer");
  MOE_REQUIRE(vec_bytes(x, out, H) == 16,
              "permute_topk: rows must be 16-byte vectors (H %% 8 == 0, aligned pointers)");
  const int nvec = static_cast<int>(H / 8);
  const int vpt = (nvec + kRowThreads - 1) / kRowThreads;
  MOE_REQUIRE(vpt <= 8, "permute_topk: H=%lld above 8192", (long long)H);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const unsigned grid = static_cast<unsigned>(T);
  const uint4* xv = static_cast<const uint4*>(x);
  uint4* ov = static_cast<uint4*>(out);
  const int e = static_cast<int>(E);
#define MOE_PERMUTE_LIST_CASE(VP)                                                           \
  permute_list_kernel<VP, uint4><<<grid, kRowThreads, 0, s>>>(xv, row_id_map_te, topk_experts, \
                                                               k, probs, ov, permuted_probs, T, e, \
                                                               nvec, num_out)
  if (vpt <= 1) MOE_PERMUTE_LIST_CASE(1);
  else if (vpt <= 2) MOE_PERMUTE_LIST_CASE(2);
  else if (vpt <= 4) MOE_PERMUTE_LIST_CASE(4);
  else if (vpt <= 7) MOE_PERMUTE_LIST_CASE(7);
  else MOE_PERMUTE_LIST_CASE(8);
#undef MOE_PERMUTE_LIST_CASE
  MOE_CUDA_CHECK_LAUNCH("permute_topk launch");
  return MOE_OK;
}

extern "C" int moe_permute_mask_map(const void* x, const int64_t* row_id_map_te, const float* probs,
                                    void* out, float* permuted_probs, int64_t T, int64_t H,
                                    int64_t E, int64_t num_out, moe_stream_t stream) {
  int st = check_row_args("permute", x, out, T, H, E);
  if (st) return st;
  MOE_REQUIRE(num_out >= 0, "permute: num_out=%lld < 0", (long long)num_out);
  if (T == 0 || H == 0 || num_out == 0) return MOE_OK;
  MOE_REQUIRE((probs == nullptr) == (permuted_probs == nullptr),
              "permute: probs and permuted_probs must both be given or both be null");
  MOE_REQUIRE(x && out && row_id_map_te, "permute: null pointer");
  return launch_permute<false, int64_t>(x, row_id_map_te, probs, out, permuted_probs, T, H, E,
                                        num_out, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int moe_permute_check(moe_stream_t stream, int32_t* device_error) {
  MOE_REQUIRE(device_error != nullptr, "permute_check: null output");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  int32_t v = 0;
  MOE_CUDA_CALL(cudaMemcpyFromSymbolAsync(&v, g_rowcopy_err, sizeof(v), 0,
                                          cudaMemcpyDeviceToHost, s),
                "permute_check copy");
  MOE_CUDA_CALL(cudaStreamSynchronize(s), "permute_check sync");
  *device_error = v;
  if (v != 0) {
    const int32_t zero = 0;
    MOE_CUDA_CALL(cudaMemcpyToSymbolAsync(g_rowcopy_err, &zero, sizeof(zero), 0,
                                          cudaMemcpyHostToDevice, s),
                  "permute_check clear");
    MOE_CUDA_CALL(cudaStreamSynchronize(s), "permute_check sync");
  }
  return v == 0 ? MOE_OK : MOE_ERR_DEVICE;
}

extern "C" int moe_permute_mask_map_trans(const void* x, const void* row_id_map_et,
                                          int32_t idx_bits, const float* probs, void* out,
                                          float* permuted_probs, int64_t T, int64_t H, int64_t E,
                                          int64_t num_out, moe_stream_t stream) {
  int st = check_row_args("permute_trans", x, out, T, H, E);
  if (st) return st;
  MOE_REQUIRE(idx_bits == 32 || idx_bits == 64, "permute_trans: idx_bits must be 32 or 64");
  MOE_REQUIRE(num_out >= 0, "permute_trans: num_out=%lld < 0", (long long)num_out);
  if (T == 0 || H == 0 || num_out == 0) return MOE_OK;
  MOE_REQUIRE((probs == nullptr) == (permuted_probs == nullptr),
              "permute_trans: probs and permuted_probs must both be given or both be null");
  MOE_REQUIRE(x && out && row_id_map_et, "permute_trans: null pointer");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (idx_bits == 64)
    return launch_permute<true, int64_t>(x, static_cast<const int64_t*>(row_id_map_et), probs, out,
                                         permuted_probs, T, H, E, num_out, s);
  return launch_permute<true, int32_t>(x, static_cast<const int32_t*>(row_id_map_et), probs, out,
                                       permuted_probs, T, H, E, num_out, s);
}

extern "C" int moe_unpermute_mask(const void* pin, const void* row_id_map_et, int32_t idx_bits,
                                  const float* probs, int32_t probs_mode, void* out,
                                  float* acc_out, int64_t T, int64_t H, int64_t E,
                                  int64_t num_rows, moe_stream_t stream) {
  int st = check_row_args("unpermute", pin, out, T, H, E);
  if (st) return st;
  MOE_REQUIRE(idx_bits == 32 || idx_bits == 64, "unpermute: idx_bits must be 32 or 64");
  MOE_REQUIRE(probs == nullptr || probs_mode == 0 || probs_mode == 1,
              "unpermute: probs_mode must be 0 ([T,E]) or 1 (permuted)");
  MOE_REQUIRE(num_rows >= 0, "unpermute: num_rows=%lld < 0", (long long)num_rows);
  MOE_REQUIRE(acc_out == nullptr || (reinterpret_cast<uintptr_t>(acc_out) & 3) == 0,
              "unpermute: acc_out must be 4-byte aligned");
  if (T == 0 || H == 0) return MOE_OK;
  MOE_REQUIRE(out && row_id_map_et && (pin || num_rows == 0), "unpermute: null pointer");
  const int mode = probs ? probs_mode : -1;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (idx_bits == 64)
    return launch_unpermute<int64_t>(pin, static_cast<const int64_t*>(row_id_map_et), probs, mode,
                                     out, acc_out, T, H, E, num_rows, s);
  return launch_unpermute<int32_t>(pin, static_cast<const int32_t*>(row_id_map_et), probs, mode,
                                   out, acc_out, T, H, E, num_rows, s);
}

extern "C" int moe_permute_backward(const void* grad_permuted, const void* row_id_map_et,
                                    int32_t idx_bits, const float* permuted_probs_grad,
                                    void* grad_x, float* acc_out, float* grad_probs, int64_t T,
                                    int64_t H, int64_t E, int64_t num_rows, moe_stream_t stream) {
  int st = check_row_args("permute_backward", grad_permuted, grad_x, T, H, E);
  if (st) return st;
  MOE_REQUIRE(idx_bits == 32 || idx_bits == 64, "permute_backward: idx_bits must be 32 or 64");
  MOE_REQUIRE(num_rows >= 0, "permute_backward: num_rows=%lld < 0", (long long)num_rows);
  MOE_REQUIRE((grad_probs == nullptr) == (permuted_probs_grad == nullptr),
              "permute_backward: grad_probs and permuted_probs_grad go together");
  MOE_REQUIRE(((reinterpret_cast<uintptr_t>(acc_out) | reinterpret_cast<uintptr_t>(grad_probs)) &
               3) == 0,
              "permute_backward: acc_out and grad_probs must be 4-byte aligned");
  if (T == 0) return MOE_OK;
  MOE_REQUIRE(row_id_map_et && (grad_permuted || num_rows == 0) && (grad_x || H == 0),
              "permute_backward: null pointer");
  if (H == 0 && grad_probs == nullptr) return MOE_OK;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (idx_bits == 64)
    return launch_unpermute<int64_t>(grad_permuted, static_cast<const int64_t*>(row_id_map_et),
                                     nullptr, -1, grad_x, acc_out, T, H, E, num_rows, s,
                                     permuted_probs_grad, grad_probs);
  return launch_unpermute<int32_t>(grad_permuted, static_cast<const int32_t*>(row_id_map_et),
                                   nullptr, -1, grad_x, acc_out, T, H, E, num_rows, s,
                                   permuted_probs_grad, grad_probs);
}

extern "C" int moe_swiglu(const void* y, void* h, int64_t M, int64_t F, moe_stream_t stream) {
  MOE_REQUIRE(M >= 0 && F >= 0 && F % 8 == 0, "swiglu: F=%lld must be a multiple of 8",
              (long long)F);
  if (M == 0 || F == 0) return MOE_OK;
  MOE_REQUIRE(y && h && aligned16(y) && aligned16(h), "swiglu: null or misaligned pointer");
  const int fvec = static_cast<int>(F / 8);
  const int64_t n = M * fvec;
  const int threads = 256;
  swiglu_kernel<<<static_cast<unsigned>((n + threads - 1) / threads), threads, 0,
                  reinterpret_cast<cudaStream_t>(stream)>>>(static_cast<const uint4*>(y),
                                                            static_cast<uint4*>(h), M, fvec);
  MOE_CUDA_CHECK_LAUNCH("swiglu launch");
  return MOE_OK;
}

extern "C" int moe_unpermute_mask_token_major(const void* pin, const int64_t* row_id_map_te,
                                              const float* probs, int32_t probs_mode, void* out,
                                              float* acc_out, int64_t T, int64_t H, int64_t E,
                                              int64_t num_rows, moe_stream_t stream) {
  int st = check_row_args("unpermute_token_major", pin, out, T, H, E);
  if (st) return st;
  MOE_REQUIRE(E <= kCombineMaxE, "unpermute_token_major: E=%lld above %d", (long long)E,
              kCombineMaxE);
  MOE_REQUIRE(probs == nullptr || probs_mode == 0 || probs_mode == 1,
              "unpermute_token_major: probs_mode must be 0 ([T,E]) or 1 (permuted)");
  MOE_REQUIRE(num_rows >= 0, "unpermute_token_major: num_rows=%lld < 0", (long long)num_rows);
  MOE_REQUIRE(acc_out == nullptr || (reinterpret_cast<uintptr_t>(acc_out) & 3) == 0,
              "unpermute_token_major: acc_out must be 4-byte aligned");
  if (T == 0 || H == 0) return MOE_OK;
  MOE_REQUIRE(out && row_id_map_te && (pin || num_rows == 0),
              "unpermute_token_major: null pointer");
  return launch_combine<false, int64_t>(pin, row_id_map_te, probs, probs ? probs_mode : -1, out,
                                        acc_out, T, H, E, num_rows,
                                        reinterpret_cast<cudaStream_t>(stream));
}
