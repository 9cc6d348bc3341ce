// Routing stage of the MoE expert layer on B200:
//   * row-wise top-k (aten::topk contract) and the fused router
//     (score -> top-k -> gate weights -> routing map + dense probs), one warp
//     per token, selection by warp-wide argmax with a lower-index tie-break;
//   * row_id_map construction in three launches: per-chunk expert counts,
//     one-block scan (expert offsets + chunk bases), and an ordered fill that
//     writes both the [T,E] and the [E,T] int64 maps with coalesced stores.
//
// Reference behaviour: kernel_cases/case23_ref_aten_topk.py:47-62 (stable
// descending sort, first k), kernel_cases/case12_moe_row_id_map_pass2.py:43-61
// (cumsum-based map, both layouts returned).
#include <float.h>
#include <math.h>

#include "moe_common.cuh"

namespace moe {
namespace {

constexpr int kTopkMaxK = 16;

// One warp per row. Lane l owns columns l, l+32, ..., l+32*(VPL-1).
// mode 0: plain top-k of the input (values = input values).
// mode 1: router with softmax gates; mode 2: router with raw-logit gates.
template <int VPL, int KMAX>
__global__ void __launch_bounds__(256) topk_router_kernel(
    const float* __restrict__ in, const float* __restrict__ bias, const int32_t* __restrict__ perm,
    int64_t T, int N, int k, int mode, int renorm, float* __restrict__ out_vals,
    int64_t* __restrict__ out_idx, uint8_t* __restrict__ routing_map, float* __restrict__ probs) {
  const int lane = lane_id();
  const int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + warp_id();
  if (row >= T) return;
  const float* rin = in + row * N;

  float v[VPL];
  uint64_t key[VPL];
#pragma unroll
  for (int j = 0; j < VPL; ++j) {
    const int c = lane + 32 * j;
    float x = -INFINITY;
    key[j] = 0;
    if (c < N) {
      const int src = perm ? __ldg(perm + c) : c;  // placement slot c reads column perm[c]
      x = __ldg(rin + src);
      if (bias != nullptr) x += __ldg(bias + src);
      key[j] = rank_key(x, c);
    }
    v[j] = x;
  }

  auto local_best = [&]() {
    uint64_t b = 0;
#pragma unroll
    for (int j = 0; j < VPL; ++j) b = key[j] > b ? key[j] : b;
    return b;
  };

  uint64_t taken = 0;  // bit j: column lane+32j selected
  uint64_t sel[KMAX];
  uint64_t best = local_best();
#pragma unroll
  for (int r = 0; r < KMAX; ++r) {
    if (r < k) {
      uint64_t w = best;
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) {
        const uint64_t o = __shfl_xor_sync(0xffffffffu, w, off);
        w = o > w ? o : w;
      }
      sel[r] = w;
      if (w == best && w != 0) {  // this lane owns the winner (keys are unique)
#pragma unroll
        for (int j = 0; j < VPL; ++j)
          if (key[j] == w) {
            key[j] = 0;
            taken |= 1ull << j;
          }
        best = local_best();
      }
    }
  }

  // Softmax statistics: row max and the normaliser.
  float m = 0.f, denom = 1.f, gsum = 1.f;
  if (mode == 1) {
    m = -INFINITY;
#pragma unroll
    for (int j = 0; j < VPL; ++j) m = fmaxf(m, v[j]);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
    float sacc = 0.f;
    if (renorm) {
#pragma unroll
      for (int r = 0; r < KMAX; ++r)
        if (r < k) sacc += expf(key_value(sel[r]) - m);
    } else {
#pragma unroll
      for (int j = 0; j < VPL; ++j)
        if (lane + 32 * j < N) sacc += expf(v[j] - m);
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) sacc += __shfl_xor_sync(0xffffffffu, sacc, off);
    }
    denom = sacc;
  } else if (mode == 2 && renorm) {
    float sacc = 0.f;
#pragma unroll
    for (int r = 0; r < KMAX; ++r)
      if (r < k) sacc += key_value(sel[r]);
    gsum = sacc;
  }
  auto gate_of = [&](float x) {
    if (mode == 1) return expf(x - m) / denom;
    if (mode == 2 && renorm) return x / gsum;
    return x;
  };

  if (lane < k) {
    uint64_t mine = 0;
#pragma unroll
    for (int r = 0; r < KMAX; ++r)
      if (r == lane) mine = sel[r];
    const int c = key_column(mine);
    const int src = perm ? __ldg(perm + c) : c;
    float x = __ldg(rin + src);  // exact input value (keeps -0.0 and NaN payloads)
    if (bias != nullptr) x += __ldg(bias + src);
    if (out_vals) out_vals[row * k + lane] = gate_of(x);
    if (out_idx) out_idx[row * k + lane] = c;
  }
  if (routing_map != nullptr || probs != nullptr) {
#pragma unroll
    for (int j = 0; j < VPL; ++j) {
      const int c = lane + 32 * j;
      if (c < N) {
        const bool t = (taken >> j) & 1ull;
        if (routing_map) routing_map[row * N + c] = t ? 1 : 0;
        if (probs) probs[row * N + c] = t ? gate_of(v[j]) : 0.f;
      }
    }
  }
}

template <int VPL>
void launch_topk(const float* in, const float* bias, const int32_t* perm, int64_t T, int N, int k,
                 int mode, int renorm, float* vals, int64_t* idx, uint8_t* rmap, float* probs,
                 cudaStream_t s) {
  const int rows_per_block = 8;
  const int64_t blocks = (T + rows_per_block - 1) / rows_per_block;
  if (k <= 8)
    topk_router_kernel<VPL, 8><<<static_cast<unsigned>(blocks), 32 * rows_per_block, 0, s>>>(
        in, bias, perm, T, N, k, mode, renorm, vals, idx, rmap, probs);
  else
    topk_router_kernel<VPL, kTopkMaxK><<<static_cast<unsigned>(blocks), 32 * rows_per_block, 0,
                                         s>>>(in, bias, perm, T, N, k, mode, renorm, vals, idx,
                                              rmap, probs);
}

int run_topk(const float* in, const float* bias, const int32_t* perm, int64_t T, int64_t N, int k,
             int mode, int renorm, float* vals, int64_t* idx, uint8_t* rmap, float* probs,
             cudaStream_t s) {
  MOE_REQUIRE(T >= 0 && N >= 1, "topk: bad shape T=%lld N=%lld", (long long)T, (long long)N);
  MOE_REQUIRE(k >= 1 && k <= N, "topk: k=%d out of range for N=%lld", k, (long long)N);
  if (k > kTopkMaxK || N > 2048) {
    set_last_error("topk: k=%d N=%lld exceeds this build (k <= %d, N <= 2048)", k, (long long)N,
                   kTopkMaxK);
    return MOE_ERR_UNSUPPORTED;
  }
  MOE_REQUIRE(in != nullptr, "topk: null input");
  if (T == 0) return MOE_OK;
  MOE_REQUIRE(T <= (int64_t)0x7fffffff * 8, "topk: T too large");
  const int vpl = static_cast<int>((N + 31) / 32);
  if (vpl <= 1)
    launch_topk<1>(in, bias, perm, T, (int)N, k, mode, renorm, vals, idx, rmap, probs, s);
  else if (vpl <= 2)
    launch_topk<2>(in, bias, perm, T, (int)N, k, mode, renorm, vals, idx, rmap, probs, s);
  else if (vpl <= 4)
    launch_topk<4>(in, bias, perm, T, (int)N, k, mode, renorm, vals, idx, rmap, probs, s);
  else if (vpl <= 8)
    launch_topk<8>(in, bias, perm, T, (int)N, k, mode, renorm, vals, idx, rmap, probs, s);
  else if (vpl <= 16)
    launch_topk<16>(in, bias, perm, T, (int)N, k, mode, renorm, vals, idx, rmap, probs, s);
  else if (vpl <= 32)
    launch_topk<32>(in, bias, perm, T, (int)N, k, mode, renorm, vals, idx, rmap, probs, s);
  else
    launch_topk<64>(in, bias, perm, T, (int)N, k, mode, renorm, vals, idx, rmap, probs, s);
  MOE_CUDA_CHECK_LAUNCH("topk launch");
  return MOE_OK;
}

// ---------------------------------------------------------------------------
// row_id_map
// ---------------------------------------------------------------------------
constexpr int kRimChunk = 64;     // tokens per chunk
constexpr int kRimThreads = 256;  // experts per block (grid.y covers the rest)

// counts[e * C + c] = number of tokens of chunk c routed to expert e.
__global__ void __launch_bounds__(kRimThreads) rim_count_kernel(const uint8_t* __restrict__ rmap,
                                                               int64_t T, int E, int C,
                                                               int32_t* __restrict__ counts) {
  const int c = blockIdx.x;
  const int e = blockIdx.y * kRimThreads + threadIdx.x;
  if (e >= E) return;
  const int64_t t0 = static_cast<int64_t>(c) * kRimChunk;
  const int nt = static_cast<int>((T - t0) < kRimChunk ? (T - t0) : kRimChunk);
  int cnt = 0;
  const uint8_t* p = rmap + t0 * E + e;
#pragma unroll 8
  for (int i = 0; i < nt; ++i) cnt += (__ldg(p + static_cast<int64_t>(i) * E) != 0);
  counts[static_cast<int64_t>(e) * C + c] = cnt;
}

// One block of 1024 threads. Turns counts[e][c] into absolute chunk bases:
// base[e][c] = offset[e] + sum_{c' < c} counts[e][c'], with
// offset[e] = sum_{e' < e} roundup(total[e'], align).
__global__ void __launch_bounds__(1024) rim_scan_kernel(int32_t* __restrict__ counts, int E, int C,
                                                        int64_t align,
                                                        int64_t* __restrict__ offsets_ws,
                                                        int32_t* __restrict__ expert_counts,
                                                        int64_t* __restrict__ num_out) {
  __shared__ int64_t warp_sums[32];
  __shared__ int64_t carry_s;
  const int lane = lane_id(), wid = warp_id();
  // 1) per-expert exclusive scan over chunks, one warp per expert.
  for (int e = wid; e < E; e += 32) {
    int32_t* col = counts + static_cast<int64_t>(e) * C;
    int carry = 0;
    for (int c0 = 0; c0 < C; c0 += 32) {
      const int c = c0 + lane;
      const int x = (c < C) ? col[c] : 0;
      int incl = x;
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, incl, off);
        if (lane >= off) incl += y;
      }
      if (c < C) col[c] = carry + incl - x;
      carry += __shfl_sync(0xffffffffu, incl, 31);
    }
    if (lane == 0) offsets_ws[e] = carry;  // total for now
  }
  __syncthreads();
  // 2) exclusive scan of padded totals over experts (chunks of 1024).
  if (threadIdx.x == 0) carry_s = 0;
  __syncthreads();
  for (int e0 = 0; e0 < E; e0 += 1024) {
    const int e = e0 + threadIdx.x;
    int64_t tot = 0, padded = 0;
    if (e < E) {
      tot = offsets_ws[e];
      padded = (align > 1) ? ((tot + align - 1) / align) * align : tot;
    }
    int64_t incl = padded;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int64_t y = __shfl_up_sync(0xffffffffu, incl, off);
      if (lane >= off) incl += y;
    }
    if (lane == 31) warp_sums[wid] = incl;
    __syncthreads();
    if (wid == 0) {
      int64_t ws = warp_sums[lane];
      int64_t wincl = ws;
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const int64_t y = __shfl_up_sync(0xffffffffu, wincl, off);
        if (lane >= off) wincl += y;
      }
      warp_sums[lane] = wincl - ws;  // exclusive prefix of warp sums
    }
    __syncthreads();
    const int64_t base = carry_s;
    if (e < E) {
      offsets_ws[e] = base + warp_sums[wid] + incl - padded;
      if (expert_counts) expert_counts[e] = static_cast<int32_t>(tot);
    }
    __syncthreads();
    if (threadIdx.x == 1023) carry_s = base + warp_sums[wid] + incl;
    __syncthreads();
  }
  if (threadIdx.x == 0 && num_out) *num_out = carry_s;
  __syncthreads();
  // 3) absolute chunk bases.
  for (int64_t i = threadIdx.x; i < static_cast<int64_t>(E) * C; i += 1024) {
    const int e = static_cast<int>(i / C);
    counts[i] += static_cast<int32_t>(offsets_ws[e]);
  }
}

// Parallel variant for E <= kRimFastMaxE: one warp per expert turns
// counts[e][c] into chunk bases local to the expert (exclusive scan over
// chunks) and writes the expert's total; the expert offsets are then formed
// inside every fill block from the totals (rim_fill_offsets_kernel).
constexpr int kRimFastMaxE = 2048;

__global__ void __launch_bounds__(1024) rim_scan_experts_kernel(int32_t* __restrict__ counts, int E,
                                                                int C,
                                                                int64_t* __restrict__ totals) {
  const int lane = lane_id();
  const int e = blockIdx.x * 32 + warp_id();
  if (e >= E) return;
  int32_t* col = counts + static_cast<int64_t>(e) * C;
  int carry = 0;
  for (int c0 = 0; c0 < C; c0 += 32) {
    const int c = c0 + lane;
    const int x = (c < C) ? col[c] : 0;
    int incl = x;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, incl, off);
      if (lane >= off) incl += y;
    }
    if (c < C) col[c] = carry + incl - x;
    carry += __shfl_sync(0xffffffffu, incl, 31);
  }
  if (lane == 0) totals[e] = carry;
}

// Exclusive scan of the padded expert totals into s_off[0..E) by one block of
// kRimThreads threads; block (0,0) also publishes expert_counts and num_out.
MOE_DEVICE void rim_block_offsets(const int64_t* __restrict__ totals, int E, int64_t align,
                                  int32_t* s_off, int64_t* s_warp, int32_t* __restrict__ expert_counts,
                                  int64_t* __restrict__ num_out, bool publish) {
  const int lane = lane_id(), wid = warp_id();
  constexpr int kWarps = kRimThreads / 32;
  int64_t carry = 0;
  for (int e0 = 0; e0 < E; e0 += kRimThreads) {
    const int e = e0 + threadIdx.x;
    int64_t tot = 0, padded = 0;
    if (e < E) {
      tot = totals[e];
      padded = (align > 1) ? ((tot + align - 1) / align) * align : tot;
      if (publish && expert_counts) expert_counts[e] = static_cast<int32_t>(tot);
    }
    int64_t incl = padded;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int64_t y = __shfl_up_sync(0xffffffffu, incl, off);
      if (lane >= off) incl += y;
    }
    if (lane == 31) s_warp[wid] = incl;
    __syncthreads();
    int64_t before = 0, all = 0;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) {
      const int64_t v = s_warp[w];
      before += (w < wid) ? v : 0;
      all += v;
    }
    if (e < E) s_off[e] = static_cast<int32_t>(carry + before + incl - padded);
    carry += all;
    __syncthreads();
  }
  if (publish && threadIdx.x == 0 && num_out) *num_out = carry;
}

// Ordered fill (see rim_fill_kernel) with the expert offsets computed in-block.
__global__ void __launch_bounds__(kRimThreads) rim_fill_offsets_kernel(
    const uint8_t* __restrict__ rmap, int64_t T, int E, int C, const int32_t* __restrict__ bases,
    const int64_t* __restrict__ totals, int64_t align, int64_t* __restrict__ row_et,
    int64_t* __restrict__ row_te, int32_t* __restrict__ expert_counts,
    int64_t* __restrict__ num_out) {
  __shared__ int32_t tile[kRimThreads][33];
  __shared__ int32_t s_off[kRimFastMaxE];
  __shared__ int64_t s_warp[kRimThreads / 32];
  rim_block_offsets(totals, E, align, s_off, s_warp, expert_counts, num_out,
                    blockIdx.x == 0 && blockIdx.y == 0);
  const int c = blockIdx.x;
  const int e0 = blockIdx.y * kRimThreads;
  const int e = e0 + threadIdx.x;
  const bool active = e < E;
  int running = active ? s_off[e] + bases[static_cast<int64_t>(e) * C + c] : 0;
  const int64_t tc0 = static_cast<int64_t>(c) * kRimChunk;
  if (row_et == nullptr && row_te == nullptr) return;
  for (int sub = 0; sub < kRimChunk; sub += 32) {
    const int64_t t0 = tc0 + sub;
    if (t0 >= T) break;
    const int nt = static_cast<int>((T - t0) < 32 ? (T - t0) : 32);
    uint8_t m[32];
#pragma unroll
    for (int i = 0; i < 32; ++i)
      m[i] = (active && i < nt) ? __ldg(rmap + (t0 + i) * E + e) : 0;
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      if (i < nt) {
        int32_t val = -1;
        if (m[i]) val = running++;
        if (active && row_te) row_te[(t0 + i) * E + e] = val;
        tile[threadIdx.x][i] = val;
      }
    }
    __syncthreads();
    if (row_et) {
      const int lane = lane_id(), wid = warp_id();
      for (int el = wid; el < kRimThreads; el += kRimThreads / 32) {
        const int ee = e0 + el;
        if (ee < E && lane < nt) row_et[static_cast<int64_t>(ee) * T + t0 + lane] = tile[el][lane];
      }
    }
    __syncthreads();
  }
}

// Launch sequence shared by both row_id_map entry points: `counts` holds
// E*C int32 chunk counts, `offs` E int64 (totals / offsets).
int rim_launch(const uint8_t* routing_map, int64_t T, int64_t E, int64_t align,
               int64_t* row_id_map_et, int64_t* row_id_map_te, int32_t* expert_counts,
               int64_t* num_out, int32_t* counts, int64_t* offs, cudaStream_t s, const char* who);

// Ordered fill. Block (c, eb): tokens of chunk c, experts eb*256 + tid.
// Each thread walks its expert column in token order (a running counter),
// writing row_te row-wise (coalesced over experts) and staging a 32-token
// tile in shared memory for the transposed [E,T] store (coalesced over tokens).
__global__ void __launch_bounds__(kRimThreads) rim_fill_kernel(
    const uint8_t* __restrict__ rmap, int64_t T, int E, int C, const int32_t* __restrict__ bases,
    int64_t* __restrict__ row_et, int64_t* __restrict__ row_te) {
  __shared__ int32_t tile[kRimThreads][33];
  const int c = blockIdx.x;
  const int e0 = blockIdx.y * kRimThreads;
  const int e = e0 + threadIdx.x;
  const bool active = e < E;
  int running = active ? bases[static_cast<int64_t>(e) * C + c] : 0;
  const int64_t tc0 = static_cast<int64_t>(c) * kRimChunk;
  for (int sub = 0; sub < kRimChunk; sub += 32) {
    const int64_t t0 = tc0 + sub;
    if (t0 >= T) break;
    const int nt = static_cast<int>((T - t0) < 32 ? (T - t0) : 32);
    uint8_t m[32];
#pragma unroll
    for (int i = 0; i < 32; ++i)
      m[i] = (active && i < nt) ? __ldg(rmap + (t0 + i) * E + e) : 0;
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      if (i < nt) {
        int32_t val = -1;
        if (m[i]) val = running++;
        if (active && row_te) row_te[(t0 + i) * E + e] = val;
        tile[threadIdx.x][i] = val;
      }
    }
    __syncthreads();
    if (row_et) {
      const int lane = lane_id(), wid = warp_id();
      for (int el = wid; el < kRimThreads; el += kRimThreads / 32) {
        const int ee = e0 + el;
        if (ee < E && lane < nt) row_et[static_cast<int64_t>(ee) * T + t0 + lane] = tile[el][lane];
      }
    }
    __syncthreads();
  }
}

int rim_launch(const uint8_t* routing_map, int64_t T, int64_t E, int64_t align,
               int64_t* row_id_map_et, int64_t* row_id_map_te, int32_t* expert_counts,
               int64_t* num_out, int32_t* counts, int64_t* offs, cudaStream_t s, const char* who) {
  const int C = static_cast<int>((T + kRimChunk - 1) / kRimChunk);
  const int eblocks = static_cast<int>((E + kRimThreads - 1) / kRimThreads);
  if (C > 0) {
    rim_count_kernel<<<dim3(C, eblocks), kRimThreads, 0, s>>>(routing_map, T, (int)E, C, counts);
    MOE_CUDA_CHECK_LAUNCH(who);
  }
  const bool want_maps = row_id_map_et != nullptr || row_id_map_te != nullptr;
  if (C > 0 && E <= kRimFastMaxE) {
    rim_scan_experts_kernel<<<static_cast<unsigned>((E + 31) / 32), 1024, 0, s>>>(counts, (int)E,
                                                                                  C, offs);
    MOE_CUDA_CHECK_LAUNCH(who);
    rim_fill_offsets_kernel<<<dim3(want_maps ? C : 1, want_maps ? eblocks : 1), kRimThreads, 0,
                              s>>>(routing_map, T, (int)E, C, counts, offs, align,
                                   want_maps ? row_id_map_et : nullptr,
                                   want_maps ? row_id_map_te : nullptr, expert_counts, num_out);
    MOE_CUDA_CHECK_LAUNCH(who);
    return MOE_OK;
  }
  rim_scan_kernel<<<1, 1024, 0, s>>>(counts, (int)E, C, align, offs, expert_counts, num_out);
  MOE_CUDA_CHECK_LAUNCH(who);
  if (C > 0 && want_maps) {
    rim_fill_kernel<<<dim3(C, eblocks), kRimThreads, 0, s>>>(routing_map, T, (int)E, C, counts,
                                                             row_id_map_et, row_id_map_te);
    MOE_CUDA_CHECK_LAUNCH(who);
  }
  return MOE_OK;
}

}  // namespace
}  // namespace moe

using namespace moe;

extern "C" int moe_topk_f32(const float* input, float* values, int64_t* indices, int64_t M,
                            int64_t N, int32_t k, moe_stream_t stream) {
  MOE_REQUIRE(values != nullptr && indices != nullptr, "topk: null output");
  return run_topk(input, nullptr, nullptr, M, N, k, 0, 0, values, indices, nullptr, nullptr,
                  reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int moe_router_topk(const float* logits, const float* bias, int64_t T, int64_t E,
                               int32_t k, int32_t score_mode, int32_t renorm, float* topk_vals,
                               int64_t* topk_idx, uint8_t* routing_map, float* probs,
                               moe_stream_t stream) {
  MOE_REQUIRE(score_mode == 0 || score_mode == 1, "router: score_mode must be 0 or 1");
  const int mode = score_mode == 1 ? 1 : 2;
  return run_topk(logits, bias, nullptr, T, E, k, mode, renorm, topk_vals, topk_idx, routing_map,
                  probs, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int moe_router_topk_placed(const float* logits, const float* bias,
                                      const int32_t* placement, int64_t T, int64_t E, int32_t k,
                                      int32_t score_mode, int32_t renorm, float* topk_vals,
                                      int64_t* topk_idx, uint8_t* routing_map, float* probs,
                                      moe_stream_t stream) {
  MOE_REQUIRE(score_mode == 0 || score_mode == 1, "router_placed: score_mode must be 0 or 1");
  MOE_REQUIRE(placement != nullptr || T == 0, "router_placed: null placement");
  const int mode = score_mode == 1 ? 1 : 2;
  return run_topk(logits, bias, placement, T, E, k, mode, renorm, topk_vals, topk_idx,
                  routing_map, probs, reinterpret_cast<cudaStream_t>(stream));
}

static size_t rim_ws_bytes(int64_t T, int64_t E) {
  const int64_t C = (T + kRimChunk - 1) / kRimChunk;
  size_t counts = static_cast<size_t>(E) * static_cast<size_t>(C) * 4;
  counts = (counts + 255) & ~static_cast<size_t>(255);
  size_t offs = static_cast<size_t>(E) * 8;
  offs = (offs + 255) & ~static_cast<size_t>(255);
  return counts + offs;
}

extern "C" int moe_row_id_map_workspace_size(int64_t T, int64_t E, size_t* bytes) {
  MOE_REQUIRE(bytes != nullptr, "row_id_map_workspace_size: null output");
  MOE_REQUIRE(T >= 0 && E >= 1, "row_id_map: bad shape T=%lld E=%lld", (long long)T,
              (long long)E);
  *bytes = rim_ws_bytes(T, E);
  return MOE_OK;
}

extern "C" int moe_row_id_map(const uint8_t* routing_map, int64_t T, int64_t E, int64_t align,
                              int64_t* row_id_map_et, int64_t* row_id_map_te,
                              int32_t* expert_counts, int64_t* num_out, void* workspace,
                              size_t workspace_bytes, moe_stream_t stream) {
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  MOE_REQUIRE(T >= 0 && E >= 1 && E <= 65536, "row_id_map: bad shape T=%lld E=%lld",
              (long long)T, (long long)E);
  MOE_REQUIRE(align >= 1 && align <= 4096, "row_id_map: align=%lld out of [1,4096]",
              (long long)align);
  MOE_REQUIRE(T * E < (int64_t)0x7fffffff, "row_id_map: T*E=%lld must stay below 2^31",
              (long long)(T * E));
  MOE_REQUIRE(T == 0 || routing_map != nullptr, "row_id_map: null routing_map");
  MOE_REQUIRE(workspace != nullptr && workspace_bytes >= rim_ws_bytes(T, E),
              "row_id_map: workspace too small (%zu < %zu)", workspace_bytes, rim_ws_bytes(T, E));
  MOE_REQUIRE((reinterpret_cast<uintptr_t>(workspace) & 255) == 0,
              "row_id_map: workspace must be 256-byte aligned");
  const int C = static_cast<int>((T + kRimChunk - 1) / kRimChunk);
  int32_t* counts = static_cast<int32_t*>(workspace);
  size_t counts_bytes = (static_cast<size_t>(E) * C * 4 + 255) & ~static_cast<size_t>(255);
  int64_t* offs = reinterpret_cast<int64_t*>(static_cast<char*>(workspace) + counts_bytes);
  return rim_launch(routing_map, T, E, align, row_id_map_et, row_id_map_te, expert_counts, num_out,
                    counts, offs, s, "row_id_map launch");
}

// ---------------------------------------------------------------------------
// row_id_map without a caller-provided workspace.
//
// Some callers cannot allocate device memory at the point where they build
// the routing maps: for example a serving runtime that hands each request a
// fixed, pre-partitioned slice of HBM and forbids further cudaMalloc, or a
// latency-critical loop where cudaMalloc's implicit synchronisation is not
// acceptable. For them the scratch lives in a file-scope device array of
// kRimStaticScratchBytes (1 MiB): it is part of this library's device image,
// so every GPU that loads the library holds it until the process exits.
//
// Host code cannot pass the array's name to a kernel (on the host it is only
// a stand-in symbol, not a device address), so the first call on each device
// looks up the real address with cudaGetSymbolAddress, with that device
// current, and caches it for the life of the process. That first call should
// therefore happen before any stream capture, and the library must not be
// used across a cudaDeviceReset of the device (the cached address would be
// that of the destroyed context).
//
// A call needs roundup(E * ceil(T/64) * 4, 256) bytes of per-chunk counts plus
// roundup(E * 8, 256) bytes of expert offsets; at E = 256 that fits for
// T <= 65408 tokens.
//
// All calls on a device share the one array and it keeps whatever the last
// call left there. Nothing in it needs to start at zero: the count kernel
// writes every count slot and the scan writes every offset before anything
// reads them. Calls whose kernels overlap on the GPU (different streams, or
// different host threads without ordering) race on the array; serialise them.
// ---------------------------------------------------------------------------
#include <mutex>
#include <vector>

namespace {
constexpr size_t kRimStaticScratchBytes = size_t(1) << 20;
static __device__ __align__(256) unsigned char g_rim_static_scratch[kRimStaticScratchBytes];

std::mutex g_rim_static_mu;
std::vector<void*> g_rim_static_addr;  // per device, filled on first use

int rim_static_scratch_address(void** out) {
  int dev = 0;
  MOE_CUDA_CALL(cudaGetDevice(&dev), "row_id_map_static_scratch: cudaGetDevice");
  std::lock_guard<std::mutex> lock(g_rim_static_mu);
  if (static_cast<size_t>(dev) >= g_rim_static_addr.size())
    g_rim_static_addr.resize(static_cast<size_t>(dev) + 1, nullptr);
  if (g_rim_static_addr[dev] == nullptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_rim_static_scratch);
    if (e != cudaSuccess || p == nullptr) {
      moe::set_last_error("row_id_map_static_scratch: cudaGetSymbolAddress failed on device %d: %s",
                          dev, cudaGetErrorString(e));
      return MOE_ERR_CUDA;
    }
    g_rim_static_addr[dev] = p;
  }
  *out = g_rim_static_addr[dev];
  return MOE_OK;
}
}  // namespace

extern "C" int moe_row_id_map_static_scratch(const uint8_t* routing_map, int64_t T, int64_t E,
                                             int64_t align, int64_t* row_id_map_et,
                                             int64_t* row_id_map_te, int32_t* expert_counts,
                                             int64_t* num_out, moe_stream_t stream) {
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  MOE_REQUIRE(T >= 0 && E >= 1 && E <= 65536, "row_id_map_static_scratch: bad shape T=%lld E=%lld",
              (long long)T, (long long)E);
  MOE_REQUIRE(align >= 1 && align <= 4096,
              "row_id_map_static_scratch: align=%lld out of [1,4096]", (long long)align);
  MOE_REQUIRE(T * E < (int64_t)0x7fffffff,
              "row_id_map_static_scratch: T*E=%lld must stay below 2^31", (long long)(T * E));
  const size_t need = rim_ws_bytes(T, E);
  MOE_REQUIRE(need <= kRimStaticScratchBytes,
              "row_id_map_static_scratch: T=%lld E=%lld needs %zu bytes of scratch, more than the "
              "%zu-byte static array; use moe_row_id_map with a workspace",
              (long long)T, (long long)E, need, kRimStaticScratchBytes);
  MOE_REQUIRE(T == 0 || routing_map != nullptr, "row_id_map_static_scratch: null routing_map");
  void* scratch = nullptr;
  int st = rim_static_scratch_address(&scratch);
  if (st) return st;
  const int C = static_cast<int>((T + kRimChunk - 1) / kRimChunk);
  int32_t* counts = static_cast<int32_t*>(scratch);
  const size_t counts_bytes = (static_cast<size_t>(E) * C * 4 + 255) & ~static_cast<size_t>(255);
  int64_t* offs = reinterpret_cast<int64_t*>(static_cast<char*>(scratch) + counts_bytes);
  return rim_launch(routing_map, T, E, align, row_id_map_et, row_id_map_te, expert_counts, num_out,
                    counts, offs, s, "row_id_map_static_scratch launch");
}
