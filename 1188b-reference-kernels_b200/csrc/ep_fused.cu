// Expert-parallel dispatch and combine fused with the NVLink exchange.
//
// The permuted rows of this rank that belong to expert e form one contiguous
// block (the permuted layout is expert-major), and that block lands in the
// buffer of its owner d = e / experts_per_rank at a fixed row shift
// expert_delta[e], computed on the host from every rank's per-expert counts.
// With an expert-major receive layout (each local expert's rows from all
// sources one after another) every local expert is one GEMM group. So:
//   dispatch: permute, but write row r of expert e straight into rank d's
//             buffer at row r + expert_delta[e] (stores over NVLink into the
//             peer mapping);
//   combine:  unpermute, but read the source row of (t, e) from rank d's
//             fc2 output at row r + expert_delta[e] (loads over NVLink).
// No local permuted copy and no separate all-to-all. Each access is checked
// against the buffers' row capacity, so a corrupt map cannot reach outside
// them; entries that fail the check are skipped.
//
// The reference names this hop (deep_ep intranode FusedDispatch /
// FusedCombine, kernel_cases/case22_ref_moe_permute_mask_kernel_true.py:3-6,
// case24_ref_moe_unpermute_mask_kernel_false.py:3-6) but does not contain it.
#include <algorithm>

#include "moe_common.cuh"
#include "rowcopy.cuh"

namespace moe {
namespace {

using namespace rowcopy;

constexpr int kMaxRanks = 8;

struct PeerRows {
  long long base[kMaxRanks];  // address of rank d's buffer in this process
  const long long* delta;     // [E] row shift from a local row id into the owner's buffer
  long long cap_rows;         // rows every rank's buffer holds
  int experts_per_rank;
  int ranks;
};

MOE_DEVICE bool peer_row(const PeerRows& pr, int e, int64_t r, long long& base, int64_t& rr) {
  const int d = e / pr.experts_per_rank;
  if (d >= pr.ranks) return false;
  rr = r + __ldg(pr.delta + e);
  base = pr.base[d];
  return rr >= 0 && rr < pr.cap_rows;
}

template <int VPT, typename V>
__global__ void __launch_bounds__(kRowThreads) ep_dispatch_kernel(
    const V* __restrict__ x, const int64_t* __restrict__ map_te, const PeerRows pr, int64_t T,
    int E, int nvec, int64_t num_rows) {
  __shared__ long long s_dst[kRowThreads];  // destination row address
  __shared__ int s_wcnt[kRowWarps];
  const int64_t t = blockIdx.x;
  const int tid = threadIdx.x;
  const V* src = x + t * nvec;
  V r[VPT];
#pragma unroll
  for (int v = 0; v < VPT; ++v) {
    const int i = tid + v * kRowThreads;
    if (i < nvec) r[v] = __ldg(src + i);
  }
  for (int e0 = 0; e0 < E; e0 += kRowThreads) {
    const int e = e0 + tid;
    int64_t row = -1;
    if (e < E) row = __ldg(map_te + t * E + e);
    long long base = 0;
    int64_t rr = 0;
    const bool valid = row >= 0 && row < num_rows && peer_row(pr, e, row, base, rr);
    int pos;
    const int total = compact_window(valid, s_wcnt, pos);
    if (valid) s_dst[pos] = base + rr * nvec * static_cast<long long>(sizeof(V));
    __syncthreads();
    for (int j = 0; j < total; ++j) {
      V* o = reinterpret_cast<V*>(s_dst[j]);
#pragma unroll
      for (int v = 0; v < VPT; ++v) {
        const int i = tid + v * kRowThreads;
        if (i < nvec) o[i] = r[v];
      }
    }
    __syncthreads();
  }
}

// One chunk of the dispatch: as ep_dispatch_kernel, but only the (t, e) whose
// local expert index e % experts_per_rank lies in [le_lo, le_hi) are sent, and
// the grid is persistent over tokens (blockIdx.x, blockIdx.x + gridDim.x, ...).
// With a grid of about one 128-thread CTA per SM and ~1 KB of shared memory,
// its CTAs fit on the SMs beside a running grouped-GEMM CTA, so the next
// chunk's rows can move over NVLink while the GEMMs of this chunk run (the
// two launches share no data and neither waits for the other). A token
// whose map has no entry in the chunk is not read.
template <int VPT, typename V>
__global__ void __launch_bounds__(kRowThreads) ep_dispatch_range_kernel(
    const V* __restrict__ x, const int64_t* __restrict__ map_te, const PeerRows pr, int64_t T,
    int E, int nvec, int64_t num_rows, int le_lo, int le_hi) {
  __shared__ long long s_dst[kRowThreads];  // destination row address
  __shared__ int s_wcnt[kRowWarps];
  const int tid = threadIdx.x;
  const int el = pr.experts_per_rank;
  for (int64_t t = blockIdx.x; t < T; t += gridDim.x) {
    const V* src = x + t * nvec;
    V r[VPT];
    bool loaded = false;
    for (int e0 = 0; e0 < E; e0 += kRowThreads) {
      const int e = e0 + tid;
      int64_t row = -1;
      if (e < E) {
        const int le = e % el;
        if (le >= le_lo && le < le_hi) row = __ldg(map_te + t * E + e);
      }
      long long base = 0;
      int64_t rr = 0;
      const bool valid = row >= 0 && row < num_rows && peer_row(pr, e, row, base, rr);
      int pos;
      const int total = compact_window(valid, s_wcnt, pos);
      if (valid) s_dst[pos] = base + rr * nvec * static_cast<long long>(sizeof(V));
      __syncthreads();
      if (total > 0 && !loaded) {  // block-uniform
#pragma unroll
        for (int v = 0; v < VPT; ++v) {
          const int i = tid + v * kRowThreads;
          if (i < nvec) r[v] = __ldg(src + i);
        }
        loaded = true;
      }
      for (int j = 0; j < total; ++j) {
        V* o = reinterpret_cast<V*>(s_dst[j]);
#pragma unroll
        for (int v = 0; v < VPT; ++v) {
          const int i = tid + v * kRowThreads;
          if (i < nvec) o[i] = r[v];
        }
      }
      __syncthreads();
    }
  }
}

// ---------------------------------------------------------------------------
// Pull dispatch: the receiver loads its rows from the sources instead of the
// sources storing them. Each source first stages its token rows and, for each
// of its permuted (expert-major) rows, the token it comes from, in two
// peer-shared buffers (ep_pull_stage_kernel). After a barrier every receiver
// walks its expert-major receive rows: row rr of the group (local expert le,
// source s) is the source's permuted row src_row0[g] + (rr - start[g]), whose
// token the receiver reads from the source's index, then the row itself;
// the two loads cross NVLink, the store is local. The receive rows come out
// exactly as the push dispatch writes them.
// ---------------------------------------------------------------------------
constexpr int kPullMaxGroups = 1024;

template <int VPT, typename V>
__global__ void __launch_bounds__(kRowThreads) ep_pull_stage_kernel(
    const V* __restrict__ x, const int64_t* __restrict__ map_te, int64_t T, int E, int nvec,
    int64_t num_rows, V* __restrict__ xs, int32_t* __restrict__ inv) {
  const int64_t t = blockIdx.x;
  const int tid = threadIdx.x;
#pragma unroll
  for (int v = 0; v < VPT; ++v) {
    const int i = tid + v * kRowThreads;
    if (i < nvec) xs[t * nvec + i] = __ldg(x + t * nvec + i);
  }
  for (int e = tid; e < E; e += kRowThreads) {
    const int64_t row = __ldg(map_te + t * E + e);
    if (row >= 0 && row < num_rows) inv[row] = static_cast<int32_t>(t);
  }
}

struct PullSrc {
  long long xs[kMaxRanks];   // rank s's staged token rows, this process's address
  long long inv[kMaxRanks];  // rank s's permuted row -> token index
  long long tok_cap;         // rows of each staging buffer
  long long row_cap;         // entries of each index
  int ranks;
};

template <int VPT, typename V>
__global__ void __launch_bounds__(kRowThreads) ep_pull_kernel(
    const PullSrc ps, const int32_t* __restrict__ table, int ng, V* __restrict__ recv,
    int64_t nrecv, int64_t cap_rows, int nvec) {
  __shared__ int32_t s_start[kPullMaxGroups];
  __shared__ int32_t s_cnt[kPullMaxGroups];
  __shared__ int32_t s_src0[kPullMaxGroups];
  __shared__ long long s_src;
  const int tid = threadIdx.x;
  for (int g = tid; g < ng; g += kRowThreads) {
    s_start[g] = __ldg(table + g);
    s_cnt[g] = __ldg(table + ng + g);
    s_src0[g] = __ldg(table + 2 * ng + g);
  }
  __syncthreads();
  for (int64_t rr = blockIdx.x; rr < nrecv && rr < cap_rows; rr += gridDim.x) {
    if (tid == 0) {
      // the last group starting at or before rr (empty groups share the next
      // group's start, so this lands on the group that holds rr)
      int lo = 0, hi = ng - 1;
      while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (s_start[mid] <= rr) lo = mid;
        else hi = mid - 1;
      }
      const int s = lo % ps.ranks;
      const int64_t j = rr - s_start[lo];
      const int64_t srow = static_cast<int64_t>(s_src0[lo]) + j;
      long long a = -1;
      if (j >= 0 && j < s_cnt[lo] && srow >= 0 && srow < ps.row_cap) {
        const int32_t tok = reinterpret_cast<const int32_t*>(ps.inv[s])[srow];
        if (tok >= 0 && tok < ps.tok_cap)
          a = ps.xs[s] + static_cast<long long>(tok) * nvec * static_cast<long long>(sizeof(V));
      }
      s_src = a;
    }
    __syncthreads();
    const long long a = s_src;
    if (a >= 0) {
      const V* src = reinterpret_cast<const V*>(a);
      V r[VPT];
#pragma unroll
      for (int v = 0; v < VPT; ++v) {
        const int i = tid + v * kRowThreads;
        if (i < nvec) r[v] = src[i];
      }
#pragma unroll
      for (int v = 0; v < VPT; ++v) {
        const int i = tid + v * kRowThreads;
        if (i < nvec) recv[rr * nvec + i] = r[v];
      }
    }
    __syncthreads();
  }
}

constexpr int kEpCombineMaxE = 1024;

template <typename V>
__global__ void __launch_bounds__(kRowThreads) ep_combine_kernel(
    const PeerRows pr, const int64_t* __restrict__ map_te, const float* __restrict__ probs,
    V* __restrict__ out, int64_t T, int E, int nvec, int64_t num_rows) {
  constexpr int kE = VecTraits<V>::kElems;
  __shared__ long long s_src[kEpCombineMaxE];  // source row address
  __shared__ float s_w[kEpCombineMaxE];
  __shared__ int s_wcnt[kRowWarps];
  __shared__ int s_n;
  const int64_t t = blockIdx.x;
  const int tid = threadIdx.x;
  const bool weighted = probs != nullptr;
  if (tid == 0) s_n = 0;
  for (int e0 = 0; e0 < E; e0 += kRowThreads) {
    const int e = e0 + tid;
    int64_t row = -1;
    if (e < E) row = __ldg(map_te + t * E + e);
    long long base = 0;
    int64_t rr = 0;
    const bool valid = row >= 0 && row < num_rows && peer_row(pr, e, row, base, rr);
    int pos;
    const int total = compact_window(valid, s_wcnt, pos);
    const int b = s_n;
    if (valid) {
      s_src[b + pos] = base + rr * nvec * static_cast<long long>(sizeof(V));
      s_w[b + pos] = weighted ? __ldg(probs + t * E + e) : 1.f;
    }
    __syncthreads();
    if (tid == 0) s_n = b + total;
  }
  __syncthreads();
  const int n = s_n;
  for (int i = tid; i < nvec; i += kRowThreads) {
    float acc[kE];
#pragma unroll
    for (int q = 0; q < kE; ++q) acc[q] = 0.f;
    int j = 0;
    for (; j + 8 <= n; j += 8) {
      const V* pa[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) pa[u] = reinterpret_cast<const V*>(s_src[j + u]) + i;
      V v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) v[u] = __ldg(pa[u]);  // 8 independent row loads in flight
#pragma unroll
      for (int u = 0; u < 8; ++u) accum_vec<V>(acc, v[u], s_w[j + u], weighted);
    }
    for (; j < n; ++j)
      accum_vec<V>(acc, reinterpret_cast<const V*>(s_src[j])[i], s_w[j], weighted);
    out[t * nvec + i] = VecTraits<V>::pack(acc);
  }
}

// Backward of the fused combine for one source rank: for each routed (t, e)
// in ascending e, with owner d = e / experts_per_rank and row rr = map[t,e] +
// delta[e], grad_probs[t,e] = <grad_out[t], y_d[rr]> (fp32, the forward rows
// loaded from the owner's fc2 output over NVLink) and dy_d[rr] =
// bf16(probs[t,e] * grad_out[t]) (stored into the owner's gradient buffer
// over NVLink). The arithmetic and the reduction order (per-thread FMA chain,
// xor butterfly, warps in order) are those of the single-GPU
// combine_backward_kernel, so the results are the same bits.
template <typename V>
__global__ void __launch_bounds__(kRowThreads) ep_combine_backward_kernel(
    const V* __restrict__ grad_out, const int64_t* __restrict__ map_te,
    const float* __restrict__ probs, const PeerRows pr, const PeerRows pw,
    float* __restrict__ grad_probs, int64_t T, int E, int nvec, int64_t num_rows) {
  constexpr int kE = VecTraits<V>::kElems;
  __shared__ long long s_src[kEpCombineMaxE];  // forward row address (owner's fc2 output)
  __shared__ long long s_dst[kEpCombineMaxE];  // gradient row address (owner's buffer)
  __shared__ int s_e[kEpCombineMaxE];
  __shared__ float s_w[kEpCombineMaxE];
  __shared__ int s_wcnt[kRowWarps];
  __shared__ float s_red[kRowWarps];
  __shared__ int s_n;
  const int64_t t = blockIdx.x;
  const int tid = threadIdx.x;
  if (tid == 0) s_n = 0;
  for (int e0 = 0; e0 < E; e0 += kRowThreads) {
    const int e = e0 + tid;
    int64_t row = -1;
    if (e < E) row = __ldg(map_te + t * E + e);
    long long rb = 0, wb = 0;
    int64_t rr = 0, wr = 0;
    const bool valid = row >= 0 && row < num_rows && peer_row(pr, e, row, rb, rr) &&
                       peer_row(pw, e, row, wb, wr);
    if (e < E && !valid) grad_probs[t * E + e] = 0.f;
    int pos;
    const int total = compact_window(valid, s_wcnt, pos);
    const int b = s_n;
    if (valid) {
      s_src[b + pos] = rb + rr * nvec * static_cast<long long>(sizeof(V));
      s_dst[b + pos] = wb + wr * nvec * static_cast<long long>(sizeof(V));
      s_e[b + pos] = e;
      s_w[b + pos] = __ldg(probs + t * E + e);
    }
    __syncthreads();
    if (tid == 0) s_n = b + total;
  }
  __syncthreads();
  const int n = s_n;
  const V* g_row = grad_out + t * nvec;
  for (int j = 0; j < n; ++j) {
    const V* yr = reinterpret_cast<const V*>(s_src[j]);
    V* dr = reinterpret_cast<V*>(s_dst[j]);
    const float w = s_w[j];
    float part = 0.f;
    for (int i = tid; i < nvec; i += kRowThreads) {
      float g[kE], y[kE], o[kE];
      VecTraits<V>::unpack(__ldg(g_row + i), g);
      VecTraits<V>::unpack(yr[i], y);
#pragma unroll
      for (int q = 0; q < kE; ++q) {
        o[q] = __fmul_rn(w, g[q]);
        part = __fmaf_rn(g[q], y[q], part);
      }
      dr[i] = VecTraits<V>::pack(o);
    }
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

// ---------------------------------------------------------------------------
// Deduplicated dispatch: a token row crosses NVLink once per destination rank
// instead of once per (token, expert). Each rank owns a staging block per
// source rank ([T rows] of token rows + [T x E_loc] int32 destination rows,
// -1 = not routed there) and a per-source row counter that the sources bump
// with remote atomics. Rows for this rank's own experts are written straight
// into the receive buffer. After the barrier, ep_expand_kernel copies every
// staged row to its listed receive rows; the receive layout (and so the
// GEMMs and the combine) is the same as without deduplication.
// ---------------------------------------------------------------------------
struct StageRows {
  long long stage[kMaxRanks];  // rank d's staging rows, this process's address
  long long meta[kMaxRanks];   // rank d's destination-row table
  long long count[kMaxRanks];  // rank d's per-source counters (int32 [ranks])
  long long rows_per_src;      // staging rows per source (T)
  int my_rank;
};

constexpr int kDedupMaxE = 1024;

template <int VPT, typename V>
__global__ void __launch_bounds__(kRowThreads) ep_dispatch_dedup_kernel(
    const V* __restrict__ x, const int64_t* __restrict__ map_te, const PeerRows pr,
    const StageRows sr, int64_t T, int E, int nvec, int64_t num_rows) {
  __shared__ long long s_dest[kDedupMaxE];  // receive row per expert (-1: not routed)
  __shared__ int s_has[kMaxRanks];
  __shared__ int s_slot;
  const int64_t t = blockIdx.x;
  const int tid = threadIdx.x;
  const int el = pr.experts_per_rank;
  const V* src = x + t * nvec;
  V r[VPT];
#pragma unroll
  for (int v = 0; v < VPT; ++v) {
    const int i = tid + v * kRowThreads;
    if (i < nvec) r[v] = __ldg(src + i);
  }
  if (tid < kMaxRanks) s_has[tid] = 0;
  __syncthreads();
  for (int e = tid; e < E; e += kRowThreads) {
    const int64_t row = __ldg(map_te + t * E + e);
    long long base = 0;
    int64_t rr = -1;
    const bool valid = row >= 0 && row < num_rows && peer_row(pr, e, row, base, rr);
    s_dest[e] = valid ? rr : -1;
    if (valid) s_has[e / el] = 1;
  }
  __syncthreads();
  for (int d = 0; d < pr.ranks; ++d) {
    if (!s_has[d]) continue;  // block-uniform
    if (d == sr.my_rank) {
      // own experts: straight into this rank's receive buffer, one copy per expert
      for (int le = 0; le < el; ++le) {
        const long long rr = s_dest[d * el + le];
        if (rr < 0) continue;
        V* o = reinterpret_cast<V*>(pr.base[d]) + rr * nvec;
#pragma unroll
        for (int v = 0; v < VPT; ++v) {
          const int i = tid + v * kRowThreads;
          if (i < nvec) o[i] = r[v];
        }
      }
      continue;
    }
    if (tid == 0) s_slot = atomicAdd(reinterpret_cast<int*>(sr.count[d]) + sr.my_rank, 1);
    __syncthreads();
    const long long slot = s_slot;
    __syncthreads();
    if (slot >= sr.rows_per_src) continue;  // cannot happen for a valid map; never overrun
    const long long srow = static_cast<long long>(sr.my_rank) * sr.rows_per_src + slot;
    V* o = reinterpret_cast<V*>(sr.stage[d]) + srow * nvec;
#pragma unroll
    for (int v = 0; v < VPT; ++v) {
      const int i = tid + v * kRowThreads;
      if (i < nvec) o[i] = r[v];
    }
    int* m = reinterpret_cast<int*>(sr.meta[d]) + srow * el;
    for (int le = tid; le < el; le += kRowThreads)
      m[le] = static_cast<int>(s_dest[d * el + le]);
  }
}

// Receiver side: each staged row (of every other source) is read once and
// written to the receive rows its table lists. Grid-stride over all slots.
template <int VPT, typename V>
__global__ void __launch_bounds__(kRowThreads) ep_expand_kernel(
    const V* __restrict__ stage, const int* __restrict__ meta, const int* __restrict__ count,
    V* __restrict__ recv, int ranks, int my_rank, int el, long long rows_per_src,
    long long cap_rows, int nvec) {
  const long long total = static_cast<long long>(ranks) * rows_per_src;
  for (long long i = blockIdx.x; i < total; i += gridDim.x) {
    const int s = static_cast<int>(i / rows_per_src);
    const long long j = i - s * rows_per_src;
    if (s == my_rank || j >= __ldg(count + s)) continue;  // block-uniform
    const V* src = stage + i * nvec;
    V r[VPT];
#pragma unroll
    for (int v = 0; v < VPT; ++v) {
      const int q = threadIdx.x + v * kRowThreads;
      if (q < nvec) r[v] = __ldg(src + q);
    }
    const int* m = meta + i * el;
    for (int le = 0; le < el; ++le) {
      const long long rr = __ldg(m + le);
      if (rr < 0 || rr >= cap_rows) continue;
      V* o = recv + rr * nvec;
#pragma unroll
      for (int v = 0; v < VPT; ++v) {
        const int q = threadIdx.x + v * kRowThreads;
        if (q < nvec) o[q] = r[v];
      }
    }
  }
}

int make_peer_rows(PeerRows& pr, const int64_t* bases, const int64_t* expert_deltas, int ranks,
                   int experts_per_rank, int64_t cap_rows, int64_t E, int64_t H, int& vbytes,
                   const char* who) {
  MOE_REQUIRE(ranks >= 1 && ranks <= kMaxRanks, "%s: ranks=%d out of [1,%d]", who, ranks,
              kMaxRanks);
  MOE_REQUIRE(experts_per_rank >= 1 && experts_per_rank * static_cast<int64_t>(ranks) == E,
              "%s: experts_per_rank * ranks must equal E", who);
  MOE_REQUIRE(bases != nullptr && expert_deltas != nullptr, "%s: null peer table", who);
  MOE_REQUIRE(cap_rows >= 0, "%s: bad capacity", who);
  uintptr_t m = (H * 2) & 15 ? 2 : 16;
  for (int d = 0; d < ranks; ++d) {
    MOE_REQUIRE(bases[d] != 0, "%s: null buffer for rank %d", who, d);
    pr.base[d] = bases[d];
    if ((static_cast<uintptr_t>(bases[d]) & 15) != 0) m = 2;
  }
  for (int d = ranks; d < kMaxRanks; ++d) pr.base[d] = 0;
  pr.delta = reinterpret_cast<const long long*>(expert_deltas);
  pr.cap_rows = cap_rows;
  pr.experts_per_rank = experts_per_rank;
  pr.ranks = ranks;
  vbytes = static_cast<int>(m);
  return MOE_OK;
}

}  // namespace
}  // namespace moe

using namespace moe;

extern "C" int moe_ep_dispatch(const void* x, const int64_t* row_id_map_te,
                               const int64_t* peer_bases, const int64_t* expert_deltas,
                               int32_t ranks, int32_t experts_per_rank, int64_t cap_rows,
                               int64_t T, int64_t H, int64_t E, int64_t num_rows,
                               moe_stream_t stream) {
  MOE_REQUIRE(T >= 0 && H >= 0 && E >= 1, "ep_dispatch: bad shape");
  if (T == 0 || H == 0) return MOE_OK;
  MOE_REQUIRE(x && row_id_map_te, "ep_dispatch: null pointer");
  PeerRows pr;
  int vb = 16;
  int st = make_peer_rows(pr, peer_bases, expert_deltas, ranks, experts_per_rank, cap_rows, E, H,
                          vb, "ep_dispatch");
  if (st) return st;
  if ((reinterpret_cast<uintptr_t>(x) & 15) != 0) vb = 2;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const unsigned grid = static_cast<unsigned>(T);
  if (vb == 16) {
    const int nvec = static_cast<int>(H / 8);
    const int vpt = (nvec + kRowThreads - 1) / kRowThreads;
    MOE_REQUIRE(vpt <= 8, "ep_dispatch: H=%lld above 8192", (long long)H);
    const uint4* xv = static_cast<const uint4*>(x);
    if (vpt <= 1) ep_dispatch_kernel<1, uint4><<<grid, kRowThreads, 0, s>>>(xv, row_id_map_te, pr, T, (int)E, nvec, num_rows);
    else if (vpt <= 2) ep_dispatch_kernel<2, uint4><<<grid, kRowThreads, 0, s>>>(xv, row_id_map_te, pr, T, (int)E, nvec, num_rows);
    else if (vpt <= 4) ep_dispatch_kernel<4, uint4><<<grid, kRowThreads, 0, s>>>(xv, row_id_map_te, pr, T, (int)E, nvec, num_rows);
    else ep_dispatch_kernel<8, uint4><<<grid, kRowThreads, 0, s>>>(xv, row_id_map_te, pr, T, (int)E, nvec, num_rows);
  } else {
    const int nvec = static_cast<int>(H);
    const int vpt = (nvec + kRowThreads - 1) / kRowThreads;
    MOE_REQUIRE(vpt <= 16, "ep_dispatch: H=%lld above 2048 for unaligned rows", (long long)H);
    const uint16_t* xv = static_cast<const uint16_t*>(x);
    ep_dispatch_kernel<16, uint16_t><<<grid, kRowThreads, 0, s>>>(xv, row_id_map_te, pr, T, (int)E, nvec, num_rows);
  }
  MOE_CUDA_CHECK_LAUNCH("ep_dispatch launch");
  return MOE_OK;
}

extern "C" int moe_ep_dispatch_range(const void* x, const int64_t* row_id_map_te,
                                     const int64_t* peer_bases, const int64_t* expert_deltas,
                                     int32_t ranks, int32_t experts_per_rank, int64_t cap_rows,
                                     int64_t T, int64_t H, int64_t E, int64_t num_rows,
                                     int32_t local_lo, int32_t local_hi, int32_t max_ctas,
                                     moe_stream_t stream) {
  MOE_REQUIRE(T >= 0 && H >= 0 && E >= 1, "ep_dispatch_range: bad shape");
  MOE_REQUIRE(local_lo >= 0 && local_lo <= local_hi && local_hi <= experts_per_rank,
              "ep_dispatch_range: local expert range [%d,%d) outside [0,%d)", local_lo, local_hi,
              experts_per_rank);
  MOE_REQUIRE(max_ctas >= 0, "ep_dispatch_range: max_ctas=%d", max_ctas);
  if (T == 0 || H == 0 || local_lo == local_hi) return MOE_OK;
  MOE_REQUIRE(x && row_id_map_te, "ep_dispatch_range: null pointer");
  PeerRows pr;
  int vb = 16;
  int st = make_peer_rows(pr, peer_bases, expert_deltas, ranks, experts_per_rank, cap_rows, E, H,
                          vb, "ep_dispatch_range");
  if (st) return st;
  if ((reinterpret_cast<uintptr_t>(x) & 15) != 0) vb = 2;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const unsigned grid = static_cast<unsigned>(
      max_ctas > 0 ? std::min<int64_t>(T, max_ctas) : T);
  const int lo = local_lo, hi = local_hi;
  if (vb == 16) {
    const int nvec = static_cast<int>(H / 8);
    const int vpt = (nvec + kRowThreads - 1) / kRowThreads;
    MOE_REQUIRE(vpt <= 8, "ep_dispatch_range: H=%lld above 8192", (long long)H);
    const uint4* xv = static_cast<const uint4*>(x);
    if (vpt <= 2) ep_dispatch_range_kernel<2, uint4><<<grid, kRowThreads, 0, s>>>(xv, row_id_map_te, pr, T, (int)E, nvec, num_rows, lo, hi);
    else if (vpt <= 4) ep_dispatch_range_kernel<4, uint4><<<grid, kRowThreads, 0, s>>>(xv, row_id_map_te, pr, T, (int)E, nvec, num_rows, lo, hi);
    else ep_dispatch_range_kernel<8, uint4><<<grid, kRowThreads, 0, s>>>(xv, row_id_map_te, pr, T, (int)E, nvec, num_rows, lo, hi);
  } else {
    const int nvec = static_cast<int>(H);
    const int vpt = (nvec + kRowThreads - 1) / kRowThreads;
    MOE_REQUIRE(vpt <= 16, "ep_dispatch_range: H=%lld above 2048 for unaligned rows",
                (long long)H);
    ep_dispatch_range_kernel<16, uint16_t><<<grid, kRowThreads, 0, s>>>(
        static_cast<const uint16_t*>(x), row_id_map_te, pr, T, (int)E, nvec, num_rows, lo, hi);
  }
  MOE_CUDA_CHECK_LAUNCH("ep_dispatch_range launch");
  return MOE_OK;
}

extern "C" int moe_ep_pull_stage(const void* x, const int64_t* row_id_map_te, int64_t T,
                                 int64_t H, int64_t E, int64_t num_rows, void* staged_rows,
                                 int32_t* row_tokens, moe_stream_t stream) {
  MOE_REQUIRE(T >= 0 && H >= 0 && E >= 1 && num_rows >= 0, "ep_pull_stage: bad shape");
  MOE_REQUIRE(T < (1ll << 31), "ep_pull_stage: T=%lld above 2^31", (long long)T);
  if (T == 0 || H == 0) return MOE_OK;
  MOE_REQUIRE(x && row_id_map_te && staged_rows && row_tokens, "ep_pull_stage: null pointer");
  MOE_REQUIRE(H % 8 == 0 && ((reinterpret_cast<uintptr_t>(x) |
                              reinterpret_cast<uintptr_t>(staged_rows)) & 15) == 0,
              "ep_pull_stage: rows must be 16-byte vectors (H %% 8 == 0, aligned pointers)");
  const int nvec = static_cast<int>(H / 8);
  const int vpt = (nvec + kRowThreads - 1) / kRowThreads;
  MOE_REQUIRE(vpt <= 8, "ep_pull_stage: H=%lld above 8192", (long long)H);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const unsigned grid = static_cast<unsigned>(T);
  const uint4* xv = static_cast<const uint4*>(x);
  uint4* sv = static_cast<uint4*>(staged_rows);
  if (vpt <= 2) ep_pull_stage_kernel<2, uint4><<<grid, kRowThreads, 0, s>>>(xv, row_id_map_te, T, (int)E, nvec, num_rows, sv, row_tokens);
  else if (vpt <= 4) ep_pull_stage_kernel<4, uint4><<<grid, kRowThreads, 0, s>>>(xv, row_id_map_te, T, (int)E, nvec, num_rows, sv, row_tokens);
  else ep_pull_stage_kernel<8, uint4><<<grid, kRowThreads, 0, s>>>(xv, row_id_map_te, T, (int)E, nvec, num_rows, sv, row_tokens);
  MOE_CUDA_CHECK_LAUNCH("ep_pull_stage launch");
  return MOE_OK;
}

extern "C" int moe_ep_dispatch_pull(const int64_t* peer_staged_rows, const int64_t* peer_row_tokens,
                                    int32_t ranks, int64_t tokens_cap, int64_t rows_cap,
                                    const int32_t* group_table, int32_t num_groups, void* recv,
                                    int64_t num_recv, int64_t cap_rows, int64_t H,
                                    moe_stream_t stream) {
  MOE_REQUIRE(ranks >= 1 && ranks <= kMaxRanks, "ep_dispatch_pull: ranks=%d out of [1,%d]", ranks,
              kMaxRanks);
  MOE_REQUIRE(num_groups >= 1 && num_groups <= kPullMaxGroups && num_groups % ranks == 0,
              "ep_dispatch_pull: num_groups=%d must be a multiple of ranks up to %d", num_groups,
              kPullMaxGroups);
  MOE_REQUIRE(num_recv >= 0 && cap_rows >= 0 && H >= 0 && tokens_cap >= 0 && rows_cap >= 0,
              "ep_dispatch_pull: bad sizes");
  if (num_recv == 0 || H == 0) return MOE_OK;
  MOE_REQUIRE(peer_staged_rows && peer_row_tokens && group_table && recv,
              "ep_dispatch_pull: null pointer");
  MOE_REQUIRE(H % 8 == 0 && (reinterpret_cast<uintptr_t>(recv) & 15) == 0,
              "ep_dispatch_pull: rows must be 16-byte vectors (H %% 8 == 0, aligned pointers)");
  PullSrc ps;
  for (int d = 0; d < kMaxRanks; ++d) {
    const bool in = d < ranks;
    MOE_REQUIRE(!in || (peer_staged_rows[d] && peer_row_tokens[d]),
                "ep_dispatch_pull: null buffer for rank %d", d);
    MOE_REQUIRE(!in || ((peer_staged_rows[d] & 15) == 0 && (peer_row_tokens[d] & 3) == 0),
                "ep_dispatch_pull: misaligned buffer for rank %d", d);
    ps.xs[d] = in ? peer_staged_rows[d] : 0;
    ps.inv[d] = in ? peer_row_tokens[d] : 0;
  }
  ps.tok_cap = tokens_cap;
  ps.row_cap = rows_cap;
  ps.ranks = ranks;
  const int nvec = static_cast<int>(H / 8);
  const int vpt = (nvec + kRowThreads - 1) / kRowThreads;
  MOE_REQUIRE(vpt <= 8, "ep_dispatch_pull: H=%lld above 8192", (long long)H);
  int dev = 0;
  MOE_CUDA_CALL(cudaGetDevice(&dev), "cudaGetDevice");
  const int64_t rows = std::min<int64_t>(num_recv, cap_rows);
  const unsigned grid = static_cast<unsigned>(std::min<int64_t>(rows, 16ll * num_sms(dev)));
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  uint4* rv = static_cast<uint4*>(recv);
  if (vpt <= 2) ep_pull_kernel<2, uint4><<<grid, kRowThreads, 0, s>>>(ps, group_table, num_groups, rv, num_recv, cap_rows, nvec);
  else if (vpt <= 4) ep_pull_kernel<4, uint4><<<grid, kRowThreads, 0, s>>>(ps, group_table, num_groups, rv, num_recv, cap_rows, nvec);
  else ep_pull_kernel<8, uint4><<<grid, kRowThreads, 0, s>>>(ps, group_table, num_groups, rv, num_recv, cap_rows, nvec);
  MOE_CUDA_CHECK_LAUNCH("ep_dispatch_pull launch");
  return MOE_OK;
}

extern "C" int moe_ep_combine(const int64_t* peer_bases, const int64_t* expert_deltas,
                              int32_t ranks, int32_t experts_per_rank, int64_t cap_rows,
                              const int64_t* row_id_map_te, const float* probs, void* out,
                              int64_t T, int64_t H, int64_t E, int64_t num_rows,
                              moe_stream_t stream) {
  MOE_REQUIRE(T >= 0 && H >= 0 && E >= 1, "ep_combine: bad shape");
  MOE_REQUIRE(E <= kEpCombineMaxE, "ep_combine: E=%lld above %d", (long long)E, kEpCombineMaxE);
  if (T == 0 || H == 0) return MOE_OK;
  MOE_REQUIRE(out && row_id_map_te, "ep_combine: null pointer");
  PeerRows pr;
  int vb = 16;
  int st = make_peer_rows(pr, peer_bases, expert_deltas, ranks, experts_per_rank, cap_rows, E, H,
                          vb, "ep_combine");
  if (st) return st;
  if ((reinterpret_cast<uintptr_t>(out) & 15) != 0) vb = 2;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const unsigned grid = static_cast<unsigned>(T);
  if (vb == 16)
    ep_combine_kernel<uint4><<<grid, kRowThreads, 0, s>>>(pr, row_id_map_te, probs,
                                                          static_cast<uint4*>(out), T, (int)E,
                                                          static_cast<int>(H / 8), num_rows);
  else
    ep_combine_kernel<uint16_t><<<grid, kRowThreads, 0, s>>>(pr, row_id_map_te, probs,
                                                             static_cast<uint16_t*>(out), T,
                                                             (int)E, static_cast<int>(H),
                                                             num_rows);
  MOE_CUDA_CHECK_LAUNCH("ep_combine launch");
  return MOE_OK;
}

extern "C" int moe_ep_combine_backward(const void* grad_out, const int64_t* row_id_map_te,
                                       const float* probs, const int64_t* peer_rows,
                                       const int64_t* peer_grad_rows,
                                       const int64_t* expert_deltas, int32_t ranks,
                                       int32_t experts_per_rank, int64_t cap_rows,
                                       float* grad_probs, int64_t T, int64_t H, int64_t E,
                                       int64_t num_rows, moe_stream_t stream) {
  MOE_REQUIRE(T >= 0 && H >= 0 && E >= 1, "ep_combine_backward: bad shape");
  MOE_REQUIRE(E <= kEpCombineMaxE, "ep_combine_backward: E=%lld above %d", (long long)E,
              kEpCombineMaxE);
  if (T == 0) return MOE_OK;
  MOE_REQUIRE(grad_out && row_id_map_te && probs && grad_probs,
              "ep_combine_backward: null pointer");
  PeerRows pr, pw;
  int vb = 16, vw = 16;
  int st = make_peer_rows(pr, peer_rows, expert_deltas, ranks, experts_per_rank, cap_rows, E, H,
                          vb, "ep_combine_backward");
  if (st) return st;
  st = make_peer_rows(pw, peer_grad_rows, expert_deltas, ranks, experts_per_rank, cap_rows, E, H,
                      vw, "ep_combine_backward");
  if (st) return st;
  if (H == 0) return MOE_OK;
  if ((reinterpret_cast<uintptr_t>(grad_out) & 15) != 0 || vw != 16) vb = 2;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const unsigned grid = static_cast<unsigned>(T);
  if (vb == 16)
    ep_combine_backward_kernel<uint4><<<grid, kRowThreads, 0, s>>>(
        static_cast<const uint4*>(grad_out), row_id_map_te, probs, pr, pw, grad_probs, T, (int)E,
        static_cast<int>(H / 8), num_rows);
  else
    ep_combine_backward_kernel<uint16_t><<<grid, kRowThreads, 0, s>>>(
        static_cast<const uint16_t*>(grad_out), row_id_map_te, probs, pr, pw, grad_probs, T,
        (int)E, static_cast<int>(H), num_rows);
  MOE_CUDA_CHECK_LAUNCH("ep_combine_backward launch");
  return MOE_OK;
}

extern "C" int moe_ep_dispatch_dedup(const void* x, const int64_t* row_id_map_te,
                                     const int64_t* peer_bases, const int64_t* expert_deltas,
                                     const int64_t* peer_stage, const int64_t* peer_meta,
                                     const int64_t* peer_count, int32_t ranks, int32_t my_rank,
                                     int32_t experts_per_rank, int64_t cap_rows, int64_t T,
                                     int64_t H, int64_t E, int64_t num_rows,
                                     moe_stream_t stream) {
  MOE_REQUIRE(T >= 0 && H >= 0 && E >= 1, "ep_dispatch_dedup: bad shape");
  MOE_REQUIRE(E <= kDedupMaxE, "ep_dispatch_dedup: E=%lld above %d", (long long)E, kDedupMaxE);
  if (T == 0 || H == 0) return MOE_OK;
  MOE_REQUIRE(x && row_id_map_te && peer_stage && peer_meta && peer_count,
              "ep_dispatch_dedup: null pointer");
  MOE_REQUIRE(my_rank >= 0 && my_rank < ranks, "ep_dispatch_dedup: my_rank out of range");
  PeerRows pr;
  int vb = 16;
  int st = make_peer_rows(pr, peer_bases, expert_deltas, ranks, experts_per_rank, cap_rows, E, H,
                          vb, "ep_dispatch_dedup");
  if (st) return st;
  StageRows sr;
  for (int d = 0; d < kMaxRanks; ++d) {
    const bool in = d < ranks;
    MOE_REQUIRE(!in || (peer_stage[d] && peer_meta[d] && peer_count[d]),
                "ep_dispatch_dedup: null staging buffer for rank %d", d);
    sr.stage[d] = in ? peer_stage[d] : 0;
    sr.meta[d] = in ? peer_meta[d] : 0;
    sr.count[d] = in ? peer_count[d] : 0;
    if (in && (static_cast<uintptr_t>(peer_stage[d]) & 15) != 0) vb = 2;
  }
  sr.rows_per_src = T;
  sr.my_rank = my_rank;
  if ((reinterpret_cast<uintptr_t>(x) & 15) != 0) vb = 2;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const unsigned grid = static_cast<unsigned>(T);
  if (vb == 16) {
    const int nvec = static_cast<int>(H / 8);
    const int vpt = (nvec + kRowThreads - 1) / kRowThreads;
    MOE_REQUIRE(vpt <= 8, "ep_dispatch_dedup: H=%lld above 8192", (long long)H);
    const uint4* xv = static_cast<const uint4*>(x);
    if (vpt <= 2) ep_dispatch_dedup_kernel<2, uint4><<<grid, kRowThreads, 0, s>>>(xv, row_id_map_te, pr, sr, T, (int)E, nvec, num_rows);
    else if (vpt <= 4) ep_dispatch_dedup_kernel<4, uint4><<<grid, kRowThreads, 0, s>>>(xv, row_id_map_te, pr, sr, T, (int)E, nvec, num_rows);
    else ep_dispatch_dedup_kernel<8, uint4><<<grid, kRowThreads, 0, s>>>(xv, row_id_map_te, pr, sr, T, (int)E, nvec, num_rows);
  } else {
    const int nvec = static_cast<int>(H);
    const int vpt = (nvec + kRowThreads - 1) / kRowThreads;
    MOE_REQUIRE(vpt <= 16, "ep_dispatch_dedup: H=%lld above 2048 for unaligned rows", (long long)H);
    ep_dispatch_dedup_kernel<16, uint16_t><<<grid, kRowThreads, 0, s>>>(
        static_cast<const uint16_t*>(x), row_id_map_te, pr, sr, T, (int)E, nvec, num_rows);
  }
  MOE_CUDA_CHECK_LAUNCH("ep_dispatch_dedup launch");
  return MOE_OK;
}

extern "C" int moe_ep_expand(const void* stage, const int32_t* meta, int32_t* count, void* recv,
                             int32_t ranks, int32_t my_rank, int32_t experts_per_rank,
                             int64_t rows_per_src, int64_t cap_rows, int64_t H,
                             moe_stream_t stream) {
  MOE_REQUIRE(ranks >= 1 && ranks <= kMaxRanks && my_rank >= 0 && my_rank < ranks,
              "ep_expand: bad ranks=%d my_rank=%d", ranks, my_rank);
  MOE_REQUIRE(experts_per_rank >= 1 && rows_per_src >= 0 && cap_rows >= 0 && H >= 0,
              "ep_expand: bad sizes");
  MOE_REQUIRE(stage && meta && count && recv, "ep_expand: null pointer");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (rows_per_src > 0 && H > 0) {
    int dev = 0;
    MOE_CUDA_CALL(cudaGetDevice(&dev), "cudaGetDevice");
    const long long total = static_cast<long long>(ranks) * rows_per_src;
    const unsigned grid = static_cast<unsigned>(std::min<long long>(total, 16ll * num_sms(dev)));
    const bool al = ((reinterpret_cast<uintptr_t>(stage) | reinterpret_cast<uintptr_t>(recv)) & 15) == 0 &&
                    H % 8 == 0;
    if (al) {
      const int nvec = static_cast<int>(H / 8);
      const int vpt = (nvec + kRowThreads - 1) / kRowThreads;
      MOE_REQUIRE(vpt <= 8, "ep_expand: H=%lld above 8192", (long long)H);
      const uint4* sv = static_cast<const uint4*>(stage);
      uint4* rv = static_cast<uint4*>(recv);
      if (vpt <= 2) ep_expand_kernel<2, uint4><<<grid, kRowThreads, 0, s>>>(sv, meta, count, rv, ranks, my_rank, experts_per_rank, rows_per_src, cap_rows, nvec);
      else if (vpt <= 4) ep_expand_kernel<4, uint4><<<grid, kRowThreads, 0, s>>>(sv, meta, count, rv, ranks, my_rank, experts_per_rank, rows_per_src, cap_rows, nvec);
      else ep_expand_kernel<8, uint4><<<grid, kRowThreads, 0, s>>>(sv, meta, count, rv, ranks, my_rank, experts_per_rank, rows_per_src, cap_rows, nvec);
    } else {
      const int nvec = static_cast<int>(H);
      MOE_REQUIRE(nvec <= 16 * kRowThreads, "ep_expand: H=%lld above 2048 for unaligned rows",
                  (long long)H);
      ep_expand_kernel<16, uint16_t><<<grid, kRowThreads, 0, s>>>(
          static_cast<const uint16_t*>(stage), meta, count, static_cast<uint16_t*>(recv), ranks,
          my_rank, experts_per_rank, rows_per_src, cap_rows, nvec);
    }
    MOE_CUDA_CHECK_LAUNCH("ep_expand launch");
  }
  // the counters start from zero for the next forward's dispatch
  MOE_CUDA_CALL(cudaMemsetAsync(count, 0, static_cast<size_t>(ranks) * sizeof(int32_t), s),
                "ep_expand: clear counters");
  return MOE_OK;
}
