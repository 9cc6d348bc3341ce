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
