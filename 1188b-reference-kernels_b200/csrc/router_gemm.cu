// Router gate GEMM fused with the softmax / top-k router on B200 tensor cores.
//
//   logits[t, :] = x[t, :] @ W^T                        (fp32, accumulated in TMEM)
//   score        = logits + bias                        (bias optional)
//   top-k of score (largest, lower column on ties, NaN ranked first)
//   gates        = softmax(score)[sel] (renormalised over sel when renorm), or
//                  the raw scores (renormalised by their sum when renorm)
//   -> topk values / indices [T,k], routing map [T,E] and dense probs [T,E]
//
// x is [T, H] bf16, W is [E, H] bf16 (both K-major). This is the router of
// the expert layer: the GEMM of kernel_cases/case38_ref_musa_asm_bf16_ssgemm_
// nt_320x256.py:51-59 followed by the routing of moe_router_topk (softmax,
// top-k with the case23 ordering, renormalisation), in one kernel, so the
// [T,E] fp32 logits never travel through HBM unless the caller asks for them.
//
// A CTA pair (cluster of 2, tcgen05 cta_group::2) owns 256 tokens and ALL E
// experts of them: each CTA stages its own 128 x-rows and half of W's rows per
// k-block (so W crosses L2 once per pair, not once per CTA), the leader issues
// M=256 MMAs (N = E in pieces of <= 256, K=16) and each CTA's TMEM receives
// its 128 rows x E fp32 columns (two accumulators when E <= 256, so the
// epilogue of one tile overlaps the mainloop of the next). Warp 0 is the TMA
// producer, warp 1 owns TMEM and (in the leader) issues the MMAs, warps 2-17
// are the epilogue: four warps per TMEM lane quadrant, each reading a quarter
// of the columns of its 32 rows (tcgen05.ld 32x32b, one row per thread) and
// keeping a register-resident sorted top-k of them (for k <= 8 through a
// branch-free sort-and-merge network, eight columns at a time, so the rows
// of a warp never diverge; for larger k by insertion). The quarters meet on a
// per-quadrant mbarrier; the first merges the other three lists (keys are
// unique, so the merged selection is exact), forms the normalisers and writes
// the outputs. Selection, softmax maximum, normalisers (with their summation
// order) and the gate formula are those of the warp-per-row router kernel in
// routing.cu, so both produce the same bits from the same logits. Dense
// outputs are zero-filled by the quadrant's warps with coalesced 16-byte
// stores over its 32 contiguous rows before the selected entries are placed.
//
// Every wait is bounded (2 s); on timeout the kernel records an error code in
// the caller's device word, drains its own copies and MMAs, frees TMEM after a
// cluster barrier and returns.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <math.h>

#include <mutex>

#include "moe_common.cuh"

namespace moe {
namespace gg {
// Defined in grouped_gemm.cu: 2-D tensor map over a row-major [outer, inner]
// bf16 (or fp32) matrix with the given box and swizzle.
int make_tmap_box(CUtensorMap* m, const void* ptr, uint64_t inner, uint64_t outer,
                  uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle swz, bool fp32);
}  // namespace gg

namespace rg {

constexpr int BM = 128;            // token rows per CTA; a pair covers 256
constexpr int kPairRows = 256;
constexpr int BK = 64;
constexpr int kEpiWarps = 16;      // 4 per TMEM lane quadrant (column quarters)
constexpr int kThreads = 64 + 32 * kEpiWarps;
constexpr int kMaxE = 512;
constexpr int kMaxStages = 8;
constexpr uint32_t kABytes = BM * BK * 2;  // 16 KB: this CTA's x rows
constexpr size_t kSmemMax = 232448;       // dynamic shared memory per block on sm_100
constexpr size_t kSmemTail = 512;         // barriers, TMEM slot, abort flag

constexpr int kErrTimeoutProducer = 1;
constexpr int kErrTimeoutMma = 2;
constexpr int kErrTimeoutEpilogue = 3;

// Merge area: quarters 1-3 hand their top-k lists (key, exact score) and
// maxima to quarter 0; [quarter-1][slot][row] so a warp's accesses are
// contiguous. One buffer: a quarter writes the next tile's list only after
// quarter 0 has released this one (per-quadrant "free" barrier).
__host__ __device__ inline size_t merge_bytes(int k) {
  return static_cast<size_t>(3 * k * BM) * (8 + 4) + static_cast<size_t>(3 * BM) * 4;
}

struct Params {
  const float* bias;  // [E] or null
  float* logits;      // [T,E] unbiased GEMM output, or null
  float* vals;        // [T,k] gates, or null
  int64_t* idx;       // [T,k] expert ids, or null
  uint8_t* rmap;      // [T,E] 0/1, or null
  float* probs;       // [T,E] dense gates, or null
  int32_t* err;
  int64_t T;
  int E;
  int k;
  int mode;    // 1 softmax gates, 2 raw-score gates
  int renorm;
  int route;   // 0: logits only (no selection work)
  int num_kb;
  int m_tiles;      // pair tiles of 256 rows
  int stages;
  int n_pieces;     // MMAs per k-slice (N = piece_n each)
  int piece_n;      // columns per piece; each CTA stages piece_n / 2 W rows of it
  int acc_stride;   // TMEM columns between the two accumulators
  int n_acc;        // 1 or 2
  uint32_t tmem_cols;
};

MOE_DEVICE void raise_abort(volatile int* abort_flag, int32_t* err, int code) {
  atomicCAS(err, 0, code);
  *abort_flag = 1;
  __threadfence_block();
}

MOE_DEVICE bool wait_drain(uint32_t bar, uint32_t parity) {
  const unsigned long long t0 = globaltimer_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer_ns() - t0 > kWaitTimeoutNs) return false;
  }
  return true;
}

// Register-resident descending top-KMAX of (key, exact score). Keys are unique
// (the column is part of the key), so the order is total.
template <int KMAX>
MOE_DEVICE void topk_insert(uint64_t (&sel)[KMAX], float (&sv)[KMAX], uint64_t key, float v) {
  if (key > sel[KMAX - 1]) {
    sel[KMAX - 1] = key;
    sv[KMAX - 1] = v;
#pragma unroll
    for (int j = KMAX - 1; j > 0; --j) {
      if (sel[j] > sel[j - 1]) {
        const uint64_t tk = sel[j];
        sel[j] = sel[j - 1];
        sel[j - 1] = tk;
        const float tv = sv[j];
        sv[j] = sv[j - 1];
        sv[j - 1] = tv;
      }
    }
  }
}

// Compare-exchange of two (key, score) pairs: the larger key first.
MOE_DEVICE void ce_desc(uint64_t& ka, float& va, uint64_t& kb, float& vb) {
  const bool sw = kb > ka;
  const uint64_t k0 = sw ? kb : ka, k1 = sw ? ka : kb;
  const float v0 = sw ? vb : va, v1 = sw ? va : vb;
  ka = k0;
  kb = k1;
  va = v0;
  vb = v1;
}

// Sorting network for 8 elements (19 comparators, depth 6) and the bitonic
// half-cleaner cascade that sorts an 8-element bitonic sequence (12).
__device__ constexpr int kSort8[19][2] = {{0, 2}, {1, 3}, {4, 6}, {5, 7}, {0, 4}, {1, 5}, {2, 6},
                                          {3, 7}, {0, 1}, {2, 3}, {4, 5}, {6, 7}, {2, 4}, {3, 5},
                                          {1, 4}, {3, 6}, {1, 2}, {3, 4}, {5, 6}};
__device__ constexpr int kBitonic8[12][2] = {{0, 4}, {1, 5}, {2, 6}, {3, 7}, {0, 2}, {1, 3},
                                             {4, 6}, {5, 7}, {0, 1}, {2, 3}, {4, 5}, {6, 7}};

// Merges 8 (key, score) pairs, sorted descending, into the descending top-8
// (sel, sv): the larger of sel[i] and new[7-i] form a bitonic sequence that
// holds the top 8 of both lists, which the cascade sorts. Branch-free, so the
// 32 rows of a warp never diverge.
MOE_DEVICE void top8_merge_sorted(uint64_t (&sel)[8], float (&sv)[8], const uint64_t (&nk)[8],
                                  const float (&nv)[8]) {
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const bool t = nk[7 - i] > sel[i];
    sel[i] = t ? nk[7 - i] : sel[i];
    sv[i] = t ? nv[7 - i] : sv[i];
  }
#pragma unroll
  for (int c = 0; c < 12; ++c)
    ce_desc(sel[kBitonic8[c][0]], sv[kBitonic8[c][0]], sel[kBitonic8[c][1]], sv[kBitonic8[c][1]]);
}

// Same for 8 unsorted pairs (sorted first by the 19-comparator network).
MOE_DEVICE void top8_merge8(uint64_t (&sel)[8], float (&sv)[8], uint64_t (&nk)[8], float (&nv)[8]) {
#pragma unroll
  for (int c = 0; c < 19; ++c)
    ce_desc(nk[kSort8[c][0]], nv[kSort8[c][0]], nk[kSort8[c][1]], nv[kSort8[c][1]]);
  top8_merge_sorted(sel, sv, nk, nv);
}

template <int KMAX>
__global__ void __launch_bounds__(kThreads, 1)
    router_gemm_topk_kernel(const __grid_constant__ CUtensorMap tmap_x,
                            const __grid_constant__ CUtensorMap tmap_w, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  const uint32_t base = (raw_addr + 1023u) & ~1023u;
  uint8_t* base_ptr = smem_raw + (base - raw_addr);
  const int E = p.E;
  const uint32_t half_rows = static_cast<uint32_t>(p.piece_n / 2);
  const uint32_t stage_bytes = kABytes + static_cast<uint32_t>(E / 2) * (BK * 2);
  const int S = p.stages;
  const int K = p.k;
  uint8_t* merge_ptr = base_ptr + static_cast<size_t>(S) * stage_bytes;
  uint64_t* m_keys = reinterpret_cast<uint64_t*>(merge_ptr);  // [3][K][BM]
  float* m_vals = reinterpret_cast<float*>(m_keys + 3 * K * BM);  // [3][K][BM]
  float* m_max = m_vals + 3 * K * BM;                             // [3][BM]
  uint64_t* bars = reinterpret_cast<uint64_t*>(merge_ptr + ((merge_bytes(K) + 7) & ~size_t(7)));
  const uint32_t bar0 = smem_u32(bars);
  auto full_bar = [&](int s) { return bar0 + 8u * s; };
  auto empty_bar = [&](int s) { return bar0 + 8u * (kMaxStages + s); };
  auto tfull_bar = [&](int a) { return bar0 + 8u * (2 * kMaxStages + a); };
  auto tempty_bar = [&](int a) { return bar0 + 8u * (2 * kMaxStages + 2 + a); };
  auto quad_bar = [&](int q) { return bar0 + 8u * (2 * kMaxStages + 4 + q); };
  auto free_bar = [&](int q) { return bar0 + 8u * (2 * kMaxStages + 8 + q); };
  const uint32_t drain_bar = bar0 + 8u * (2 * kMaxStages + 12);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * kMaxStages + 13);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int cid = static_cast<int>(cluster_id_x());
  const int ncl = static_cast<int>(num_clusters_x());
  const int warp = warp_id();
  const int lane = lane_id();

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(tfull_bar(a), 1);
      mbar_init(tempty_bar(a), 2 * kEpiWarps);  // every epilogue warp of both CTAs
    }
    for (int q = 0; q < 4; ++q) {
      mbar_init(quad_bar(q), 4);
      mbar_init(free_bar(q), 1);
    }
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmap_x);
    tma_prefetch_desc(&tmap_w);
  }
  if (warp == 1) {
    tmem_alloc_pair(smem_u32(tmem_slot), p.tmem_cols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // barriers of both CTAs initialised before any remote use
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer (both CTAs)
    if (lane == 0) {
      const uint64_t pol_x = l2_policy_evict_first();  // every x row is read once
      const uint64_t pol_w = l2_policy_evict_last();   // W is read by every pair
      int stage = 0;
      uint32_t phase = 0;
      int issued[kMaxStages];
#pragma unroll
      for (int s = 0; s < kMaxStages; ++s) issued[s] = -1;
      bool ok = true;
      // Both CTAs' bytes per stage land on the leader's full barrier.
      const uint32_t tx = 2u * stage_bytes;
      for (int t = cid; ok && t < p.m_tiles; t += ncl) {
        const int row0 = t * kPairRows + static_cast<int>(rank) * BM;
        for (int kb = 0; kb < p.num_kb; ++kb) {
          if (!mbar_wait(empty_bar(stage), phase ^ 1u, abort_flag)) {
            ok = false;
            break;
          }
          const uint32_t sa = base + static_cast<uint32_t>(stage) * stage_bytes;
          const uint32_t sb = sa + kABytes;
          const uint32_t leader_full = map_to_rank(full_bar(stage), 0);
          if (leader) mbar_arrive_expect_tx(full_bar(stage), tx);
          tma_load_2d_pair(sa, &tmap_x, kb * BK, row0, leader_full, pol_x);
          for (int pc = 0; pc < p.n_pieces; ++pc)  // this CTA's half of each piece's W rows
            tma_load_2d_pair(sb + static_cast<uint32_t>(pc) * half_rows * (BK * 2), &tmap_w,
                             kb * BK, pc * p.piece_n + static_cast<int>(rank * half_rows),
                             leader_full, pol_w);
          issued[stage] = static_cast<int>(phase);
          if (++stage == S) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (ok) {
        // The pair's MMA releases every stage with a commit that lands in this
        // CTA's shared memory; wait for the last ones before exiting.
        for (int s = 0; s < S; ++s)
          if (issued[s] >= 0) wait_drain(empty_bar(s), static_cast<uint32_t>(issued[s]));
      } else {
        raise_abort(abort_flag, p.err, kErrTimeoutProducer);
        if (leader) {
          for (int s = 0; s < S; ++s)
            if (issued[s] >= 0) wait_drain(full_bar(s), static_cast<uint32_t>(issued[s]));
        } else {
          // Copies count on the leader's barrier; give them a bounded time to land.
          const unsigned long long t0 = globaltimer_ns();
          while (globaltimer_ns() - t0 < 200000ull) {
          }
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (leader)
    if (leader && lane == 0) {
      const uint32_t idesc = umma_idesc_bf16_f32(kPairRows, p.piece_n);
      int stage = 0;
      uint32_t phase = 0;
      int it = 0;
      bool ok = true;
      bool issued_any = false;
      for (int t = cid; ok && t < p.m_tiles; t += ncl) {
        const int acc = p.n_acc == 2 ? (it & 1) : 0;
        const uint32_t aph = static_cast<uint32_t>(p.n_acc == 2 ? ((it >> 1) & 1) : (it & 1));
        if (!mbar_wait_cluster(tempty_bar(acc), aph ^ 1u, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * p.acc_stride);
        for (int kb = 0; kb < p.num_kb; ++kb) {
          if (!mbar_wait_cluster(full_bar(stage), phase, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = base + static_cast<uint32_t>(stage) * stage_bytes;
          const uint32_t sb = sa + kABytes;
          const uint64_t ad = umma_desc_k_sw128(sa);
          for (int pc = 0; pc < p.n_pieces; ++pc) {
            const uint64_t bd =
                umma_desc_k_sw128(sb + static_cast<uint32_t>(pc) * half_rows * (BK * 2));
            const uint32_t dcol = d_tmem + static_cast<uint32_t>(pc * p.piece_n);
#pragma unroll
            for (int k = 0; k < BK / 16; ++k)
              umma_bf16_pair(dcol, ad + 2ull * k, bd + 2ull * k, idesc, (kb | k) != 0 ? 1u : 0u);
          }
          issued_any = true;
          umma_commit_pair(empty_bar(stage), 0x3);
          if (++stage == S) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit_pair(tfull_bar(acc), 0x3);
        ++it;
      }
      if (!ok) {
        raise_abort(abort_flag, p.err, kErrTimeoutMma);
        if (issued_any) {
          umma_commit_pair(drain_bar, 0x1);
          wait_drain(drain_bar, 0);
        }
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue (both CTAs)
    const int quad = warp & 3;                 // TMEM lanes 32*quad .. 32*quad+31
    const int quarter = (warp - 2) >> 2;       // column quarter of this warp
    const int r_in_cta = quad * 32 + lane;
    const int nch = E / 32;
    const int c_begin = (quarter * nch) / 4;
    const int c_end = ((quarter + 1) * nch) / 4;
    const uint32_t leader_tempty0 = map_to_rank(tempty_bar(0), 0);
    const uint32_t leader_tempty1 = map_to_rank(tempty_bar(1), 0);
    const bool full_sum = p.route && p.mode == 1 && !p.renorm;  // needs every column in order
    int it = 0;
    bool ok = true;
    auto release_acc = [&](int acc) {
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(acc == 0 ? leader_tempty0 : leader_tempty1);
    };
    for (int t = cid; t < p.m_tiles; t += ncl) {
      const int acc = p.n_acc == 2 ? (it & 1) : 0;
      const uint32_t aph = static_cast<uint32_t>(p.n_acc == 2 ? ((it >> 1) & 1) : (it & 1));
      if (!mbar_wait_cluster(tfull_bar(acc), aph, abort_flag)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const int64_t wrow0 = static_cast<int64_t>(t) * kPairRows + rank * BM + quad * 32;
      const int64_t row = wrow0 + lane;
      const bool rvalid = row < p.T;
      const uint32_t tbase = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) +
                             static_cast<uint32_t>(acc * p.acc_stride);

      uint64_t sel[KMAX];
      float sv[KMAX];
#pragma unroll
      for (int j = 0; j < KMAX; ++j) {
        sel[j] = 0;
        sv[j] = 0.f;
      }
      float m = -INFINITY;
      // Pass 1 over this quarter's columns: logits out, selection, maximum.
#pragma unroll 1
      for (int ch = c_begin; ch < c_end; ++ch) {
        const int c0 = ch * 32;
        uint32_t r[32];
        tmem_ld_32x32b_x32(tbase + static_cast<uint32_t>(c0), r);
        tmem_ld_wait();
        if (rvalid && p.logits != nullptr) {
          float* lrow = p.logits + row * E + c0;
#pragma unroll
          for (int v = 0; v < 8; ++v)
            *reinterpret_cast<uint4*>(lrow + v * 4) =
                make_uint4(r[v * 4], r[v * 4 + 1], r[v * 4 + 2], r[v * 4 + 3]);
        }
        if (p.route) {
          if constexpr (KMAX == 8) {
            // eight columns at a time through the branch-free merge network
#pragma unroll
            for (int g8 = 0; g8 < 4; ++g8) {
              uint64_t nk[8];
              float nv[8];
#pragma unroll
              for (int j = 0; j < 8; ++j) {
                const int c = c0 + 8 * g8 + j;
                float x = __uint_as_float(r[8 * g8 + j]);
                if (p.bias != nullptr) x += __ldg(p.bias + c);
                m = fmaxf(m, x);
                nk[j] = rank_key(x, c);
                nv[j] = x;
              }
              top8_merge8(sel, sv, nk, nv);
            }
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              float x = __uint_as_float(r[j]);
              if (p.bias != nullptr) x += __ldg(p.bias + c0 + j);
              m = fmaxf(m, x);
              topk_insert<KMAX>(sel, sv, rank_key(x, c0 + j), x);
            }
          }
        }
      }
      if (!(quarter == 0 && full_sum)) release_acc(acc);
      if (!p.route) {
        ++it;
        continue;
      }

      // Hand the list over, zero this quarter's share of the dense rows.
      if (quarter != 0) {
        // quarter 0 has finished reading the previous tile's lists
        if (it > 0 && !mbar_wait(free_bar(quad), static_cast<uint32_t>((it - 1) & 1), abort_flag)) {
          ok = false;
          break;
        }
        const int q = quarter - 1;
#pragma unroll
        for (int j = 0; j < KMAX; ++j) {
          if (j < K) {
            m_keys[(q * K + j) * BM + r_in_cta] = sel[j];
            m_vals[(q * K + j) * BM + r_in_cta] = sv[j];
          }
        }
        m_max[q * BM + r_in_cta] = m;
      }
      const int64_t nrows = min(static_cast<int64_t>(32), p.T - wrow0);
      if (nrows > 0) {
        const uint4 z = make_uint4(0u, 0u, 0u, 0u);
        if (p.probs != nullptr) {
          uint4* dst = reinterpret_cast<uint4*>(p.probs + wrow0 * E);
          const int64_t n16 = nrows * E / 4;
          for (int64_t i = quarter * 32 + lane; i < n16; i += 128) dst[i] = z;
        }
        if (p.rmap != nullptr) {
          uint4* dst = reinterpret_cast<uint4*>(p.rmap + wrow0 * E);
          const int64_t n16 = nrows * E / 16;
          for (int64_t i = quarter * 32 + lane; i < n16; i += 128) dst[i] = z;
        }
      }
      // Quadrant barrier (bounded): lists, maxima and zeros of all four
      // quarters are visible to quarter 0 after it.
      __threadfence_block();
      __syncwarp();
      if (lane == 0) mbar_arrive(quad_bar(quad));
      if (!mbar_wait(quad_bar(quad), static_cast<uint32_t>(it & 1), abort_flag)) {
        ok = false;
        break;
      }
      ++it;
      if (quarter != 0) continue;

#pragma unroll 1
      for (int q = 0; q < 3; ++q) {
        m = fmaxf(m, m_max[q * BM + r_in_cta]);
        if constexpr (KMAX == 8) {
          uint64_t nk[8];
          float nv[8];
#pragma unroll
          for (int j = 0; j < 8; ++j) {  // a sorted list; slots past k are empty
            nk[j] = j < K ? m_keys[(q * K + j) * BM + r_in_cta] : 0ull;
            nv[j] = j < K ? m_vals[(q * K + j) * BM + r_in_cta] : 0.f;
          }
          top8_merge_sorted(sel, sv, nk, nv);
        } else {
#pragma unroll
          for (int j = 0; j < KMAX; ++j) {
            if (j < K) {
              const uint64_t key = m_keys[(q * K + j) * BM + r_in_cta];
              const float v = m_vals[(q * K + j) * BM + r_in_cta];
              topk_insert<KMAX>(sel, sv, key, v);
            }
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(free_bar(quad));  // the lists may be overwritten
      // Normalisers, in the summation order of the warp-per-row router:
      // lane l of that kernel sums columns l, l+32, ... in turn, then the 32
      // partial sums meet in an xor butterfly (offsets 16, 8, 4, 2, 1).
      float denom = 1.f, gsum = 1.f;
      if (p.mode == 1) {
        if (p.renorm) {
          float s = 0.f;
#pragma unroll
          for (int j = 0; j < KMAX; ++j)
            if (j < p.k) s += expf(key_value(sel[j]) - m);
          denom = s;
        } else {
          float part[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) part[j] = 0.f;
#pragma unroll 1
          for (int c0 = 0; c0 < E; c0 += 32) {
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
              uint32_t r[16];
              tmem_ld_32x32b_x16(tbase + static_cast<uint32_t>(c0 + 16 * hh), r);
              tmem_ld_wait();
#pragma unroll
              for (int j = 0; j < 16; ++j) {
                float x = __uint_as_float(r[j]);
                if (p.bias != nullptr) x += __ldg(p.bias + c0 + 16 * hh + j);
                part[16 * hh + j] += expf(x - m);
              }
            }
          }
          release_acc(acc);
#pragma unroll
          for (int off = 16; off > 0; off >>= 1) {
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              if (j < (j ^ off)) {
                const float a = part[j], b = part[j ^ off];
                part[j] = a + b;
                part[j ^ off] = b + a;
              }
            }
          }
          denom = part[0];
        }
      } else if (p.mode == 2 && p.renorm) {
        float s = 0.f;
#pragma unroll
        for (int j = 0; j < KMAX; ++j)
          if (j < p.k) s += key_value(sel[j]);
        gsum = s;
      }
      auto gate_of = [&](float x) {
        if (p.mode == 1) return expf(x - m) / denom;
        if (p.mode == 2 && p.renorm) return x / gsum;
        return x;
      };
      if (rvalid) {
#pragma unroll
        for (int j = 0; j < KMAX; ++j) {
          if (j < p.k) {
            const int c = key_column(sel[j]);
            const float gte = gate_of(sv[j]);
            if (p.vals != nullptr) p.vals[row * p.k + j] = gte;
            if (p.idx != nullptr) p.idx[row * p.k + j] = c;
            if (p.probs != nullptr) p.probs[row * E + c] = gte;
            if (p.rmap != nullptr) p.rmap[row * E + c] = 1;
          }
        }
      }
    }
    if (!ok && lane == 0) raise_abort(abort_flag, p.err, kErrTimeoutEpilogue);
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync();  // no CTA leaves while its partner may still touch its memory
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, p.tmem_cols);
  }
}

size_t smem_bytes(int stages, int E, int k) {
  return 1024 + static_cast<size_t>(stages) * (kABytes + static_cast<size_t>(E / 2) * BK * 2) +
         ((merge_bytes(k) + 7) & ~size_t(7)) + kSmemTail;
}

// Clusters of 2 that can be resident at once for this kernel and smem size.
template <int KMAX>
int max_clusters(size_t smem) {
  int n = 0;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * 74);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaOccupancyMaxActiveClusters(&n, router_gemm_topk_kernel<KMAX>, &cfg) != cudaSuccess)
    n = 0;
  cudaGetLastError();  // clear a non-sticky error from an unsupported query
  return n;
}

int ensure_attr() {
  int dev = 0;
  MOE_CUDA_CALL(cudaGetDevice(&dev), "cudaGetDevice");
  static std::mutex mu;
  static bool done[64] = {};
  std::lock_guard<std::mutex> lock(mu);
  if (dev < 64 && done[dev]) return MOE_OK;
  MOE_CUDA_CALL(cudaFuncSetAttribute(router_gemm_topk_kernel<8>,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     static_cast<int>(kSmemMax)),
                "cudaFuncSetAttribute(router_gemm_topk<8>)");
  MOE_CUDA_CALL(cudaFuncSetAttribute(router_gemm_topk_kernel<16>,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     static_cast<int>(kSmemMax)),
                "cudaFuncSetAttribute(router_gemm_topk<16>)");
  if (dev < 64) done[dev] = true;
  return MOE_OK;
}

template <int KMAX>
int launch(const CUtensorMap& tx, const CUtensorMap& tw, Params p, cudaStream_t s) {
  // Stages: as many x-tile + half-W-tile stages as fit beside the merge area.
  const size_t stage_bytes = kABytes + static_cast<size_t>(p.E / 2) * (BK * 2);
  const size_t merge = (merge_bytes(p.k) + 7) & ~size_t(7);
  int stages = static_cast<int>((kSmemMax - 1024 - kSmemTail - merge) / stage_bytes);
  stages = stages > kMaxStages ? kMaxStages : stages;
  MOE_REQUIRE(stages >= 2, "router_gemm_topk: E=%d leaves fewer than two stages", p.E);
  p.stages = stages;
  const size_t smem = smem_bytes(stages, p.E, p.k);
  int dev = 0;
  MOE_CUDA_CALL(cudaGetDevice(&dev), "cudaGetDevice");
  static std::mutex mu;
  // Resident clusters depend only on the shared memory per CTA (one CTA per
  // SM either way); cached per device and size.
  static int cache[64][4];
  static size_t cache_smem[64][4];
  static int cache_n[64] = {};
  int ncl = -1;
  {
    std::lock_guard<std::mutex> lock(mu);
    if (dev >= 0 && dev < 64)
      for (int i = 0; i < cache_n[dev]; ++i)
        if (cache_smem[dev][i] == smem) ncl = cache[dev][i];
    if (ncl < 0) {
      ncl = max_clusters<KMAX>(smem);
      if (dev >= 0 && dev < 64) {
        const int i = cache_n[dev] < 4 ? cache_n[dev]++ : 3;
        cache[dev][i] = ncl;
        cache_smem[dev][i] = smem;
      }
    }
  }
  if (ncl <= 0) {
    set_last_error("router_gemm_topk: CTA pairs cannot be scheduled (smem %zu)", smem);
    return MOE_ERR_UNSUPPORTED;
  }
  const int clusters = p.m_tiles < ncl ? p.m_tiles : ncl;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * clusters);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  MOE_CUDA_CALL(cudaLaunchKernelEx(&cfg, router_gemm_topk_kernel<KMAX>, tx, tw, p),
                "router_gemm_topk launch");
  return MOE_OK;
}

}  // namespace rg
}  // namespace moe

using namespace moe;

extern "C" int moe_router_gemm_topk(const void* x, const void* w, const float* bias, int64_t T,
                                    int64_t H, int64_t E, int32_t k, int32_t score_mode,
                                    int32_t renorm, float* logits, float* topk_vals,
                                    int64_t* topk_idx, uint8_t* routing_map, float* probs,
                                    int32_t* device_error, moe_stream_t stream) {
  MOE_REQUIRE(T >= 0 && T < (1ll << 31), "router_gemm_topk: T=%lld out of range", (long long)T);
  MOE_REQUIRE(H >= 8 && H % 8 == 0, "router_gemm_topk: H=%lld must be a positive multiple of 8",
              (long long)H);
  MOE_REQUIRE(E >= 32 && E <= rg::kMaxE && E % 32 == 0,
              "router_gemm_topk: E=%lld must be a multiple of 32 in [32, %d]", (long long)E,
              rg::kMaxE);
  MOE_REQUIRE(score_mode == 0 || score_mode == 1, "router_gemm_topk: score_mode must be 0 or 1");
  MOE_REQUIRE(k >= 1 && k <= 16 && k <= E, "router_gemm_topk: k=%d out of range [1, min(E, 16)]",
              k);
  MOE_REQUIRE(device_error != nullptr, "router_gemm_topk: null device_error");
  if (T == 0) return MOE_OK;  // (empty outputs may have null data pointers)
  const bool route = topk_vals || topk_idx || routing_map || probs;
  MOE_REQUIRE(route || logits != nullptr, "router_gemm_topk: no output requested");
  MOE_REQUIRE(x != nullptr && w != nullptr, "router_gemm_topk: null x or w");
  MOE_REQUIRE(((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(w) |
                reinterpret_cast<uintptr_t>(logits) | reinterpret_cast<uintptr_t>(probs) |
                reinterpret_cast<uintptr_t>(routing_map)) & 15) == 0,
              "router_gemm_topk: x, w, logits, probs and routing_map must be 16-byte aligned");
  int st = rg::ensure_attr();
  if (st) return st;

  // N pieces of at most 256 columns; each CTA of the pair stages half of a
  // piece's W rows (a multiple of 8 rows, whole 128-byte swizzle atoms).
  const int n_pieces = static_cast<int>((E + 255) / 256);
  const int piece_n = static_cast<int>(E / n_pieces);

  CUtensorMap tx, tw;
  st = gg::make_tmap_box(&tx, x, static_cast<uint64_t>(H), static_cast<uint64_t>(T),
                         static_cast<uint32_t>(rg::BK), static_cast<uint32_t>(rg::BM),
                         CU_TENSOR_MAP_SWIZZLE_128B, false);
  if (st) return st;
  st = gg::make_tmap_box(&tw, w, static_cast<uint64_t>(H), static_cast<uint64_t>(E),
                         static_cast<uint32_t>(rg::BK), static_cast<uint32_t>(piece_n / 2),
                         CU_TENSOR_MAP_SWIZZLE_128B, false);
  if (st) return st;

  rg::Params p;
  p.bias = bias;
  p.logits = logits;
  p.vals = topk_vals;
  p.idx = topk_idx;
  p.rmap = routing_map;
  p.probs = probs;
  p.err = device_error;
  p.T = T;
  p.E = static_cast<int>(E);
  p.k = k;
  p.mode = score_mode == 1 ? 1 : 2;
  p.renorm = renorm ? 1 : 0;
  p.route = route ? 1 : 0;
  p.num_kb = static_cast<int>((H + rg::BK - 1) / rg::BK);
  p.m_tiles = static_cast<int>((T + rg::kPairRows - 1) / rg::kPairRows);
  p.stages = 0;
  p.n_pieces = n_pieces;
  p.piece_n = piece_n;
  int acc = 32;
  while (acc < E) acc <<= 1;
  p.acc_stride = acc;
  p.n_acc = 2 * acc <= 512 ? 2 : 1;
  p.tmem_cols = static_cast<uint32_t>(p.n_acc * acc);

  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  return k <= 8 ? rg::launch<8>(tx, tw, p, s) : rg::launch<16>(tx, tw, p, s);
}
