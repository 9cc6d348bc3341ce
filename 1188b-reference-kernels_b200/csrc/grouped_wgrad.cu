// Grouped weight gradient on B200 tensor cores (the wgrad of the expert FFN):
//
//   dW[g] = dy[rows of g]^T @ x[rows of g]      dW [G, N, K] bf16, fp32 accumulation
//
// dy [R, N] and x [R, K] are the row-major activations of the forward, groups
// are contiguous row ranges. The reference computes this as a Python loop of
// torch.mm(dy[seg].t(), x[seg]) (kernel_cases/case05_moe_grouped_gemm_fc2_
// wgrad.py:49-64, case09_moe_grouped_gemm_fc1_wgrad.py:49-64, "TN").
//
// Both MMA operands are MN-major: a 64-row slice of dy (or x) staged by TMA as
// 64-column x 64-row boxes is a [64 reduction rows x 64 MN columns] tile with
// the MN columns contiguous, which tcgen05 reads directly (instruction bits 15
// and 16). The reduction runs over a group's rows only: every group has its
// own pair of tensor maps (built on the host from the host-side splits, stored
// in the workspace) whose outer extent is that group's row count, so the last
// partial 64-row block is zero-filled by TMA instead of reaching into the next
// group. A group with no rows gets a zero dW[g], like torch.mm over zero rows.
//
// Two kernels, chosen per call from the mean rows per group:
//   grouped_wgrad_pair_kernel (deep groups): CTA pairs (cta_group::2) on
//     256 x 256 tiles of dW[g], 5-stage ring of 32 KB per CTA;
//   grouped_wgrad_kernel (shallow groups, where writing dW dominates): one
//     persistent CTA per SM on 128 x 256 tiles, 3-stage ring of 16 KB dy +
//     32 KB x.
// Both: warp 0 TMA producer, warp 1 TMEM owner and single-thread MMA issuer,
// warps 2-5 epilogue. The epilogue moves 64 columns per step (two TMEM loads
// under one wait, one 32 x 64 TMA tile store from a 128B-swizzled buffer,
// four stores in flight per warp). Every wait is bounded (2 s).
#include <cuda.h>
#include <cudaTypedefs.h>
#include <string.h>

#include <algorithm>
#include <mutex>
#include <vector>

#include "moe_common.cuh"

namespace moe {
namespace gw {

constexpr int BM = 128;  // dW rows per tile (columns of dy)
constexpr int BN = 256;  // dW columns per tile (columns of x)
constexpr int BK = 64;   // reduction rows per stage
constexpr int kStages = 3;  // K-loops are a group's rows / 64: short for most groups
constexpr int kThreads = 192;
constexpr uint32_t kBox = 64 * 64 * 2;          // one 64-column x 64-row bf16 box
constexpr uint32_t kABytes = (BM / 64) * kBox;  // 16 KB of dy
constexpr uint32_t kBBytes = (BN / 64) * kBox;  // 32 KB of x
constexpr uint32_t kStageBytes = kABytes + kBBytes;
constexpr uint32_t kTmemCols = 2 * BN;
constexpr uint32_t kEpiBoxBytes = 32 * 64 * 2;  // 32 rows x 64 bf16 columns, 128B-swizzled
constexpr int kEpiBufs = 4;                     // tile stores in flight per epilogue warp
constexpr size_t kSmemBytes = 1024 + kStages * kStageBytes + 1024 + 4 * kEpiBufs * kEpiBoxBytes;
constexpr int kErrTimeoutProducer = 1;
constexpr int kErrTimeoutMma = 2;
constexpr int kErrTimeoutEpilogue = 3;

// Only groups with rows are walked (their dW slices of empty groups are
// zeroed by the host with memsets); entry i of the tables is group gid[i].
struct Params {
  const CUtensorMap* maps;  // [2Gnz] in global memory: rows of group gid[i] of dy, then of x
  const int32_t* rows;      // [Gnz] rows of those groups
  const int32_t* gid;       // [Gnz] their group ids
  int32_t* err;
  __nv_bfloat16* out;  // dW [G, N, K]
  int G, N, K;         // G = groups with rows (when gnz is null)
  int m_tiles, n_tiles;
  const int32_t* gnz;  // device count of groups with rows (built by wgrad_table_kernel), or null
};

// Groups with rows: from the device table when it was built on the device.
MOE_DEVICE int groups_with_rows(const Params& p) { return p.gnz != nullptr ? __ldg(p.gnz) : p.G; }

MOE_DEVICE void tensormap_acquire(const void* tmap) {
  asm volatile("fence.proxy.tensormap::generic.acquire.gpu [%0], 128;" ::"l"(
                   reinterpret_cast<uint64_t>(tmap))
               : "memory");
}

MOE_DEVICE bool wait_drain(uint32_t bar, uint32_t parity) {
  const unsigned long long t0 = globaltimer_ns();
  while (!mbar_try_wait(bar, parity))
    if (globaltimer_ns() - t0 > kWaitTimeoutNs) return false;
  return true;
}

MOE_DEVICE void raise_abort(volatile int* abort_flag, int32_t* err, int code) {
  atomicCAS(err, 0, code);
  *abort_flag = 1;
  __threadfence_block();
}

__global__ void __launch_bounds__(kThreads, 1)
    grouped_wgrad_kernel(const __grid_constant__ CUtensorMap tmap_out, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  const uint32_t base = (raw_addr + 1023u) & ~1023u;
  uint8_t* base_ptr = smem_raw + (base - raw_addr);
  uint64_t* bars = reinterpret_cast<uint64_t*>(base_ptr + kStages * kStageBytes);
  const uint32_t bar0 = smem_u32(bars);
  auto full_bar = [&](int s) { return bar0 + 8u * s; };
  auto empty_bar = [&](int s) { return bar0 + 8u * (kStages + s); };
  auto tfull_bar = [&](int a) { return bar0 + 8u * (2 * kStages + a); };
  auto tempty_bar = [&](int a) { return bar0 + 8u * (2 * kStages + 2 + a); };
  const uint32_t drain_bar = bar0 + 8u * (2 * kStages + 4);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * kStages + 5);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = warp_id();
  const int lane = lane_id();
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(tfull_bar(a), 1);
      mbar_init(tempty_bar(a), 4);
    }
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const long long per_g = static_cast<long long>(p.m_tiles) * p.n_tiles;
  const long long total = per_g * groups_with_rows(p);
  // g: index into the tables (and maps); p.gid[g] is the group's id in dW.
  auto locate = [&](long long t, int& g, int& mi, int& ni) {
    g = static_cast<int>(t / per_g);
    const int r = static_cast<int>(t - g * per_g);
    mi = r / p.n_tiles;
    ni = r - mi * p.n_tiles;
  };
  auto nkb_of = [&](int g) { return (max(p.rows[g], 0) + BK - 1) / BK; };

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      const uint64_t pol = l2_policy_evict_normal();
      int stage = 0;
      uint32_t phase = 0;
      int issued[kStages];
#pragma unroll
      for (int s = 0; s < kStages; ++s) issued[s] = -1;
      bool ok = true;
      int last_g = -1;
      for (long long t = blockIdx.x; t < total && ok; t += gridDim.x) {
        int g, mi, ni;
        locate(t, g, mi, ni);
        const CUtensorMap* ma = p.maps + 2 * g;  // dy rows of group g
        const CUtensorMap* mb = ma + 1;          // x rows of group g
        if (g != last_g) {
          tensormap_acquire(ma);
          tensormap_acquire(mb);
          last_g = g;
        }
        const int nkb = nkb_of(g);
        for (int kb = 0; kb < nkb; ++kb) {
          if (!mbar_wait(empty_bar(stage), phase ^ 1u, abort_flag)) {
            ok = false;
            break;
          }
          const uint32_t sa = base + stage * kStageBytes;
          const uint32_t sb = sa + kABytes;
          mbar_arrive_expect_tx(full_bar(stage), kStageBytes);
#pragma unroll
          for (int j = 0; j < BM / 64; ++j)
            tma_load_2d(sa + j * kBox, ma, mi * BM + j * 64, kb * BK, full_bar(stage), pol);
#pragma unroll
          for (int j = 0; j < BN / 64; ++j)
            tma_load_2d(sb + j * kBox, mb, ni * BN + j * 64, kb * BK, full_bar(stage), pol);
          issued[stage] = static_cast<int>(phase);
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok) {
        raise_abort(abort_flag, p.err, kErrTimeoutProducer);
        for (int s = 0; s < kStages; ++s)
          if (issued[s] >= 0) wait_drain(full_bar(s), static_cast<uint32_t>(issued[s]));
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc = umma_idesc_bf16_f32(BM, BN) | (1u << 15) | kIdescBMajorMN;
      int stage = 0;
      uint32_t phase = 0;
      int it = 0;
      bool ok = true;
      bool issued_any = false;
      for (long long t = blockIdx.x; t < total && ok; t += gridDim.x) {
        int g, mi, ni;
        locate(t, g, mi, ni);
        const int acc = it & 1;
        const uint32_t aph = static_cast<uint32_t>((it >> 1) & 1);
        if (!mbar_wait(tempty_bar(acc), aph ^ 1u, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
        const int nkb = nkb_of(g);
        for (int kb = 0; kb < nkb; ++kb) {
          if (!mbar_wait(full_bar(stage), phase, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = base + stage * kStageBytes;
          const uint32_t sb = sa + kABytes;
          // MN-major operands: 64-column chunks 8 KB apart, 8-row groups 1 KB
          // apart; each K=16 slice moves two row groups (+2 KB = +128).
          const uint64_t ad = umma_desc_mn_sw128(sa, kBox);
          const uint64_t bd = umma_desc_mn_sw128(sb, kBox);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k)
            umma_bf16(d_tmem, ad + 128ull * k, bd + 128ull * k, idesc, (kb | k) != 0 ? 1u : 0u);
          issued_any = true;
          umma_commit(empty_bar(stage));
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit(tfull_bar(acc));  // also for a group without rows: the epilogue writes zeros
        ++it;
      }
      if (!ok) {
        raise_abort(abort_flag, p.err, kErrTimeoutMma);
        if (issued_any) {
          umma_commit(drain_bar);
          wait_drain(drain_bar, 0);
        }
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue
    const int quad = warp & 3;  // TMEM lanes this warp may access: 32*quad ..
    const uint32_t epi_base = ((bar0 + 512u + 1023u) & ~1023u) +
                              static_cast<uint32_t>(quad) * kEpiBufs * kEpiBoxBytes;
    uint32_t chunk_no = 0;
    int it = 0;
    bool ok = true;
    for (long long t = blockIdx.x; t < total; t += gridDim.x) {
      int g, mi, ni;
      locate(t, g, mi, ni);
      const int acc = it & 1;
      const uint32_t aph = static_cast<uint32_t>((it >> 1) & 1);
      if (!mbar_wait(tfull_bar(acc), aph, abort_flag)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const bool no_rows = p.rows[g] <= 0;
      const int rowl = mi * BM + quad * 32 + lane;  // row of dW[g]
      const bool rvalid = rowl < p.N;
      const bool tma = __all_sync(0xffffffffu, rvalid);
      const int gd = p.gid[g];                               // group id in dW
      const int warp_row0 = gd * p.N + mi * BM + quad * 32;  // in the [G*N, K] view
      __nv_bfloat16* orow = p.out + (static_cast<int64_t>(gd) * p.N + rowl) * p.K;
      const uint32_t tbase =
          tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + static_cast<uint32_t>(acc * BN);
#pragma unroll 1
      for (int c = 0; c < BN / 64; ++c) {
        const int col = ni * BN + c * 64;
        if (col >= p.K) break;  // warp-uniform
        uint32_t r[64];
        if (!no_rows) {
          uint32_t (&r0)[32] = *reinterpret_cast<uint32_t(*)[32]>(&r[0]);
          uint32_t (&r1)[32] = *reinterpret_cast<uint32_t(*)[32]>(&r[32]);
          tmem_ld_32x32b_x32(tbase + c * 64, r0);
          tmem_ld_32x32b_x32(tbase + c * 64 + 32, r1);
          tmem_ld_wait();
        } else {
#pragma unroll
          for (int q = 0; q < 64; ++q) r[q] = 0u;
        }
        uint32_t o[32];  // this lane's row: 64 bf16 = 128 bytes
#pragma unroll
        for (int q = 0; q < 32; ++q)
          o[q] = pack_bf16x2(__uint_as_float(r[2 * q]), __uint_as_float(r[2 * q + 1]));
        if (tma) {
          const uint32_t buf = epi_base + (chunk_no % kEpiBufs) * kEpiBoxBytes;
          ++chunk_no;
          if (lane == 0) bulk_wait_read<kEpiBufs - 1>();
          __syncwarp();
          // 128-byte swizzle: 16-byte chunk j of row r lives at chunk j ^ (r & 7).
          const uint32_t sw = static_cast<uint32_t>(lane & 7);
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const uint32_t dst =
                buf + static_cast<uint32_t>(lane) * 128u + ((static_cast<uint32_t>(j) ^ sw) << 4);
            asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(dst), "r"(o[4 * j]),
                         "r"(o[4 * j + 1]), "r"(o[4 * j + 2]), "r"(o[4 * j + 3])
                         : "memory");
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_2d(&tmap_out, col, warp_row0, buf);
            bulk_commit();
          }
        } else if (rvalid) {
#pragma unroll
          for (int v = 0; v < 8; ++v)
            if (col + v * 8 + 8 <= p.K)
              *reinterpret_cast<uint4*>(orow + col + v * 8) =
                  make_uint4(o[4 * v], o[4 * v + 1], o[4 * v + 2], o[4 * v + 3]);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(tempty_bar(acc));
      ++it;
    }
    if (lane == 0) bulk_wait_all();
    __syncwarp();
    if (!ok && lane == 0) raise_abort(abort_flag, p.err, kErrTimeoutEpilogue);
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

// ---------------------------------------------------------------------------
// CTA-pair variant (tcgen05 cta_group::2, clusters of 2): a pair owns a
// 256 x 256 tile of dW[g]. Each CTA stages 128 columns of dy (its 128 dW
// rows) and half of the tile's 256 x columns per reduction block, 32 KB a
// stage, so per SM the operand traffic is two thirds of the single-CTA
// kernel's and the ring is five stages deep beside the same epilogue buffers.
// The leader issues M=256, N=256 MMAs with both operands MN-major; each CTA's
// TMEM receives its 128 dW rows. TMA bytes of both CTAs count on the leader's
// full barrier, the commits release both CTAs' stages, both CTAs' epilogue
// warps arrive on the leader's accumulator-empty barrier. Waits bounded as in
// the single-CTA kernel; a cluster barrier precedes the pair TMEM release.
// ---------------------------------------------------------------------------
constexpr int kPairTile = 256;
constexpr int kPairStages = 5;
constexpr int64_t kPairMinRows = 384;  // mean rows per group with rows for the pair kernel
constexpr uint32_t kPairHalfBytes = 2 * kBox;                    // 128 columns x 64 rows
constexpr uint32_t kPairStageBytes = 2 * kPairHalfBytes;          // dy half + x half: 32 KB
constexpr size_t kPairSmemBytes =
    1024 + kPairStages * kPairStageBytes + 1024 + 4 * kEpiBufs * kEpiBoxBytes;

__global__ void __launch_bounds__(kThreads, 1)
    grouped_wgrad_pair_kernel(const __grid_constant__ CUtensorMap tmap_out, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  const uint32_t base = (raw_addr + 1023u) & ~1023u;
  uint8_t* base_ptr = smem_raw + (base - raw_addr);
  uint64_t* bars = reinterpret_cast<uint64_t*>(base_ptr + kPairStages * kPairStageBytes);
  const uint32_t bar0 = smem_u32(bars);
  auto full_bar = [&](int s) { return bar0 + 8u * s; };
  auto empty_bar = [&](int s) { return bar0 + 8u * (kPairStages + s); };
  auto tfull_bar = [&](int a) { return bar0 + 8u * (2 * kPairStages + a); };
  auto tempty_bar = [&](int a) { return bar0 + 8u * (2 * kPairStages + 2 + a); };
  const uint32_t drain_bar = bar0 + 8u * (2 * kPairStages + 4);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * kPairStages + 5);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const long long cid = cluster_id_x();
  const long long ncl = num_clusters_x();
  const int warp = warp_id();
  const int lane = lane_id();
  if (threadIdx.x == 0) {
    for (int s = 0; s < kPairStages; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(tfull_bar(a), 1);
      mbar_init(tempty_bar(a), 8);  // 4 epilogue warps in each of the 2 CTAs
    }
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc_pair(smem_u32(tmem_slot), kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // barriers of both CTAs initialised before any remote use
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const long long per_g = static_cast<long long>(p.m_tiles) * p.n_tiles;
  const long long total = per_g * groups_with_rows(p);
  auto locate = [&](long long t, int& g, int& mi, int& ni) {
    g = static_cast<int>(t / per_g);
    const int r = static_cast<int>(t - g * per_g);
    mi = r / p.n_tiles;
    ni = r - mi * p.n_tiles;
  };
  auto nkb_of = [&](int g) { return (max(p.rows[g], 0) + BK - 1) / BK; };

  if (warp == 0) {
    // ------------------------------------------------------------ producer (both CTAs)
    if (lane == 0) {
      const uint64_t pol = l2_policy_evict_normal();
      int stage = 0;
      uint32_t phase = 0;
      int issued[kPairStages];
#pragma unroll
      for (int s = 0; s < kPairStages; ++s) issued[s] = -1;
      bool ok = true;
      int last_g = -1;
      const int half = static_cast<int>(rank) * (kPairTile / 2);
      for (long long t = cid; t < total && ok; t += ncl) {
        int g, mi, ni;
        locate(t, g, mi, ni);
        const CUtensorMap* ma = p.maps + 2 * g;  // dy rows of group g
        const CUtensorMap* mb = ma + 1;          // x rows of group g
        if (g != last_g) {
          tensormap_acquire(ma);
          tensormap_acquire(mb);
          last_g = g;
        }
        const int nkb = nkb_of(g);
        for (int kb = 0; kb < nkb; ++kb) {
          if (!mbar_wait(empty_bar(stage), phase ^ 1u, abort_flag)) {
            ok = false;
            break;
          }
          const uint32_t sa = base + stage * kPairStageBytes;
          const uint32_t sb = sa + kPairHalfBytes;
          const uint32_t leader_full = map_to_rank(full_bar(stage), 0);
          if (leader) mbar_arrive_expect_tx(full_bar(stage), 2u * kPairStageBytes);
#pragma unroll
          for (int j = 0; j < 2; ++j) {
            tma_load_2d_pair(sa + j * kBox, ma, mi * kPairTile + half + j * 64, kb * BK,
                             leader_full, pol);
            tma_load_2d_pair(sb + j * kBox, mb, ni * kPairTile + half + j * 64, kb * BK,
                             leader_full, pol);
          }
          issued[stage] = static_cast<int>(phase);
          if (++stage == kPairStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (ok) {
        // The pair's MMA releases every stage with a commit that lands in this
        // CTA's shared memory; wait for the last ones before exiting.
        for (int s = 0; s < kPairStages; ++s)
          if (issued[s] >= 0) wait_drain(empty_bar(s), static_cast<uint32_t>(issued[s]));
      } else {
        raise_abort(abort_flag, p.err, kErrTimeoutProducer);
        if (leader) {
          for (int s = 0; s < kPairStages; ++s)
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
      const uint32_t idesc =
          umma_idesc_bf16_f32(kPairTile, kPairTile) | (1u << 15) | kIdescBMajorMN;
      int stage = 0;
      uint32_t phase = 0;
      int it = 0;
      bool ok = true;
      bool issued_any = false;
      for (long long t = cid; t < total && ok; t += ncl) {
        int g, mi, ni;
        locate(t, g, mi, ni);
        const int acc = it & 1;
        const uint32_t aph = static_cast<uint32_t>((it >> 1) & 1);
        if (!mbar_wait_cluster(tempty_bar(acc), aph ^ 1u, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
        const int nkb = nkb_of(g);
        for (int kb = 0; kb < nkb; ++kb) {
          if (!mbar_wait_cluster(full_bar(stage), phase, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = base + stage * kPairStageBytes;
          const uint32_t sb = sa + kPairHalfBytes;
          const uint64_t ad = umma_desc_mn_sw128(sa, kBox);
          const uint64_t bd = umma_desc_mn_sw128(sb, kBox);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k)
            umma_bf16_pair(d_tmem, ad + 128ull * k, bd + 128ull * k, idesc,
                           (kb | k) != 0 ? 1u : 0u);
          issued_any = true;
          umma_commit_pair(empty_bar(stage), 0x3);
          if (++stage == kPairStages) {
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
    const int quad = warp & 3;  // TMEM lanes this warp may access: 32*quad ..
    const uint32_t epi_base = ((bar0 + 512u + 1023u) & ~1023u) +
                              static_cast<uint32_t>(quad) * kEpiBufs * kEpiBoxBytes;
    const uint32_t leader_tempty0 = map_to_rank(tempty_bar(0), 0);
    const uint32_t leader_tempty1 = map_to_rank(tempty_bar(1), 0);
    uint32_t chunk_no = 0;
    int it = 0;
    bool ok = true;
    for (long long t = cid; t < total; t += ncl) {
      int g, mi, ni;
      locate(t, g, mi, ni);
      const int acc = it & 1;
      const uint32_t aph = static_cast<uint32_t>((it >> 1) & 1);
      if (!mbar_wait_cluster(tfull_bar(acc), aph, abort_flag)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const int row_in_tile = static_cast<int>(rank) * 128 + quad * 32;
      const int rowl = mi * kPairTile + row_in_tile + lane;  // row of dW[g]
      const bool rvalid = rowl < p.N;
      const bool tma = __all_sync(0xffffffffu, rvalid);
      const int gd = p.gid[g];
      const int warp_row0 = gd * p.N + mi * kPairTile + row_in_tile;  // in the [G*N, K] view
      __nv_bfloat16* orow = p.out + (static_cast<int64_t>(gd) * p.N + rowl) * p.K;
      const uint32_t tbase =
          tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + static_cast<uint32_t>(acc * BN);
#pragma unroll 1
      for (int c = 0; c < BN / 64; ++c) {
        const int col = ni * kPairTile + c * 64;
        if (col >= p.K) break;  // warp-uniform
        uint32_t r[64];
        uint32_t (&r0)[32] = *reinterpret_cast<uint32_t(*)[32]>(&r[0]);
        uint32_t (&r1)[32] = *reinterpret_cast<uint32_t(*)[32]>(&r[32]);
        tmem_ld_32x32b_x32(tbase + c * 64, r0);
        tmem_ld_32x32b_x32(tbase + c * 64 + 32, r1);
        tmem_ld_wait();
        uint32_t o[32];  // this lane's row: 64 bf16 = 128 bytes
#pragma unroll
        for (int q = 0; q < 32; ++q)
          o[q] = pack_bf16x2(__uint_as_float(r[2 * q]), __uint_as_float(r[2 * q + 1]));
        if (tma) {
          const uint32_t buf = epi_base + (chunk_no % kEpiBufs) * kEpiBoxBytes;
          ++chunk_no;
          if (lane == 0) bulk_wait_read<kEpiBufs - 1>();
          __syncwarp();
          // 128-byte swizzle: 16-byte chunk j of row r lives at chunk j ^ (r & 7).
          const uint32_t sw = static_cast<uint32_t>(lane & 7);
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const uint32_t dst =
                buf + static_cast<uint32_t>(lane) * 128u + ((static_cast<uint32_t>(j) ^ sw) << 4);
            asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(dst), "r"(o[4 * j]),
                         "r"(o[4 * j + 1]), "r"(o[4 * j + 2]), "r"(o[4 * j + 3])
                         : "memory");
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_2d(&tmap_out, col, warp_row0, buf);
            bulk_commit();
          }
        } else if (rvalid) {
#pragma unroll
          for (int v = 0; v < 8; ++v)
            if (col + v * 8 + 8 <= p.K)
              *reinterpret_cast<uint4*>(orow + col + v * 8) =
                  make_uint4(o[4 * v], o[4 * v + 1], o[4 * v + 2], o[4 * v + 3]);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(acc == 0 ? leader_tempty0 : leader_tempty1);
      ++it;
    }
    if (lane == 0) bulk_wait_all();
    __syncwarp();
    if (!ok && lane == 0) raise_abort(abort_flag, p.err, kErrTimeoutEpilogue);
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync();  // no CTA leaves while its partner may still touch its memory
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, kTmemCols);
  }
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* q = nullptr;
    cudaDriverEntryPointQueryResult r;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &q, cudaEnableDefault, &r) ==
            cudaSuccess &&
        r == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(q);
  });
  return fn;
}

// bf16 row-major [outer, inner] at ptr; box box_inner x box_outer.
int encode_bf16(CUtensorMap* m, const void* ptr, uint64_t inner, uint64_t outer,
                uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle swz) {
  auto encode = encode_fn();
  if (encode == nullptr) {
    set_last_error("grouped_wgrad: cuTensorMapEncodeTiled unavailable");
    return MOE_ERR_CUDA;
  }
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {inner * 2};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1u, 1u};
  const CUresult r = encode(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims,
                            strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_last_error("grouped_wgrad: cuTensorMapEncodeTiled failed (%d)", static_cast<int>(r));
    return MOE_ERR_CUDA;
  }
  return MOE_OK;
}

// ---------------------------------------------------------------------------
// Group table built on the device, so no call waits for the stream: the host
// encodes one tensor map over all of dy and one over all of x (templates);
// wgrad_table_kernel compacts the groups with rows and writes, for each, a copy
// of both templates whose global address and outer extent it replaces
// (tensormap.replace) with the group's first row and row count. The splits
// come from device memory or, for the host-array entry point, by value in the
// kernel parameters (at most kHostSplitsMax groups).
// ---------------------------------------------------------------------------
constexpr int kHostSplitsMax = 4096;
struct HostSplits {
  int32_t v[kHostSplitsMax];
};
constexpr int kErrBadSplits = 4;  // device error word: a negative count or sum(m) > rows

MOE_DEVICE int32_t split_of(const int32_t* m_dev, const HostSplits& hs, int g) {
  return m_dev != nullptr ? __ldg(m_dev + g) : hs.v[g];
}

// Writes the template map to dst (global), then points it at `addr` with
// `rows` rows. tensormap.replace works on the object in the generic proxy,
// after this thread's own stores of the template.
MOE_DEVICE void store_group_map(CUtensorMap* dst, const CUtensorMap& tmpl, uint64_t addr,
                                uint32_t rows) {
  const uint4* src = reinterpret_cast<const uint4*>(&tmpl);
  uint4* d = reinterpret_cast<uint4*>(dst);
#pragma unroll
  for (int i = 0; i < 8; ++i) d[i] = src[i];
  asm volatile("tensormap.replace.tile.global_address.global.b1024.b64 [%0], %1;" ::"l"(dst),
               "l"(addr)
               : "memory");
  asm volatile("tensormap.replace.tile.global_dim.global.b1024.b32 [%0], 1, %1;" ::"l"(dst),
               "r"(rows)
               : "memory");
}

__global__ void __launch_bounds__(1024) wgrad_table_kernel(
    const int32_t* __restrict__ m_dev, const __grid_constant__ HostSplits hs, int G,
    int64_t rows_total, const __grid_constant__ CUtensorMap tmpl_dy,
    const __grid_constant__ CUtensorMap tmpl_x, const char* dy, const char* x, int64_t N,
    int64_t K, int32_t* __restrict__ rows_out, int32_t* __restrict__ gid_out,
    CUtensorMap* __restrict__ maps_out, int32_t* __restrict__ gnz_out, int32_t* __restrict__ err) {
  __shared__ int64_t w_rows[32];
  __shared__ int w_nz[32];
  __shared__ int64_t carry_rows;
  __shared__ int carry_nz;
  __shared__ int bad;
  const int lane = lane_id(), wid = warp_id();
  if (threadIdx.x == 0) {
    carry_rows = 0;
    carry_nz = 0;
    bad = 0;
  }
  __syncthreads();
  for (int g0 = 0; g0 < G; g0 += 1024) {
    const int g = g0 + static_cast<int>(threadIdx.x);
    int32_t m = g < G ? split_of(m_dev, hs, g) : 0;
    if (m < 0) {
      bad = 1;
      m = 0;
    }
    int64_t r_incl = m;
    int nz_incl = m > 0 ? 1 : 0;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int64_t yr = __shfl_up_sync(0xffffffffu, r_incl, off);
      const int yn = __shfl_up_sync(0xffffffffu, nz_incl, off);
      if (lane >= off) {
        r_incl += yr;
        nz_incl += yn;
      }
    }
    if (lane == 31) {
      w_rows[wid] = r_incl;
      w_nz[wid] = nz_incl;
    }
    __syncthreads();
    if (wid == 0) {
      int64_t a = w_rows[lane];
      int b = w_nz[lane];
      const int64_t a0 = a;
      const int b0 = b;
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const int64_t ya = __shfl_up_sync(0xffffffffu, a, off);
        const int yb = __shfl_up_sync(0xffffffffu, b, off);
        if (lane >= off) {
          a += ya;
          b += yb;
        }
      }
      w_rows[lane] = a - a0;  // exclusive prefix of the warps before
      w_nz[lane] = b - b0;
    }
    __syncthreads();
    const int64_t start = carry_rows + w_rows[wid] + r_incl - m;
    const int idx = carry_nz + w_nz[wid] + nz_incl - (m > 0 ? 1 : 0);
    if (m > 0) {
      if (start + m > rows_total) {
        bad = 1;  // the maps would reach past dy / x: emit nothing
      } else {
        rows_out[idx] = m;
        gid_out[idx] = g;
        store_group_map(maps_out + 2 * idx, tmpl_dy,
                        reinterpret_cast<uint64_t>(dy) + static_cast<uint64_t>(start * N * 2),
                        static_cast<uint32_t>(m));
        store_group_map(maps_out + 2 * idx + 1, tmpl_x,
                        reinterpret_cast<uint64_t>(x) + static_cast<uint64_t>(start * K * 2),
                        static_cast<uint32_t>(m));
      }
    }
    __syncthreads();
    if (threadIdx.x == 1023) {
      carry_rows = start + m;
      carry_nz = idx + (m > 0 ? 1 : 0);
    }
    __syncthreads();
  }
  asm volatile("fence.proxy.tensormap::generic.release.gpu;" ::: "memory");
  if (threadIdx.x == 0) {
    *gnz_out = bad ? 0 : carry_nz;
    if (bad) atomicCAS(err, 0, kErrBadSplits);
  }
}

// dW[g] = 0 for every group without rows (torch.mm over zero rows).
__global__ void __launch_bounds__(256) wgrad_zero_empty_kernel(
    uint4* __restrict__ dw, const int32_t* __restrict__ m_dev, const __grid_constant__ HostSplits hs,
    int64_t slice_vec) {
  const int g = static_cast<int>(blockIdx.y);
  if (split_of(m_dev, hs, g) != 0) return;
  uint4* d = dw + static_cast<int64_t>(g) * slice_vec;
  const uint4 z = make_uint4(0u, 0u, 0u, 0u);
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < slice_vec;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    d[i] = z;
}

size_t rows_bytes(int64_t G) { return (static_cast<size_t>(G) * 4 + 255) & ~static_cast<size_t>(255); }
size_t ws_bytes(int64_t G) {
  return 256 + 2 * rows_bytes(G) + 2 * static_cast<size_t>(G) * sizeof(CUtensorMap);
}

int ensure_smem_attr() {
  int dev = 0;
  MOE_CUDA_CALL(cudaGetDevice(&dev), "cudaGetDevice");
  static std::mutex mu;
  static bool done[64] = {};
  std::lock_guard<std::mutex> lock(mu);
  if (dev < 64 && done[dev]) return MOE_OK;
  MOE_CUDA_CALL(cudaFuncSetAttribute(grouped_wgrad_kernel,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     static_cast<int>(kSmemBytes)),
                "cudaFuncSetAttribute(grouped_wgrad)");
  MOE_CUDA_CALL(cudaFuncSetAttribute(grouped_wgrad_pair_kernel,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     static_cast<int>(kPairSmemBytes)),
                "cudaFuncSetAttribute(grouped_wgrad_pair)");
  if (dev < 64) done[dev] = true;
  return MOE_OK;
}

// Clusters of 2 that can be resident at once (0: the pair kernel cannot run,
// or MOE_WGRAD_PAIR=0 asks for the single-CTA kernel).
int pair_clusters(int dev) {
  static std::mutex mu;
  static int cache[64];
  static bool init[64] = {};
  const char* e = getenv("MOE_WGRAD_PAIR");
  if (e != nullptr && e[0] == '0') return 0;
  std::lock_guard<std::mutex> lock(mu);
  if (dev >= 0 && dev < 64 && init[dev]) return cache[dev];
  int n = 0;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * 74);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = kPairSmemBytes;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaOccupancyMaxActiveClusters(&n, grouped_wgrad_pair_kernel, &cfg) != cudaSuccess) n = 0;
  cudaGetLastError();  // clear a non-sticky error from an unsupported query
  if (dev >= 0 && dev < 64) {
    cache[dev] = n;
    init[dev] = true;
  }
  return n;
}

}  // namespace gw
}  // namespace moe

using namespace moe;

extern "C" int moe_grouped_wgrad_workspace_size(int64_t G, size_t* bytes) {
  MOE_REQUIRE(bytes != nullptr, "grouped_wgrad_workspace_size: null output");
  MOE_REQUIRE(G >= 1 && G <= (1 << 20), "grouped_wgrad: G=%lld out of range", (long long)G);
  *bytes = gw::ws_bytes(G);
  return MOE_OK;
}

// dW of both entry points: m_dev (device) or m_host (host array, G <= 4096,
// passed by value), never both. Nothing here waits for the stream.
static int grouped_wgrad_run(const void* dy, const void* x, void* dw, int64_t rows_total,
                             int64_t G, int64_t N, int64_t K, const int32_t* m_dev,
                             const int32_t* m_host, void* workspace, size_t workspace_bytes,
                             moe_stream_t stream, const char* who) {
  MOE_REQUIRE(rows_total >= 0 && rows_total < (1ll << 31), "%s: rows=%lld out of range", who,
              (long long)rows_total);
  MOE_REQUIRE(N >= 8 && N % 8 == 0 && K >= 8 && K % 8 == 0,
              "%s: N=%lld and K=%lld must be positive multiples of 8", who, (long long)N,
              (long long)K);
  MOE_REQUIRE(G * N < (1ll << 31), "%s: G*N too large", who);
  MOE_REQUIRE(workspace != nullptr && workspace_bytes >= gw::ws_bytes(G) &&
                  (reinterpret_cast<uintptr_t>(workspace) & 255) == 0,
              "%s: workspace must hold %zu bytes, 256-byte aligned", who, gw::ws_bytes(G));
  MOE_REQUIRE(dy && x && dw, "%s: null pointer", who);
  MOE_REQUIRE(((reinterpret_cast<uintptr_t>(dy) | reinterpret_cast<uintptr_t>(x) |
                reinterpret_cast<uintptr_t>(dw)) & 15) == 0,
              "%s: dy, x and dw must be 16-byte aligned", who);
  gw::HostSplits hs{};
  int64_t sum = rows_total;  // device splits: the rows are the estimate below
  int64_t gnz_host = G;
  if (m_host != nullptr) {
    sum = 0;
    gnz_host = 0;
    for (int64_t g = 0; g < G; ++g) {
      MOE_REQUIRE(m_host[g] >= 0, "%s: m_splits[%lld] < 0", who, (long long)g);
      sum += m_host[g];
      gnz_host += m_host[g] > 0 ? 1 : 0;
      hs.v[g] = m_host[g];
    }
    MOE_REQUIRE(sum <= rows_total, "%s: sum(m_splits)=%lld exceeds rows=%lld", who,
                (long long)sum, (long long)rows_total);
  }
  int st = gw::ensure_smem_attr();
  if (st) return st;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  char* ws = static_cast<char*>(workspace);
  const size_t rb = gw::rows_bytes(G);
  int32_t* err = reinterpret_cast<int32_t*>(ws);
  int32_t* gnz = reinterpret_cast<int32_t*>(ws + 4);
  MOE_CUDA_CALL(cudaMemsetAsync(ws, 0, 8, s), "grouped_wgrad: clear error word");
  int dev = 0;
  MOE_CUDA_CALL(cudaGetDevice(&dev), "cudaGetDevice");
  // dW of the groups without rows: zeros.
  const int64_t slice_vec = N * K * 2 / 16;
  const unsigned zx = static_cast<unsigned>(std::min<int64_t>((slice_vec + 255) / 256, 64));
  gw::wgrad_zero_empty_kernel<<<dim3(zx, static_cast<unsigned>(G)), 256, 0, s>>>(
      static_cast<uint4*>(dw), m_dev, hs, slice_vec);
  MOE_CUDA_CHECK_LAUNCH("grouped_wgrad zero launch");
  if (rows_total == 0 || gnz_host == 0 || sum == 0) return MOE_OK;
  CUtensorMap tdy, tx, tout;
  if ((st = gw::encode_bf16(&tdy, dy, static_cast<uint64_t>(N), static_cast<uint64_t>(rows_total),
                            64u, 64u, CU_TENSOR_MAP_SWIZZLE_128B)) ||
      (st = gw::encode_bf16(&tx, x, static_cast<uint64_t>(K), static_cast<uint64_t>(rows_total),
                            64u, 64u, CU_TENSOR_MAP_SWIZZLE_128B)) ||
      (st = gw::encode_bf16(&tout, dw, static_cast<uint64_t>(K), static_cast<uint64_t>(G * N),
                            64u, 32u, CU_TENSOR_MAP_SWIZZLE_128B)))
    return st;
  gw::Params p;
  p.maps = reinterpret_cast<const CUtensorMap*>(ws + 256 + 2 * rb);
  p.rows = reinterpret_cast<const int32_t*>(ws + 256);
  p.gid = reinterpret_cast<const int32_t*>(ws + 256 + rb);
  p.err = err;
  p.out = static_cast<__nv_bfloat16*>(dw);
  p.G = static_cast<int>(G);  // upper bound; the kernels read the device count
  p.gnz = gnz;
  p.N = static_cast<int>(N);
  p.K = static_cast<int>(K);
  gw::wgrad_table_kernel<<<1, 1024, 0, s>>>(
      m_dev, hs, static_cast<int>(G), rows_total, tdy, tx, static_cast<const char*>(dy),
      static_cast<const char*>(x), N, K, const_cast<int32_t*>(p.rows), const_cast<int32_t*>(p.gid),
      reinterpret_cast<CUtensorMap*>(ws + 256 + 2 * rb), gnz, err);
  MOE_CUDA_CHECK_LAUNCH("grouped_wgrad table launch");
  // CTA pairs when the groups are deep enough for the MMA to dominate (a
  // 256 x 256 pair tile moves two thirds of the operand bytes per SM of the
  // single-CTA tile); with a few k-blocks per tile the kernel is bound by
  // writing dW, where the single-CTA kernel measured faster (case09's ~100
  // rows per group: 686 vs 1016 us). Host splits give the exact mean rows of
  // the groups with rows; device splits, the mean over all G groups.
  const int clusters = gw::pair_clusters(dev);
  if (clusters > 0 && sum >= gw::kPairMinRows * gnz_host) {  // 256 x 256 tiles on CTA pairs
    p.m_tiles = static_cast<int>((N + gw::kPairTile - 1) / gw::kPairTile);
    p.n_tiles = static_cast<int>((K + gw::kPairTile - 1) / gw::kPairTile);
    const int64_t tiles = static_cast<int64_t>(p.m_tiles) * p.n_tiles * gnz_host;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(2 * std::min<int64_t>(tiles, clusters)));
    cfg.blockDim = dim3(gw::kThreads);
    cfg.dynamicSmemBytes = gw::kPairSmemBytes;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    MOE_CUDA_CALL(cudaLaunchKernelEx(&cfg, gw::grouped_wgrad_pair_kernel, tout, p),
                  "grouped_wgrad pair launch");
    return MOE_OK;
  }
  p.m_tiles = static_cast<int>((N + gw::BM - 1) / gw::BM);
  p.n_tiles = static_cast<int>((K + gw::BN - 1) / gw::BN);
  const int64_t tiles = static_cast<int64_t>(p.m_tiles) * p.n_tiles * gnz_host;
  const int grid = static_cast<int>(std::min<int64_t>(tiles, num_sms(dev)));
  gw::grouped_wgrad_kernel<<<grid, gw::kThreads, gw::kSmemBytes, s>>>(tout, p);
  MOE_CUDA_CHECK_LAUNCH("grouped_wgrad launch");
  return MOE_OK;
}

extern "C" int moe_grouped_wgrad(const void* dy, const void* x, void* dw, int64_t rows_total,
                                 int64_t G, int64_t N, int64_t K, const int32_t* m_splits,
                                 void* workspace, size_t workspace_bytes, moe_stream_t stream) {
  MOE_REQUIRE(G >= 1 && G <= gw::kHostSplitsMax,
              "grouped_wgrad: G=%lld out of [1,%d] (larger G: moe_grouped_wgrad_dev)",
              (long long)G, gw::kHostSplitsMax);
  MOE_REQUIRE(m_splits != nullptr, "grouped_wgrad: null m_splits (host array of G counts)");
  return grouped_wgrad_run(dy, x, dw, rows_total, G, N, K, nullptr, m_splits, workspace,
                           workspace_bytes, stream, "grouped_wgrad");
}

extern "C" int moe_grouped_wgrad_dev(const void* dy, const void* x, void* dw, int64_t rows_total,
                                     int64_t G, int64_t N, int64_t K, const int32_t* m_splits,
                                     void* workspace, size_t workspace_bytes,
                                     moe_stream_t stream) {
  MOE_REQUIRE(G >= 1 && G <= (1 << 20), "grouped_wgrad_dev: G=%lld out of range", (long long)G);
  MOE_REQUIRE(m_splits != nullptr, "grouped_wgrad_dev: null m_splits (device array of G counts)");
  return grouped_wgrad_run(dy, x, dw, rows_total, G, N, K, m_splits, nullptr, workspace,
                           workspace_bytes, stream, "grouped_wgrad_dev");
}
