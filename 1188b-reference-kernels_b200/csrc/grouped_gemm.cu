// Grouped (per-expert) GEMM for the MoE expert FFN on B200 tensor cores.
//
//   out[r, :] = x[r, :] @ W[widx(g)]^T     for every row r of group g
//
// x is [rows, K] bf16 (K contiguous), W is [num_w, N, K] bf16 ("[out,in]",
// K contiguous), i.e. both operands are K-major, which is the native operand
// form of tcgen05.mma. The reference computes the same thing as a Python loop
// of torch.mm over uniform splits (kernel_cases/case03_moe_grouped_gemm_fc1_fwd
// .py:57-64, case04_moe_grouped_gemm_fc2_fwd.py:57-64); here the groups are
// ragged and described by a device-side table, so no host sync is needed.
// moe_grouped_gemm_nn takes W as [num_w, K, N] instead (out = x @ W[g], the
// dgrad of case07/08 with the forward weight as stored): its B tiles are
// staged MN-major and described to tcgen05 as such.
// Epilogues: bf16 out, SwiGLU (fc1: gate|up -> silu(gate)*up), or the fp32
// accumulator (the router logits GEMM of case38 with one group).
//
// Two kernels share the group table, the raster order and the epilogues:
//   grouped_gemm_pair_kernel (default): CTA pairs (cta_group::2, clusters of
//     2) on 256-row tiles, epilogue through 64B-swizzled shared buffers and
//     TMA tile stores; it takes every group of at least 256 rows, its last
//     partial tile row-predicated. Inside a group it walks the N-tiles in
//     chunks of at most 32 MB of weights, all M-tiles per chunk. Its tiles
//     are 256 columns wide with two alternating accumulators, or, for deep
//     reductions (K >= 4096), 512 columns wide (two MMAs per K step sharing
//     the A tile, a quarter fewer operand bytes per flop) with one
//     accumulator that is handed to the epilogue half by half.
//   grouped_gemm_kernel: one CTA per SM on 128-row tiles; it takes the groups
//     of fewer than 256 rows after the pair kernel, or everything when CTA
//     pairs cannot be scheduled.
// Single-CTA kernel structure (one persistent CTA per SM, 192 threads):
//   warp 0      TMA producer: 128x64 A tile + 2 x 128x64 B half-tiles per
//               stage, 128-byte swizzle, 4-stage mbarrier ring.
//   warp 1      TMEM owner (512 columns = two 128x256 fp32 accumulators) and
//               single-thread tcgen05.mma issuer (M=128, N=256, K=16).
//   warps 2-5   epilogue: tcgen05.ld (32 lanes x 32 columns), bf16 convert
//               (or SwiGLU for fc1, or fp32), predicated 16-byte global stores.
// Two accumulators let the epilogue of tile i overlap the mainloop of i+1.
// Tiles are walked group by group; inside a group, super-rows of M-tiles
// sweep all N-tiles so that concurrently running CTAs share both the weight
// slab and the activation rows in L2.
//
// Every wait is bounded (2 s); on timeout the kernel records an error word in
// the workspace, drains its own in-flight copies and MMAs, frees TMEM and
// returns. Every CTA loads only its own tiles.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <stdlib.h>

#include <algorithm>
#include <mutex>

#include "moe_common.cuh"
#include "swiglu.cuh"

namespace moe {
namespace gg {

constexpr int BM = 128;
constexpr int BN = 256;
constexpr int BK = 64;
constexpr int kStages = 4;
constexpr int kSuperRow = 16;  // M-tiles per raster super-row
constexpr int kThreads = 192;
constexpr uint32_t kABytes = BM * BK * 2;           // 16 KB
constexpr uint32_t kBHalfBytes = 128 * BK * 2;      // 16 KB
constexpr uint32_t kBBytes = BN * BK * 2;           // 32 KB
constexpr uint32_t kStageBytes = kABytes + kBBytes;  // 48 KB
constexpr uint32_t kTmemCols = 2 * BN;              // 512
constexpr size_t kSmemBytes = 1024 + kStages * kStageBytes + 256;

// Device error codes written to the workspace error word.
constexpr int kErrTimeoutProducer = 1;
constexpr int kErrTimeoutMma = 2;
constexpr int kErrTimeoutEpilogue = 3;

struct Params {
  const int32_t* row_start;
  const int32_t* rows;
  const int32_t* widx;
  int32_t* err;
  void* out;        // bf16 [x_rows, n_out], or fp32 for epilogue 2
  int64_t x_rows;
  int G;
  int n_w;     // rows of one weight matrix (N)
  int n_out;   // output columns (N, or N/2 for SwiGLU)
  int f_half;  // N/2 (SwiGLU up-row offset)
  int num_kb;
  int n_tiles;
  int bn;        // pair kernel: N-tile width (256; narrower for epilogues 0/2 when N % 256 != 0)
  int b_mn;      // 1: w is [num_w, K, N] (out = x @ w[g]), B staged MN-major
  int k_rows;    // K: reduction rows of one weight matrix when b_mn
  int epilogue;  // 0 bf16 out, 1 SwiGLU -> bf16, 2 fp32 out
  int raster;   // pair kernel: pair M-tiles per raster super-row
  int n_chunk;  // pair kernel: N-tiles per weight-slab chunk (0: super-rows of `raster`)
  int l2_mode;  // pair kernel: 0 both evict_normal, 1 B evict_first, 2 A evict_last + B evict_first,
                //   3 A evict_first + B evict_last, 4 B evict_last
};

struct Tile {
  int g;
  int m_idx;
  int n_idx;
};

// Maps a linear tile index to (group, m-tile, n-tile). Tile indices handed to
// one CTA (or CTA pair) increase monotonically, so the walker only moves
// forward. kTileM rows per M-tile; inside a group, super-rows of kRaster
// M-tiles sweep all N-tiles.
template <int kTileM, int kRaster>
struct WalkerT {
  const int32_t* rows;
  int G;
  int n_tiles;
  int g = 0;
  int mt = -1;
  long long base = 0;

  __device__ bool locate(long long t, Tile& tile) {
    while (g < G) {
      if (mt < 0) mt = (max(rows[g], 0) + kTileM - 1) / kTileM;
      const long long cnt = static_cast<long long>(mt) * n_tiles;
      if (t < base + cnt) break;
      base += cnt;
      ++g;
      mt = -1;
    }
    if (g >= G) return false;
    const long long local = t - base;
    const long long sr_tiles = static_cast<long long>(kRaster) * n_tiles;
    const int sr = static_cast<int>(local / sr_tiles);
    const int within = static_cast<int>(local - sr * sr_tiles);
    const int mg = min(kRaster, mt - sr * kRaster);
    tile.g = g;
    tile.n_idx = within / mg;
    tile.m_idx = sr * kRaster + within % mg;
    return true;
  }
};
using Walker = WalkerT<BM, kSuperRow>;

// Same walk with the super-row height chosen at run time.
// n_chunk > 0 replaces the super-rows by N-chunks: a group's tiles are walked
// chunk by chunk of n_chunk N-tiles, and inside a chunk M-tile by M-tile
// (every N-tile of the chunk for one M-tile, then the next M-tile). The CTA
// pairs running at once then share one M-tile of rows and one chunk of the
// weight slab, which is sized to stay in L2 while all of the group's M-tiles
// stream past it; rows are read once per chunk.
template <int kTileM>
struct WalkerRT {
  const int32_t* rows;
  int G;
  int n_tiles;
  int raster;
  int n_chunk;
  int g = 0;
  int mt = -1;
  long long base = 0;

  __device__ bool locate(long long t, Tile& tile) {
    while (g < G) {
      if (mt < 0) mt = (max(rows[g], 0) + kTileM - 1) / kTileM;
      const long long cnt = static_cast<long long>(mt) * n_tiles;
      if (t < base + cnt) break;
      base += cnt;
      ++g;
      mt = -1;
    }
    if (g >= G) return false;
    const long long local = t - base;
    tile.g = g;
    if (n_chunk > 0) {
      const long long full = static_cast<long long>(mt) * n_chunk;  // tiles of a whole chunk
      const int ci = static_cast<int>(local / full);
      const int rem = static_cast<int>(local - ci * full);
      const int nc = min(n_chunk, n_tiles - ci * n_chunk);  // the last chunk may be narrower
      tile.m_idx = rem / nc;
      tile.n_idx = ci * n_chunk + rem % nc;
      return true;
    }
    const long long sr_tiles = static_cast<long long>(raster) * n_tiles;
    const int sr = static_cast<int>(local / sr_tiles);
    const int within = static_cast<int>(local - sr * sr_tiles);
    const int mg = min(raster, mt - sr * raster);
    tile.n_idx = within / mg;
    tile.m_idx = sr * raster + within % mg;
    return true;
  }
};

MOE_DEVICE bool wait_drain(uint32_t bar, uint32_t parity) {
  const unsigned long long t0 = globaltimer_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer_ns() - t0 > kWaitTimeoutNs) return false;
  }
  return true;
}

MOE_DEVICE void raise_abort(volatile int* abort_flag, int32_t* err, int code) {
  atomicCAS(err, 0, code);
  *abort_flag = 1;
  __threadfence_block();
}

__global__ void __launch_bounds__(kThreads, 1)
    grouped_gemm_kernel(const __grid_constant__ CUtensorMap tmap_a,
                        const __grid_constant__ CUtensorMap tmap_b, const Params p) {
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
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmap_a);
    tma_prefetch_desc(&tmap_b);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  Walker walker{p.rows, p.G, p.n_tiles};

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      const uint64_t pol_a = l2_policy_evict_normal();
      const uint64_t pol_b = l2_policy_evict_normal();
      int stage = 0;
      uint32_t phase = 0;
      int issued[kStages];
#pragma unroll
      for (int s = 0; s < kStages; ++s) issued[s] = -1;
      bool ok = true;
      for (long long t = blockIdx.x; ok; t += gridDim.x) {
        Tile tile;
        if (!walker.locate(t, tile)) break;
        const int row0 = p.row_start[tile.g] + tile.m_idx * BM;
        const int wbase = p.widx[tile.g] * (p.b_mn ? p.k_rows : p.n_w);
        int b0, b1;
        if (p.b_mn) {
          b0 = tile.n_idx * BN;  // first output column; rows follow kb
          b1 = 0;
        } else if (p.epilogue == 1) {
          b0 = wbase + tile.n_idx * 128;
          b1 = b0 + p.f_half;
        } else {
          b0 = wbase + tile.n_idx * BN;
          b1 = b0 + 128;
        }
        for (int kb = 0; kb < p.num_kb; ++kb) {
          if (!mbar_wait(empty_bar(stage), phase ^ 1u, abort_flag)) {
            ok = false;
            break;
          }
          const uint32_t sa = base + stage * kStageBytes;
          const uint32_t sb = sa + kABytes;
          mbar_arrive_expect_tx(full_bar(stage), kStageBytes);
          tma_load_2d(sa, &tmap_a, kb * BK, row0, full_bar(stage), pol_a);
          if (p.b_mn) {
            // four 64-column x 64-row boxes of w[g] (rows = reduction index)
#pragma unroll
            for (int j = 0; j < BN / 64; ++j)
              tma_load_2d(sb + j * 8192u, &tmap_b, b0 + j * 64, wbase + kb * BK, full_bar(stage),
                          pol_b);
          } else {
            tma_load_2d(sb, &tmap_b, kb * BK, b0, full_bar(stage), pol_b);
            tma_load_2d(sb + kBHalfBytes, &tmap_b, kb * BK, b1, full_bar(stage), pol_b);
          }
          issued[stage] = static_cast<int>(phase);
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok) {
        raise_abort(abort_flag, p.err, kErrTimeoutProducer);
        // Let every copy this thread started land before shared memory goes away.
        for (int s = 0; s < kStages; ++s)
          if (issued[s] >= 0) wait_drain(full_bar(s), static_cast<uint32_t>(issued[s]));
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc = umma_idesc_bf16_f32(BM, BN) | (p.b_mn ? kIdescBMajorMN : 0u);
      int stage = 0;
      uint32_t phase = 0;
      int it = 0;
      bool ok = true;
      bool issued_any = false;
      for (long long t = blockIdx.x; ok; t += gridDim.x) {
        Tile tile;
        if (!walker.locate(t, tile)) break;
        const int acc = it & 1;
        const uint32_t aph = static_cast<uint32_t>((it >> 1) & 1);
        if (!mbar_wait(tempty_bar(acc), aph ^ 1u, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
        for (int kb = 0; kb < p.num_kb; ++kb) {
          if (!mbar_wait(full_bar(stage), phase, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = base + stage * kStageBytes;
          const uint32_t sb = sa + kABytes;
          const uint64_t ad = umma_desc_k_sw128(sa);
          const uint64_t bd = p.b_mn ? umma_desc_mn_sw128(sb, 8192u) : umma_desc_k_sw128(sb);
          // K-major: +32 bytes along K inside the 128-byte swizzle atom (+2 in
          // 16-byte units); MN-major B: +16 rows = two 1024-byte K groups (+128).
          const uint64_t bstep = p.b_mn ? 128ull : 2ull;
#pragma unroll
          for (int k = 0; k < BK / 16; ++k)
            umma_bf16(d_tmem, ad + 2ull * k, bd + bstep * k, idesc, (kb | k) != 0 ? 1u : 0u);
          issued_any = true;
          umma_commit(empty_bar(stage));
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit(tfull_bar(acc));
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
    const int r_in_tile = quad * 32 + lane;
    int it = 0;
    bool ok = true;
    for (long long t = blockIdx.x;; t += gridDim.x) {
      Tile tile;
      if (!walker.locate(t, tile)) break;
      const int acc = it & 1;
      const uint32_t aph = static_cast<uint32_t>((it >> 1) & 1);
      if (!mbar_wait(tfull_bar(acc), aph, abort_flag)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const int m_local = tile.m_idx * BM + r_in_tile;
      const int64_t row = static_cast<int64_t>(p.row_start[tile.g]) + m_local;
      const bool rvalid = m_local < p.rows[tile.g] && row < p.x_rows;
      const uint32_t tbase =
          tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + static_cast<uint32_t>(acc * BN);
      if (p.epilogue == 2) {
        const int n0 = tile.n_idx * BN;
        float* orow = static_cast<float*>(p.out) + row * p.n_out;
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(tbase + c * 32, r);
          tmem_ld_wait();
          if (rvalid) {
#pragma unroll
            for (int v = 0; v < 8; ++v) {
              const int col = n0 + c * 32 + v * 4;
              if (col + 4 <= p.n_out)
                *reinterpret_cast<uint4*>(orow + col) =
                    make_uint4(r[v * 4], r[v * 4 + 1], r[v * 4 + 2], r[v * 4 + 3]);
            }
          }
        }
      } else if (p.epilogue == 0) {
        const int n0 = tile.n_idx * BN;
        __nv_bfloat16* orow = static_cast<__nv_bfloat16*>(p.out) + row * p.n_out;
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(tbase + c * 32, r);
          tmem_ld_wait();
          if (rvalid) {
#pragma unroll
            for (int v = 0; v < 4; ++v) {
              const int col = n0 + c * 32 + v * 8;
              if (col + 8 <= p.n_out) {
                uint4 o;
                o.x = pack_bf16x2(__uint_as_float(r[v * 8 + 0]), __uint_as_float(r[v * 8 + 1]));
                o.y = pack_bf16x2(__uint_as_float(r[v * 8 + 2]), __uint_as_float(r[v * 8 + 3]));
                o.z = pack_bf16x2(__uint_as_float(r[v * 8 + 4]), __uint_as_float(r[v * 8 + 5]));
                o.w = pack_bf16x2(__uint_as_float(r[v * 8 + 6]), __uint_as_float(r[v * 8 + 7]));
                *reinterpret_cast<uint4*>(orow + col) = o;
              }
            }
          }
        }
      } else {
        const int n0 = tile.n_idx * 128;
        __nv_bfloat16* orow = static_cast<__nv_bfloat16*>(p.out) + row * p.n_out;
#pragma unroll 1
        for (int c = 0; c < 128 / 32; ++c) {
          uint32_t gr[32], ur[32];
          tmem_ld_32x32b_x32(tbase + c * 32, gr);
          tmem_ld_32x32b_x32(tbase + 128 + c * 32, ur);
          tmem_ld_wait();
          if (rvalid) {
#pragma unroll
            for (int v = 0; v < 4; ++v) {
              const int col = n0 + c * 32 + v * 8;
              if (col + 8 <= p.n_out) {
                uint32_t o[4];
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                  const int j = v * 8 + 2 * q;
                  const float2 h = swiglu2_f32(
                      make_float2(round_bf16(__uint_as_float(gr[j])),
                                  round_bf16(__uint_as_float(gr[j + 1]))),
                      make_float2(round_bf16(__uint_as_float(ur[j])),
                                  round_bf16(__uint_as_float(ur[j + 1]))));
                  o[q] = pack_bf16x2(h.x, h.y);
                }
                *reinterpret_cast<uint4*>(orow + col) = make_uint4(o[0], o[1], o[2], o[3]);
              }
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(tempty_bar(acc));
      ++it;
    }
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
// CTA-pair variant (tcgen05 cta_group::2), launched as clusters of 2 CTAs.
//
// A pair owns a 256-row x 256-column output tile. Each CTA stages only its own
// 128 A rows and its half of the B rows (128 of 256) per k-block, 32 KB a
// stage instead of 48 KB, so per SM the L2->shared traffic and the shared
// memory operand reads are a third lower than the single-CTA kernel's. The
// leader CTA (rank 0) issues M=256, N=256 MMAs that read both CTAs' shared
// memory and write both CTAs' TMEM; its commits arrive on the barrier at the
// same offset in both CTAs. Both CTAs' TMA loads count their bytes on the
// leader's full barrier; both CTAs' epilogue warps arrive on the leader's
// accumulator-empty barrier. All waits are bounded as in the 1-CTA kernel,
// and a cluster barrier precedes the pair TMEM release.
// ---------------------------------------------------------------------------
namespace pairk {
constexpr int kPairTileM = 256;
constexpr int kPairStages = 6;
constexpr int kPairRaster = 8;                            // pair M-tiles per super-row
constexpr uint32_t kPairABytes = 128 * BK * 2;            // 16 KB: this CTA's rows
constexpr uint32_t kPairBBytes = 128 * BK * 2;            // 16 KB: this CTA's half of B
constexpr uint32_t kPairStageBytes = kPairABytes + kPairBBytes;   // 32 KB
constexpr uint32_t kEpiBoxBytes = 32 * 32 * 2;            // 32 rows x 32 bf16 columns
constexpr uint32_t kEpiBytes = 4 * 2 * kEpiBoxBytes;        // 4 warps x 2 buffers = 16 KB
constexpr size_t kPairSmemBytes = 1024 + kPairStages * kPairStageBytes + 1024 + kEpiBytes;
// Wide tiles: 256 rows x 512 columns per pair (two N=256 MMAs per K step that
// share the A tile), one 128x512 fp32 accumulator per CTA (all 512 TMEM
// columns, so the epilogue does not overlap the next tile's mainloop), and a
// quarter fewer operand bytes per flop than the 256x256 tile.
constexpr int kWideStages = 4;
constexpr int kWideOverlap = 2;  // k-blocks issued half by half at each end of a tile
constexpr uint32_t kWideBBytes = 256 * BK * 2;                     // 32 KB: this CTA's 256 B rows
constexpr uint32_t kWideStageBytes = kPairABytes + kWideBBytes;    // 48 KB
constexpr size_t kWideSmemBytes = 1024 + kWideStages * kWideStageBytes + 1024 + kEpiBytes;
static_assert(kPairSmemBytes <= 232448 && kWideSmemBytes <= 232448, "shared memory per CTA");
}  // namespace pairk

template <bool kWide>
__global__ void __launch_bounds__(kThreads, 1)
    grouped_gemm_pair_kernel(const __grid_constant__ CUtensorMap tmap_a,
                             const __grid_constant__ CUtensorMap tmap_b,
                             const __grid_constant__ CUtensorMap tmap_out, const Params p) {
  constexpr int kS = kWide ? pairk::kWideStages : pairk::kPairStages;
  constexpr uint32_t kSB = kWide ? pairk::kWideStageBytes : pairk::kPairStageBytes;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  const uint32_t base = (raw_addr + 1023u) & ~1023u;
  uint8_t* base_ptr = smem_raw + (base - raw_addr);
  uint64_t* bars = reinterpret_cast<uint64_t*>(base_ptr + kS * kSB);
  const uint32_t bar0 = smem_u32(bars);
  auto full_bar = [&](int s) { return bar0 + 8u * s; };
  auto empty_bar = [&](int s) { return bar0 + 8u * (kS + s); };
  auto tfull_bar = [&](int a) { return bar0 + 8u * (2 * kS + a); };
  auto tempty_bar = [&](int a) { return bar0 + 8u * (2 * kS + 2 + a); };
  const uint32_t drain_bar = bar0 + 8u * (2 * kS + 4);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * kS + 5);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const long long cid = cluster_id_x();
  const long long ncl = num_clusters_x();
  const int warp = warp_id();
  const int lane = lane_id();

  if (threadIdx.x == 0) {
    for (int s = 0; s < kS; ++s) {
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
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmap_a);
    tma_prefetch_desc(&tmap_b);
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

  WalkerRT<pairk::kPairTileM> walker{p.rows, p.G, p.n_tiles, p.raster, p.n_chunk};

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      // Weight slabs are read by the few M-tiles of one super-row and then not
      // again until the next super-row; activation rows are reused by every
      // N-tile of the super-row. Mode 1/2 let L2 drop the weights first;
      // modes 3/4 keep them (with one-M-tile super-rows every M-tile of a
      // group reads the whole weight slab, while its rows die after the
      // group's N-tiles, which run at about the same time).
      const uint64_t pol_a = p.l2_mode == 2   ? l2_policy_evict_last()
                             : p.l2_mode == 3 ? l2_policy_evict_first()
                                              : l2_policy_evict_normal();
      const uint64_t pol_b = (p.l2_mode == 1 || p.l2_mode == 2) ? l2_policy_evict_first()
                             : p.l2_mode >= 3                  ? l2_policy_evict_last()
                                                               : l2_policy_evict_normal();
      int stage = 0;
      uint32_t phase = 0;
      int issued[kS];
#pragma unroll
      for (int s = 0; s < kS; ++s) issued[s] = -1;
      bool ok = true;
      // Coordinates of this CTA's A rows and B rows for a tile.
      auto coords = [&](const Tile& tl, int& ra, int& rb) {
        ra = p.row_start[tl.g] + tl.m_idx * pairk::kPairTileM + static_cast<int>(rank) * 128;
        if (p.b_mn) {  // first output column of this CTA's half; rows follow kb
          rb = kWide ? tl.n_idx * 512 + static_cast<int>(rank) * 256
                     : tl.n_idx * p.bn + static_cast<int>(rank) * (p.bn / 2);
          return;
        }
        const int wb = p.widx[tl.g] * p.n_w;
        if (kWide)  // SwiGLU: 256 gate rows (rank 0) / 256 up rows (rank 1); else 256 of 512 rows
          rb = (p.epilogue == 1) ? wb + tl.n_idx * 256 + static_cast<int>(rank) * p.f_half
                                 : wb + tl.n_idx * 512 + static_cast<int>(rank) * 256;
        else
          rb = (p.epilogue == 1) ? wb + tl.n_idx * 128 + static_cast<int>(rank) * p.f_half
                                 : wb + tl.n_idx * p.bn + static_cast<int>(rank) * (p.bn / 2);
      };
      // Both CTAs' bytes per stage: 128 A rows each, bn/2 B rows each.
      const uint32_t tx =
          kWide ? 2u * (pairk::kPairABytes + pairk::kWideBBytes)
                : 2u * (pairk::kPairABytes + static_cast<uint32_t>(p.bn / 2) * (BK * 2));
      for (long long t = cid; ok; t += ncl) {
        Tile tile;
        if (!walker.locate(t, tile)) break;
        int row0, b0;
        coords(tile, row0, b0);
        const int wrow0 = p.b_mn ? p.widx[tile.g] * p.k_rows : 0;  // first reduction row of w[g]
        for (int kb = 0; kb < p.num_kb; ++kb) {
          if (!mbar_wait(empty_bar(stage), phase ^ 1u, abort_flag)) {
            ok = false;
            break;
          }
          const uint32_t sa = base + stage * kSB;
          const uint32_t sb = sa + pairk::kPairABytes;
          const uint32_t leader_full = map_to_rank(full_bar(stage), 0);
          if (leader) mbar_arrive_expect_tx(full_bar(stage), tx);
          tma_load_2d_pair(sa, &tmap_a, kb * BK, row0, leader_full, pol_a);
          if (p.b_mn) {
            const int wrow = wrow0 + kb * BK;
            // this CTA's 128 (wide: 256) columns as 64-column boxes
#pragma unroll
            for (int j = 0; j < (kWide ? 4 : 2); ++j)
              tma_load_2d_pair(sb + j * 8192u, &tmap_b, b0 + j * 64, wrow, leader_full, pol_b);
          } else {
            tma_load_2d_pair(sb, &tmap_b, kb * BK, b0, leader_full, pol_b);
          }
          issued[stage] = static_cast<int>(phase);
          if (++stage == kS) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (ok) {
        // The pair's MMA releases every stage with a commit that lands in this
        // CTA's shared memory; wait for the last ones before exiting.
        for (int s = 0; s < kS; ++s)
          if (issued[s] >= 0) wait_drain(empty_bar(s), static_cast<uint32_t>(issued[s]));
      } else {
        raise_abort(abort_flag, p.err, kErrTimeoutProducer);
        if (leader) {
          for (int s = 0; s < kS; ++s)
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
      const uint32_t idesc = umma_idesc_bf16_f32(pairk::kPairTileM, kWide ? 256 : p.bn) |
                             (p.b_mn ? kIdescBMajorMN : 0u);
      int stage = 0;
      uint32_t phase = 0;
      int it = 0;
      bool ok = true;
      bool issued_any = false;
      if (kWide) {
        // One accumulator of two 256-column halves, handed to the epilogue
        // half by half: the last kWideOverlap k-blocks of a tile are issued
        // for half 0 first (its epilogue then runs while half 1 finishes), and
        // the first kWideOverlap k-blocks of the next tile for half 0 first
        // (while the epilogue drains half 1). A stage is released once both
        // halves have read it. Barriers tfull/tempty(h) belong to half h.
        long long q0 = 0;  // k-blocks consumed before this tile
        const int nkb = p.num_kb;
        const int h_end = min(pairk::kWideOverlap, nkb);
        const int t_beg = max(h_end, nkb - pairk::kWideOverlap);
        auto slot = [&](int kb, int& s, uint32_t& ph) {
          const long long q = q0 + kb;
          s = static_cast<int>(q % kS);
          ph = static_cast<uint32_t>((q / kS) & 1);
        };
        auto wait_full = [&](int kb) {
          int s;
          uint32_t ph;
          slot(kb, s, ph);
          if (!mbar_wait_cluster(full_bar(s), ph, abort_flag)) return false;
          tc_fence_after();
          return true;
        };
        auto mma = [&](int kb, int h0, int h1) {  // halves h0..h1 of k-block kb
          int s;
          uint32_t ph;
          slot(kb, s, ph);
          const uint32_t sa = base + static_cast<uint32_t>(s) * kSB;
          const uint32_t sb = sa + pairk::kPairABytes;
          const uint64_t ad = umma_desc_k_sw128(sa);
          // half h reads this CTA's B rows (or MN-major columns) h*128.. at +16 KB
          const uint64_t bstep = p.b_mn ? 128ull : 2ull;
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            const uint32_t accum = (kb | k) != 0 ? 1u : 0u;
            for (int h = h0; h <= h1; ++h) {
              const uint32_t sbh = sb + static_cast<uint32_t>(h) * 16384u;
              const uint64_t bd = p.b_mn ? umma_desc_mn_sw128(sbh, 8192u) : umma_desc_k_sw128(sbh);
              umma_bf16_pair(tmem_base + static_cast<uint32_t>(h * 256), ad + 2ull * k,
                             bd + bstep * k, idesc, accum);
            }
          }
          issued_any = true;
        };
        auto release = [&](int kb) {
          int s;
          uint32_t ph;
          slot(kb, s, ph);
          umma_commit_pair(empty_bar(s), 0x3);
        };
        for (long long t = cid; ok; t += ncl) {
          Tile tile;
          if (!walker.locate(t, tile)) break;
          const uint32_t tph = static_cast<uint32_t>(it & 1);
          // head: k-blocks [0, h_end), half 0 then half 1
          ok = mbar_wait_cluster(tempty_bar(0), tph ^ 1u, abort_flag);
          if (!ok) break;
          tc_fence_after();
          for (int kb = 0; kb < h_end && ok; ++kb) {
            ok = wait_full(kb);
            if (ok) mma(kb, 0, 0);
          }
          if (!ok) break;
          if (h_end == nkb) umma_commit_pair(tfull_bar(0), 0x3);
          ok = mbar_wait_cluster(tempty_bar(1), tph ^ 1u, abort_flag);
          if (!ok) break;
          tc_fence_after();
          for (int kb = 0; kb < h_end; ++kb) {
            mma(kb, 1, 1);
            release(kb);
          }
          // body: both halves per k-block
          for (int kb = h_end; kb < t_beg && ok; ++kb) {
            ok = wait_full(kb);
            if (!ok) break;
            mma(kb, 0, 1);
            release(kb);
          }
          if (!ok) break;
          // tail: k-blocks [t_beg, nkb), half 0 then half 1
          if (t_beg < nkb) {
            for (int kb = t_beg; kb < nkb && ok; ++kb) {
              ok = wait_full(kb);
              if (ok) mma(kb, 0, 0);
            }
            if (!ok) break;
            umma_commit_pair(tfull_bar(0), 0x3);
            for (int kb = t_beg; kb < nkb; ++kb) {
              mma(kb, 1, 1);
              release(kb);
            }
          }
          umma_commit_pair(tfull_bar(1), 0x3);
          q0 += nkb;
          ++it;
        }
      }
      for (long long t = cid; ok && !kWide; t += ncl) {
        Tile tile;
        if (!walker.locate(t, tile)) break;
        const int acc = it & 1;
        const uint32_t aph = static_cast<uint32_t>((it >> 1) & 1);
        if (!mbar_wait_cluster(tempty_bar(acc), aph ^ 1u, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
        for (int kb = 0; kb < p.num_kb; ++kb) {
          if (!mbar_wait_cluster(full_bar(stage), phase, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = base + stage * kSB;
          const uint32_t sb = sa + pairk::kPairABytes;
          const uint64_t ad = umma_desc_k_sw128(sa);
          const uint64_t bd = p.b_mn ? umma_desc_mn_sw128(sb, 8192u) : umma_desc_k_sw128(sb);
          const uint64_t bstep = p.b_mn ? 128ull : 2ull;  // see grouped_gemm_kernel
#pragma unroll
          for (int k = 0; k < BK / 16; ++k)
            umma_bf16_pair(d_tmem, ad + 2ull * k, bd + bstep * k, idesc, (kb | k) != 0 ? 1u : 0u);
          issued_any = true;
          umma_commit_pair(empty_bar(stage), 0x3);
          if (++stage == kS) {
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
    // Each warp owns 32 TMEM lanes (rows). When all 32 rows are inside the
    // group, every 32-column chunk is staged in a 64B-swizzled shared buffer
    // (conflict-free) and written by one TMA tile store; otherwise the rows
    // are stored individually with row predicates.
    const int quad = warp & 3;  // TMEM lanes this warp may access: 32*quad ..
    const int r_in_cta = quad * 32 + lane;
    const uint32_t leader_tempty0 = map_to_rank(tempty_bar(0), 0);
    const uint32_t leader_tempty1 = map_to_rank(tempty_bar(1), 0);
    const uint32_t epi_base = ((bar0 + 512u + 1023u) & ~1023u) + static_cast<uint32_t>(quad) * 2u * pairk::kEpiBoxBytes;
    uint32_t chunk_no = 0;
    int it = 0;
    bool ok = true;
    // One 32-row chunk of 64 bytes per row (32 bf16 or 16 fp32 columns) of
    // this lane's row, as 16 32-bit words; col counts output elements.
    const int elem_bytes = p.epilogue == 2 ? 4 : 2;
    const int chunk_cols = 64 / elem_bytes;
    auto emit = [&](const uint32_t (&o)[16], bool tma, int64_t row, int col, int warp_row0,
                    char* orow, bool rvalid) {
      if (tma) {
        const uint32_t buf = epi_base + (chunk_no & 1u) * pairk::kEpiBoxBytes;
        ++chunk_no;
        if (lane == 0) bulk_wait_read<1>();  // the store that used this buffer has read it
        __syncwarp();
        const uint32_t sw = static_cast<uint32_t>((lane >> 1) & 3);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const uint32_t dst = buf + static_cast<uint32_t>(lane) * 64u + ((static_cast<uint32_t>(j) ^ sw) << 4);
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
        const int vcols = chunk_cols / 4;  // columns per 16-byte vector
#pragma unroll
        for (int v = 0; v < 4; ++v)
          if (col + (v + 1) * vcols <= p.n_out)
            *reinterpret_cast<uint4*>(orow + static_cast<int64_t>(col + v * vcols) * elem_bytes) =
                make_uint4(o[4 * v], o[4 * v + 1], o[4 * v + 2], o[4 * v + 3]);
      }
      (void)row;
    };
    for (long long t = cid;; t += ncl) {
      Tile tile;
      if (!walker.locate(t, tile)) break;
      const int acc = kWide ? 0 : (it & 1);
      const uint32_t aph = static_cast<uint32_t>((it >> 1) & 1);
      if (!kWide) {
        if (!mbar_wait_cluster(tfull_bar(acc), aph, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
      }
      const int m_local = tile.m_idx * pairk::kPairTileM + static_cast<int>(rank) * 128 + r_in_cta;
      const int64_t row = static_cast<int64_t>(p.row_start[tile.g]) + m_local;
      const bool rvalid = m_local < p.rows[tile.g] && row < p.x_rows;
      const bool tma = __all_sync(0xffffffffu, rvalid);
      const int warp_row0 = static_cast<int>(row) - lane;
      const uint32_t tbase =
          tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + static_cast<uint32_t>(acc * BN);
      char* orow = static_cast<char*>(p.out) + row * p.n_out * elem_bytes;
      // Wide tiles, plain epilogue: accumulator columns h*256 + [0,128) hold
      // output columns n0 + h*128 + [0,128) (rank 0's B rows), h*256 +
      // [128,256) hold n0 + 256 + h*128 + [0,128) (rank 1's B rows).
      auto wide_plain_half = [&](int h) {
        const int n0 = tile.n_idx * 512;
#pragma unroll 1
        for (int q8 = 0; q8 < 8; ++q8) {
          const int col = n0 + ((q8 >> 2) << 8) + h * 128 + (q8 & 3) * 32;
          if (col >= p.n_out) continue;  // warp-uniform
          uint32_t r[32];
          tmem_ld_32x32b_x32(tbase + h * 256 + q8 * 32, r);
          tmem_ld_wait();
          uint32_t o[16];
#pragma unroll
          for (int q = 0; q < 16; ++q)
            o[q] = pack_bf16x2(__uint_as_float(r[2 * q]), __uint_as_float(r[2 * q + 1]));
          emit(o, tma, row, col, warp_row0, orow, rvalid);
        }
      };
      // Wide tiles, SwiGLU: accumulator columns h*256 + [0,128) are gate and
      // h*256 + [128,256) up of output columns n0 + h*128 + [0,128).
      auto wide_swiglu_half = [&](int h) {
        const int n0 = tile.n_idx * 256;
#pragma unroll 1
        for (int q4 = 0; q4 < 4; ++q4) {
          const int col = n0 + h * 128 + q4 * 32;
          if (col >= p.n_out) continue;  // warp-uniform
          uint32_t gr[32], ur[32];
          tmem_ld_32x32b_x32(tbase + h * 256 + q4 * 32, gr);
          tmem_ld_32x32b_x32(tbase + h * 256 + 128 + q4 * 32, ur);
          tmem_ld_wait();
          uint32_t o[16];
#pragma unroll
          for (int q = 0; q < 16; ++q) {
            const float2 h = swiglu2_f32(
                make_float2(round_bf16(__uint_as_float(gr[2 * q])),
                            round_bf16(__uint_as_float(gr[2 * q + 1]))),
                make_float2(round_bf16(__uint_as_float(ur[2 * q])),
                            round_bf16(__uint_as_float(ur[2 * q + 1]))));
            o[q] = pack_bf16x2(h.x, h.y);
          }
          emit(o, tma, row, col, warp_row0, orow, rvalid);
        }
      };
      if (kWide) {
        // Half h of the accumulator (columns h*256 ..) as soon as the MMA
        // hands it over; its columns are free for the next tile once this
        // CTA's four warps and the partner's have arrived.
        const uint32_t tph = static_cast<uint32_t>(it & 1);
        for (int h = 0; h < 2; ++h) {
          if (!mbar_wait_cluster(tfull_bar(h), tph, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          if (p.epilogue == 0)
            wide_plain_half(h);
          else
            wide_swiglu_half(h);
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive_cluster(h == 0 ? leader_tempty0 : leader_tempty1);
        }
        if (!ok) break;
        ++it;
        continue;
      }
      if (p.epilogue == 2) {
        const int n0 = tile.n_idx * p.bn;
#pragma unroll 1
        for (int c = 0; c < p.bn / 32; ++c) {
          const int col = n0 + c * 32;
          if (col >= p.n_out) break;  // warp-uniform
          uint32_t r[32];
          tmem_ld_32x32b_x32(tbase + c * 32, r);
          tmem_ld_wait();
          uint32_t o[16];
#pragma unroll
          for (int q = 0; q < 16; ++q) o[q] = r[q];
          emit(o, tma, row, col, warp_row0, orow, rvalid);
          if (col + 16 < p.n_out) {
#pragma unroll
            for (int q = 0; q < 16; ++q) o[q] = r[16 + q];
            emit(o, tma, row, col + 16, warp_row0, orow, rvalid);
          }
        }
      } else if (p.epilogue == 0) {
        const int n0 = tile.n_idx * p.bn;
#pragma unroll 1
        for (int c = 0; c < p.bn / 32; ++c) {
          const int col = n0 + c * 32;
          if (col >= p.n_out) break;  // warp-uniform
          uint32_t r[32];
          tmem_ld_32x32b_x32(tbase + c * 32, r);
          tmem_ld_wait();
          uint32_t o[16];
#pragma unroll
          for (int q = 0; q < 16; ++q)
            o[q] = pack_bf16x2(__uint_as_float(r[2 * q]), __uint_as_float(r[2 * q + 1]));
          emit(o, tma, row, col, warp_row0, orow, rvalid);
        }
      } else {
        const int n0 = tile.n_idx * 128;
#pragma unroll 1
        for (int c = 0; c < 128 / 32; ++c) {
          const int col = n0 + c * 32;
          if (col >= p.n_out) break;  // warp-uniform
          uint32_t gr[32], ur[32];
          tmem_ld_32x32b_x32(tbase + c * 32, gr);
          tmem_ld_32x32b_x32(tbase + 128 + c * 32, ur);
          tmem_ld_wait();
          uint32_t o[16];
#pragma unroll
          for (int q = 0; q < 16; ++q) {
            const float2 h = swiglu2_f32(
                make_float2(round_bf16(__uint_as_float(gr[2 * q])),
                            round_bf16(__uint_as_float(gr[2 * q + 1]))),
                make_float2(round_bf16(__uint_as_float(ur[2 * q])),
                            round_bf16(__uint_as_float(ur[2 * q + 1]))));
            o[q] = pack_bf16x2(h.x, h.y);
          }
          emit(o, tma, row, col, warp_row0, orow, rvalid);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(acc == 0 ? leader_tempty0 : leader_tempty1);
      ++it;
    }
    if (lane == 0) bulk_wait_all();  // every tile store has finished
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

// ---------------------------------------------------------------------------
// Group-table construction (single block).
// mode 0: contiguous groups from splits, group g starts at the padded prefix.
// mode 1: expert-parallel receive layout, see moe_grouped_gemm_plan_ep.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(1024) plan_kernel(const int32_t* __restrict__ counts, int n,
                                                    int mode, int num_src, int num_w,
                                                    int64_t align, int32_t* __restrict__ err,
                                                    int32_t* __restrict__ row_start,
                                                    int32_t* __restrict__ rows,
                                                    int32_t* __restrict__ widx,
                                                    int32_t* __restrict__ tmp,
                                                    int32_t* __restrict__ rows_body,
                                                    int32_t* __restrict__ tail_start,
                                                    int32_t* __restrict__ rows_tail,
                                                    int fold_min) {
  __shared__ int64_t warp_sums[32];
  __shared__ int64_t carry_s;
  const int lane = lane_id(), wid = warp_id();
  if (threadIdx.x == 0) {
    *err = 0;
    carry_s = 0;
  }
  __syncthreads();
  for (int i0 = 0; i0 < n; i0 += 1024) {
    const int i = i0 + threadIdx.x;
    int64_t padded = 0;
    if (i < n) {
      const int64_t c = max(counts[i], 0);
      padded = (align > 1) ? ((c + align - 1) / align) * align : c;
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
      const int64_t ws = warp_sums[lane];
      int64_t wincl = ws;
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const int64_t y = __shfl_up_sync(0xffffffffu, wincl, off);
        if (lane >= off) wincl += y;
      }
      warp_sums[lane] = wincl - ws;
    }
    __syncthreads();
    const int64_t cbase = carry_s;
    if (i < n) tmp[i] = static_cast<int32_t>(cbase + warp_sums[wid] + incl - padded);
    __syncthreads();
    if (threadIdx.x == 1023) carry_s = cbase + warp_sums[wid] + incl;
    __syncthreads();
  }
  for (int g = threadIdx.x; g < n; g += 1024) {
    int f = g, w = g;
    if (mode == 1) {
      const int e = g / num_src, s = g - e * num_src;
      f = s * num_w + e;
      w = e;
    }
    const int32_t m = max(counts[f], 0);
    // A group of at least fold_min rows keeps its remainder on the pair
    // kernel as a row-predicated last tile, computed while its weight slab is
    // still in L2; smaller groups split as below.
    const int32_t body = m >= fold_min ? m : (m / pairk::kPairTileM) * pairk::kPairTileM;
    row_start[g] = tmp[f];
    rows[g] = m;
    widx[g] = w;
    // Whole 256-row tiles go to the CTA-pair kernel, the rest (< 256 rows) to
    // the single-CTA kernel's 128-row tiles, which pads at most 127 rows.
    rows_body[g] = body;
    tail_start[g] = tmp[f] + body;
    rows_tail[g] = m - body;
  }
}

struct WsLayout {
  int32_t* err;
  int32_t* row_start;
  int32_t* rows;
  int32_t* widx;
  int32_t* tmp;
  int32_t* rows_body;   // whole 256-row tiles of each group (CTA-pair kernel)
  int32_t* tail_start;  // first row after them
  int32_t* rows_tail;   // remaining rows (single-CTA kernel)
};

size_t ws_array_bytes(int64_t G) {
  return (static_cast<size_t>(G) * 4 + 255) & ~static_cast<size_t>(255);
}
size_t ws_bytes(int64_t G) { return 256 + 7 * ws_array_bytes(G); }

WsLayout ws_layout(const void* ws, int64_t G) {
  char* b = static_cast<char*>(const_cast<void*>(ws));
  const size_t a = ws_array_bytes(G);
  WsLayout l;
  l.err = reinterpret_cast<int32_t*>(b);
  l.row_start = reinterpret_cast<int32_t*>(b + 256);
  l.rows = reinterpret_cast<int32_t*>(b + 256 + a);
  l.widx = reinterpret_cast<int32_t*>(b + 256 + 2 * a);
  l.tmp = reinterpret_cast<int32_t*>(b + 256 + 3 * a);
  l.rows_body = reinterpret_cast<int32_t*>(b + 256 + 4 * a);
  l.tail_start = reinterpret_cast<int32_t*>(b + 256 + 5 * a);
  l.rows_tail = reinterpret_cast<int32_t*>(b + 256 + 6 * a);
  return l;
}

PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

int make_tmap_box(CUtensorMap* m, const void* ptr, uint64_t inner, uint64_t outer,
                  uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle swz,
                  bool fp32 = false);

// 2-D bf16 tensor map over a row-major [outer, inner] matrix, box 64 x 128,
// 128-byte swizzle (one box row = one 128-byte swizzle row).
int make_tmap(CUtensorMap* m, const void* ptr, uint64_t inner, uint64_t outer) {
  return make_tmap_box(m, ptr, inner, outer, static_cast<uint32_t>(BK), 128u,
                       CU_TENSOR_MAP_SWIZZLE_128B);
}

// 2-D tensor map over a row-major [outer, inner] bf16 (or fp32) matrix.
int make_tmap_box(CUtensorMap* m, const void* ptr, uint64_t inner, uint64_t outer,
                  uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle swz, bool fp32) {
  auto encode = get_encode_fn();
  if (encode == nullptr) {
    set_last_error("grouped_gemm: cuTensorMapEncodeTiled unavailable");
    return MOE_ERR_CUDA;
  }
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {inner * (fp32 ? 4 : 2)};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1u, 1u};
  const CUresult r = encode(m, fp32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16,
                            2, const_cast<void*>(ptr), dims,
                            strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_last_error("grouped_gemm: cuTensorMapEncodeTiled failed (%d)", static_cast<int>(r));
    return MOE_ERR_CUDA;
  }
  return MOE_OK;
}

// Clusters of 2 that can be resident at once (0 if the pair kernel cannot run).
int pair_clusters(int dev) {
  static std::mutex mu;
  static int cache[64];
  static bool init[64] = {};
  std::lock_guard<std::mutex> lock(mu);
  if (dev >= 0 && dev < 64 && init[dev]) return cache[dev];
  int n = 0;
  if (cudaFuncSetAttribute(grouped_gemm_pair_kernel<false>,
                           cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(pairk::kPairSmemBytes)) == cudaSuccess &&
      cudaFuncSetAttribute(grouped_gemm_pair_kernel<true>,
                           cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(pairk::kWideSmemBytes)) == cudaSuccess) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * 74);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = pairk::kPairSmemBytes;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int nw = 0;
    if (cudaOccupancyMaxActiveClusters(&n, grouped_gemm_pair_kernel<false>, &cfg) != cudaSuccess ||
        cudaOccupancyMaxActiveClusters(&nw, grouped_gemm_pair_kernel<true>, &cfg) != cudaSuccess)
      n = 0;
    n = std::min(n, nw);
  }
  cudaGetLastError();  // clear a non-sticky error from an unsupported query
  if (dev >= 0 && dev < 64) {
    cache[dev] = n;
    init[dev] = true;
  }
  return n;
}

// Weight bytes of one slab chunk of the N-chunk walk: about a quarter of L2,
// so the chunk stays resident while a group's M-tiles stream past it (the
// measured fc1 slab of 58.7 MB did not, the fc2 slab of 29.4 MB did).
constexpr int64_t kSlabChunkBytes = 32ll << 20;
constexpr int kNChunkDefault = -1;
// Wide pair tiles (256x512) against square ones (256x256), measured in the
// layer at the 1 kW cap, interleaved in one process: fc1 (K=7168) 6.82-6.86
// against 7.28 ms, fc2 (K=2048) 3.78 against 3.55-3.73 ms. With a single
// accumulator the epilogue overlaps only the first and last k-blocks of a
// tile, which hides it when the reduction is long.
constexpr int kWideDefault = 1;
constexpr int64_t kWideMinK = 4096;

int env_int(const char* name, int def, int lo, int hi) {
  const char* e = getenv(name);
  if (e == nullptr || e[0] == 0) return def;
  const int v = atoi(e);
  return (v < lo || v > hi) ? def : v;
}

// Smallest group whose remainder (rows beyond its whole 256-row tiles) stays
// on the pair kernel: MOE_GEMM_FOLD=1 (default) folds the remainder of every
// group that has whole tiles, computed right after that group's other tiles
// while its weight slab is still in L2; 0 hands every remainder to the
// single-CTA kernel, which then streams those slabs from HBM once more.
int fold_min() {
  static const int v = env_int("MOE_GEMM_FOLD", 1, 0, 1) == 1 ? pairk::kPairTileM : 0x7fffffff;
  return v;
}

bool pair_enabled() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("MOE_GEMM_PAIR");
    v = (e != nullptr && e[0] == '0') ? 0 : 1;
  }
  return v == 1;
}

int ensure_smem_attr() {
  int dev = 0;
  MOE_CUDA_CALL(cudaGetDevice(&dev), "cudaGetDevice");
  static std::mutex mu;
  static bool done[64] = {};
  std::lock_guard<std::mutex> lock(mu);
  if (dev < 64 && done[dev]) return MOE_OK;
  MOE_CUDA_CALL(cudaFuncSetAttribute(grouped_gemm_kernel,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     static_cast<int>(kSmemBytes)),
                "cudaFuncSetAttribute(grouped_gemm)");
  if (dev < 64) done[dev] = true;
  return MOE_OK;
}

}  // namespace gg
}  // namespace moe

using namespace moe;

extern "C" int moe_grouped_gemm_workspace_size(int64_t G, size_t* bytes) {
  MOE_REQUIRE(bytes != nullptr, "grouped_gemm_workspace_size: null output");
  MOE_REQUIRE(G >= 1 && G <= (1 << 24), "grouped_gemm: G=%lld out of range", (long long)G);
  *bytes = gg::ws_bytes(G);
  return MOE_OK;
}

static int check_ws(const void* ws, size_t bytes, int64_t G) {
  MOE_REQUIRE(ws != nullptr && bytes >= gg::ws_bytes(G),
              "grouped_gemm: workspace too small (%zu < %zu)", bytes, gg::ws_bytes(G));
  MOE_REQUIRE((reinterpret_cast<uintptr_t>(ws) & 255) == 0,
              "grouped_gemm: workspace must be 256-byte aligned");
  return MOE_OK;
}

extern "C" int moe_grouped_gemm_plan_splits(const int32_t* m_splits, int64_t G, int64_t align,
                                            void* workspace, size_t workspace_bytes,
                                            moe_stream_t stream) {
  MOE_REQUIRE(G >= 1 && G <= (1 << 24), "grouped_gemm_plan: G=%lld out of range", (long long)G);
  MOE_REQUIRE(align >= 1 && align <= 4096, "grouped_gemm_plan: align=%lld out of [1,4096]",
              (long long)align);
  MOE_REQUIRE(m_splits != nullptr, "grouped_gemm_plan: null m_splits");
  int st = check_ws(workspace, workspace_bytes, G);
  if (st) return st;
  gg::WsLayout l = gg::ws_layout(workspace, G);
  gg::plan_kernel<<<1, 1024, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      m_splits, static_cast<int>(G), 0, 1, static_cast<int>(G), align, l.err, l.row_start, l.rows,
      l.widx, l.tmp, l.rows_body, l.tail_start, l.rows_tail, gg::fold_min());
  MOE_CUDA_CHECK_LAUNCH("grouped_gemm plan");
  return MOE_OK;
}

extern "C" int moe_grouped_gemm_plan_ep(const int32_t* counts, int64_t num_src, int64_t num_w,
                                        void* workspace, size_t workspace_bytes,
                                        moe_stream_t stream) {
  MOE_REQUIRE(num_src >= 1 && num_w >= 1 && num_src * num_w <= (1 << 24),
              "grouped_gemm_plan_ep: bad num_src=%lld num_w=%lld", (long long)num_src,
              (long long)num_w);
  MOE_REQUIRE(counts != nullptr, "grouped_gemm_plan_ep: null counts");
  const int64_t G = num_src * num_w;
  int st = check_ws(workspace, workspace_bytes, G);
  if (st) return st;
  gg::WsLayout l = gg::ws_layout(workspace, G);
  gg::plan_kernel<<<1, 1024, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      counts, static_cast<int>(G), 1, static_cast<int>(num_src), static_cast<int>(num_w), 1,
      l.err, l.row_start, l.rows, l.widx, l.tmp, l.rows_body, l.tail_start, l.rows_tail,
      gg::fold_min());
  MOE_CUDA_CHECK_LAUNCH("grouped_gemm plan_ep");
  return MOE_OK;
}

// b_mn = 0: w [num_w, N, K], out = x @ w[g]^T; b_mn = 1: w [num_w, K, N],
// out = x @ w[g] (B staged MN-major; bf16 or fp32 output, no SwiGLU).
static int grouped_gemm_run(const void* x, const void* w, void* out, int64_t x_rows, int64_t G,
                            int64_t num_w, int64_t N, int64_t K, int32_t epilogue,
                            const void* workspace, size_t workspace_bytes, moe_stream_t stream,
                            int b_mn) {
  MOE_REQUIRE(epilogue >= 0 && epilogue <= 2, "grouped_gemm: epilogue must be 0, 1 or 2");
  MOE_REQUIRE(!b_mn || epilogue != 1, "grouped_gemm_nn: no SwiGLU epilogue");
  MOE_REQUIRE(!b_mn || num_w * K < (1ll << 31), "grouped_gemm_nn: num_w*K too large");
  MOE_REQUIRE(G >= 1 && num_w >= 1, "grouped_gemm: G=%lld num_w=%lld", (long long)G,
              (long long)num_w);
  MOE_REQUIRE(x_rows >= 0 && x_rows < (1ll << 31), "grouped_gemm: x_rows=%lld out of range",
              (long long)x_rows);
  MOE_REQUIRE(K >= 8 && K % 8 == 0, "grouped_gemm: K=%lld must be a positive multiple of 8",
              (long long)K);
  MOE_REQUIRE(N >= 8 && N % 8 == 0, "grouped_gemm: N=%lld must be a positive multiple of 8",
              (long long)N);
  MOE_REQUIRE(epilogue != 1 || N % 16 == 0, "grouped_gemm: SwiGLU needs N=2F with F %% 8 == 0");
  MOE_REQUIRE(num_w * N < (1ll << 31), "grouped_gemm: num_w*N too large");
  int st = check_ws(workspace, workspace_bytes, G);
  if (st) return st;
  if (x_rows == 0) return MOE_OK;
  MOE_REQUIRE(x && w && out, "grouped_gemm: null pointer");
  MOE_REQUIRE(((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(w) |
                reinterpret_cast<uintptr_t>(out)) & 15) == 0,
              "grouped_gemm: x, w and out must be 16-byte aligned");
  st = gg::ensure_smem_attr();
  if (st) return st;

  CUtensorMap ta, tb;
  st = gg::make_tmap(&ta, x, static_cast<uint64_t>(K), static_cast<uint64_t>(x_rows));
  if (st) return st;
  if (b_mn)  // w viewed as [num_w*K, N]: 64-column x 64-row boxes, rows = reduction index
    st = gg::make_tmap_box(&tb, w, static_cast<uint64_t>(N), static_cast<uint64_t>(num_w * K), 64u,
                           64u, CU_TENSOR_MAP_SWIZZLE_128B);
  else
    st = gg::make_tmap(&tb, w, static_cast<uint64_t>(K), static_cast<uint64_t>(num_w * N));
  if (st) return st;

  gg::WsLayout l = gg::ws_layout(workspace, G);
  gg::Params p;
  p.row_start = l.row_start;
  p.rows = l.rows;
  p.widx = l.widx;
  p.err = l.err;
  p.out = out;
  p.x_rows = x_rows;
  p.G = static_cast<int>(G);
  p.n_w = static_cast<int>(N);
  p.epilogue = epilogue;
  if (epilogue == 1) {
    p.f_half = static_cast<int>(N / 2);
    p.n_out = p.f_half;
    p.n_tiles = (p.f_half + 127) / 128;
  } else {
    p.f_half = 0;
    p.n_out = static_cast<int>(N);
    p.n_tiles = static_cast<int>((N + gg::BN - 1) / gg::BN);
  }
  p.bn = gg::BN;
  p.b_mn = b_mn;
  p.k_rows = static_cast<int>(K);
  p.num_kb = static_cast<int>((K + gg::BK - 1) / gg::BK);
  static const int raster = gg::env_int("MOE_GEMM_RASTER", gg::pairk::kPairRaster, 1, 64);
  static const int l2_mode = gg::env_int("MOE_GEMM_L2", 0, 0, 4);
  p.raster = raster;
  p.l2_mode = l2_mode;
  p.n_chunk = 0;

  int dev = 0;
  MOE_CUDA_CALL(cudaGetDevice(&dev), "cudaGetDevice");
  const int clusters = gg::pair_enabled() ? gg::pair_clusters(dev) : 0;
  if (clusters > 0) {
    // Epilogue tile stores: 32 rows x 64 bytes (32 bf16 or 16 fp32 columns).
    CUtensorMap to;
    st = gg::make_tmap_box(&to, out, static_cast<uint64_t>(p.n_out), static_cast<uint64_t>(x_rows),
                           epilogue == 2 ? 16u : 32u, 32u, CU_TENSOR_MAP_SWIZZLE_64B, epilogue == 2);
    if (st) return st;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * clusters);
    cfg.blockDim = dim3(gg::kThreads);
    cfg.dynamicSmemBytes = gg::pairk::kPairSmemBytes;
    cfg.stream = reinterpret_cast<cudaStream_t>(stream);
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    static const bool split = gg::env_int("MOE_GEMM_SPLIT", 1, 0, 1) == 1;
    gg::Params pb = p;
    if (split) pb.rows = l.rows_body;
    // Without SwiGLU, N is cut into equal N-tiles of at most 256 columns (a
    // multiple of 32), e.g. 320 -> 2 x 160 rather than 256 + a 64-column tile
    // padded to 256. The B box of the pair then holds bn/2 rows per CTA.
    CUtensorMap tbp = tb;
    if (epilogue != 1 && !b_mn) {
      const int nt = static_cast<int>((N + gg::BN - 1) / gg::BN);
      const int per = static_cast<int>((N + nt - 1) / nt);
      pb.bn = std::min(gg::BN, (per + 31) / 32 * 32);
      pb.n_tiles = static_cast<int>((N + pb.bn - 1) / pb.bn);
      if (pb.bn != gg::BN) {
        st = gg::make_tmap_box(&tbp, w, static_cast<uint64_t>(K), static_cast<uint64_t>(num_w * N),
                               static_cast<uint32_t>(gg::BK), static_cast<uint32_t>(pb.bn / 2),
                               CU_TENSOR_MAP_SWIZZLE_128B);
        if (st) return st;
      }
    }
    // Wide 256x512 tiles where N (or F for SwiGLU) is a whole number of them
    // and the reduction is deep enough to hide most of their epilogue:
    // MOE_GEMM_WIDE=1 (default) for K >= kWideMinK, 2 for every K, 0 never.
    static const int wide_env = gg::env_int("MOE_GEMM_WIDE", gg::kWideDefault, 0, 2);
    const bool wide = wide_env != 0 && (wide_env == 2 || K >= gg::kWideMinK) &&
                      ((epilogue == 0 && N % 512 == 0) ||
                       (epilogue == 1 && !b_mn && p.f_half % 256 == 0));
    if (wide && !b_mn) {  // one 256-row box per CTA; MN-major B keeps its 64x64 boxes
      st = gg::make_tmap_box(&tbp, w, static_cast<uint64_t>(K), static_cast<uint64_t>(num_w * N),
                             static_cast<uint32_t>(gg::BK), 256u, CU_TENSOR_MAP_SWIZZLE_128B);
      if (st) return st;
    }
    if (wide) {
      pb.bn = 512;
      pb.n_tiles = epilogue == 1 ? p.f_half / 256 : static_cast<int>(N / 512);
      cfg.dynamicSmemBytes = gg::pairk::kWideSmemBytes;
    }
    // Weight-slab chunks: MOE_GEMM_NCHUNK=-1 picks the most N-tiles whose
    // weight rows fit in kSlabChunkBytes, k > 0 takes k N-tiles, 0 keeps the
    // super-rows of MOE_GEMM_RASTER.
    static const int nchunk_env = gg::env_int("MOE_GEMM_NCHUNK", gg::kNChunkDefault, -1, 1024);
    if (nchunk_env != 0) {
      const int64_t ntile_bytes = (wide ? 512 : epilogue == 1 ? 256 : pb.bn) * K * 2;
      const int64_t fit = std::max<int64_t>(1, gg::kSlabChunkBytes / ntile_bytes);
      pb.n_chunk = static_cast<int>(
          std::min<int64_t>(pb.n_tiles, nchunk_env > 0 ? nchunk_env : fit));
    }
    if (wide)
      MOE_CUDA_CALL(cudaLaunchKernelEx(&cfg, gg::grouped_gemm_pair_kernel<true>, ta, tbp, to, pb),
                    "grouped_gemm wide pair launch");
    else
      MOE_CUDA_CALL(cudaLaunchKernelEx(&cfg, gg::grouped_gemm_pair_kernel<false>, ta, tbp, to, pb),
                    "grouped_gemm pair launch");
    if (!split) return MOE_OK;
    // Remainders of every group (< 256 rows) on 128-row single-CTA tiles.
    gg::Params pt = p;
    pt.row_start = l.tail_start;
    pt.rows = l.rows_tail;
    gg::grouped_gemm_kernel<<<num_sms(dev), gg::kThreads, gg::kSmemBytes,
                              reinterpret_cast<cudaStream_t>(stream)>>>(ta, tb, pt);
    MOE_CUDA_CHECK_LAUNCH("grouped_gemm tail launch");
    return MOE_OK;
  }
  const int grid = num_sms(dev);
  gg::grouped_gemm_kernel<<<grid, gg::kThreads, gg::kSmemBytes,
                            reinterpret_cast<cudaStream_t>(stream)>>>(ta, tb, p);
  MOE_CUDA_CHECK_LAUNCH("grouped_gemm launch");
  return MOE_OK;
}

extern "C" int moe_grouped_gemm(const void* x, const void* w, void* out, int64_t x_rows, int64_t G,
                                int64_t num_w, int64_t N, int64_t K, int32_t epilogue,
                                const void* workspace, size_t workspace_bytes,
                                moe_stream_t stream) {
  return grouped_gemm_run(x, w, out, x_rows, G, num_w, N, K, epilogue, workspace,
                          workspace_bytes, stream, 0);
}

extern "C" int moe_grouped_gemm_nn(const void* x, const void* w, void* out, int64_t x_rows,
                                   int64_t G, int64_t num_w, int64_t N, int64_t K,
                                   int32_t epilogue, const void* workspace,
                                   size_t workspace_bytes, moe_stream_t stream) {
  return grouped_gemm_run(x, w, out, x_rows, G, num_w, N, K, epilogue, workspace,
                          workspace_bytes, stream, 1);
}

extern "C" int moe_grouped_gemm_check(const void* workspace, size_t workspace_bytes,
                                      moe_stream_t stream, int32_t* device_error) {
  MOE_REQUIRE(device_error != nullptr, "grouped_gemm_check: null output");
  MOE_REQUIRE(workspace != nullptr && workspace_bytes >= 256, "grouped_gemm_check: bad workspace");
  int32_t v = 0;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  MOE_CUDA_CALL(cudaMemcpyAsync(&v, workspace, sizeof(v), cudaMemcpyDeviceToHost, s),
                "grouped_gemm_check copy");
  MOE_CUDA_CALL(cudaStreamSynchronize(s), "grouped_gemm_check sync");
  *device_error = v;
  return v == 0 ? MOE_OK : MOE_ERR_DEVICE;
}
