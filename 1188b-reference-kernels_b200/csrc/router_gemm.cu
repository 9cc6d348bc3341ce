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
// One CTA owns 128 tokens and ALL E experts of them: E <= 512 fp32 columns of
// TMEM (two accumulators when E <= 256, so the epilogue of one tile overlaps
// the mainloop of the next). Warp 0 is the TMA producer (128 x 64 x-tile plus
// E x 64 W-tile per stage, 128-byte swizzle, as many stages as fit), warp 1
// allocates TMEM and issues tcgen05.mma (M=128, N = E in pieces of <= 256,
// K=16), warps 2-5 are the epilogue: each thread owns one token's row of the
// accumulator and reads it 32 columns at a time (tcgen05.ld 32x32b), keeping a
// register-resident sorted top-k. The selection, the softmax maximum, the
// normalisers (including their summation order) and the gate formula are
// those of the warp-per-row router kernel in routing.cu, so both produce the
// same bits from the same logits. Dense outputs are zero-filled by each warp
// with coalesced 16-byte stores over its 32 contiguous rows, then each thread
// writes its k selected entries.
//
// Every wait is bounded (2 s); on timeout the kernel records an error code in
// the caller's device word, drains its own copies and MMAs, frees TMEM and
// returns.
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

constexpr int BM = 128;
constexpr int BK = 64;
constexpr int kThreads = 192;
constexpr int kMaxE = 512;
constexpr int kMaxStages = 8;
constexpr uint32_t kABytes = BM * BK * 2;  // 16 KB
constexpr size_t kSmemMax = 232448;       // dynamic shared memory per block on sm_100
constexpr size_t kSmemTail = 512;         // barriers, TMEM slot, abort flag

constexpr int kErrTimeoutProducer = 1;
constexpr int kErrTimeoutMma = 2;
constexpr int kErrTimeoutEpilogue = 3;

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
  int m_tiles;
  int stages;
  int b_box_rows;
  int b_boxes;
  int acc_stride;  // TMEM columns between the two accumulators
  int n_acc;       // 1 or 2
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

template <int KMAX>
__global__ void __launch_bounds__(kThreads, 1)
    router_gemm_topk_kernel(const __grid_constant__ CUtensorMap tmap_x,
                            const __grid_constant__ CUtensorMap tmap_w, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  const uint32_t base = (raw_addr + 1023u) & ~1023u;
  uint8_t* base_ptr = smem_raw + (base - raw_addr);
  const uint32_t stage_bytes = kABytes + static_cast<uint32_t>(p.E) * (BK * 2);
  const int S = p.stages;
  uint64_t* bars = reinterpret_cast<uint64_t*>(base_ptr + static_cast<size_t>(S) * stage_bytes);
  const uint32_t bar0 = smem_u32(bars);
  auto full_bar = [&](int s) { return bar0 + 8u * s; };
  auto empty_bar = [&](int s) { return bar0 + 8u * (kMaxStages + s); };
  auto tfull_bar = [&](int a) { return bar0 + 8u * (2 * kMaxStages + a); };
  auto tempty_bar = [&](int a) { return bar0 + 8u * (2 * kMaxStages + 2 + a); };
  const uint32_t drain_bar = bar0 + 8u * (2 * kMaxStages + 4);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * kMaxStages + 5);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = warp_id();
  const int lane = lane_id();

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
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
    tma_prefetch_desc(&tmap_x);
    tma_prefetch_desc(&tmap_w);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), p.tmem_cols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      const uint64_t pol_x = l2_policy_evict_first();   // every x row is read once
      const uint64_t pol_w = l2_policy_evict_last();    // W is read by every CTA
      int stage = 0;
      uint32_t phase = 0;
      int issued[kMaxStages];
#pragma unroll
      for (int s = 0; s < kMaxStages; ++s) issued[s] = -1;
      bool ok = true;
      for (int t = blockIdx.x; ok && t < p.m_tiles; t += gridDim.x) {
        const int row0 = t * BM;
        for (int kb = 0; kb < p.num_kb; ++kb) {
          if (!mbar_wait(empty_bar(stage), phase ^ 1u, abort_flag)) {
            ok = false;
            break;
          }
          const uint32_t sa = base + static_cast<uint32_t>(stage) * stage_bytes;
          const uint32_t sb = sa + kABytes;
          mbar_arrive_expect_tx(full_bar(stage), stage_bytes);
          tma_load_2d(sa, &tmap_x, kb * BK, row0, full_bar(stage), pol_x);
          for (int j = 0; j < p.b_boxes; ++j)
            tma_load_2d(sb + static_cast<uint32_t>(j * p.b_box_rows) * (BK * 2), &tmap_w, kb * BK,
                        j * p.b_box_rows, full_bar(stage), pol_w);
          issued[stage] = static_cast<int>(phase);
          if (++stage == S) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok) {
        raise_abort(abort_flag, p.err, kErrTimeoutProducer);
        for (int s = 0; s < S; ++s)
          if (issued[s] >= 0) wait_drain(full_bar(s), static_cast<uint32_t>(issued[s]));
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const int n_pieces = (p.E + 255) / 256;
      int stage = 0;
      uint32_t phase = 0;
      int it = 0;
      bool ok = true;
      bool issued_any = false;
      for (int t = blockIdx.x; ok && t < p.m_tiles; t += gridDim.x) {
        const int acc = p.n_acc == 2 ? (it & 1) : 0;
        const uint32_t aph =
            static_cast<uint32_t>(p.n_acc == 2 ? ((it >> 1) & 1) : (it & 1));
        if (!mbar_wait(tempty_bar(acc), aph ^ 1u, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * p.acc_stride);
        for (int kb = 0; kb < p.num_kb; ++kb) {
          if (!mbar_wait(full_bar(stage), phase, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = base + static_cast<uint32_t>(stage) * stage_bytes;
          const uint32_t sb = sa + kABytes;
          const uint64_t ad = umma_desc_k_sw128(sa);
          for (int pc = 0; pc < n_pieces; ++pc) {
            const int n0 = pc * 256;
            const int nw = min(256, p.E - n0);
            const uint32_t idesc = umma_idesc_bf16_f32(BM, nw);
            const uint64_t bd = umma_desc_k_sw128(sb + static_cast<uint32_t>(n0) * (BK * 2));
#pragma unroll
            for (int k = 0; k < BK / 16; ++k)
              umma_bf16(d_tmem + static_cast<uint32_t>(n0), ad + 2ull * k, bd + 2ull * k, idesc,
                        (kb | k) != 0 ? 1u : 0u);
          }
          issued_any = true;
          umma_commit(empty_bar(stage));
          if (++stage == S) {
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
    const int quad = warp & 3;  // TMEM lanes 32*quad .. 32*quad+31
    const int E = p.E;
    int it = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < p.m_tiles; t += gridDim.x) {
      const int acc = p.n_acc == 2 ? (it & 1) : 0;
      const uint32_t aph = static_cast<uint32_t>(p.n_acc == 2 ? ((it >> 1) & 1) : (it & 1));
      if (!mbar_wait(tfull_bar(acc), aph, abort_flag)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const int64_t wrow0 = static_cast<int64_t>(t) * BM + quad * 32;  // warp's first token
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
      // Pass 1: logits out, selection, row maximum of the scores.
#pragma unroll 1
      for (int c0 = 0; c0 < E; c0 += 32) {
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
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            float x = __uint_as_float(r[j]);
            if (p.bias != nullptr) x += __ldg(p.bias + c0 + j);
            m = fmaxf(m, x);
            topk_insert<KMAX>(sel, sv, rank_key(x, c0 + j), x);
          }
        }
      }
      // Normalisers, in the summation order of the warp-per-row router:
      // lane l of that kernel sums columns l, l+32, ... in turn, then the 32
      // partial sums meet in an xor butterfly (offsets 16, 8, 4, 2, 1).
      float denom = 1.f, gsum = 1.f;
      if (p.route && p.mode == 1) {
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
            uint32_t r[32];
            tmem_ld_32x32b_x32(tbase + static_cast<uint32_t>(c0), r);
            tmem_ld_wait();
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              float x = __uint_as_float(r[j]);
              if (p.bias != nullptr) x += __ldg(p.bias + c0 + j);
              part[j] += expf(x - m);
            }
          }
#pragma unroll
          for (int off = 16; off > 0; off >>= 1) {
            float nxt[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) nxt[j] = part[j] + part[j ^ off];
#pragma unroll
            for (int j = 0; j < 32; ++j) part[j] = nxt[j];
          }
          denom = part[0];
        }
      } else if (p.route && p.mode == 2 && p.renorm) {
        float s = 0.f;
#pragma unroll
        for (int j = 0; j < KMAX; ++j)
          if (j < p.k) s += key_value(sel[j]);
        gsum = s;
      }
      // The accumulator is no longer needed: hand it back to the MMA warp.
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(tempty_bar(acc));
      ++it;

      if (p.route) {
        auto gate_of = [&](float x) {
          if (p.mode == 1) return expf(x - m) / denom;
          if (p.mode == 2 && p.renorm) return x / gsum;
          return x;
        };
        if (rvalid) {
#pragma unroll
          for (int j = 0; j < KMAX; ++j) {
            if (j < p.k) {
              if (p.vals != nullptr) p.vals[row * p.k + j] = gate_of(sv[j]);
              if (p.idx != nullptr) p.idx[row * p.k + j] = key_column(sel[j]);
            }
          }
        }
        if (p.rmap != nullptr || p.probs != nullptr) {
          // Zero the warp's contiguous rows with coalesced stores, then place
          // each token's k entries (ordered after the zeros by __syncwarp).
          const int64_t nrows = min(static_cast<int64_t>(32), p.T - wrow0);
          if (nrows > 0) {
            const uint4 z = make_uint4(0u, 0u, 0u, 0u);
            if (p.probs != nullptr) {
              uint4* dst = reinterpret_cast<uint4*>(p.probs + wrow0 * E);
              const int64_t n16 = nrows * E / 4;
              for (int64_t i = lane; i < n16; i += 32) dst[i] = z;
            }
            if (p.rmap != nullptr) {
              uint4* dst = reinterpret_cast<uint4*>(p.rmap + wrow0 * E);
              const int64_t n16 = nrows * E / 16;
              for (int64_t i = lane; i < n16; i += 32) dst[i] = z;
            }
          }
          __syncwarp();
          if (rvalid) {
#pragma unroll
            for (int j = 0; j < KMAX; ++j) {
              if (j < p.k) {
                const int c = key_column(sel[j]);
                if (p.probs != nullptr) p.probs[row * E + c] = gate_of(sv[j]);
                if (p.rmap != nullptr) p.rmap[row * E + c] = 1;
              }
            }
          }
        }
      }
    }
    if (!ok && lane == 0) raise_abort(abort_flag, p.err, kErrTimeoutEpilogue);
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, p.tmem_cols);
  }
}

size_t smem_bytes(int stages, int E) {
  return 1024 + static_cast<size_t>(stages) * (kABytes + static_cast<size_t>(E) * BK * 2) +
         kSmemTail;
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

  // Stages: as many x-tile + W-tile stages as fit in shared memory.
  const uint32_t stage_bytes = rg::kABytes + static_cast<uint32_t>(E) * (rg::BK * 2);
  int stages = static_cast<int>((rg::kSmemMax - 1024 - rg::kSmemTail) / stage_bytes);
  stages = stages > rg::kMaxStages ? rg::kMaxStages : stages;
  MOE_REQUIRE(stages >= 2, "router_gemm_topk: E=%lld leaves fewer than two stages",
              (long long)E);
  // W boxes: the largest power of two <= 256 rows that divides E.
  int bbr = 256;
  while (E % bbr != 0) bbr >>= 1;

  CUtensorMap tx, tw;
  st = gg::make_tmap_box(&tx, x, static_cast<uint64_t>(H), static_cast<uint64_t>(T),
                         static_cast<uint32_t>(rg::BK), static_cast<uint32_t>(rg::BM),
                         CU_TENSOR_MAP_SWIZZLE_128B, false);
  if (st) return st;
  st = gg::make_tmap_box(&tw, w, static_cast<uint64_t>(H), static_cast<uint64_t>(E),
                         static_cast<uint32_t>(rg::BK), static_cast<uint32_t>(bbr),
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
  p.m_tiles = static_cast<int>((T + rg::BM - 1) / rg::BM);
  p.stages = stages;
  p.b_box_rows = bbr;
  p.b_boxes = static_cast<int>(E / bbr);
  int acc = 32;
  while (acc < E) acc <<= 1;
  p.acc_stride = acc;
  p.n_acc = 2 * acc <= 512 ? 2 : 1;
  p.tmem_cols = static_cast<uint32_t>(p.n_acc * acc);

  int dev = 0;
  MOE_CUDA_CALL(cudaGetDevice(&dev), "cudaGetDevice");
  const int sms = num_sms(dev);
  const int grid = p.m_tiles < sms ? p.m_tiles : sms;
  const size_t smem = rg::smem_bytes(stages, p.E);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (k <= 8)
    rg::router_gemm_topk_kernel<8><<<grid, rg::kThreads, smem, s>>>(tx, tw, p);
  else
    rg::router_gemm_topk_kernel<16><<<grid, rg::kThreads, smem, s>>>(tx, tw, p);
  MOE_CUDA_CHECK_LAUNCH("router_gemm_topk launch");
  return MOE_OK;
}
