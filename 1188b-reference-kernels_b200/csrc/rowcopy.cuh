// Row-copy building blocks shared by the permute / combine kernels and the
// fused expert-parallel dispatch / combine kernels: one 128-thread CTA per
// token, map entries compacted in ascending expert order with a warp ballot,
// rows moved as 16-, 4- or 2-byte vectors of bf16.
#pragma once

#include "moe_common.cuh"

namespace moe {
namespace rowcopy {

constexpr int kRowThreads = 128;
constexpr int kRowWarps = kRowThreads / 32;

template <typename IdxT, bool kTrans>
MOE_DEVICE int64_t load_map(const IdxT* map, int64_t T, int E, int64_t t, int e) {
  return kTrans ? static_cast<int64_t>(__ldg(map + static_cast<int64_t>(e) * T + t))
                : static_cast<int64_t>(__ldg(map + t * E + e));
}

// Ordered compaction of one window of up to 128 map entries: valid entries are
// written to s_idx[0..n) in ascending thread (= expert) order. Returns n.
MOE_DEVICE int compact_window(bool valid, int* s_wcnt, int& pos) {
  const int lane = lane_id(), wid = warp_id();
  const unsigned b = __ballot_sync(0xffffffffu, valid);
  if (lane == 0) s_wcnt[wid] = __popc(b);
  __syncthreads();
  int before = 0, total = 0;
#pragma unroll
  for (int w = 0; w < kRowWarps; ++w) {
    const int c = s_wcnt[w];
    before += (w < wid) ? c : 0;
    total += c;
  }
  pos = before + __popc(b & ((1u << lane) - 1u));
  return total;
}

// A row moves as vectors V of 8 (uint4), 2 (uint32_t) or 1 (uint16_t) bf16
// values; the widest one that the row length and pointer alignment allow.
template <typename V>
struct VecTraits;
template <>
struct VecTraits<uint4> {
  static constexpr int kElems = 8;
  MOE_DEVICE static void unpack(const uint4& q, float (&f)[8]) {
    const uint32_t u[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      f[2 * i] = bf16_lo(u[i]);
      f[2 * i + 1] = bf16_hi(u[i]);
    }
  }
  MOE_DEVICE static uint4 pack(const float (&f)[8]) {
    return make_uint4(pack_bf16x2(f[0], f[1]), pack_bf16x2(f[2], f[3]), pack_bf16x2(f[4], f[5]),
                      pack_bf16x2(f[6], f[7]));
  }
};
template <>
struct VecTraits<uint32_t> {
  static constexpr int kElems = 2;
  MOE_DEVICE static void unpack(const uint32_t& q, float (&f)[2]) {
    f[0] = bf16_lo(q);
    f[1] = bf16_hi(q);
  }
  MOE_DEVICE static uint32_t pack(const float (&f)[2]) { return pack_bf16x2(f[0], f[1]); }
};
template <>
struct VecTraits<uint16_t> {
  static constexpr int kElems = 1;
  MOE_DEVICE static void unpack(const uint16_t& q, float (&f)[1]) {
    f[0] = __uint_as_float(static_cast<uint32_t>(q) << 16);
  }
  MOE_DEVICE static uint16_t pack(const float (&f)[1]) {
    return static_cast<uint16_t>(pack_bf16x2(f[0], 0.f) & 0xFFFFu);
  }
};

template <typename V>
MOE_DEVICE void accum_vec(float (&acc)[VecTraits<V>::kElems], const V& q, float w, bool weighted) {
  constexpr int kE = VecTraits<V>::kElems;
  float f[kE];
  VecTraits<V>::unpack(q, f);
#pragma unroll
  for (int i = 0; i < kE; ++i)
    acc[i] = weighted ? __fadd_rn(acc[i], __fmul_rn(w, f[i])) : __fadd_rn(acc[i], f[i]);
}

// Widest vector the row length and both row pointers allow: 16, 4 or 2 bytes.
inline int vec_bytes(const void* a, const void* b, int64_t H) {
  const uintptr_t m = reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b);
  if (H % 8 == 0 && (m & 15) == 0) return 16;
  if (H % 2 == 0 && (m & 3) == 0) return 4;
  return 2;
}


}  // namespace rowcopy
}  // namespace moe
