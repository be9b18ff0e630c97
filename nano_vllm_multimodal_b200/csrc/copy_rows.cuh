// Row copies with the widest vector that every address and stride allows.
#pragma once

#include "nib_common.cuh"

namespace nib {

template <int VW> struct VecOf;
template <> struct VecOf<16> { using type = uint4; };
template <> struct VecOf<8> { using type = uint2; };
template <> struct VecOf<4> { using type = uint32_t; };
template <> struct VecOf<2> { using type = uint16_t; };

// Largest vector width (16/8/4/2 bytes) dividing every value in `vals`
// (addresses and byte strides/sizes).
inline int pick_vec_width(std::initializer_list<uint64_t> vals) {
  uint64_t acc = 0;
  for (uint64_t v : vals) acc |= v;
  if ((acc & 15u) == 0) return 16;
  if ((acc & 7u) == 0) return 8;
  if ((acc & 3u) == 0) return 4;
  return 2;
}

// One warp copies one row of `units` VW-byte vectors, 4 vectors per lane in
// flight (all loads of a round are issued before its stores).
template <int VW>
__device__ __forceinline__ void warp_copy_row(char* __restrict__ dst, const char* __restrict__ src,
                                              int units, int lane) {
  using V = typename VecOf<VW>::type;
  const V* s = reinterpret_cast<const V*>(src);
  V* d = reinterpret_cast<V*>(dst);
  for (int base = 0; base < units; base += 128) {
    V buf[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int u = base + i * 32 + lane;
      if (u < units) buf[i] = __ldg(s + u);
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int u = base + i * 32 + lane;
      if (u < units) d[u] = buf[i];
    }
  }
}

template <int VW>
__device__ __forceinline__ void warp_zero_row(char* __restrict__ dst, int units, int lane) {
  using V = typename VecOf<VW>::type;
  V* d = reinterpret_cast<V*>(dst);
  for (int u = lane; u < units; u += 32) d[u] = V{};
}

#define NIB_VW_SWITCH(vw, VW_, ...)                  \
  switch (vw) {                                      \
    case 16: { constexpr int VW_ = 16; __VA_ARGS__; break; } \
    case 8: { constexpr int VW_ = 8; __VA_ARGS__; break; }   \
    case 4: { constexpr int VW_ = 4; __VA_ARGS__; break; }   \
    default: { constexpr int VW_ = 2; __VA_ARGS__; break; } \
  }

}  // namespace nib
