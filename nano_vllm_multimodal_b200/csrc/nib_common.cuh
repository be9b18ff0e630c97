// Shared device helpers for the sm_100a elementwise kernels.
//
// All HBM traffic goes through 16-byte vectors (one LDG.128 / STG.128 per
// lane); element conversions are explicit so the rounding points match the
// reference's PyTorch code exactly (fp32 math, round-to-nearest-even to the
// storage dtype where PyTorch rounds).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <utility>

#include "../../include/nib_b200.h"

namespace nib {

// ---------------------------------------------------------------- host side
void set_error(const char* fmt, ...);
int launch_status(const char* what);  // NIB_OK or NIB_ERR_CUDA after a launch
inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

// number of SMs of the current device (cached per device)
int sm_count();

// Programmatic dependent launch (opt-in: NIB_B200_PDL=1). Every kernel of this
// library can be launched with the programmatic-stream-serialization
// attribute: it may then be scheduled while the kernel before it on the stream
// is still finishing, so its launch latency and block set-up overlap that
// tail. Each kernel therefore starts with pdl_enter(), which waits for the
// preceding grid to complete (and its memory to be visible) before touching
// global memory, then lets the next kernel launch early in turn. Without the
// attribute pdl_enter() returns at once.
bool pdl_enabled();
void note_launch_error(cudaError_t e);  // reported by the next launch_status()

template <typename... KArgs, typename... Args>
inline void launch_k_pdl(bool pdl, void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                         Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
  if (e != cudaSuccess) note_launch_error(e);
}

template <typename... KArgs, typename... Args>
inline void launch_k(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                     Args&&... args) {
  launch_k_pdl(pdl_enabled(), kernel, grid, block, smem, st, std::forward<Args>(args)...);
}

// The second kernel of one entry point, whose only input is its predecessor's
// output (a split merge after the splits): launched as a programmatic dependent
// whatever NIB_B200_PDL says, so its CTAs wait at pdl_enter() in the
// predecessor's tail instead of behind a launch gap. The predecessor triggers
// its dependents only once all of its CTAs have started, so the waiting CTAs
// never keep one of them from running.
template <typename... KArgs, typename... Args>
inline void launch_k_after(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                           Args&&... args) {
  launch_k_pdl(true, kernel, grid, block, smem, st, std::forward<Args>(args)...);
}

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
// first statement of every kernel: wait for the predecessor grid, then allow the successor's launch
__device__ __forceinline__ void pdl_enter() {
  pdl_wait();
  pdl_launch_dependents();
}

// Largest grid.x a one-shot launch uses; kernels grid-stride past it.
constexpr int64_t kMaxGrid = 0x7fffffff;

#define NIB_REQUIRE(cond, ...)                 \
  do {                                         \
    if (!(cond)) {                             \
      ::nib::set_error(__VA_ARGS__);           \
      return NIB_ERR_INVALID;                  \
    }                                          \
  } while (0)

#define NIB_SUPPORT(cond, ...)                 \
  do {                                         \
    if (!(cond)) {                             \
      ::nib::set_error(__VA_ARGS__);           \
      return NIB_ERR_UNSUPPORTED;              \
    }                                          \
  } while (0)

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
inline int elem_size(int dtype) { return dtype == NIB_F32 ? 4 : 2; }

// ---------------------------------------------------------------- element traits
template <typename T> struct Elem;
template <> struct Elem<float> {
  static constexpr int kPerVec = 4;
  __device__ __forceinline__ static float to_f(float v) { return v; }
  __device__ __forceinline__ static float from_f(float v) { return v; }
};
template <> struct Elem<__nv_bfloat16> {
  static constexpr int kPerVec = 8;
  __device__ __forceinline__ static float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
  __device__ __forceinline__ static __nv_bfloat16 from_f(float v) { return __float2bfloat16_rn(v); }
};
template <> struct Elem<__half> {
  static constexpr int kPerVec = 8;
  __device__ __forceinline__ static float to_f(__half v) { return __half2float(v); }
  __device__ __forceinline__ static __half from_f(float v) { return __float2half_rn(v); }
};

// two adjacent elements rounded from fp32 (round to nearest each), one store
template <typename T> struct Vec2;
template <> struct Vec2<float> {
  using type = float2;
  __device__ __forceinline__ static float2 make(float a, float b) { return make_float2(a, b); }
};
template <> struct Vec2<__nv_bfloat16> {
  using type = __nv_bfloat162;
  __device__ __forceinline__ static __nv_bfloat162 make(float a, float b) { return __floats2bfloat162_rn(a, b); }
};
template <> struct Vec2<__half> {
  using type = __half2;
  __device__ __forceinline__ static __half2 make(float a, float b) { return __floats2half2_rn(a, b); }
};

// round an fp32 value to T and back (identity for float)
template <typename T>
__device__ __forceinline__ float round_to(float v) {
  return Elem<T>::to_f(Elem<T>::from_f(v));
}

// ---------------------------------------------------------------- 16-byte vectors
__device__ __forceinline__ uint4 ld_vec(const void* p) {
  return __ldg(reinterpret_cast<const uint4*>(p));
}
// read-once streaming input: no L1 allocation, L2 fetches whole 256-byte
// blocks (the neighbouring 16-byte vectors of the row are read next). A
// coherent load: in-place callers write the same rows after reading them.
__device__ __forceinline__ uint4 ld_stream(const void* p) {
  uint4 v;
  asm volatile("ld.global.L1::no_allocate.L2::256B.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}
__device__ __forceinline__ void st_vec(void* p, const uint4& v) {
  *reinterpret_cast<uint4*>(p) = v;
}
__device__ __forceinline__ uint4 zero_vec() { return make_uint4(0u, 0u, 0u, 0u); }

// unpack one 16-byte vector of T into kPerVec floats
template <typename T>
__device__ __forceinline__ void unpack(const uint4& v, float* f);

template <>
__device__ __forceinline__ void unpack<float>(const uint4& v, float* f) {
  f[0] = __uint_as_float(v.x); f[1] = __uint_as_float(v.y);
  f[2] = __uint_as_float(v.z); f[3] = __uint_as_float(v.w);
}
template <>
__device__ __forceinline__ void unpack<__nv_bfloat16>(const uint4& v, float* f) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(w[i] << 16);
    f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
  }
}
template <>
__device__ __forceinline__ void unpack<__half>(const uint4& v, float* f) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __half2 h = *reinterpret_cast<const __half2*>(&w[i]);
    float2 t = __half22float2(h);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}

// pack kPerVec floats into one 16-byte vector of T (round to nearest even)
template <typename T>
__device__ __forceinline__ uint4 pack(const float* f);

template <>
__device__ __forceinline__ uint4 pack<float>(const float* f) {
  return make_uint4(__float_as_uint(f[0]), __float_as_uint(f[1]), __float_as_uint(f[2]),
                    __float_as_uint(f[3]));
}
template <>
__device__ __forceinline__ uint4 pack<__nv_bfloat16>(const float* f) {
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __nv_bfloat162 h = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
    w[i] = *reinterpret_cast<uint32_t*>(&h);
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}
template <>
__device__ __forceinline__ uint4 pack<__half>(const float* f) {
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __half2 h = __floats2half2_rn(f[2 * i], f[2 * i + 1]);
    w[i] = *reinterpret_cast<uint32_t*>(&h);
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}

// load kPerVec<T> weights starting at element i as floats (W = T or float)
template <typename T, typename W>
__device__ __forceinline__ void load_weights(const W* w, int64_t i, float* f) {
  constexpr int E = Elem<T>::kPerVec;
  if constexpr (sizeof(W) == sizeof(T)) {
    unpack<T>(ld_vec(w + i), f);
  } else {
    // fp32 weights with 16-bit activations: two 16-byte loads
#pragma unroll
    for (int j = 0; j < E; j += 4) unpack<float>(ld_vec(w + i + j), f + j);
  }
}

// Sum of squares of one 16-byte vector's E values: squares rounded to fp32,
// then a pairwise tree ((s0+s1)+(s2+s3))+... . This is the fixed summation
// order of every RMSNorm statistic in this library (lanes then add their
// vectors' sums in order and combine by an xor butterfly).
template <int E>
__device__ __forceinline__ float sumsq_tree(const float* v) {
  float s[E];
#pragma unroll
  for (int e = 0; e < E; ++e) s[e] = __fmul_rn(v[e], v[e]);
#pragma unroll
  for (int w = E / 2; w >= 1; w /= 2) {
#pragma unroll
    for (int e = 0; e < w; ++e) s[e] = __fadd_rn(s[2 * e], s[2 * e + 1]);
  }
  return s[0];
}

// 1/sqrt(x) as the reference computes it in fp32: the correctly rounded square
// root, then the correctly rounded reciprocal (IEEE sqrt.rn and rcp.rn, the
// same two roundings as `1.0f / sqrtf(x)` without fast math).
__device__ __forceinline__ float inv_sqrt_rn(float x) { return __frcp_rn(__fsqrt_rn(x)); }

__device__ __forceinline__ void flag(unsigned int* status, unsigned int bit) {
  if (status != nullptr) atomicOr(status, bit);
}

}  // namespace nib
