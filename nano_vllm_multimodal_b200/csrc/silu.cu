// SiluAndMul: y = silu(x[:, :I]) * x[:, I:] (nanovllm/layers/activation.py:8-11).
//
// One CTA works on two rows at a time (rows r and r + gridDim.x of its
// grid-strided sequence): every thread issues all of its gate/up 16-byte loads
// for both rows before any math, so a CTA keeps 4 * KU * 16 B per thread in
// flight. The expression is evaluated in fp32 and rounded once, as the
// reference's compiled (GPU) SiluAndMul does:
//   silu(g) = g / (1 + exp(-g))
// 16-bit activations: when every |g| of a 16-byte vector is <= 80, the vector
// takes the fast form g * rcp(1 + 2^(-g*log2 e)) with the hardware ex2/rcp
// approximations. Their arguments and results stay in the normal fp32 range
// there, and their relative error (< 1e-5) is far below half a bf16/fp16 ulp,
// so the rounded result stays within one ulp of the exactly rounded value.
// Other vectors use the IEEE expf / divide form, which reproduces the
// reference's saturation (silu -> -0 once exp overflows). float32 activations
// always use the IEEE form.
#include "dispatch.cuh"

namespace nib {

__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float rcp_approx(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ float silu_ieee(float g) { return g / (1.0f + expf(-g)); }

// y[e] = round(silu(g[e]) * u[e]) for one 16-byte vector
template <typename T>
__device__ __forceinline__ uint4 silu_mul_vec(const uint4& gv, const uint4& uv) {
  constexpr int E = Elem<T>::kPerVec;
  float g[E], u[E], o[E];
  unpack<T>(gv, g);
  unpack<T>(uv, u);
  bool fast = false;
  if constexpr (sizeof(T) == 2) {
    float m = fabsf(g[0]);
#pragma unroll
    for (int e = 1; e < E; ++e) m = fmaxf(m, fabsf(g[e]));
    fast = m <= 80.0f;  // a NaN lane is ignored by fmax: NaN in, NaN out on either path
  }
  if (fast) {
    constexpr float kNegLog2e = -1.4426950408889634f;
#pragma unroll
    for (int e = 0; e < E; ++e)
      o[e] = __fmul_rn(__fmul_rn(g[e], rcp_approx(1.0f + ex2_approx(g[e] * kNegLog2e))), u[e]);
  } else {
#pragma unroll
    for (int e = 0; e < E; ++e) o[e] = __fmul_rn(silu_ieee(g[e]), u[e]);
  }
  return pack<T>(o);
}

template <typename T, int KU>
__global__ void __launch_bounds__(256)
silu_mul_rows(const T* __restrict__ x, int64_t x_rs, T* __restrict__ y, int64_t rows, int inter) {
  constexpr int E = Elem<T>::kPerVec;
  const int upr = inter / E;
  const int64_t stride = gridDim.x;
  for (int64_t r0 = blockIdx.x; r0 < rows; r0 += 2 * stride) {
    const int64_t r1 = r0 + stride;
    const bool two = r1 < rows;
    const T* x0 = x + r0 * x_rs;
    const T* x1 = x + (two ? r1 : r0) * x_rs;
    uint4 g0[KU], u0[KU], g1[KU], u1[KU];
#pragma unroll
    for (int k = 0; k < KU; ++k) {
      const int j = k * blockDim.x + threadIdx.x;
      const bool ok = j < upr;
      g0[k] = ok ? ld_stream(x0 + j * E) : zero_vec();
      u0[k] = ok ? ld_stream(x0 + inter + j * E) : zero_vec();
      g1[k] = (ok && two) ? ld_stream(x1 + j * E) : zero_vec();
      u1[k] = (ok && two) ? ld_stream(x1 + inter + j * E) : zero_vec();
    }
#pragma unroll
    for (int k = 0; k < KU; ++k) {
      const int j = k * blockDim.x + threadIdx.x;
      if (j >= upr) continue;
      st_vec(y + r0 * inter + j * E, silu_mul_vec<T>(g0[k], u0[k]));
      if (two) st_vec(y + r1 * inter + j * E, silu_mul_vec<T>(g1[k], u1[k]));
    }
  }
}

template <typename T>
static int launch_silu(const void* x, int64_t x_rs, int64_t rows, int64_t inter, void* y,
                       cudaStream_t st) {
  constexpr int E = Elem<T>::kPerVec;
  const int upr = static_cast<int>(inter / E);
  int threads = 256;
  int ku = (upr + threads - 1) / threads;
  if (upr <= 128) {
    threads = ((upr + 31) / 32) * 32;
    ku = 1;
  }
  NIB_SUPPORT(ku <= 8, "silu_and_mul: intermediate size %lld is larger than this build supports",
              (long long)inter);
  int64_t blocks = (rows + 1) / 2;
  const int64_t cap = static_cast<int64_t>(sm_count()) * (2048 / threads) * 2;
  if (blocks > cap) blocks = cap;
  const T* xp = static_cast<const T*>(x);
  T* yp = static_cast<T*>(y);
  const unsigned nb = static_cast<unsigned>(blocks);
  switch (ku) {
#define NIB_SILU_KU(K) \
    case K: silu_mul_rows<T, K><<<nb, threads, 0, st>>>(xp, x_rs, yp, rows, static_cast<int>(inter)); break;
    NIB_SILU_KU(1) NIB_SILU_KU(2) NIB_SILU_KU(3) NIB_SILU_KU(4)
    NIB_SILU_KU(5) NIB_SILU_KU(6) NIB_SILU_KU(7) NIB_SILU_KU(8)
#undef NIB_SILU_KU
  }
  return launch_status("silu_and_mul");
}

}  // namespace nib

using namespace nib;

extern "C" int nib_silu_and_mul(int dtype, const void* x, int64_t x_row_stride, int64_t rows,
                                int64_t inter, void* y, void* stream) {
  NIB_REQUIRE(rows >= 0 && inter >= 1, "silu_and_mul: bad sizes");
  if (rows == 0) return NIB_OK;
  NIB_REQUIRE(x && y, "silu_and_mul: null pointer");
  const int E = 16 / elem_size(dtype);
  NIB_SUPPORT(aligned16(x) && aligned16(y), "silu_and_mul: pointers must be 16-byte aligned");
  NIB_SUPPORT(inter % E == 0 && x_row_stride % E == 0,
              "silu_and_mul: intermediate size and row stride must be multiples of %d elements", E);
  NIB_DISPATCH(dtype, T, return launch_silu<T>(x, x_row_stride, rows, inter, y, as_stream(stream)));
  return NIB_OK;
}
