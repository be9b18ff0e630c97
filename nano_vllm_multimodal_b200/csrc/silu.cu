// SiluAndMul: y = silu(x[:, :I]) * x[:, I:] (nanovllm/layers/activation.py:8-11).
//
// One CTA per row (grid-strided); every thread issues all of its gate/up
// 16-byte loads for the row before any math, so a CTA keeps
// 2 * KU * 16 B per thread in flight. The expression is evaluated in fp32 and
// rounded once, as the reference's compiled (GPU) SiluAndMul does:
//   silu(g) = g / (1 + exp(-g))
// For 2^-100 <= |g| <= 80 the exponential and the quotient use the hardware
// approximations (ex2.approx, rcp.approx): their relative error (< 1e-5) is far
// below half a bf16/fp16 ulp, so the rounded result stays within one ulp of
// the exactly rounded value. Outside that range the IEEE expf / divide path
// reproduces the reference's saturation (silu -> -0 once exp overflows).
// float32 activations always take the IEEE path.
#include "dispatch.cuh"

namespace nib {

template <typename T>
__device__ __forceinline__ float silu_f32(float g) {
  // float32 outputs keep full precision: IEEE expf and divide throughout
  if constexpr (sizeof(T) == 4) return g / (1.0f + expf(-g));
  const float a = fabsf(g);
  if (a <= 80.0f && a >= 0x1p-100f) return __fdividef(g, 1.0f + __expf(-g));
  return g / (1.0f + expf(-g));  // saturating tails, tiny and subnormal inputs
}

template <typename T, int KU>
__global__ void __launch_bounds__(256)
silu_mul_rows(const T* __restrict__ x, int64_t x_rs, T* __restrict__ y, int64_t rows, int inter) {
  constexpr int E = Elem<T>::kPerVec;
  const int upr = inter / E;
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
    const T* xr = x + r * x_rs;
    uint4 g[KU], u[KU];
#pragma unroll
    for (int k = 0; k < KU; ++k) {
      const int j = k * blockDim.x + threadIdx.x;
      const bool ok = j < upr;
      g[k] = ok ? ld_stream(xr + j * E) : zero_vec();
      u[k] = ok ? ld_stream(xr + inter + j * E) : zero_vec();
    }
#pragma unroll
    for (int k = 0; k < KU; ++k) {
      const int j = k * blockDim.x + threadIdx.x;
      if (j >= upr) continue;
      float gf[E], uf[E], o[E];
      unpack<T>(g[k], gf);
      unpack<T>(u[k], uf);
#pragma unroll
      for (int e = 0; e < E; ++e) o[e] = __fmul_rn(silu_f32<T>(gf[e]), uf[e]);
      st_vec(y + r * inter + j * E, pack<T>(o));
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
  int64_t blocks = rows;
  const int64_t cap = static_cast<int64_t>(sm_count()) * (2048 / threads) * 4;
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
