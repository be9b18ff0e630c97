// SiluAndMul: y = silu(x[:, :I]) * x[:, I:] (nanovllm/layers/activation.py:8-11).
//
// One CTA row (threadIdx.y) per token row: every thread issues all of its
// gate/up 16-byte loads before any math. The grid covers every row once
// (one-shot CTAs, no grid-stride loop unless rows exceed the grid limit):
// finished CTAs retire while their stores drain and the block scheduler starts
// new ones, whose loads overlap that drain. On B200 this moves 12% more bytes
// per second than persistent CTAs looping over rows (16 per SM), and reaches
// more than a plain 1:1 copy since the traffic is two reads per write.
// The expression is evaluated in fp32 and rounded once, as the
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

// 4 resident CTAs (1024 threads) per SM while the row buffers allow it
template <int KU>
constexpr int silu_min_blocks() { return KU <= 3 ? 4 : (KU == 4 ? 3 : (KU <= 6 ? 2 : 1)); }

template <typename T, int KU>
__global__ void __launch_bounds__(256, silu_min_blocks<KU>())
silu_mul_rows(const T* __restrict__ x, int64_t x_rs, T* __restrict__ y, int64_t rows, int inter) {
  ::nib::pdl_enter();
  constexpr int E = Elem<T>::kPerVec;
  const int upr = inter / E;
  const int64_t step = static_cast<int64_t>(gridDim.x) * blockDim.y;
  for (int64_t r = static_cast<int64_t>(blockIdx.x) * blockDim.y + threadIdx.y; r < rows; r += step) {
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
      if (j < upr) st_vec(y + r * inter + j * E, silu_mul_vec<T>(g[k], u[k]));
    }
  }
}

template <typename T>
static int launch_silu(const void* x, int64_t x_rs, int64_t rows, int64_t inter, void* y,
                       cudaStream_t st) {
  constexpr int E = Elem<T>::kPerVec;
  const int upr = static_cast<int>(inter / E);
  // 256 threads per CTA: a row of >= 256 vectors takes the whole CTA (KU
  // vectors per thread); shorter rows are packed several to a CTA.
  int tx = 256, ty = 1, ku = (upr + 255) / 256;
  if (upr < 256) {
    tx = ((upr + 31) / 32) * 32;
    ty = 256 / tx;
    ku = 1;
  }
  NIB_SUPPORT(ku <= 8, "silu_and_mul: intermediate size %lld is larger than this build supports",
              (long long)inter);
  int64_t blocks = (rows + ty - 1) / ty;
  if (blocks > kMaxGrid) blocks = kMaxGrid;
  const T* xp = static_cast<const T*>(x);
  T* yp = static_cast<T*>(y);
  const unsigned nb = static_cast<unsigned>(blocks);
  const dim3 block(tx, ty);
  switch (ku) {
#define NIB_SILU_KU(K) \
    case K: ::nib::launch_k(silu_mul_rows<T, K>, nb, block, 0, st, xp, x_rs, yp, rows, static_cast<int>(inter)); break;
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
