// Per-lane math of the attention prologue, shared by both prologue kernels.
//
// Lane layout ("paired halves"): a head of D elements is covered by
// L = D / (2E) lanes; lane l holds E elements of the first half
// (d = l*E + e) and the E elements of the second half that pair with them
// under rotate-half (d + D/2). Both halves use the same E frequencies, so the
// rotation needs no data exchange, and a warp covers 32 / L heads at once.
//
// Rounding points (reference: nanovllm/layers/layernorm.py:16-26,
// nanovllm/models/qwen3_vl.py:74-79, nanovllm/layers/rotary_embedding.py:6-14,
// nanovllm/layers/multimodal_rotary_embedding.py:12-45):
//   norm:          n = T(x * rs); y = T(n * w)
//   1-D / chunked: fp32 x*c -/+ p*s, one rounding to T
//   interleaved:   T(T(x*c) -/+ T(p*s))
// For 16-bit T the products and sums of two T values use packed bf16x2/f16x2
// instructions, which round the exact result once - identical to the fp32
// operation followed by a rounding to T.
#pragma once

#include "nib_common.cuh"

namespace nib {

template <typename T> struct Packed;
template <> struct Packed<__nv_bfloat16> {
  using P = __nv_bfloat162;
  __device__ __forceinline__ static P mul(P a, P b) { return __hmul2_rn(a, b); }
  __device__ __forceinline__ static P add(P a, P b) { return __hadd2_rn(a, b); }
  __device__ __forceinline__ static P sub(P a, P b) { return __hsub2_rn(a, b); }
  __device__ __forceinline__ static P make(float lo, float hi) { return __floats2bfloat162_rn(lo, hi); }
};
template <> struct Packed<__half> {
  using P = __half2;
  __device__ __forceinline__ static P mul(P a, P b) { return __hmul2_rn(a, b); }
  __device__ __forceinline__ static P add(P a, P b) { return __hadd2_rn(a, b); }
  __device__ __forceinline__ static P sub(P a, P b) { return __hsub2_rn(a, b); }
  __device__ __forceinline__ static P make(float lo, float hi) { return __floats2half2_rn(lo, hi); }
};

template <typename P>
__device__ __forceinline__ uint32_t pbits(P v) { return *reinterpret_cast<uint32_t*>(&v); }
template <typename P>
__device__ __forceinline__ P pfrom(uint32_t w) { return *reinterpret_cast<P*>(&w); }

__device__ __forceinline__ uint4 as_u4(const uint32_t* w) { return make_uint4(w[0], w[1], w[2], w[3]); }
__device__ __forceinline__ void from_u4(const uint4& v, uint32_t* w) {
  w[0] = v.x; w[1] = v.y; w[2] = v.z; w[3] = v.w;
}

// Per-lane constants of one norm weight vector in the paired layout.
template <typename T, typename W>
struct HeadWeights {
  static constexpr int E = Elem<T>::kPerVec;
  float fa[E], fb[E];    // float copies (fp32 weights or fp32 activations)
  uint32_t pa[4], pb[4]; // packed 16-bit copies when W == T is 16-bit

  __device__ __forceinline__ void load(const W* w, int l, int half) {
    load_weights<T, W>(w, l * E, fa);
    load_weights<T, W>(w, half + l * E, fb);
    if constexpr (sizeof(T) == 2 && sizeof(W) == 2) {
      from_u4(ld_vec(w + l * E), pa);
      from_u4(ld_vec(w + half + l * E), pb);
    }
  }
};

// n = T(x * rs); y = T(n * w) for one vector (E elements); writes packed words
// and refreshes the float copies.
template <typename T, typename W>
__device__ __forceinline__ void normalize_vec(float* x, uint32_t* words, float rs, const float* wf,
                                              const uint32_t* wp) {
  constexpr int E = Elem<T>::kPerVec;
  if constexpr (sizeof(T) == 2) {
    using PK = Packed<T>;
    using P = typename PK::P;
#pragma unroll
    for (int k = 0; k < E / 2; ++k) {
      const P nn = PK::make(__fmul_rn(x[2 * k], rs), __fmul_rn(x[2 * k + 1], rs));
      P y;
      if constexpr (sizeof(W) == 2) {
        y = PK::mul(nn, pfrom<P>(wp[k]));
      } else {
        y = PK::make(__fmul_rn(Elem<T>::to_f(reinterpret_cast<const T*>(&nn)[0]), wf[2 * k]),
                     __fmul_rn(Elem<T>::to_f(reinterpret_cast<const T*>(&nn)[1]), wf[2 * k + 1]));
      }
      words[k] = pbits(y);
    }
    unpack<T>(as_u4(words), x);
  } else {
#pragma unroll
    for (int e = 0; e < E; ++e) x[e] = __fmul_rn(__fmul_rn(x[e], rs), wf[e]);
    from_u4(pack<T>(x), words);
  }
}

// Rotate-half of the pair (a = first-half elements, b = their partners).
// inter: interleaved M-RoPE rounding (T arithmetic); else fp32 math.
template <typename T>
__device__ __forceinline__ void rotate_pair(const float* a, const float* b, uint32_t* wa, uint32_t* wb,
                                            const float* c, const float* s, const uint32_t* c2,
                                            const uint32_t* s2, bool inter) {
  constexpr int E = Elem<T>::kPerVec;
  if (inter) {
    if constexpr (sizeof(T) == 2) {
      using PK = Packed<T>;
      using P = typename PK::P;
#pragma unroll
      for (int k = 0; k < E / 2; ++k) {
        const P xa = pfrom<P>(wa[k]), xb = pfrom<P>(wb[k]);
        const P cc = pfrom<P>(c2[k]), ss = pfrom<P>(s2[k]);
        wa[k] = pbits(PK::sub(PK::mul(xa, cc), PK::mul(xb, ss)));
        wb[k] = pbits(PK::add(PK::mul(xb, cc), PK::mul(xa, ss)));
      }
    } else {
      float ya[E], yb[E];
#pragma unroll
      for (int e = 0; e < E; ++e) {
        ya[e] = __fsub_rn(__fmul_rn(a[e], c[e]), __fmul_rn(b[e], s[e]));
        yb[e] = __fadd_rn(__fmul_rn(b[e], c[e]), __fmul_rn(a[e], s[e]));
      }
      from_u4(pack<T>(ya), wa);
      from_u4(pack<T>(yb), wb);
    }
  } else {
    float ya[E], yb[E];
#pragma unroll
    for (int e = 0; e < E; ++e) {
      ya[e] = __fsub_rn(__fmul_rn(a[e], c[e]), __fmul_rn(b[e], s[e]));
      yb[e] = __fadd_rn(__fmul_rn(b[e], c[e]), __fmul_rn(a[e], s[e]));
    }
    from_u4(pack<T>(ya), wa);
    from_u4(pack<T>(yb), wb);
  }
}

// Interleaved M-RoPE cos/sin as packed T pairs (the values are already T).
template <typename T>
__device__ __forceinline__ void pack_trig(const float* c, const float* s, uint32_t* c2, uint32_t* s2) {
  constexpr int E = Elem<T>::kPerVec;
  if constexpr (sizeof(T) == 2) {
    using PK = Packed<T>;
#pragma unroll
    for (int k = 0; k < E / 2; ++k) {
      c2[k] = pbits(PK::make(c[2 * k], c[2 * k + 1]));
      s2[k] = pbits(PK::make(s[2 * k], s[2 * k + 1]));
    }
  }
}

// M-RoPE frequency -> position axis (multimodal_rotary_embedding.py:120-147)
__device__ __forceinline__ int mrope_axis(int j, bool inter, const int32_t* sec) {
  if (inter) {
    const int r = j % 3;
    return (r == 1 && j < 3 * sec[1]) ? 1 : (r == 2 && j < 3 * sec[2]) ? 2 : 0;
  }
  return j < sec[0] ? 0 : (j < sec[0] + sec[1] ? 1 : 2);
}

}  // namespace nib
