// Attention prologue: per-head q/k RMSNorm + RoPE / M-RoPE + paged KV store.
//
// Reference composition (each stage's numerics kept exactly):
//   q_norm/k_norm   RMSNorm.rms_forward (nanovllm/layers/layernorm.py:16-26) or
//                   Qwen3VLTextRMSNorm (nanovllm/models/qwen3_vl.py:74-79)
//   1-D RoPE        nanovllm/layers/rotary_embedding.py:6-14,37-48 - fp32 math
//                   on the fp32 cos|sin table, one rounding at the end
//   M-RoPE          nanovllm/layers/multimodal_rotary_embedding.py:12-45,89-147
//                   cos/sin = dtype(cos/sin(fp32(pos) * inv_freq));
//                   chunked: fp32 math, one rounding;
//                   interleaved: dtype arithmetic, every product and the sum
//                   rounded (round(round(x*c) + round(rot(x)*s)))
//   store           rotated k and raw v to flat slot slot_mapping[t]
//                   (nanovllm/layers/attention.py:87-93), -1 skipped.
//
// Layout (prologue_math.cuh): a head spans L = head_dim / 16 lanes (bf16/fp16;
// head_dim / 8 for fp32), each holding a 16-byte vector of the first half and
// its rotate-half partner vector of the second half, so a warp covers 32 / L
// heads per step and the rotation needs no shuffles. A work item is
// (token, chunk of up to CH head groups); all its loads are issued before any
// math. M-RoPE cos/sin are computed once per item for the head_dim/2
// frequencies and shared through shared memory. This register-staged kernel
// takes any q/k/v strides; prologue_pipe.cu is the bulk-copy variant for the
// fused-qkv layout, with bit-identical results.
#include <type_traits>

#include "dispatch.cuh"
#include "prologue.cuh"
#include "prologue_math.cuh"

namespace nib {

constexpr int kPrologueWarps = 4;
// Head groups per work item: 4 (all loads of up to 16 heads in flight at
// once) for large batches; 1 for batches of at most kFewItems single-group
// items, where a work item's chain of dependent steps, not bandwidth, sets the
// time (C2 decode, 256 tokens: 3.96 -> 2.93 us per launch on B200).
constexpr int kChunk = 4;
constexpr int64_t kFewItems = 4096;

template <typename T, typename W, int D, int CH>
__global__ void __launch_bounds__(kPrologueWarps * 32)
qk_prologue_kernel(const nib_qk_prologue_args a) {
  ::nib::pdl_enter();
  constexpr int E = Elem<T>::kPerVec;
  constexpr int L = D / (2 * E);  // lanes per head (paired-halves layout)
  static_assert(L >= 1 && L <= 32, "head must span 1..32 lanes");
  constexpr int HPW = 32 / L;     // heads per warp step
  constexpr int NF = D / 2;
  __shared__ float s_cos[kPrologueWarps][NF];
  __shared__ float s_sin[kPrologueWarps][NF];

  const int lane = threadIdx.x & 31;
  const int wib = threadIdx.x >> 5;
  const int hs = lane / L;
  const int l = lane % L;
  const int fb = l * E;

  const int nq = a.num_heads, nkv = a.num_kv_heads;
  const int Uq = (nq + HPW - 1) / HPW;
  const int Uk = (nkv + HPW - 1) / HPW;
  const bool store = a.key_cache != nullptr;
  const int Uv = store ? Uk : 0;
  const int U = Uq + Uk + Uv;
  const int nchunks = (U + CH - 1) / CH;
  const int64_t items = a.tokens * nchunks;
  const bool inter = a.rope_mode == NIB_ROPE_MROPE_INTERLEAVED;

  const T* q = static_cast<const T*>(a.q);
  const T* k = static_cast<const T*>(a.k);
  const T* v = static_cast<const T*>(a.v);
  T* q_out = static_cast<T*>(a.q_out);
  T* k_out = static_cast<T*>(a.k_out);
  T* kc = static_cast<T*>(a.key_cache);
  T* vc = static_cast<T*>(a.value_cache);

  HeadWeights<T, W> wq, wk;
  if (a.norm) {
    wq.load(static_cast<const W*>(a.q_weight), l, NF);
    wk.load(static_cast<const W*>(a.k_weight), l, NF);
  }

  const int64_t warp = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;

  for (int64_t it = warp; it < items; it += nwarps) {
    const int64_t t = it / nchunks;
    const int chunk = static_cast<int>(it - t * nchunks);
    const int u0 = chunk * CH;

    // The slot and the 1-D table position are loaded together, and the v
    // vectors are loaded whatever the slot, so that only the table row waits
    // on a load (position -> row): two memory round trips per item, which is
    // what bounds small decode batches.
    const bool rotates = a.rope_mode != NIB_ROPE_NONE && u0 < Uq + Uk;
    const int32_t sv = store ? __ldg(a.slot_mapping + t) : -1;
    const int64_t tp = (rotates && a.rope_mode == NIB_ROPE_TABLE)
                           ? __ldg(a.positions + t * a.positions_token_stride) : 0;
    // M-RoPE: the positions and inverse frequencies of this lane's frequencies
    // (j = lane, lane + 32, ...) are loaded here too, so sincosf waits on one load
    constexpr int FPL = (NF + 31) / 32;
    float mp[FPL], mf[FPL];
    const bool mrope = rotates && a.rope_mode != NIB_ROPE_TABLE;
#pragma unroll
    for (int m = 0; m < FPL; ++m) {
      const int j = lane + 32 * m;
      mp[m] = mf[m] = 0.f;
      if (mrope && j < NF) {
        const int axis = mrope_axis(j, inter, a.sections);
        mp[m] = static_cast<float>(__ldg(a.positions + axis * a.positions_axis_stride + t * a.positions_token_stride));
        mf[m] = __ldg(a.inv_freq + j);
      }
    }

    // ---- issue every load of this item first (two vectors per lane per head)
    uint4 ba[CH], bb[CH];
#pragma unroll
    for (int i = 0; i < CH; ++i) {
      const int u = u0 + i;
      ba[i] = bb[i] = zero_vec();
      const T* src = nullptr;
      if (u < Uq) {
        const int head = u * HPW + hs;
        if (head < nq) src = q + t * a.q_token_stride + head * a.q_head_stride;
      } else if (u < Uq + Uk) {
        const int head = (u - Uq) * HPW + hs;
        if (head < nkv) src = k + t * a.k_token_stride + head * a.k_head_stride;
      } else if (u < U) {
        const int head = (u - Uq - Uk) * HPW + hs;
        if (head < nkv) src = v + t * a.v_token_stride + head * a.v_head_stride;
      }
      if (src) {
        ba[i] = ld_stream(src + fb);
        bb[i] = ld_stream(src + NF + fb);
      }
    }

    int64_t slot = -1;
    if (sv >= 0 && sv < a.num_slots) {
      slot = sv;
    } else if (store && sv != -1 && chunk == 0 && lane == 0) {
      flag(a.status, NIB_DEV_BAD_SLOT);
    }

    // ---- cos / sin of this lane's E frequencies (only if the item rotates something)
    float c[E], s[E];
    uint32_t c2[4], s2[4];
    if (rotates) {
      if (a.rope_mode == NIB_ROPE_TABLE) {
        const int64_t p = tp;
        if (p >= 0 && p < a.table_rows) {
          const float* row = a.cos_sin_table + p * D;
#pragma unroll
          for (int e = 0; e < E; e += 4) {
            unpack<float>(ld_vec(row + fb + e), c + e);
            unpack<float>(ld_vec(row + NF + fb + e), s + e);
          }
        } else {
          if (lane == 0 && chunk == 0) flag(a.status, NIB_DEV_BAD_POSITION);
#pragma unroll
          for (int e = 0; e < E; ++e) c[e] = s[e] = 0.f;
        }
      } else {
        __syncwarp();
#pragma unroll
        for (int m = 0; m < FPL; ++m) {
          const int j = lane + 32 * m;
          if (j < NF) {
            float sn, cs;
            sincosf(__fmul_rn(mp[m], mf[m]), &sn, &cs);
            s_cos[wib][j] = round_to<T>(cs);
            s_sin[wib][j] = round_to<T>(sn);
          }
        }
        __syncwarp();
#pragma unroll
        for (int e = 0; e < E; ++e) {
          c[e] = s_cos[wib][fb + e];
          s[e] = s_sin[wib][fb + e];
        }
      }
      if (inter) pack_trig<T>(c, s, c2, s2);
    }

    // ---- per head group: norm, rotate, write
#pragma unroll
    for (int i = 0; i < CH; ++i) {
      const int u = u0 + i;
      if (u >= U) break;
      if (u < Uq + Uk) {
        const bool is_q = u < Uq;
        const int head = is_q ? u * HPW + hs : (u - Uq) * HPW + hs;
        const bool head_ok = head < (is_q ? nq : nkv);
        float xa[E], xb[E];
        uint32_t wa[4], wb[4];
        unpack<T>(ba[i], xa);
        unpack<T>(bb[i], xb);
        from_u4(ba[i], wa);
        from_u4(bb[i], wb);
        if (a.norm) {
          float ss = __fadd_rn(sumsq_tree<E>(xa), sumsq_tree<E>(xb));
#pragma unroll
          for (int off = L / 2; off > 0; off >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, off));
          const float rs = inv_sqrt_rn(__fadd_rn(__fmul_rn(ss, 1.0f / D), a.eps));
          const HeadWeights<T, W>& hw = is_q ? wq : wk;
          normalize_vec<T, W>(xa, wa, rs, hw.fa, hw.pa);
          normalize_vec<T, W>(xb, wb, rs, hw.fb, hw.pb);
        }
        if (a.rope_mode != NIB_ROPE_NONE) rotate_pair<T>(xa, xb, wa, wb, c, s, c2, s2, inter);
        if (head_ok) {
          const uint4 oa = as_u4(wa), ob = as_u4(wb);
          T* dst = is_q ? q_out + (t * nq + head) * D : (k_out ? k_out + (t * nkv + head) * D : nullptr);
          if (dst) {
            st_vec(dst + fb, oa);
            st_vec(dst + NF + fb, ob);
          }
          if (!is_q && slot >= 0) {
            T* cd = kc + slot * a.cache_slot_stride + head * D;
            st_vec(cd + fb, oa);
            st_vec(cd + NF + fb, ob);
          }
        }
      } else {
        const int head = (u - Uq - Uk) * HPW + hs;
        if (slot >= 0 && head < nkv) {
          T* cd = vc + slot * a.cache_slot_stride + head * D;
          st_vec(cd + fb, ba[i]);
          st_vec(cd + NF + fb, bb[i]);
        }
      }
    }
  }
}

// ---------------------------------------------------------------- generic M-RoPE apply
// apply_multimodal_rotary_emb with given cos/sin [3, T, D] (any even D, any
// dtypes). One thread per output element; TO is the arithmetic dtype of the
// interleaved strategy (the promoted dtype of x and cos).
template <typename TX, typename TC, typename TO>
__global__ void __launch_bounds__(256)
mrope_apply_kernel(const TX* __restrict__ x, int64_t xts, int64_t xhs, int64_t tokens,
                   int64_t heads, int D, const TC* __restrict__ cos, const TC* __restrict__ sin,
                   int s0, int s1, int s2, int interleaved, TX* __restrict__ out) {
  ::nib::pdl_enter();
  const int64_t total = tokens * heads * D;
  const int half = D / 2;
  for (int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; idx < total;
       idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int d = static_cast<int>(idx % D);
    const int64_t th = idx / D;
    const int64_t h = th % heads;
    const int64_t t = th / heads;
    const int j = d % half;
    int axis;
    if (interleaved) {
      const int m = j % 3;
      axis = (m == 1 && j < 3 * s1) ? 1 : (m == 2 && j < 3 * s2) ? 2 : 0;
    } else {
      axis = j < s0 ? 0 : (j < s0 + s1 ? 1 : 2);
    }
    // chunked selects over the full head dim (sections repeated), so element d
    // reads column d; interleaved selects on the first half and repeats that
    // selection for the second half, so both halves read column j
    const int64_t ci = (axis * tokens + t) * D + (interleaved ? j : d);
    const float cv = Elem<TC>::to_f(cos[ci]);
    const float sv = Elem<TC>::to_f(sin[ci]);
    const TX* xr = x + t * xts + h * xhs;
    const float xv = Elem<TX>::to_f(xr[d]);
    const float pv = Elem<TX>::to_f(xr[d < half ? d + half : d - half]);
    const float rot = d < half ? -pv : pv;
    float y;
    if (interleaved) {
      const float t1 = round_to<TO>(__fmul_rn(xv, cv));
      const float t2 = round_to<TO>(__fmul_rn(rot, sv));
      y = round_to<TO>(__fadd_rn(t1, t2));
    } else {
      y = __fadd_rn(__fmul_rn(xv, cv), __fmul_rn(rot, sv));
    }
    out[idx] = Elem<TX>::from_f(y);
  }
}

// Vectorised apply_multimodal_rotary_emb for head_dim 64/128/256 with cos/sin in
// the activation dtype, a warp per token. Paired-halves layout: lane l of a head
// holds the E columns fb = l*E.. of the first half and their rotate-half
// partners of the second half. Every load of the token is issued before any
// math: the head vectors of up to kApplyGroups head groups, and one 16-byte
// vector of each of the three axes' cos and sin rows at the lane's columns
// (plus the second-half columns for the chunked strategy). The axis of each
// column is fixed per lane, so selecting it is a register move, with no shared
// memory. Same arithmetic as mrope_apply_kernel: chunked in fp32 with one
// rounding, interleaved in T with every product and the sum rounded. The
// second half reads column d for chunked and column j = d - D/2 for
// interleaved (multimodal_rotary_embedding.py:33-45).
constexpr int kApplyWarps = 4;
constexpr int kApplyGroups = 4;  // head groups whose vectors are in flight together

template <typename T>
__device__ __forceinline__ void select_axis(const uint4* v, uint32_t axes, float* f) {
  constexpr int E = Elem<T>::kPerVec;
  float a0[E], a1[E], a2[E];
  unpack<T>(v[0], a0);
  unpack<T>(v[1], a1);
  unpack<T>(v[2], a2);
#pragma unroll
  for (int e = 0; e < E; ++e) {
    const uint32_t ax = (axes >> (2 * e)) & 3u;
    f[e] = ax == 0 ? a0[e] : (ax == 1 ? a1[e] : a2[e]);
  }
}

template <typename T, int D, bool INTER>
__global__ void __launch_bounds__(kApplyWarps * 32, INTER ? 6 : 4)
mrope_apply_vec_kernel(const T* __restrict__ x, int64_t xts, int64_t xhs, int64_t tokens, int heads,
                       const T* __restrict__ cos, const T* __restrict__ sin, int s0, int s1, int s2,
                       T* __restrict__ out) {
  ::nib::pdl_enter();
  constexpr int E = Elem<T>::kPerVec;
  constexpr int L = D / (2 * E);
  constexpr int HPW = 32 / L;
  constexpr int NF = D / 2;
  constexpr bool inter = INTER;
  const int lane = threadIdx.x & 31;
  const int hs = lane / L, fb = (lane % L) * E;
  const int32_t sec[3] = {s0, s1, s2};
  uint32_t axes = 0;  // 2 bits per column of this lane
#pragma unroll
  for (int e = 0; e < E; ++e) axes |= static_cast<uint32_t>(mrope_axis(fb + e, inter, sec)) << (2 * e);
  const int groups = (heads + HPW - 1) / HPW;
  const int64_t warp = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  for (int64_t t = warp; t < tokens; t += nwarps) {
    const T* xt = x + t * xts;
    uint4 va[kApplyGroups], vb[kApplyGroups];
    auto load_heads = [&](int g0) {
#pragma unroll
      for (int g = 0; g < kApplyGroups; ++g) {
        const int h = (g0 + g) * HPW + hs;
        va[g] = vb[g] = zero_vec();
        if (g0 + g < groups && h < heads) {
          const T* src = xt + static_cast<int64_t>(h) * xhs;
          va[g] = ld_stream(src + fb);
          vb[g] = ld_stream(src + NF + fb);
        }
      }
    };
    uint4 cv[3], sv[3], cw[inter ? 1 : 3], sw[inter ? 1 : 3];
#pragma unroll
    for (int ax = 0; ax < 3; ++ax) {
      const int64_t o = (ax * tokens + t) * D + fb;
      cv[ax] = ld_vec(cos + o);
      sv[ax] = ld_vec(sin + o);
      if constexpr (!inter) {
        cw[ax] = ld_vec(cos + o + NF);
        sw[ax] = ld_vec(sin + o + NF);
      }
    }
    load_heads(0);
    float ca[E], sa[E], cb[E], sb[E];
    select_axis<T>(cv, axes, ca);
    select_axis<T>(sv, axes, sa);
    if constexpr (inter) {
#pragma unroll
      for (int e = 0; e < E; ++e) {
        cb[e] = ca[e];
        sb[e] = sa[e];
      }
    } else {
      select_axis<T>(cw, axes, cb);
      select_axis<T>(sw, axes, sb);
    }
    uint32_t c2[4], s2[4];
    pack_trig<T>(ca, sa, c2, s2);
    T* ot = out + t * heads * static_cast<int64_t>(D);
    for (int g0 = 0; g0 < groups; g0 += kApplyGroups) {
      if (g0 > 0) load_heads(g0);
#pragma unroll
      for (int g = 0; g < kApplyGroups; ++g) {
        const int h = (g0 + g) * HPW + hs;
        if (g0 + g >= groups || h >= heads) continue;
        uint32_t wa[4], wb[4];
        from_u4(va[g], wa);
        from_u4(vb[g], wb);
        if constexpr (sizeof(T) == 2 && inter) {
          {
            using PK = Packed<T>;
            using P = typename PK::P;
#pragma unroll
            for (int k = 0; k < E / 2; ++k) {
              const P xa = pfrom<P>(wa[k]), xb = pfrom<P>(wb[k]);
              const P cc = pfrom<P>(c2[k]), ss = pfrom<P>(s2[k]);
              wa[k] = pbits(PK::sub(PK::mul(xa, cc), PK::mul(xb, ss)));
              wb[k] = pbits(PK::add(PK::mul(xb, cc), PK::mul(xa, ss)));
            }
            T* dst = ot + static_cast<int64_t>(h) * D;
            st_vec(dst + fb, as_u4(wa));
            st_vec(dst + NF + fb, as_u4(wb));
            continue;
          }
        }
        float xa[E], xb[E], ya[E], yb[E];
        unpack<T>(va[g], xa);
        unpack<T>(vb[g], xb);
#pragma unroll
        for (int e = 0; e < E; ++e) {
          ya[e] = __fsub_rn(__fmul_rn(xa[e], ca[e]), __fmul_rn(xb[e], sa[e]));
          yb[e] = __fadd_rn(__fmul_rn(xb[e], cb[e]), __fmul_rn(xa[e], sb[e]));
        }
        T* dst = ot + static_cast<int64_t>(h) * D;
        st_vec(dst + fb, pack<T>(ya));
        st_vec(dst + NF + fb, pack<T>(yb));
      }
    }
  }
}

template <typename TO>
__global__ void __launch_bounds__(256)
mrope_cos_sin_any_kernel(const int64_t* __restrict__ pos, int64_t pas, int64_t pts, int64_t tokens,
                     const float* __restrict__ inv_freq, int D, TO* __restrict__ cos,
                     TO* __restrict__ sin) {
  ::nib::pdl_enter();
  const int half = D / 2;
  const int64_t total = 3 * tokens * half;
  for (int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; idx < total;
       idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int j = static_cast<int>(idx % half);
    const int64_t at = idx / half;
    const int64_t t = at % tokens;
    const int64_t ax = at / tokens;
    const float f = __fmul_rn(static_cast<float>(__ldg(pos + ax * pas + t * pts)), __ldg(inv_freq + j));
    float sn, cs;
    sincosf(f, &sn, &cs);
    const int64_t o = (ax * tokens + t) * D + j;
    cos[o] = cos[o + half] = Elem<TO>::from_f(cs);
    sin[o] = sin[o + half] = Elem<TO>::from_f(sn);
  }
}

// Even half-widths: a thread computes frequencies j and j+1 of kCosSinTok
// consecutive tokens and writes each of cos/sin as packed 2-element stores into
// the first and second half of head_dim; the axis is blockIdx.y. HP = pairs per
// token when it is a compile-time constant (head_dim 64/128/256), else 0.
// All position loads are issued before the 2*kCosSinTok independent sincosf.
constexpr int kCosSinTok = 4;
template <typename TO, int HP>
__global__ void __launch_bounds__(256)
mrope_cos_sin_pair_kernel(const int64_t* __restrict__ pos, int64_t pas, int64_t pts, int64_t tokens,
                          const float* __restrict__ inv_freq, int D, TO* __restrict__ cos,
                          TO* __restrict__ sin) {
  ::nib::pdl_enter();
  using P2 = typename Vec2<TO>::type;
  const int half = D / 2;
  const int hp = HP > 0 ? HP : half / 2;
  const int64_t ax = blockIdx.y;
  const int64_t groups = (tokens + kCosSinTok - 1) / kCosSinTok;
  const int64_t total = groups * hp;
  for (int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; idx < total;
       idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t tg = idx / hp;
    const int j = 2 * static_cast<int>(idx - tg * hp);
    const int64_t t0 = tg * kCosSinTok;
    const float f0 = __ldg(inv_freq + j), f1 = __ldg(inv_freq + j + 1);
    float p[kCosSinTok];
#pragma unroll
    for (int k = 0; k < kCosSinTok; ++k)
      p[k] = t0 + k < tokens ? static_cast<float>(__ldg(pos + ax * pas + (t0 + k) * pts)) : 0.f;
#pragma unroll
    for (int k = 0; k < kCosSinTok; ++k) {
      if (t0 + k >= tokens) break;
      float s0, c0, s1, c1;
      sincosf(__fmul_rn(p[k], f0), &s0, &c0);
      sincosf(__fmul_rn(p[k], f1), &s1, &c1);
      const int64_t o = (ax * tokens + t0 + k) * D + j;
      const P2 cv = Vec2<TO>::make(c0, c1), sv = Vec2<TO>::make(s0, s1);
      *reinterpret_cast<P2*>(cos + o) = cv;
      *reinterpret_cast<P2*>(cos + o + half) = cv;
      *reinterpret_cast<P2*>(sin + o) = sv;
      *reinterpret_cast<P2*>(sin + o + half) = sv;
    }
  }
}

// per_sm = 0: one thread per item (one-shot grid)
static unsigned flat_grid(int64_t total, int per_sm) {
  int64_t blocks = (total + 255) / 256;
  const int64_t cap = per_sm > 0 ? static_cast<int64_t>(sm_count()) * per_sm : kMaxGrid;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  return static_cast<unsigned>(blocks);
}

template <typename T, typename W>
static int launch_prologue(const nib_qk_prologue_args& a, cudaStream_t st) {
  constexpr int E = Elem<T>::kPerVec;
  const int D = a.head_dim;
  const int lph = D / (2 * E);
  NIB_SUPPORT(D == 64 || D == 128 || D == 256, "qk_prologue: head_dim %d not supported (64/128/256)", D);
  const int hpw = 32 / lph;
  const int Uq = (a.num_heads + hpw - 1) / hpw;
  const int Uk = (a.num_kv_heads + hpw - 1) / hpw;
  const int U = Uq + Uk + (a.key_cache ? Uk : 0);
  const bool few = a.tokens * U <= kFewItems;
  const int ch = few ? 1 : kChunk;
  const int64_t items = a.tokens * ((U + ch - 1) / ch);
  int64_t blocks = (items + kPrologueWarps - 1) / kPrologueWarps;
  const int64_t cap = static_cast<int64_t>(sm_count()) * 64;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  const unsigned nb = static_cast<unsigned>(blocks);
  const int threads = kPrologueWarps * 32;
  auto run = [&](auto dtag) {
    constexpr int DD = decltype(dtag)::value;
    if (few) ::nib::launch_k(qk_prologue_kernel<T, W, DD, 1>, nb, threads, 0, st, a);
    else ::nib::launch_k(qk_prologue_kernel<T, W, DD, kChunk>, nb, threads, 0, st, a);
  };
  if (D == 64) run(std::integral_constant<int, 64>{});
  else if (D == 128) run(std::integral_constant<int, 128>{});
  else run(std::integral_constant<int, 256>{});
  return launch_status("qk_prologue");
}

}  // namespace nib

using namespace nib;

extern "C" int nib_qk_prologue(const nib_qk_prologue_args* args, void* stream) {
  NIB_REQUIRE(args != nullptr, "qk_prologue: null args");
  NIB_REQUIRE(args->struct_size == static_cast<int32_t>(sizeof(nib_qk_prologue_args)),
              "qk_prologue: struct_size %d does not match this library (%d)", args->struct_size,
              static_cast<int>(sizeof(nib_qk_prologue_args)));
  const nib_qk_prologue_args& a = *args;
  NIB_REQUIRE(a.tokens >= 0 && a.num_heads >= 1 && a.num_kv_heads >= 1, "qk_prologue: bad sizes");
  if (a.tokens == 0) return NIB_OK;
  NIB_REQUIRE(a.q && a.k && a.q_out, "qk_prologue: null q/k pointer");
  const int E = 16 / elem_size(a.dtype);
  const bool store = a.key_cache != nullptr;
  NIB_REQUIRE(a.k_out || store, "qk_prologue: k_out may be NULL only when storing into the caches");
  NIB_REQUIRE(!store || (a.value_cache && a.v && a.slot_mapping), "qk_prologue: store needs v, caches and slot_mapping");
  NIB_REQUIRE(!a.norm || (a.q_weight && a.k_weight), "qk_prologue: norm needs q/k weights");
  NIB_REQUIRE(a.rope_mode >= NIB_ROPE_NONE && a.rope_mode <= NIB_ROPE_MROPE_INTERLEAVED, "qk_prologue: bad rope mode");
  NIB_REQUIRE(a.rope_mode == NIB_ROPE_NONE || a.positions, "qk_prologue: rope needs positions");
  NIB_REQUIRE(a.rope_mode != NIB_ROPE_TABLE || a.cos_sin_table, "qk_prologue: table rope needs the cos/sin table");
  if (a.rope_mode == NIB_ROPE_MROPE_CHUNKED || a.rope_mode == NIB_ROPE_MROPE_INTERLEAVED) {
    NIB_REQUIRE(a.inv_freq, "qk_prologue: M-RoPE needs inv_freq");
    NIB_REQUIRE(a.sections[0] > 0 && a.sections[1] > 0 && a.sections[2] > 0 &&
                    a.sections[0] + a.sections[1] + a.sections[2] == a.head_dim / 2,
                "qk_prologue: sections must be positive and sum to head_dim/2");
  }
  const void* vec_ptrs[] = {a.q, a.k, a.q_out, a.k_out ? a.k_out : a.q, store ? a.v : a.q,
                            store ? a.key_cache : a.q, store ? a.value_cache : a.q};
  for (const void* p : vec_ptrs) NIB_SUPPORT(aligned16(p), "qk_prologue: tensors must be 16-byte aligned");
  const int64_t strides[] = {a.q_token_stride, a.q_head_stride, a.k_token_stride, a.k_head_stride,
                             store ? a.v_token_stride : 0, store ? a.v_head_stride : 0,
                             store ? a.cache_slot_stride : 0};
  for (int64_t s : strides) NIB_SUPPORT(s % E == 0, "qk_prologue: strides must be multiples of %d elements", E);
  if (a.rope_mode == NIB_ROPE_TABLE) NIB_SUPPORT(aligned16(a.cos_sin_table), "qk_prologue: table must be 16-byte aligned");
  if (a.norm) NIB_SUPPORT(aligned16(a.q_weight) && aligned16(a.k_weight), "qk_prologue: weights must be 16-byte aligned");
  const cudaStream_t st = as_stream(stream);
  NIB_REQUIRE(a.variant >= 0 && a.variant <= 2, "qk_prologue: bad variant %d", a.variant);
  const bool pipe_ok = prologue_pipe_eligible(a);
  NIB_SUPPORT(a.variant != 2 || pipe_ok, "qk_prologue: the pipelined variant needs q/k/v as consecutive "
              "head ranges of one 16-byte aligned bf16/fp16 row");
  // rotary alone (the rotary modules' forward): one warp per token, all loads first; the
  // pipelined kernel reached 69-81% of the copy bandwidth on these launches
  if (a.variant == 0 && rope_rows_eligible(a)) return launch_rope_rows(a, st);
  if (a.variant == 2 || (a.variant == 0 && pipe_ok && a.tokens >= kPipeMinTokens))
    return launch_prologue_pipe(a, st);
  NIB_DISPATCH(a.dtype, T, {
    if (!a.norm || a.weight_dtype == a.dtype) return launch_prologue<T, T>(a, st);
    if (a.weight_dtype == NIB_F32) return launch_prologue<T, float>(a, st);
    set_error("qk_prologue: weight dtype must equal the activation dtype or be float32");
    return NIB_ERR_UNSUPPORTED;
  });
  return NIB_OK;
}

extern "C" int nib_mrope_apply(int x_dtype, const void* x, int64_t x_token_stride,
                               int64_t x_head_stride, int64_t tokens, int64_t heads, int64_t head_dim,
                               int cos_dtype, const void* cos, const void* sin,
                               const int32_t sections[3], int interleaved, void* out, void* stream) {
  NIB_REQUIRE(tokens >= 0 && heads >= 1 && head_dim >= 2 && head_dim % 2 == 0, "mrope_apply: bad sizes");
  if (tokens == 0) return NIB_OK;
  NIB_REQUIRE(x && cos && sin && out && sections, "mrope_apply: null pointer");
  const int64_t total = tokens * heads * head_dim;
  const cudaStream_t st = as_stream(stream);
  const unsigned grid = flat_grid(total, 16);
  const int D = static_cast<int>(head_dim);
  const int E = 16 / elem_size(x_dtype);
  if (cos_dtype == x_dtype && (D == 64 || D == 128 || D == 256) && aligned16(x) && aligned16(out) &&
      aligned16(cos) && aligned16(sin) && x_token_stride % E == 0 && x_head_stride % E == 0 &&
      heads <= 65535) {
    // one-shot grid: 7% faster on B200 than 16 persistent CTAs per SM
    int64_t blocks = (tokens + kApplyWarps - 1) / kApplyWarps;
    const int64_t cap = kMaxGrid;
    if (blocks > cap) blocks = cap;
    const unsigned nb = static_cast<unsigned>(blocks);
    const int th = kApplyWarps * 32;
#define NIB_APPLY_VEC(TT)                                                                          \
    do {                                                                                           \
      auto run = [&](auto dtag) {                                                                  \
        constexpr int DD = decltype(dtag)::value;                                                  \
        auto kern = interleaved ? mrope_apply_vec_kernel<TT, DD, true>                             \
                                : mrope_apply_vec_kernel<TT, DD, false>;                           \
        ::nib::launch_k(kern, nb, th, 0, st,                                                                    \
            static_cast<const TT*>(x), x_token_stride, x_head_stride, tokens, static_cast<int>(heads), \
            static_cast<const TT*>(cos), static_cast<const TT*>(sin), sections[0], sections[1],   \
            sections[2], static_cast<TT*>(out));                                                  \
      };                                                                                           \
      if (D == 64) run(std::integral_constant<int, 64>{});                                         \
      else if (D == 128) run(std::integral_constant<int, 128>{});                                  \
      else run(std::integral_constant<int, 256>{});                                                \
    } while (0)
    NIB_DISPATCH(x_dtype, TX, NIB_APPLY_VEC(TX));
#undef NIB_APPLY_VEC
    return launch_status("mrope_apply");
  }
#define NIB_MROPE_APPLY(TX, TC, TO)                                                              \
  ::nib::launch_k(mrope_apply_kernel<TX, TC, TO>, grid, 256, 0, st,                                           \
      static_cast<const TX*>(x), x_token_stride, x_head_stride, tokens, heads, D,                \
      static_cast<const TC*>(cos), static_cast<const TC*>(sin), sections[0], sections[1],        \
      sections[2], interleaved, static_cast<TX*>(out))
  NIB_DISPATCH(x_dtype, TX, {
    if (cos_dtype == x_dtype) {
      NIB_MROPE_APPLY(TX, TX, TX);
    } else if (cos_dtype == NIB_F32) {
      NIB_MROPE_APPLY(TX, float, float);
    } else if (cos_dtype == NIB_F16) {
      NIB_MROPE_APPLY(TX, __half, float);
    } else if (cos_dtype == NIB_BF16) {
      NIB_MROPE_APPLY(TX, __nv_bfloat16, float);
    } else {
      set_error("mrope_apply: bad cos dtype %d", cos_dtype);
      return NIB_ERR_UNSUPPORTED;
    }
  });
#undef NIB_MROPE_APPLY
  return launch_status("mrope_apply");
}

extern "C" int nib_mrope_cos_sin(const int64_t* positions, int64_t positions_axis_stride,
                                 int64_t positions_token_stride, int64_t tokens,
                                 const float* inv_freq, int64_t head_dim, int out_dtype, void* cos,
                                 void* sin, void* stream) {
  NIB_REQUIRE(tokens >= 0 && head_dim >= 2 && head_dim % 2 == 0, "mrope_cos_sin: bad sizes");
  if (tokens == 0) return NIB_OK;
  NIB_REQUIRE(positions && inv_freq && cos && sin, "mrope_cos_sin: null pointer");
  const cudaStream_t st = as_stream(stream);
  const int D = static_cast<int>(head_dim);
  const int es = elem_size(out_dtype);
  if ((D / 2) % 2 == 0 && reinterpret_cast<uintptr_t>(cos) % (2 * es) == 0 &&
      reinterpret_cast<uintptr_t>(sin) % (2 * es) == 0) {
    // one-shot grid, axis on y
    int64_t blocks = ((tokens + kCosSinTok - 1) / kCosSinTok * (D / 4) + 255) / 256;
    if (blocks > kMaxGrid) blocks = kMaxGrid;
    const dim3 grid(static_cast<unsigned>(blocks), 3);
#define NIB_COS_SIN_PAIR(HP)                                                                    \
  NIB_DISPATCH(out_dtype, TO,                                                                   \
               ::nib::launch_k(mrope_cos_sin_pair_kernel<TO, HP>, grid, 256, 0, st,                          \
                   positions, positions_axis_stride, positions_token_stride, tokens, inv_freq, D, \
                   static_cast<TO*>(cos), static_cast<TO*>(sin)))
    if (D == 64) {
      NIB_COS_SIN_PAIR(16);
    } else if (D == 128) {
      NIB_COS_SIN_PAIR(32);
    } else if (D == 256) {
      NIB_COS_SIN_PAIR(64);
    } else {
      NIB_COS_SIN_PAIR(0);
    }
#undef NIB_COS_SIN_PAIR
    return launch_status("mrope_cos_sin");
  }
  const unsigned grid = flat_grid(3 * tokens * (head_dim / 2), 16);
  NIB_DISPATCH(out_dtype, TO,
               ::nib::launch_k(mrope_cos_sin_any_kernel<TO>, grid, 256, 0, st,
                   positions, positions_axis_stride, positions_token_stride, tokens, inv_freq, D,
                   static_cast<TO*>(cos), static_cast<TO*>(sin)));
  return launch_status("mrope_cos_sin");
}
