// Rotary embedding alone: the forward of the rotary modules
// (RotaryEmbedding.forward, nanovllm/layers/rotary_embedding.py:37-48;
// MultimodalRotaryEmbedding.forward, multimodal_rotary_embedding.py:103-117),
// i.e. nib_qk_prologue without norm and without store.
//
// A warp per token and a one-shot grid. Every head vector of the token (q and
// k, any token / head strides) is loaded before any math, so a warp has the
// whole 6 KB row of a 16/8-head token in flight at once and the SM's many
// resident warps hide the latency - the design of the vectorised M-RoPE apply
// kernel, which reaches the copy roofline. cos/sin come from the fp32 table
// row of the token's position (1-D) or, for M-RoPE, from sincosf of the
// token's three positions: each lane computes D/64 of the D/2 frequencies and
// shuffles them to the lanes that rotate with them. Same lane layout and the
// same rotation routine as the prologue kernels (prologue_math.cuh), so the
// results are bit-identical to theirs.
#include "dispatch.cuh"
#include "prologue.cuh"
#include "prologue_math.cuh"

namespace nib {

constexpr int kRopeMaxSteps = 8;  // head steps per warp: (nq + nkv) <= 8 * 32 / (D / 16)

template <typename T, int D, int MODE>
__global__ void __launch_bounds__(256)
rope_rows_kernel(const nib_qk_prologue_args a) {
  pdl_enter();
  constexpr int E = 8;            // 16-bit elements per 16-byte vector
  constexpr int L = D / (2 * E);  // lanes per head
  constexpr int HPW = 32 / L;     // heads per warp step
  constexpr int NF = D / 2;       // frequencies
  constexpr int FPL = (NF + 31) / 32;
  constexpr bool kTable = MODE == NIB_ROPE_TABLE;
  constexpr bool kInter = MODE == NIB_ROPE_MROPE_INTERLEAVED;
  const int lane = threadIdx.x & 31;
  const int hs = lane / L, l = lane % L, fb = l * E;
  const int nq = a.num_heads, nkv = a.num_kv_heads, nh = nq + nkv;
  const int steps = (nh + HPW - 1) / HPW;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  const T* q = static_cast<const T*>(a.q);
  const T* k = static_cast<const T*>(a.k);
  T* qo = static_cast<T*>(a.q_out);
  T* ko = static_cast<T*>(a.k_out);

  for (int64_t t = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); t < a.tokens;
       t += warps) {
    // ---- every load of the token first
    int64_t p0 = __ldg(a.positions + t * a.positions_token_stride), p1 = 0, p2 = 0;
    if constexpr (!kTable) {
      p1 = __ldg(a.positions + a.positions_axis_stride + t * a.positions_token_stride);
      p2 = __ldg(a.positions + 2 * a.positions_axis_stride + t * a.positions_token_stride);
    }
    uint4 va[kRopeMaxSteps], vb[kRopeMaxSteps];
#pragma unroll
    for (int u = 0; u < kRopeMaxSteps; ++u) {
      const int h = u * HPW + hs;
      va[u] = vb[u] = zero_vec();
      if (u < steps && h < nh) {
        const T* src = h < nq ? q + t * a.q_token_stride + static_cast<int64_t>(h) * a.q_head_stride
                              : k + t * a.k_token_stride + static_cast<int64_t>(h - nq) * a.k_head_stride;
        va[u] = ld_stream(src + fb);
        vb[u] = ld_stream(src + NF + fb);
      }
    }
    // ---- cos / sin of this lane's E frequencies
    float c[E], s[E];
    if constexpr (kTable) {
      if (p0 >= 0 && p0 < a.table_rows) {
        const float* tab = a.cos_sin_table + p0 * D;
#pragma unroll
        for (int e = 0; e < E; e += 4) {
          *reinterpret_cast<float4*>(c + e) = __ldg(reinterpret_cast<const float4*>(tab + fb + e));
          *reinterpret_cast<float4*>(s + e) = __ldg(reinterpret_cast<const float4*>(tab + NF + fb + e));
        }
      } else {
        if (l == 0 && hs == 0) flag(a.status, NIB_DEV_BAD_POSITION);
#pragma unroll
        for (int e = 0; e < E; ++e) c[e] = s[e] = 0.f;
      }
    } else {
      float cm[FPL], sm[FPL];  // frequency lane + 32 m
#pragma unroll
      for (int m = 0; m < FPL; ++m) {
        const int j = lane + 32 * m;
        cm[m] = sm[m] = 0.f;
        if (j < NF) {
          const int ax = mrope_axis(j, kInter, a.sections);
          const int64_t p = ax == 0 ? p0 : (ax == 1 ? p1 : p2);
          float sn, cs;
          sincosf(__fmul_rn(static_cast<float>(p), __ldg(a.inv_freq + j)), &sn, &cs);
          cm[m] = round_to<T>(cs);
          sm[m] = round_to<T>(sn);
        }
      }
#pragma unroll
      for (int e = 0; e < E; ++e) {
        const int f = fb + e;
        float cv = 0.f, sv = 0.f;
#pragma unroll
        for (int m = 0; m < FPL; ++m) {  // f / 32 is the same for the whole warp per (e, m)
          const float cx = __shfl_sync(0xffffffffu, cm[m], f & 31);
          const float sx = __shfl_sync(0xffffffffu, sm[m], f & 31);
          if (f / 32 == m) {
            cv = cx;
            sv = sx;
          }
        }
        c[e] = cv;
        s[e] = sv;
      }
    }
    uint32_t c2[4], s2[4];
    if constexpr (kInter) pack_trig<T>(c, s, c2, s2);
    // ---- rotate and store
#pragma unroll
    for (int u = 0; u < kRopeMaxSteps; ++u) {
      const int h = u * HPW + hs;
      if (u >= steps || h >= nh) continue;
      float xa[E], xb[E];
      uint32_t wa[4], wb[4];
      unpack<T>(va[u], xa);
      unpack<T>(vb[u], xb);
      from_u4(va[u], wa);
      from_u4(vb[u], wb);
      rotate_pair<T>(xa, xb, wa, wb, c, s, c2, s2, kInter);
      T* dst = h < nq ? qo + (t * nq + h) * D : ko + (t * nkv + (h - nq)) * D;
      st_vec(dst + fb, as_u4(wa));
      st_vec(dst + NF + fb, as_u4(wb));
    }
  }
}

// whether the rotary-only kernel takes this call: rotary on, no norm, no store,
// 16-bit activations, head_dim 64/128/256, at most kRopeMaxSteps head steps,
// 16-byte aligned rows and strides (checked by the caller)
bool rope_rows_eligible(const nib_qk_prologue_args& a) {
  if (a.rope_mode == NIB_ROPE_NONE || a.norm || a.key_cache) return false;
  if (a.dtype != NIB_BF16 && a.dtype != NIB_F16) return false;
  if (a.head_dim != 64 && a.head_dim != 128 && a.head_dim != 256) return false;
  if (!a.k_out) return false;
  const int hpw = 32 / (a.head_dim / 16);
  return a.num_heads + a.num_kv_heads <= kRopeMaxSteps * hpw;
}

template <typename T, int D>
static int launch_rope_d(const nib_qk_prologue_args& a, cudaStream_t st) {
  const int64_t blocks64 = (a.tokens + 7) / 8;
  const unsigned blocks = static_cast<unsigned>(blocks64 < kMaxGrid ? blocks64 : kMaxGrid);
  switch (a.rope_mode) {
    case NIB_ROPE_TABLE: ::nib::launch_k(rope_rows_kernel<T, D, NIB_ROPE_TABLE>, blocks, 256, 0, st, a); break;
    case NIB_ROPE_MROPE_CHUNKED:
      ::nib::launch_k(rope_rows_kernel<T, D, NIB_ROPE_MROPE_CHUNKED>, blocks, 256, 0, st, a);
      break;
    default: ::nib::launch_k(rope_rows_kernel<T, D, NIB_ROPE_MROPE_INTERLEAVED>, blocks, 256, 0, st, a); break;
  }
  return launch_status("qk_prologue (rotary only)");
}

template <typename T>
static int launch_rope_t(const nib_qk_prologue_args& a, cudaStream_t st) {
  switch (a.head_dim) {
    case 64: return launch_rope_d<T, 64>(a, st);
    case 128: return launch_rope_d<T, 128>(a, st);
    default: return launch_rope_d<T, 256>(a, st);
  }
}

int launch_rope_rows(const nib_qk_prologue_args& a, cudaStream_t st) {
  return a.dtype == NIB_BF16 ? launch_rope_t<__nv_bfloat16>(a, st) : launch_rope_t<__half>(a, st);
}

}  // namespace nib
