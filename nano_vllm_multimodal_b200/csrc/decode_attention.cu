// Paged decode attention: one query token per request against its cached keys
// and values, read in place from the paged cache [blocks, block_size, kv_heads,
// head_dim]. Replaces flash_attn_with_kvcache(q.unsqueeze(1), k_cache, v_cache,
// cache_seqlens=context_lens, block_table=block_tables, softmax_scale,
// causal=True) at nanovllm/layers/attention.py:122-130; the numerical contract
// is the reference's SDPA decode branch (attention.py:286-300): softmax(q K^T *
// scale) V over the request's first context_lens[b] cached tokens, grouped-query
// heads sharing kv head h / (num_heads / num_kv_heads).
//
// This file is the CUDA-core kernel: bf16/f16 at any head_dim the ABI takes,
// and every layout the tensor-core kernel (decode_attention_mma.cu, the
// default where it applies) does not take. Its arithmetic runs in fp32 and the
// design is about bytes in flight:
//   * a CTA owns (request, kv head, split of the context); its warps split
//     the q heads of that kv head (two per warp) and the tokens;
//   * a token's 16-byte K and V vectors are spread over D/8 lanes, so one warp
//     step covers 32/(D/8) tokens; each lane copies its own vectors of U steps
//     per stage with cp.async into a per-warp ring of S shared-memory stages,
//     S - 1 stages ahead of the one it computes on, so the bytes in flight do
//     not cost registers;
//   * scores are kept in the log2 domain (q pre-scaled by scale * log2 e) with
//     an online max / sum per lane group; groups, warps and (for long contexts
//     with few requests) splits are merged with the usual max-rescaled sums.
#include <type_traits>

#include "dispatch.cuh"

namespace nib {

// the tensor-core kernel (decode_attention_mma.cu)
bool decode_mma_eligible(const nib_decode_attention_args& a);
size_t decode_mma_smem(int head_dim);
int launch_decode_mma(const nib_decode_attention_args& a, int splits, cudaStream_t st);

constexpr int kDecodeWarps = 8;
constexpr int kDecodeUnroll = 2;           // token steps per stage
constexpr int kDecodeStages = 2;           // ring stages per warp
constexpr int kDecodeMinBlocks = 2;        // resident CTAs per SM the registers are sized for
constexpr int kDecodeVecs = 2;             // 16-byte vectors per lane and token (1 or 2)
constexpr int64_t kDecodeSplitTokens = 0;  // > 0: at most this many tokens per split

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, bool pred) {
  const uint32_t s = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(s), "l"(gmem), "r"(pred ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// Packed fp32 pairs (sm_100 f32x2): two fp32 FMAs or multiplies per instruction.
// Attention has no bit-exact target, so fused forms are what is wanted here.
using f2_t = unsigned long long;
__device__ __forceinline__ f2_t f2(float lo, float hi) {
  f2_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ float2 f2_split(f2_t v) {
  float2 r;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(r.x), "=f"(r.y) : "l"(v));
  return r;
}
__device__ __forceinline__ f2_t fma2(f2_t a, f2_t b, f2_t c) {
  f2_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}
__device__ __forceinline__ f2_t mul2(f2_t a, f2_t b) {
  f2_t r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
// the four element pairs of a 16-byte vector as packed fp32
template <typename T>
__device__ __forceinline__ void unpack_pairs(const uint4& v, f2_t* out) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    if constexpr (std::is_same<T, __nv_bfloat16>::value) {
      out[i] = f2(__uint_as_float(w[i] << 16), __uint_as_float(w[i] & 0xffff0000u));
    } else {
      const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
      out[i] = f2(f.x, f.y);
    }
  }
}

__device__ __forceinline__ float ex2f(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

struct DecodeParams {
  const void* q;
  int64_t q_bs, q_hs;
  const void* kc;
  const void* vc;
  int64_t c_bs, c_ss, c_hs;  // cache block / slot / head strides (elements)
  int64_t num_blocks, block_size;
  int bs_shift;  // log2(block_size) when it is a power of two, else -1
  const int32_t* tables;
  int64_t table_stride, max_blocks;
  const int32_t* lens;
  float qscale;  // softmax scale * log2(e)
  void* out;
  int64_t o_bs, o_hs;
  float* ws;     // [batch, num_heads, splits, D + 2] partials when splits > 1
  int num_heads, num_kv_heads, group, splits, head_groups, token_groups;
  unsigned int* status;
};

// merge (m, l, acc) with (mo, lo, acco): log2-domain running max and sums; acc packed
template <int P>
__device__ __forceinline__ void merge_state(float& m, float& l, f2_t* acc, float mo, float lo,
                                            const f2_t* acco) {
  const float M = fmaxf(m, mo);
  if (M == -INFINITY) return;  // both empty
  const float a = ex2f(m - M), b = ex2f(mo - M);
  l = l * a + lo * b;
  const f2_t a2 = f2(a, a), b2 = f2(b, b);
#pragma unroll
  for (int k = 0; k < P; ++k) acc[k] = fma2(acco[k], b2, mul2(acc[k], a2));
  m = M;
}

template <typename T, int D, int HPW>
__global__ void __launch_bounds__(kDecodeWarps * 32, kDecodeMinBlocks)
decode_attention_kernel(const DecodeParams p) {
  ::nib::pdl_enter();
  constexpr int V = kDecodeVecs;       // 16-byte vectors per lane and token
  constexpr int E = Elem<T>::kPerVec * V;  // elements per lane and token
  constexpr int P = E / 2;             // packed pairs per lane and token
  constexpr int GS = D / E;            // lanes per token
  constexpr int TPS = 32 / GS;         // tokens per warp step
  constexpr int U = kDecodeUnroll;
  constexpr int S = kDecodeStages;
  static_assert(S * U <= 32, "stage masks live in one 32-bit word");
  // dynamic shared memory: the warps' cp.async rings, reused after the token
  // loop (behind a CTA barrier) as the [warps][HPW][D + 2] reduction buffer
  extern __shared__ __align__(16) unsigned char dsm[];
  float* red = reinterpret_cast<float*>(dsm);

  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int grp = lane / GS, gl = lane % GS;
  const int kvh = static_cast<int>(blockIdx.x % p.num_kv_heads);
  const int64_t b = blockIdx.x / p.num_kv_heads;
  const int split = blockIdx.y;
  const int hg = w / p.token_groups, tg = w % p.token_groups;
  const bool warp_active = hg < p.head_groups;

  int64_t len = __ldg(p.lens + b);
  const int64_t cap = p.max_blocks * p.block_size;
  if (len < 0 || len > cap) {
    if (threadIdx.x == 0 && split == 0) flag(p.status, NIB_DEV_BAD_INDEX);
    len = len < 0 ? 0 : cap;
  }
  const int64_t chunk = (len + p.splits - 1) / p.splits;
  const int64_t t_begin = split * chunk;
  const int64_t t_end = t_begin + chunk < len ? t_begin + chunk : len;

  // this warp's q heads (pre-scaled), fp32
  int head[HPW];
  bool hok[HPW];
  f2_t q[HPW][P];
#pragma unroll
  for (int j = 0; j < HPW; ++j) {
    const int hl = hg * HPW + j;  // head index within the kv group
    hok[j] = warp_active && hl < p.group;
    head[j] = kvh * p.group + (hok[j] ? hl : 0);
    float qv[E];
#pragma unroll
    for (int v = 0; v < V; ++v)
      unpack<T>(hok[j] ? ld_vec(static_cast<const T*>(p.q) + b * p.q_bs + head[j] * p.q_hs + gl * E + v * 8)
                       : zero_vec(), qv + v * 8);
#pragma unroll
    for (int k = 0; k < P; ++k) q[j][k] = f2(qv[2 * k] * p.qscale, qv[2 * k + 1] * p.qscale);
  }

  float m[HPW], l[HPW];
  f2_t acc[HPW][P];
#pragma unroll
  for (int j = 0; j < HPW; ++j) {
    m[j] = -INFINITY;
    l[j] = 0.f;
#pragma unroll
    for (int k = 0; k < P; ++k) acc[j][k] = 0ull;  // (+0, +0)
  }

  const T* kc = static_cast<const T*>(p.kc);
  const T* vc = static_cast<const T*>(p.vc);
  const int32_t* table = p.tables + b * p.table_stride;
  const int64_t head_off = kvh * p.c_hs + gl * E;
  const int64_t stride = static_cast<int64_t>(p.token_groups) * TPS;  // tokens between a group's steps
  if (warp_active) {
    // ring slot of (stage, token step, K|V) for this lane; each lane reads back only
    // what it copied itself, so a lane's cp.async.wait_group is all the ordering needed
    uint4* ring = reinterpret_cast<uint4*>(dsm) + static_cast<size_t>(w) * (S * U * 2 * 32 * V);
    auto slot = [&](int st, int u, int kind) { return ring + (((st * U + u) * 2 + kind) * 32 + lane) * V; };
    const uint32_t bsz = static_cast<uint32_t>(p.block_size);
    const int64_t first = t_begin + tg * TPS;  // this warp's first step
    const int64_t step = stride * U;           // tokens between a warp's stages
    // warp-uniform iteration count (the shuffles below need every lane); a group's
    // token is t = first + it * step + u * stride + grp, masked past t_end.
    // Token indices are < 2^31 (host check).
    const int64_t n_iter = first < t_end ? (t_end - first + step - 1) / step : 0;
    uint32_t okbits = 0;  // U bits per stage: token present and its block id valid
    auto issue = [&](int64_t it) {
      const int st = static_cast<int>(it % S);
      uint32_t mask = 0;
      if (it < n_iter) {
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int64_t t = first + it * step + u * stride + grp;
          bool ok = t < t_end;
          const uint32_t ut = static_cast<uint32_t>(t);
          const uint32_t bi = p.bs_shift >= 0 ? ut >> p.bs_shift : ut / bsz;
          const uint32_t bo = p.bs_shift >= 0 ? ut & (bsz - 1) : ut - bi * bsz;
          int64_t blk = 0;
          if (ok) {
            blk = __ldg(table + bi);
            if (blk < 0 || blk >= p.num_blocks) {
              flag(p.status, NIB_DEV_BAD_BLOCK);
              ok = false;  // the token does not take part
            }
          }
          const int64_t off = ok ? blk * p.c_bs + static_cast<int64_t>(bo) * p.c_ss + head_off : 0;
#pragma unroll
          for (int v = 0; v < V; ++v) {  // not ok: nothing read, zeros written
            cp_async16(slot(st, u, 0) + v, kc + off + v * 8, ok);
            cp_async16(slot(st, u, 1) + v, vc + off + v * 8, ok);
          }
          mask |= static_cast<uint32_t>(ok) << u;
        }
      }
      okbits = (okbits & ~(((1u << U) - 1) << (st * U))) | (mask << (st * U));
      cp_async_commit();  // one group per stage, empty past the end
    };
#pragma unroll
    for (int it = 0; it < S - 1; ++it) issue(it);
    for (int64_t it = 0; it < n_iter; ++it) {
      issue(it + S - 1);
      cp_async_wait<S - 1>();  // this lane's copies of stage `it` have landed
      const int st = static_cast<int>(it % S);
      bool ok[U];
#pragma unroll
      for (int u = 0; u < U; ++u) ok[u] = (okbits >> (st * U + u)) & 1u;
      float s[U][HPW];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        f2_t kp[P];
#pragma unroll
        for (int v = 0; v < V; ++v) unpack_pairs<T>(slot(st, u, 0)[v], kp + v * 4);
#pragma unroll
        for (int j = 0; j < HPW; ++j) {
          f2_t d = 0ull;
#pragma unroll
          for (int k = 0; k < P; ++k) d = fma2(q[j][k], kp[k], d);
          const float2 dd = f2_split(d);
          s[u][j] = dd.x + dd.y;
        }
      }
#pragma unroll
      for (int off = GS / 2; off > 0; off >>= 1) {
#pragma unroll
        for (int u = 0; u < U; ++u) {
#pragma unroll
          for (int j = 0; j < HPW; ++j) s[u][j] += __shfl_xor_sync(0xffffffffu, s[u][j], off);
        }
      }
#pragma unroll
      for (int j = 0; j < HPW; ++j) {
        float mx = m[j];
#pragma unroll
        for (int u = 0; u < U; ++u)
          if (ok[u]) mx = fmaxf(mx, s[u][j]);
        if (mx == -INFINITY) continue;  // nothing seen yet
        const float r = ex2f(m[j] - mx);
        l[j] *= r;
        const f2_t r2 = f2(r, r);
#pragma unroll
        for (int k = 0; k < P; ++k) acc[j][k] = mul2(acc[j][k], r2);
        m[j] = mx;
#pragma unroll
        for (int u = 0; u < U; ++u) {
          if (!ok[u]) continue;
          const float pr = ex2f(s[u][j] - mx);
          l[j] += pr;
          const f2_t p2 = f2(pr, pr);
          f2_t vp[P];
#pragma unroll
          for (int v = 0; v < V; ++v) unpack_pairs<T>(slot(st, u, 1)[v], vp + v * 4);
#pragma unroll
          for (int k = 0; k < P; ++k) acc[j][k] = fma2(p2, vp[k], acc[j][k]);
        }
      }
    }
    cp_async_wait<0>();  // only empty groups can remain; leave none behind
  }

  // merge the TPS token groups of the warp (lanes gl, gl + GS, ...)
#pragma unroll
  for (int off = GS; off < 32; off <<= 1) {
#pragma unroll
    for (int j = 0; j < HPW; ++j) {
      const float mo = __shfl_xor_sync(0xffffffffu, m[j], off);
      const float lo = __shfl_xor_sync(0xffffffffu, l[j], off);
      f2_t ao[P];
#pragma unroll
      for (int k = 0; k < P; ++k) ao[k] = __shfl_xor_sync(0xffffffffu, acc[j][k], off);
      merge_state<P>(m[j], l[j], acc[j], mo, lo, ao);
    }
  }
  // one copy per warp into shared memory, then merge the token-group warps of each head
  constexpr int SW = D + 2;
  __syncthreads();  // every warp is done with its ring before it becomes `red`
  if (grp == 0) {
#pragma unroll
    for (int j = 0; j < HPW; ++j) {
      float* r = red + (w * HPW + j) * SW;
#pragma unroll
      for (int k = 0; k < P; ++k) {
        const float2 a2 = f2_split(acc[j][k]);
        r[gl * E + 2 * k] = a2.x;
        r[gl * E + 2 * k + 1] = a2.y;
      }
      if (gl == 0) {
        r[D] = m[j];
        r[D + 1] = l[j];
      }
    }
  }
  __syncthreads();
  const int heads_here = p.group;  // q heads of this kv head
  for (int idx = threadIdx.x; idx < heads_here * D; idx += blockDim.x) {
    const int hl = idx / D, d = idx % D;
    const int hgi = hl / HPW, j = hl % HPW;
    float M = -INFINITY;
    for (int t = 0; t < p.token_groups; ++t) M = fmaxf(M, red[((hgi * p.token_groups + t) * HPW + j) * SW + D]);
    float L = 0.f, A = 0.f;
    if (M != -INFINITY) {
      for (int t = 0; t < p.token_groups; ++t) {
        const float* r = red + ((hgi * p.token_groups + t) * HPW + j) * SW;
        const float f = ex2f(r[D] - M);
        L += r[D + 1] * f;
        A += r[d] * f;
      }
    }
    const int h = kvh * p.group + hl;
    if (p.splits == 1) {
      const float o = L > 0.f ? A / L : 0.f;
      static_cast<T*>(p.out)[b * p.o_bs + h * p.o_hs + d] = Elem<T>::from_f(o);
    } else {
      float* ws = p.ws + ((b * p.num_heads + h) * p.splits + split) * SW;
      ws[d] = A;
      if (d == 0) {
        ws[D] = M;
        ws[D + 1] = L;
      }
    }
  }
}

// out[b, h, d] from the split partials (max-rescaled sums)
constexpr int kCombineUnrolled = 8;  // split counts merged with one round of loads

template <typename T, int D>
__global__ void __launch_bounds__(D)
decode_combine_kernel(const DecodeParams p) {
  ::nib::pdl_enter();
  constexpr int SW = D + 2;
  const int64_t bh = blockIdx.x;  // b * num_heads + h
  const int64_t b = bh / p.num_heads;
  const int h = static_cast<int>(bh % p.num_heads);
  const int d = threadIdx.x;
  const float* ws = p.ws + bh * p.splits * SW;
  float M = -INFINITY;
  float L = 0.f, A = 0.f;
  if (p.splits <= kCombineUnrolled) {
    // every split's max, sum and element loaded at once: one memory round trip
    float m[kCombineUnrolled], l[kCombineUnrolled], o[kCombineUnrolled];
#pragma unroll
    for (int s = 0; s < kCombineUnrolled; ++s) {
      const bool in = s < p.splits;
      m[s] = in ? ws[s * SW + D] : -INFINITY;
      l[s] = in ? ws[s * SW + D + 1] : 0.f;
      o[s] = in ? ws[s * SW + d] : 0.f;
    }
#pragma unroll
    for (int s = 0; s < kCombineUnrolled; ++s) M = fmaxf(M, m[s]);
    if (M != -INFINITY) {
#pragma unroll
      for (int s = 0; s < kCombineUnrolled; ++s) {
        if (s < p.splits) {  // the same sums, in the same order, as the loop below
          const float f = ex2f(m[s] - M);
          L += l[s] * f;
          A += o[s] * f;
        }
      }
    }
  } else {
    for (int s = 0; s < p.splits; ++s) M = fmaxf(M, ws[s * SW + D]);
    if (M != -INFINITY) {
      for (int s = 0; s < p.splits; ++s) {
        const float f = ex2f(ws[s * SW + D] - M);
        L += ws[s * SW + D + 1] * f;
        A += ws[s * SW + d] * f;
      }
    }
  }
  static_cast<T*>(p.out)[b * p.o_bs + h * p.o_hs + d] = Elem<T>::from_f(L > 0.f ? A / L : 0.f);
}

// CTA shape and split count for a launch
struct DecodePlan {
  int hpw, head_groups, token_groups, warps, splits;
  size_t smem;
  bool mma;  // the tensor-core kernel runs
};

static DecodePlan decode_plan(const nib_decode_attention_args& a) {
  DecodePlan pl{};
  const int g = a.num_heads / a.num_kv_heads;
  pl.hpw = g >= 2 ? 2 : 1;
  pl.head_groups = (g + pl.hpw - 1) / pl.hpw;
  pl.token_groups = pl.head_groups >= kDecodeWarps ? 1 : kDecodeWarps / pl.head_groups;
  pl.warps = pl.head_groups * pl.token_groups;
  pl.mma = a.variant != 1 && decode_mma_eligible(a);
  // splits: enough CTAs for every SM, at least 256 tokens per split (tensor-core
  // kernel: at least 64, one 16-token tile per warp). The tensor-core kernel's
  // splits shrink linearly toward the last one (decode_attention_mma.cu), which
  // puts small CTAs in the grid's last wave; it asks for 12 CTAs per SM (about 4
  // waves at 3 resident) and at least 2 splits. Measured on C2's contexts
  // (U[1, 8192], ms per call, CTAs per SM wanted 8 / 12 / 16 / 24): GQA 8 with
  // 256 requests 0.191 / 0.183 / 0.184 / 0.191; 8/1 heads 0.102 / 0.104 / 0.110 /
  // 0.120; 64 requests of up to 32,768 tokens 0.183 / 0.181 / 0.185 / 0.192; GQA 2
  // with 256 requests 0.658 with one split, 0.641 with two.
  const int64_t ctas = a.batch * a.num_kv_heads;
  const int64_t want = (pl.mma ? 12LL : 4LL) * sm_count();
  int64_t s = ctas >= want ? 1 : (want + ctas - 1) / ctas;
  if (pl.mma && s < 2) s = 2;
  const int64_t max_len = a.max_context_len > 0 ? a.max_context_len : a.max_blocks_per_seq * a.block_size;
  const int64_t by_len = (max_len + (pl.mma ? 63 : 255)) / (pl.mma ? 64 : 256);
  if (kDecodeSplitTokens > 0) {
    const int64_t balance = (max_len + kDecodeSplitTokens - 1) / kDecodeSplitTokens;
    if (s < balance) s = balance;
  }
  if (s > by_len) s = by_len;
  if (s < 1) s = 1;
  if (s > 1024) s = 1024;
  pl.splits = static_cast<int>(s);
  const size_t red = static_cast<size_t>(pl.warps) * pl.hpw * (a.head_dim + 2) * sizeof(float);
  const size_t ring = static_cast<size_t>(pl.warps) * kDecodeStages * kDecodeUnroll * 2 * 32 * 16 * kDecodeVecs;
  pl.smem = red > ring ? red : ring;
  return pl;
}

static int64_t decode_workspace(const nib_decode_attention_args& a, const DecodePlan& pl) {
  return pl.splits > 1 ? a.batch * a.num_heads * pl.splits * (a.head_dim + 2) * static_cast<int64_t>(sizeof(float)) : 0;
}

static const char* decode_check(const nib_decode_attention_args* a) {
  if (a == nullptr || a->struct_size != static_cast<int32_t>(sizeof(nib_decode_attention_args)))
    return "decode_attention: args struct size mismatch";
  if (a->dtype != NIB_BF16 && a->dtype != NIB_F16) return "decode_attention: dtype must be bf16 or f16";
  if (a->head_dim != 64 && a->head_dim != 128 && a->head_dim != 256) return "decode_attention: head_dim must be 64, 128 or 256";
  if (a->batch < 0 || a->num_heads < 1 || a->num_kv_heads < 1 || a->num_heads % a->num_kv_heads != 0)
    return "decode_attention: bad head counts";
  if (a->num_heads / a->num_kv_heads > 2 * kDecodeWarps) return "decode_attention: more than 16 q heads per kv head";
  if (a->block_size < 1 || a->num_blocks < 0 || a->max_blocks_per_seq < 0) return "decode_attention: bad cache sizes";
  return nullptr;
}

template <typename T, int D, int HPW>
static int launch_decode(const nib_decode_attention_args& a, const DecodePlan& pl, cudaStream_t st) {
  DecodeParams p{};
  p.q = a.q;
  p.q_bs = a.q_batch_stride;
  p.q_hs = a.q_head_stride;
  p.kc = a.key_cache;
  p.vc = a.value_cache;
  p.c_bs = a.cache_block_stride;
  p.c_ss = a.cache_slot_stride;
  p.c_hs = a.cache_head_stride;
  p.num_blocks = a.num_blocks;
  p.block_size = a.block_size;
  p.bs_shift = -1;
  for (int k = 0; k < 31; ++k)
    if ((int64_t{1} << k) == a.block_size) p.bs_shift = k;
  p.tables = a.block_tables;
  p.table_stride = a.block_table_stride;
  p.max_blocks = a.max_blocks_per_seq;
  p.lens = a.context_lens;
  p.qscale = a.scale * 1.4426950408889634f;
  p.out = a.out;
  p.o_bs = a.out_batch_stride;
  p.o_hs = a.out_head_stride;
  p.ws = static_cast<float*>(a.workspace);
  p.num_heads = a.num_heads;
  p.num_kv_heads = a.num_kv_heads;
  p.group = a.num_heads / a.num_kv_heads;
  p.splits = pl.splits;
  p.head_groups = pl.head_groups;
  p.token_groups = pl.token_groups;
  p.status = a.status;
  const dim3 grid(static_cast<unsigned>(a.batch * a.num_kv_heads), static_cast<unsigned>(pl.splits));
  auto kernel = decode_attention_kernel<T, D, HPW>;
  static int configured[64] = {0};  // per device: dynamic shared memory opted in
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && configured[dev] < static_cast<int>(pl.smem)) {
    const cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               static_cast<int>(pl.smem));
    if (e != cudaSuccess) {
      set_error("decode_attention: cannot reserve shared memory: %s", cudaGetErrorString(e));
      return NIB_ERR_CUDA;
    }
    configured[dev] = static_cast<int>(pl.smem);
  }
  ::nib::launch_k(kernel, grid, pl.warps * 32, pl.smem, st, p);
  if (pl.splits > 1) ::nib::launch_k_after(decode_combine_kernel<T, D>, static_cast<unsigned>(a.batch * a.num_heads), D, 0, st, p);
  return launch_status("decode_attention");
}

// the split partials' combine after the tensor-core kernel (same workspace format)
template <typename T, int D>
static int launch_combine(const nib_decode_attention_args& a, int splits, cudaStream_t st) {
  DecodeParams p{};
  p.out = a.out;
  p.o_bs = a.out_batch_stride;
  p.o_hs = a.out_head_stride;
  p.ws = static_cast<float*>(a.workspace);
  p.num_heads = a.num_heads;
  p.splits = splits;
  ::nib::launch_k_after(decode_combine_kernel<T, D>, static_cast<unsigned>(a.batch * a.num_heads), D, 0, st, p);
  return launch_status("decode_attention (combine)");
}

template <typename T, int D>
static int launch_decode_d(const nib_decode_attention_args& a, const DecodePlan& pl, cudaStream_t st) {
  return pl.hpw == 2 ? launch_decode<T, D, 2>(a, pl, st) : launch_decode<T, D, 1>(a, pl, st);
}

}  // namespace nib

using namespace nib;

extern "C" int64_t nib_decode_attention_workspace_bytes(const nib_decode_attention_args* a) {
  if (decode_check(a) != nullptr) return -1;
  return decode_workspace(*a, decode_plan(*a));
}

extern "C" int nib_decode_attention(const nib_decode_attention_args* a, void* stream) {
  const char* bad = decode_check(a);
  if (bad != nullptr) {
    set_error("%s", bad);
    return NIB_ERR_INVALID;
  }
  if (a->batch == 0) return NIB_OK;
  NIB_REQUIRE(a->q && a->key_cache && a->value_cache && a->block_tables && a->context_lens && a->out,
              "decode_attention: null pointer");
  NIB_REQUIRE(a->batch * a->num_kv_heads <= 0x7fffffffLL, "decode_attention: batch too large");
  NIB_REQUIRE(a->max_blocks_per_seq * a->block_size < (int64_t{1} << 31),
              "decode_attention: block table covers 2^31 tokens or more");
  const int E = 8;
  NIB_SUPPORT(aligned16(a->q) && aligned16(a->key_cache) && aligned16(a->value_cache),
              "decode_attention: q and caches must be 16-byte aligned");
  NIB_SUPPORT(a->q_batch_stride % E == 0 && a->q_head_stride % E == 0 && a->cache_block_stride % E == 0 &&
                  a->cache_slot_stride % E == 0 && a->cache_head_stride % E == 0,
              "decode_attention: strides must be multiples of 8 elements");
  const DecodePlan pl = decode_plan(*a);
  const int64_t need = decode_workspace(*a, pl);
  NIB_REQUIRE(need == 0 || (a->workspace && a->workspace_bytes >= need && aligned16(a->workspace)),
              "decode_attention: workspace of %lld bytes needed", static_cast<long long>(need));
  const cudaStream_t st = as_stream(stream);
  NIB_REQUIRE(a->variant >= 0 && a->variant <= 2, "decode_attention: bad variant %d", a->variant);
  if (pl.mma) {
    const int rc = launch_decode_mma(*a, pl.splits, st);
    if (rc != NIB_OK || pl.splits == 1) return rc;
    if (a->dtype == NIB_BF16)
      return a->head_dim == 64 ? launch_combine<__nv_bfloat16, 64>(*a, pl.splits, st)
                               : launch_combine<__nv_bfloat16, 128>(*a, pl.splits, st);
    return a->head_dim == 64 ? launch_combine<__half, 64>(*a, pl.splits, st) : launch_combine<__half, 128>(*a, pl.splits, st);
  }
  NIB_SUPPORT(a->variant != 2, "decode_attention: the tensor-core kernel needs bf16/f16, head_dim 64 or 128, "
              "at most 16 q heads per kv head, a block size that is a multiple of 16 and 16-byte aligned strides");
  if (pl.smem > 200 * 1024) {
    set_error("decode_attention: shared-memory ring too large");
    return NIB_ERR_UNSUPPORTED;
  }
  if (a->dtype == NIB_BF16) {
    switch (a->head_dim) {
      case 64: return launch_decode_d<__nv_bfloat16, 64>(*a, pl, st);
      case 128: return launch_decode_d<__nv_bfloat16, 128>(*a, pl, st);
      default: return launch_decode_d<__nv_bfloat16, 256>(*a, pl, st);
    }
  }
  switch (a->head_dim) {
    case 64: return launch_decode_d<__half, 64>(*a, pl, st);
    case 128: return launch_decode_d<__half, 128>(*a, pl, st);
    default: return launch_decode_d<__half, 256>(*a, pl, st);
  }
}
