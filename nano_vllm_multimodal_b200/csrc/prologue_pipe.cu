// Attention prologue, pipelined variant for the fused-qkv layout.
//
// Same math and rounding points as qk_prologue_kernel (rope.cu), so results
// are bit-identical; only the data movement differs. When q, k and v are the
// three head ranges of one qkv row (the layout every NanoInfer decoder
// produces: nanovllm/models/qwen3.py:77-81), each warp owns a contiguous
// range of tokens and streams their rows [q|k|v] - plus the 1-D RoPE table row
// of the token - into a private ring of shared-memory stages with
// cp.async.bulk, `stages - 1` tokens ahead of the token it is computing. The
// bytes in flight no longer depend on registers or on how long the math
// takes. Per-token metadata (slot, positions) is fetched 32 tokens at a time
// with one coalesced load and broadcast by shuffles.
//
// Packed bf16x2 / f16x2 arithmetic is used only where it is bit-identical to
// the scalar fp32-then-round sequence: products and sums of two 16-bit values
// rounded once (the exact product of two bf16/fp16 values fits in fp32, and
// their fp32 sum never lands on a 16-bit rounding midpoint it did not hold
// exactly).
#include "bulk_copy.cuh"
#include "dispatch.cuh"
#include "prologue.cuh"

namespace nib {

template <typename T> struct Packed;
template <> struct Packed<__nv_bfloat16> {
  using P = __nv_bfloat162;
  __device__ __forceinline__ static P mul(P a, P b) { return __hmul2_rn(a, b); }
  __device__ __forceinline__ static P add(P a, P b) { return __hadd2_rn(a, b); }
  __device__ __forceinline__ static P neg(P a) { return __hneg2(a); }
  __device__ __forceinline__ static P make(float lo, float hi) { return __floats2bfloat162_rn(lo, hi); }
};
template <> struct Packed<__half> {
  using P = __half2;
  __device__ __forceinline__ static P mul(P a, P b) { return __hmul2_rn(a, b); }
  __device__ __forceinline__ static P add(P a, P b) { return __hadd2_rn(a, b); }
  __device__ __forceinline__ static P neg(P a) { return __hneg2(a); }
  __device__ __forceinline__ static P make(float lo, float hi) { return __floats2half2_rn(lo, hi); }
};

template <typename P>
__device__ __forceinline__ uint32_t bits(P v) { return *reinterpret_cast<uint32_t*>(&v); }
template <typename P>
__device__ __forceinline__ P from_bits(uint32_t w) { return *reinterpret_cast<P*>(&w); }

constexpr int kUG = 4;  // head groups per compute phase

struct TokenMeta {
  int32_t slot;
  int64_t p0, p1, p2;
};

template <typename T, typename W, int D>
__global__ void __launch_bounds__(kPipeMaxWarps * 32, 1)
qk_prologue_pipe_kernel(const nib_qk_prologue_args a, const int stages, const uint32_t row_bytes,
                        const uint32_t stage_bytes) {
  constexpr int E = 8;  // 16-bit activations: 8 per 16-byte vector
  constexpr int LPH = D / E;
  constexpr int HPW = 32 / LPH;
  constexpr int HALF = LPH / 2;
  constexpr int NF = D / 2;
  constexpr int FPL = (NF + 31) / 32;
  using PK = Packed<T>;
  using P = typename PK::P;

  extern __shared__ __align__(128) unsigned char smem[];
  const int lane = threadIdx.x & 31;
  const int wib = threadIdx.x >> 5;
  const int wpc = blockDim.x >> 5;
  unsigned char* wbuf = smem + static_cast<size_t>(wib) * stages * stage_bytes;
  unsigned char* tail = smem + static_cast<size_t>(wpc) * stages * stage_bytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(tail) + wib * stages;
  float* trig = reinterpret_cast<float*>(tail + static_cast<size_t>(wpc) * stages * 8) + wib * 2 * NF;

  const int hs = lane / LPH;
  const int l = lane % LPH;
  const bool first = l < HALF;
  const int fb = (l % HALF) * E;
  const int nq = a.num_heads, nkv = a.num_kv_heads;
  const bool store = a.key_cache != nullptr;
  const int Uq = (nq + HPW - 1) / HPW;
  const int Uk = (nkv + HPW - 1) / HPW;
  const int mode = a.rope_mode;
  const bool table = mode == NIB_ROPE_TABLE;
  const bool mrope = mode == NIB_ROPE_MROPE_CHUNKED || mode == NIB_ROPE_MROPE_INTERLEAVED;
  const bool inter = mode == NIB_ROPE_MROPE_INTERLEAVED;
  const uint32_t tab_bytes = table ? D * 4 : 0;

  const int64_t ntok = a.tokens;
  const int64_t gw = static_cast<int64_t>(blockIdx.x) * wpc + wib;
  const int64_t nw = static_cast<int64_t>(gridDim.x) * wpc;
  const int64_t tb = ntok * gw / nw;
  const int64_t n = ntok * (gw + 1) / nw - tb;
  if (n <= 0) return;

  const char* rows = static_cast<const char*>(a.q);
  const int64_t row_stride = a.q_token_stride * static_cast<int64_t>(sizeof(T));
  T* q_out = static_cast<T*>(a.q_out);
  T* k_out = static_cast<T*>(a.k_out);
  T* kc = static_cast<T*>(a.key_cache);
  T* vc = static_cast<T*>(a.value_cache);

  if (lane == 0) {
    for (int s = 0; s < stages; ++s) mbar_init(&bars[s], 1);
    fence_mbar_init();
  }
  __syncwarp();

  // ---- per-lane constants: norm weights, M-RoPE frequency layout
  float wq[E], wk[E];
  if (a.norm) {
    load_weights<T, W>(static_cast<const W*>(a.q_weight), l * E, wq);
    load_weights<T, W>(static_cast<const W*>(a.k_weight), l * E, wk);
  }
  int fax[FPL];
  float finv[FPL];
#pragma unroll
  for (int m = 0; m < FPL; ++m) {
    const int j = lane + 32 * m;
    fax[m] = 0;
    finv[m] = 0.f;
    if (mrope && j < NF) {
      if (inter) {
        const int r = j % 3;
        fax[m] = (r == 1 && j < 3 * a.sections[1]) ? 1 : (r == 2 && j < 3 * a.sections[2]) ? 2 : 0;
      } else {
        fax[m] = j < a.sections[0] ? 0 : (j < a.sections[0] + a.sections[1] ? 1 : 2);
      }
      finv[m] = __ldg(a.inv_freq + j);
    }
  }

  // ---- metadata, 32 tokens per batch (lane j holds token 32*b + j)
  auto load_meta = [&](int64_t b) {
    TokenMeta m{-1, 0, 0, 0};
    const int64_t i = 32 * b + lane;
    if (i < n) {
      const int64_t t = tb + i;
      if (store) m.slot = __ldg(a.slot_mapping + t);
      if (mode != NIB_ROPE_NONE) {
        m.p0 = __ldg(a.positions + t * a.positions_token_stride);
        if (mrope) {
          m.p1 = __ldg(a.positions + a.positions_axis_stride + t * a.positions_token_stride);
          m.p2 = __ldg(a.positions + 2 * a.positions_axis_stride + t * a.positions_token_stride);
        }
      }
    }
    return m;
  };
  TokenMeta cur = load_meta(0), nxt = load_meta(1);
  auto pick32 = [&](int32_t c, int32_t x, int idx) {
    const int32_t a0 = __shfl_sync(0xffffffffu, c, idx & 31);
    const int32_t a1 = __shfl_sync(0xffffffffu, x, idx & 31);
    return idx < 32 ? a0 : a1;
  };
  auto pick64 = [&](int64_t c, int64_t x, int idx) {
    const int64_t a0 = __shfl_sync(0xffffffffu, c, idx & 31);
    const int64_t a1 = __shfl_sync(0xffffffffu, x, idx & 31);
    return idx < 32 ? a0 : a1;
  };

  // ---- producer side: lane 0 streams row j (and its table row) into stage j % stages
  auto issue = [&](int64_t j, int64_t base) {
    const int idx = static_cast<int>(j - base);
    const int64_t p = table ? pick64(cur.p0, nxt.p0, idx) : 0;
    if (lane == 0) {
      const int st = static_cast<int>(j % stages);
      unsigned char* dst = wbuf + static_cast<size_t>(st) * stage_bytes;
      const bool tab_ok = table && p >= 0 && p < a.table_rows;
      fence_proxy_async();
      mbar_arrive_expect_tx(&bars[st], row_bytes + (tab_ok ? tab_bytes : 0u));
      bulk_load(dst, rows + (tb + j) * row_stride, row_bytes, &bars[st]);
      if (tab_ok) bulk_load(dst + row_bytes, a.cos_sin_table + p * D, tab_bytes, &bars[st]);
    }
  };

  for (int64_t j = 0; j < stages - 1 && j < n; ++j) issue(j, 0);

  for (int64_t i = 0; i < n; ++i) {
    const int64_t base = i & ~static_cast<int64_t>(31);
    if ((i & 31) == 0 && i > 0) {
      cur = nxt;
      nxt = load_meta(i / 32 + 1);
    }
    if (i + stages - 1 < n) issue(i + stages - 1, base);

    const int st = static_cast<int>(i % stages);
    const bool ok = mbar_wait(&bars[st], static_cast<uint32_t>((i / stages) & 1));
    if (!__all_sync(0xffffffffu, ok)) {
      if (lane == 0) flag(a.status, kDevTimeout);
      // let this warp's other copies land (bounded) before leaving
      for (int64_t j = i + 1; j < i + stages && j < n; ++j)
        (void)mbar_wait(&bars[j % stages], static_cast<uint32_t>((j / stages) & 1));
      return;
    }
    const int idx = static_cast<int>(i - base);
    const int64_t t = tb + i;
    const unsigned char* row = wbuf + static_cast<size_t>(st) * stage_bytes;
    const T* rq = reinterpret_cast<const T*>(row);

    int64_t slot = -1;
    if (store) {
      const int32_t sv = pick32(cur.slot, nxt.slot, idx);
      if (sv >= 0 && sv < a.num_slots) slot = sv;
      else if (sv != -1 && lane == 0) flag(a.status, NIB_DEV_BAD_SLOT);
    }

    // ---- cos / sin for this lane's E frequencies
    float c[E], s[E];
    if (table) {
      const int64_t p = pick64(cur.p0, nxt.p0, idx);
      if (p >= 0 && p < a.table_rows) {
        const float* tab = reinterpret_cast<const float*>(row + row_bytes);
#pragma unroll
        for (int e = 0; e < E; e += 4) {
          *reinterpret_cast<float4*>(c + e) = *reinterpret_cast<const float4*>(tab + fb + e);
          *reinterpret_cast<float4*>(s + e) = *reinterpret_cast<const float4*>(tab + NF + fb + e);
        }
      } else {
        if (lane == 0) flag(a.status, NIB_DEV_BAD_POSITION);
#pragma unroll
        for (int e = 0; e < E; ++e) c[e] = s[e] = 0.f;
      }
    } else if (mrope) {
      const int64_t pa0 = pick64(cur.p0, nxt.p0, idx);
      const int64_t pa1 = pick64(cur.p1, nxt.p1, idx);
      const int64_t pa2 = pick64(cur.p2, nxt.p2, idx);
#pragma unroll
      for (int m = 0; m < FPL; ++m) {
        const int j = lane + 32 * m;
        if (j < NF) {
          const int64_t p = fax[m] == 0 ? pa0 : (fax[m] == 1 ? pa1 : pa2);
          float sn, cs;
          sincosf(__fmul_rn(static_cast<float>(p), finv[m]), &sn, &cs);
          trig[j] = round_to<T>(cs);
          trig[NF + j] = round_to<T>(sn);
        }
      }
      __syncwarp();
#pragma unroll
      for (int e = 0; e < E; e += 4) {
        *reinterpret_cast<float4*>(c + e) = *reinterpret_cast<const float4*>(trig + fb + e);
        *reinterpret_cast<float4*>(s + e) = *reinterpret_cast<const float4*>(trig + NF + fb + e);
      }
    }
    P c2[E / 2], s2[E / 2];
    if (inter) {
#pragma unroll
      for (int k = 0; k < E / 2; ++k) {
        c2[k] = PK::make(c[2 * k], c[2 * k + 1]);  // exact: already rounded to T
        s2[k] = PK::make(s[2 * k], s[2 * k + 1]);
      }
    }

    // ---- q and k heads, kUG head groups per phase so that their dependency
    // chains (squares -> butterfly -> 1/sqrt -> scale -> shuffle -> rotate)
    // interleave instead of running back to back
    T* qo_t = q_out + t * nq * D + hs * D + l * E;
    T* ko_t = k_out + t * nkv * D + hs * D + l * E;
    T* kc_t = slot >= 0 ? kc + slot * a.cache_slot_stride + hs * D + l * E : nullptr;
    const T* rl = rq + hs * D + l * E;
    const int Uqk = Uq + Uk;
    for (int u0 = 0; u0 < Uqk; u0 += kUG) {
      uint32_t w32[kUG][4];
      float x[kUG][E];
      bool hok[kUG], isq[kUG];
      int hoff[kUG];  // head * D within q (or within k)
#pragma unroll
      for (int g = 0; g < kUG; ++g) {
        const int u = u0 + g;
        isq[g] = u < Uq;
        const int hg = isq[g] ? u : u - Uq;  // head group within q or k
        hoff[g] = hg * HPW * D;
        hok[g] = u < Uqk && hg * HPW + hs < (isq[g] ? nq : nkv);
        const uint4 raw = hok[g] ? *reinterpret_cast<const uint4*>(rl + (isq[g] ? 0 : nq * D) + hoff[g])
                                 : zero_vec();
        w32[g][0] = raw.x; w32[g][1] = raw.y; w32[g][2] = raw.z; w32[g][3] = raw.w;
        unpack<T>(raw, x[g]);
      }
      if (a.norm) {
        float ss[kUG];
#pragma unroll
        for (int g = 0; g < kUG; ++g) ss[g] = sumsq_tree<E>(x[g]);
#pragma unroll
        for (int off = HALF; off > 0; off >>= 1) {
#pragma unroll
          for (int g = 0; g < kUG; ++g) ss[g] = __fadd_rn(ss[g], __shfl_xor_sync(0xffffffffu, ss[g], off));
        }
#pragma unroll
        for (int g = 0; g < kUG; ++g) {
          const float rs = 1.0f / sqrtf(__fadd_rn(__fmul_rn(ss[g], 1.0f / D), a.eps));
          const float* wf = isq[g] ? wq : wk;
#pragma unroll
          for (int k = 0; k < E / 2; ++k) {
            const P nn = PK::make(__fmul_rn(x[g][2 * k], rs), __fmul_rn(x[g][2 * k + 1], rs));
            P y;
            if constexpr (sizeof(W) == sizeof(T)) {
              y = PK::mul(nn, PK::make(wf[2 * k], wf[2 * k + 1]));  // weights are T values: exact
            } else {
              y = PK::make(__fmul_rn(Elem<T>::to_f(reinterpret_cast<const T*>(&nn)[0]), wf[2 * k]),
                           __fmul_rn(Elem<T>::to_f(reinterpret_cast<const T*>(&nn)[1]), wf[2 * k + 1]));
            }
            w32[g][k] = bits(y);
          }
          if (!inter) unpack<T>(make_uint4(w32[g][0], w32[g][1], w32[g][2], w32[g][3]), x[g]);
        }
      }
      if (mode != NIB_ROPE_NONE) {
        uint32_t o32[kUG][4];
#pragma unroll
        for (int g = 0; g < kUG; ++g) {
#pragma unroll
          for (int k = 0; k < 4; ++k) o32[g][k] = __shfl_xor_sync(0xffffffffu, w32[g][k], HALF);
        }
#pragma unroll
        for (int g = 0; g < kUG; ++g) {
          if (inter) {
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              const P t1 = PK::mul(from_bits<P>(w32[g][k]), c2[k]);
              const P t2 = PK::mul(from_bits<P>(o32[g][k]), s2[k]);
              w32[g][k] = bits(PK::add(t1, first ? PK::neg(t2) : t2));
            }
          } else {
            float p[E];
            unpack<T>(make_uint4(o32[g][0], o32[g][1], o32[g][2], o32[g][3]), p);
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              const float a0 = __fmul_rn(x[g][2 * k], c[2 * k]), b0 = __fmul_rn(p[2 * k], s[2 * k]);
              const float a1 = __fmul_rn(x[g][2 * k + 1], c[2 * k + 1]), b1 = __fmul_rn(p[2 * k + 1], s[2 * k + 1]);
              w32[g][k] = bits(PK::make(first ? __fsub_rn(a0, b0) : __fadd_rn(a0, b0),
                                        first ? __fsub_rn(a1, b1) : __fadd_rn(a1, b1)));
            }
          }
        }
      }
#pragma unroll
      for (int g = 0; g < kUG; ++g) {
        if (!hok[g]) continue;
        const uint4 o = make_uint4(w32[g][0], w32[g][1], w32[g][2], w32[g][3]);
        if (isq[g]) {
          st_vec(qo_t + hoff[g], o);
        } else {
          st_vec(ko_t + hoff[g], o);
          if (kc_t) st_vec(kc_t + hoff[g], o);
        }
      }
    }
    // ---- v heads straight from the staged row into the cache
    if (slot >= 0) {
      T* vc_t = vc + slot * a.cache_slot_stride + hs * D + l * E;
      const T* rv = rl + (nq + nkv) * D;
#pragma unroll 4
      for (int u = 0; u < Uk; ++u) {
        if (u * HPW + hs < nkv)
          st_vec(vc_t + u * HPW * D, *reinterpret_cast<const uint4*>(rv + u * HPW * D));
      }
    }
    __syncwarp();  // stage `st` and the trig scratch are rewritten next
  }
}

// ------------------------------------------------------------------ host side

static bool pipe_layout(const nib_qk_prologue_args& a, PipeLayout* out) {
  const int es = elem_size(a.dtype);
  const int D = a.head_dim;
  const bool store = a.key_cache != nullptr;
  const int64_t heads = a.num_heads + a.num_kv_heads + (store ? a.num_kv_heads : 0);
  const uint32_t row_bytes = static_cast<uint32_t>(heads * D * es);
  const uint32_t tab = a.rope_mode == NIB_ROPE_TABLE ? D * 4 : 0;
  const uint32_t stage_bytes = (row_bytes + tab + 127u) / 128u * 128u;
  const uint32_t trig = (a.rope_mode == NIB_ROPE_MROPE_CHUNKED || a.rope_mode == NIB_ROPE_MROPE_INTERLEAVED)
                            ? D * 4 : 0;  // 2 * (D/2) floats
  for (int stages = kPipeStages; stages >= 2; --stages) {
    for (int warps = kPipeMaxWarps; warps >= 2; warps -= 2) {
      const uint32_t bytes = warps * (stages * stage_bytes + stages * 8 + trig);
      if (bytes <= kPipeSmemBudget) {
        *out = PipeLayout{warps, stages, row_bytes, stage_bytes, bytes};
        return true;
      }
    }
  }
  return false;
}

// The pipelined kernel applies when q, k (and v when storing) are consecutive
// head ranges of one row with a shared, 16-byte aligned token stride.
bool prologue_pipe_eligible(const nib_qk_prologue_args& a) {
  if (a.dtype != NIB_BF16 && a.dtype != NIB_F16) return false;
  if (a.head_dim != 64 && a.head_dim != 128 && a.head_dim != 256) return false;
  const int es = elem_size(a.dtype);
  const int64_t D = a.head_dim;
  const char* q = static_cast<const char*>(a.q);
  if (a.q_head_stride != D || a.k_head_stride != D) return false;
  if (static_cast<const char*>(a.k) != q + a.num_heads * D * es) return false;
  if (a.k_token_stride != a.q_token_stride) return false;
  if (a.key_cache) {
    if (a.v_head_stride != D || a.v_token_stride != a.q_token_stride) return false;
    if (static_cast<const char*>(a.v) != q + (a.num_heads + a.num_kv_heads) * D * es) return false;
  }
  if (!aligned16(q) || (a.q_token_stride * es) % 16 != 0) return false;
  if (a.rope_mode == NIB_ROPE_TABLE && !aligned16(a.cos_sin_table)) return false;
  PipeLayout lay;
  return pipe_layout(a, &lay);
}

template <typename T, typename W, int D>
static int launch_pipe_d(const nib_qk_prologue_args& a, const PipeLayout& lay, cudaStream_t st) {
  auto kernel = qk_prologue_pipe_kernel<T, W, D>;
  static int configured_bytes[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && configured_bytes[dev] < static_cast<int>(lay.smem_bytes)) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(kPipeSmemBudget));
    if (e != cudaSuccess) {
      set_error("qk_prologue: cannot reserve shared memory: %s", cudaGetErrorString(e));
      return NIB_ERR_CUDA;
    }
    configured_bytes[dev] = static_cast<int>(kPipeSmemBudget);
  }
  const int64_t warps_needed = a.tokens;  // at most one token range per warp is useful
  int64_t blocks = static_cast<int64_t>(sm_count());
  const int64_t by_tokens = (warps_needed + lay.warps - 1) / lay.warps;
  if (blocks > by_tokens) blocks = by_tokens;
  if (blocks < 1) blocks = 1;
  kernel<<<static_cast<unsigned>(blocks), lay.warps * 32, lay.smem_bytes, st>>>(
      a, lay.stages, lay.row_bytes, lay.stage_bytes);
  return launch_status("qk_prologue (pipelined)");
}

template <typename T, typename W>
static int launch_pipe_t(const nib_qk_prologue_args& a, const PipeLayout& lay, cudaStream_t st) {
  switch (a.head_dim) {
    case 64: return launch_pipe_d<T, W, 64>(a, lay, st);
    case 128: return launch_pipe_d<T, W, 128>(a, lay, st);
    default: return launch_pipe_d<T, W, 256>(a, lay, st);
  }
}

int launch_prologue_pipe(const nib_qk_prologue_args& a, cudaStream_t st) {
  PipeLayout lay;
  if (!pipe_layout(a, &lay)) {
    set_error("qk_prologue: row too large for the pipelined kernel");
    return NIB_ERR_UNSUPPORTED;
  }
  const bool w32 = a.norm && a.weight_dtype == NIB_F32;
  if (a.norm && !w32 && a.weight_dtype != a.dtype) {
    set_error("qk_prologue: weight dtype must equal the activation dtype or be float32");
    return NIB_ERR_UNSUPPORTED;
  }
  if (a.dtype == NIB_BF16)
    return w32 ? launch_pipe_t<__nv_bfloat16, float>(a, lay, st) : launch_pipe_t<__nv_bfloat16, __nv_bfloat16>(a, lay, st);
  return w32 ? launch_pipe_t<__half, float>(a, lay, st) : launch_pipe_t<__half, __half>(a, lay, st);
}

}  // namespace nib
