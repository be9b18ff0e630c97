// Attention prologue, pipelined variant for the fused-qkv layout.
//
// Same math and rounding points as qk_prologue_kernel (rope.cu), so results
// are bit-identical; only the data movement differs. When q, k and v are the
// three head ranges of one qkv row (the layout every NanoInfer decoder
// produces: nanovllm/models/qwen3.py:77-81), each warp owns every wpc-th
// token of its CTA's range and streams their rows [q|k|v] - plus the 1-D RoPE table row
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
#include "prologue_math.cuh"

namespace nib {

constexpr int kUG = 3;  // head groups per compute phase

struct TokenMeta {
  int32_t slot;
  int64_t p0, p1, p2;
};

template <typename T, typename W, int D>
__global__ void __launch_bounds__(pipe_max_warps<W>() * 32, 1)
qk_prologue_pipe_kernel(const nib_qk_prologue_args a, const int stages, const uint32_t row_bytes,
                        const uint32_t stage_bytes) {
  constexpr int E = 8;  // 16-bit activations: 8 per 16-byte vector
  constexpr int L = D / (2 * E);  // lanes per head (paired-halves layout)
  constexpr int HPW = 32 / L;
  constexpr int NF = D / 2;
  constexpr int FPL = (NF + 31) / 32;

  extern __shared__ __align__(128) unsigned char smem[];
  const int lane = threadIdx.x & 31;
  const int wib = threadIdx.x >> 5;
  const int wpc = blockDim.x >> 5;
  unsigned char* wbuf = smem + static_cast<size_t>(wib) * stages * stage_bytes;
  unsigned char* tail = smem + static_cast<size_t>(wpc) * stages * stage_bytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(tail) + wib * stages;
  float* trig = reinterpret_cast<float*>(tail + static_cast<size_t>(wpc) * stages * 8) + wib * 2 * NF;

  const int hs = lane / L;
  const int l = lane % L;
  const int fb = l * E;
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
  // The CTA owns tokens [cb, ce) and its warps take them interleaved (warp w:
  // cb + w, cb + w + wpc, ...), so each CTA streams one contiguous range of
  // rows and outputs: 148 streams per GPU instead of one per warp. On a
  // power-capped B200 that took the C5 launch from 0.836-0.842 to 0.800-0.803
  // ms; at 32,768 tokens it measured the same.
  const int64_t cb = ntok * blockIdx.x / gridDim.x;
  const int64_t ce = ntok * (blockIdx.x + 1) / gridDim.x;
  const int64_t n = (ce - cb - wib + wpc - 1) / wpc;  // this warp's tokens
  if (n <= 0) return;
  auto tok = [&](int64_t i) { return cb + wib + i * wpc; };

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
  pdl_enter();  // the barrier set-up above overlaps the previous kernel's tail

  // ---- per-lane constants: norm weights, M-RoPE frequency layout
  HeadWeights<T, W> wq, wk;
  if (a.norm) {
    wq.load(static_cast<const W*>(a.q_weight), l, NF);
    wk.load(static_cast<const W*>(a.k_weight), l, NF);
  }
  int fax[FPL];
  float finv[FPL];
#pragma unroll
  for (int m = 0; m < FPL; ++m) {
    const int j = lane + 32 * m;
    fax[m] = 0;
    finv[m] = 0.f;
    if (mrope && j < NF) {
      fax[m] = mrope_axis(j, inter, a.sections);
      finv[m] = __ldg(a.inv_freq + j);
    }
  }

  // ---- metadata, 32 tokens per batch (lane j holds token 32*b + j)
  auto load_meta = [&](int64_t b) {
    TokenMeta m{-1, 0, 0, 0};
    const int64_t i = 32 * b + lane;
    if (i < n) {
      const int64_t t = tok(i);
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
      bulk_load(dst, rows + tok(j) * row_stride, row_bytes, &bars[st]);
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
    const int64_t t = tok(i);
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
    uint32_t c2[4], s2[4];
    if (inter) pack_trig<T>(c, s, c2, s2);

    // ---- q and k heads, kUG head groups per phase so that their dependency
    // chains (squares -> butterfly -> 1/sqrt -> scale -> rotate) interleave
    const int64_t qo_base = (t * nq + hs) * D + fb;
    const int64_t ko_base = (t * nkv + hs) * D + fb;
    T* kc_t = slot >= 0 ? kc + slot * a.cache_slot_stride + hs * D + fb : nullptr;
    const T* rl = rq + hs * D + fb;
    const int Uqk = Uq + Uk;
    for (int u0 = 0; u0 < Uqk; u0 += kUG) {
      uint32_t wa[kUG][4], wb[kUG][4];
      float xa[kUG][E], xb[kUG][E];
      bool hok[kUG], isq[kUG];
      int hoff[kUG];  // head * D within q (or within k)
#pragma unroll
      for (int g = 0; g < kUG; ++g) {
        const int u = u0 + g;
        isq[g] = u < Uq;
        const int hg = isq[g] ? u : u - Uq;
        hoff[g] = hg * HPW * D;
        hok[g] = u < Uqk && hg * HPW + hs < (isq[g] ? nq : nkv);
        const T* src = rl + (isq[g] ? 0 : nq * D) + hoff[g];
        const uint4 ra = hok[g] ? *reinterpret_cast<const uint4*>(src) : zero_vec();
        const uint4 rb = hok[g] ? *reinterpret_cast<const uint4*>(src + NF) : zero_vec();
        from_u4(ra, wa[g]);
        from_u4(rb, wb[g]);
        unpack<T>(ra, xa[g]);
        unpack<T>(rb, xb[g]);
      }
      if (a.norm) {
        float ss[kUG];
#pragma unroll
        for (int g = 0; g < kUG; ++g) ss[g] = __fadd_rn(sumsq_tree<E>(xa[g]), sumsq_tree<E>(xb[g]));
#pragma unroll
        for (int off = L / 2; off > 0; off >>= 1) {
#pragma unroll
          for (int g = 0; g < kUG; ++g) ss[g] = __fadd_rn(ss[g], __shfl_xor_sync(0xffffffffu, ss[g], off));
        }
#pragma unroll
        for (int g = 0; g < kUG; ++g) {
          const float rs = inv_sqrt_rn(__fadd_rn(__fmul_rn(ss[g], 1.0f / D), a.eps));
          const HeadWeights<T, W>& hw = isq[g] ? wq : wk;
          normalize_vec<T, W>(xa[g], wa[g], rs, hw.fa, hw.pa);
          normalize_vec<T, W>(xb[g], wb[g], rs, hw.fb, hw.pb);
        }
      }
      if (mode != NIB_ROPE_NONE) {
#pragma unroll
        for (int g = 0; g < kUG; ++g) rotate_pair<T>(xa[g], xb[g], wa[g], wb[g], c, s, c2, s2, inter);
      }
#pragma unroll
      for (int g = 0; g < kUG; ++g) {
        if (!hok[g]) continue;
        const uint4 oa = as_u4(wa[g]), ob = as_u4(wb[g]);
        if (isq[g]) {
          T* dst = q_out + qo_base + hoff[g];
          st_vec(dst, oa);
          st_vec(dst + NF, ob);
        } else {
          if (k_out) {
            T* dst = k_out + ko_base + hoff[g];
            st_vec(dst, oa);
            st_vec(dst + NF, ob);
          }
          if (kc_t) {
            st_vec(kc_t + hoff[g], oa);
            st_vec(kc_t + hoff[g] + NF, ob);
          }
        }
      }
    }
    // ---- v heads: the contiguous nkv*D block of the staged row into the cache slot
    if (slot >= 0) {
      T* vd = vc + slot * a.cache_slot_stride;
      const T* vs = rq + (nq + nkv) * D;
      for (int off = lane * E; off < nkv * D; off += 32 * E)
        st_vec(vd + off, *reinterpret_cast<const uint4*>(vs + off));
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
  const bool fp32_weights = a.norm && a.weight_dtype == NIB_F32;
  int max_warps = pipe_max_warps(fp32_weights);
  // Chunked M-RoPE rotates in fp32 (more math per byte than the packed
  // interleaved rotation) and keeps 12 warps at every size: 17.4 vs 20.4 us at
  // C4's 8,312 tokens, 104 vs 128 us at 65,536.
  if (a.tokens <= kPipeFewTokens && max_warps > kPipeFewTokenWarps && a.rope_mode != NIB_ROPE_MROPE_CHUNKED)
    max_warps = kPipeFewTokenWarps;
  for (int stages = pipe_max_stages(fp32_weights); stages >= 2; --stages) {
    for (int warps = max_warps; warps >= 2; warps -= 2) {
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
  ::nib::launch_k(kernel, static_cast<unsigned>(blocks), lay.warps * 32, lay.smem_bytes, st,
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
