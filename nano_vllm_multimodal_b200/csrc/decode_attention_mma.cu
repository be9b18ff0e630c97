// Paged decode attention on the tensor cores (the default kernel of
// nib_decode_attention for bf16/f16, head_dim 64/128, up to 16 q heads per kv
// head, block sizes that are multiples of 16).
//
// Same contract as decode_attention.cu (flash_attn_with_kvcache's decode call,
// nanovllm/layers/attention.py:122-130; the reference's SDPA decode branch,
// attention.py:286-300): out[b, h] = softmax(q[b, h] . K^T * scale) V over the
// request's first context_lens[b] cached tokens, kv head h / group.
//
// A CTA owns (request, kv head, split of the context). The kv head's q heads
// (at most 16) are the M rows of mma.sync m16n8k16 tiles, the context's
// tokens the N columns: S = Q K^T per 16-token tile (D/16 k-steps x 2 n-tiles),
// then O += P V (one k-step of 16 tokens x D/8 n-tiles). q heads beyond the
// group are zero rows. With at most 16 q heads per kv head this spends the
// same tensor-core issue on grouped-query (GQA 8) as on GQA 2, so the kernel
// stays HBM-bound where the CUDA-core kernel's fp32 FMAs per cached byte grow
// with the group.
//
// Each warp owns every kMmaWarps-th tile of the CTA's range and a private ring
// of kMmaStages (2) shared-memory stages, so 3 CTAs (12 warps) fit on an SM:
// with 3 stages and 2 CTAs per SM the GQA-8 C2 decode took 0.210 ms instead of
// 0.203 ms. Lane 0 loads a tile with two TMA tensor copies per 64-element
// half of the head, one from each cache (cp.async.bulk.tensor, 5-D maps over
// [blocks, block_size, kv_heads, D/64, 64], 128-byte swizzle, no multicast),
// completing on the stage's mbarrier; the waits are bounded in wall time like every wait of this
// library (on timeout: NIB_DEV_TIMEOUT, wait for the warp's other copies,
// return). Fragments come from shared memory with ldmatrix (.trans for V);
// the swizzle keeps those reads free of bank conflicts. Scores are kept in
// the log2 domain with an online max and sum per q head; warps and splits are
// merged with max-rescaled sums (the split partials use the CUDA-core
// kernel's workspace format and its combine kernel).
#include <cuda.h>

#include <mutex>
#include <type_traits>

#include "bulk_copy.cuh"
#include "dispatch.cuh"

namespace nib {

constexpr int kMmaWarps = 4;
constexpr int kMmaStages = 2;  // ring stages per warp: 3 CTAs (12 warps) per SM fit
constexpr int kMmaTile = 16;   // tokens per tile

struct MmaDecodeParams {
  const void* q;
  int64_t q_bs, q_hs;
  const int32_t* tables;
  int64_t table_stride, max_blocks, num_blocks;
  int block_size;
  const int32_t* lens;
  float qscale;  // softmax scale * log2(e)
  void* out;
  int64_t o_bs, o_hs;
  float* ws;  // [batch, num_heads, splits, D + 2] when splits > 1
  int num_heads, num_kv_heads, group, splits;
  unsigned int* status;
};

// byte offset of (token t, element d) inside a stage's K or V tile. The tile is
// D/64 regions (one per 64-element half of the head, one tensor copy each) of
// kMmaTile 128-byte rows, row = token, whose 16-byte chunks are XOR-swizzled by
// row % 8 - how a SWIZZLE_128B tensor copy lays its box out. An ldmatrix phase
// reads the same chunk of 8 consecutive tokens: 8 different rows, 8 different
// swizzled chunks, no bank conflict. (With both halves of a token in one box,
// consecutive tokens sit 2 rows apart and every phase conflicts 2-way: 48% of
// the shared-memory wavefronts in the first version of this kernel.)
template <int D>
__device__ __forceinline__ uint32_t swz(int t, int d) {
  return static_cast<uint32_t>((d >> 6) * (kMmaTile * 128) + t * 128 + ((((d & 63) >> 3) ^ (t & 7)) << 4) +
                               (d & 7) * 2);
}

__device__ __forceinline__ void tma_load_5d(uint32_t dst, const CUtensorMap* map, int c0, int c1, int c2,
                                            int c3, int c4, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.5d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4, %5, %6}], [%7];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(c4), "r"(smem_addr(bar))
      : "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t* r) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t* r) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

// c += a (16x16, row) * b (16x8, col), fp32 accumulate
template <typename T>
__device__ __forceinline__ void mma16816(float* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9},"
        " {%0, %1, %2, %3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  } else {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9},"
        " {%0, %1, %2, %3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
}

template <typename T>
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  typename Vec2<T>::type v = Vec2<T>::make(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

__device__ __forceinline__ float ex2_fast(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Zero the K and V rows of the tokens outside [lo, hi) (tile-relative) of one
// stage, whatever the cache holds there: their scores are masked, but 0 x NaN
// would still reach the sums. The fence orders these generic writes before
// the stage's next tensor copy.
template <int D>
__device__ __forceinline__ void zero_rows(unsigned char* kg, int lo, int hi, int lane) {
  constexpr uint32_t kTileBytes = kMmaTile * D * 2;
  for (int e = lane; e < kMmaTile * (D / 8); e += 32) {  // 16-byte units of one tile
    const int t = e % kMmaTile;  // a token's row in each region (the chunk order within does not matter)
    if (t < lo || t >= hi) {
      const int u = e / kMmaTile;  // (region, chunk)
      const uint32_t at = (u >> 3) * (kMmaTile * 128) + t * 128 + (u & 7) * 16;
      *reinterpret_cast<uint4*>(kg + at) = make_uint4(0, 0, 0, 0);
      *reinterpret_cast<uint4*>(kg + kTileBytes + at) = make_uint4(0, 0, 0, 0);
    }
  }
  fence_proxy_async();
  __syncwarp();
}

// Q fragments of one (request, kv head): the A operand, rows = the kv head's q
// heads, zero past the group.
template <typename T, int D>
__device__ __forceinline__ void load_q_frags(uint32_t (&qa)[D / 16][4], const T* qb, int64_t q_hs, int first_head,
                                             int group, int lane) {
  const int r0 = lane >> 2, cq = (lane & 3) * 2;
  const bool ok0 = r0 < group, ok1 = r0 + 8 < group;
  const T* q0 = qb + static_cast<int64_t>(first_head + (ok0 ? r0 : 0)) * q_hs;
  const T* q1 = qb + static_cast<int64_t>(first_head + (ok1 ? r0 + 8 : 0)) * q_hs;
#pragma unroll
  for (int ks = 0; ks < D / 16; ++ks) {
    const int k = ks * 16 + cq;
    qa[ks][0] = ok0 ? __ldg(reinterpret_cast<const uint32_t*>(q0 + k)) : 0u;
    qa[ks][1] = ok1 ? __ldg(reinterpret_cast<const uint32_t*>(q1 + k)) : 0u;
    qa[ks][2] = ok0 ? __ldg(reinterpret_cast<const uint32_t*>(q0 + k + 8)) : 0u;
    qa[ks][3] = ok1 ? __ldg(reinterpret_cast<const uint32_t*>(q1 + k + 8)) : 0u;
  }
}

// One 16-token tile of a stage (K at kt, V at kt + tile bytes) into the online
// softmax state of rows r0 (a) and r0 + 8 (b): S = Q K^T, scores of tokens
// outside [lo, hi) (tile-relative) masked, then O += P V.
template <typename T, int D>
__device__ __forceinline__ void mma_tile(const uint32_t (&qa)[D / 16][4], uint32_t kt, int lo, int hi, float qscale,
                                         float (&o)[D / 8][4], float& m_a, float& m_b, float& l_a, float& l_b,
                                         int lane) {
  constexpr int KS = D / 16;
  constexpr int ND = D / 8;
  const uint32_t vt = kt + kMmaTile * D * 2;
  const int cq = (lane & 3) * 2;
  // ---- S = Q K^T (2 n-tiles of 8 tokens)
  float s[2][4];
#pragma unroll
  for (int nt = 0; nt < 2; ++nt) {
    s[nt][0] = s[nt][1] = s[nt][2] = s[nt][3] = 0.f;
#pragma unroll
    for (int ks = 0; ks < KS; ks += 2) {
      uint32_t kb[4];
      // matrices (tokens 8nt..8nt+7) x (d chunks 2ks .. 2ks+3): lane L gives row L%8 of matrix L/8
      ldsm_x4(kt + swz<D>(nt * 8 + (lane & 7), (ks * 2 + (lane >> 3)) * 8), kb);
      mma16816<T>(s[nt], qa[ks], kb[0], kb[1]);
      mma16816<T>(s[nt], qa[ks + 1], kb[2], kb[3]);
    }
  }
  // ---- online softmax (log2 domain); mask tokens outside the range
  float mx_a = -INFINITY, mx_b = -INFINITY;
#pragma unroll
  for (int nt = 0; nt < 2; ++nt) {
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      const int t = nt * 8 + cq + c;
      const bool in = t >= lo && t < hi;
      s[nt][c] = in ? s[nt][c] * qscale : -INFINITY;
      s[nt][c + 2] = in ? s[nt][c + 2] * qscale : -INFINITY;
      mx_a = fmaxf(mx_a, s[nt][c]);
      mx_b = fmaxf(mx_b, s[nt][c + 2]);
    }
  }
#pragma unroll
  for (int off = 1; off < 4; off <<= 1) {
    mx_a = fmaxf(mx_a, __shfl_xor_sync(0xffffffffu, mx_a, off));
    mx_b = fmaxf(mx_b, __shfl_xor_sync(0xffffffffu, mx_b, off));
  }
  const float na = fmaxf(m_a, mx_a), nb = fmaxf(m_b, mx_b);
  const float ra = na == -INFINITY ? 1.f : ex2_fast(m_a - na);
  const float rb = nb == -INFINITY ? 1.f : ex2_fast(m_b - nb);
  m_a = na;
  m_b = nb;
  float pa[2][2], pb[2][2];
#pragma unroll
  for (int nt = 0; nt < 2; ++nt) {
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      pa[nt][c] = na == -INFINITY ? 0.f : ex2_fast(s[nt][c] - na);
      pb[nt][c] = nb == -INFINITY ? 0.f : ex2_fast(s[nt][c + 2] - nb);
    }
  }
  l_a = l_a * ra + (pa[0][0] + pa[0][1]) + (pa[1][0] + pa[1][1]);
  l_b = l_b * rb + (pb[0][0] + pb[0][1]) + (pb[1][0] + pb[1][1]);
#pragma unroll
  for (int n = 0; n < ND; ++n) {
    o[n][0] *= ra;
    o[n][1] *= ra;
    o[n][2] *= rb;
    o[n][3] *= rb;
  }
  // P as the A fragment of one 16-token k-step (the C layout of two n-tiles)
  uint32_t pf[4];
  pf[0] = pack2<T>(pa[0][0], pa[0][1]);
  pf[1] = pack2<T>(pb[0][0], pb[0][1]);
  pf[2] = pack2<T>(pa[1][0], pa[1][1]);
  pf[3] = pack2<T>(pb[1][0], pb[1][1]);
  // ---- O += P V (V^T fragments by ldmatrix.trans: rows = tokens, 8 d values each)
#pragma unroll
  for (int n2 = 0; n2 < ND; n2 += 2) {
    uint32_t vb[4];
    // matrices: (tokens 0-7, d chunk n2), (tokens 8-15, n2), (0-7, n2+1), (8-15, n2+1)
    ldsm_x4_t(vt + swz<D>((lane & 7) + ((lane >> 3) & 1) * 8, (n2 + (lane >> 4)) * 8), vb);
    mma16816<T>(o[n2], pf, vb[0], vb[1]);
    mma16816<T>(o[n2 + 1], pf, vb[2], vb[3]);
  }
}

template <typename T, int D>
__global__ void __launch_bounds__(kMmaWarps * 32, 3)
decode_attention_mma_kernel(const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap,
                            const MmaDecodeParams p) {
  constexpr int KS = D / 16;          // k-steps of Q K^T
  constexpr int ND = D / 8;           // n-tiles of P V
  constexpr uint32_t kTileBytes = kMmaTile * D * 2;  // one of K or V
  constexpr uint32_t kStageBytes = 2 * kTileBytes;
  __shared__ __align__(8) uint64_t bars[kMmaWarps][kMmaStages];
  extern __shared__ unsigned char dsm_raw[];
  // the 128-byte swizzle repeats every 1,024 bytes: stages start on that boundary
  const uint32_t raw = smem_addr(dsm_raw);
  const uint32_t base_all = (raw + 1023u) & ~1023u;
  unsigned char* dsm = dsm_raw + (base_all - raw);

  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  if (lane == 0) {
    for (int s = 0; s < kMmaStages; ++s) mbar_init(&bars[w][s], 1);
    fence_mbar_init();
  }
  __syncwarp();
  pdl_enter();  // the barrier set-up above overlaps the previous kernel's tail

  const int kvh = static_cast<int>(blockIdx.x % p.num_kv_heads);
  const int64_t b = blockIdx.x / p.num_kv_heads;
  const int split = blockIdx.y;
  int64_t len = __ldg(p.lens + b);
  const int64_t cap = p.max_blocks * p.block_size;
  if (len < 0 || len > cap) {
    if (threadIdx.x == 0 && split == 0) flag(p.status, NIB_DEV_BAD_INDEX);
    len = len < 0 ? 0 : cap;
  }
  // Split boundaries: the splits of a context shrink linearly toward the last one
  // (split y gets a share s - y of s + (s-1) + ... + 1), and the grid's rows are
  // dispatched in split order, so its final wave holds the smallest CTAs.
  auto split_start = [&](int y) -> int64_t {
    const int64_t sp = p.splits;
    const int64_t before = y * sp - static_cast<int64_t>(y) * (y - 1) / 2;
    return len * before / (sp * (sp + 1) / 2);
  };
  const int64_t t_begin = split_start(split);
  const int64_t t_end = split_start(split + 1);
  const int64_t tile0 = t_begin / kMmaTile;
  const int64_t n_tiles = t_end > t_begin ? (t_end + kMmaTile - 1) / kMmaTile - tile0 : 0;
  const int64_t n_mine = n_tiles > w ? (n_tiles - w + kMmaWarps - 1) / kMmaWarps : 0;  // warp-uniform

  const int r0 = lane >> 2, cq = (lane & 3) * 2;
  uint32_t qa[KS][4];
  load_q_frags<T, D>(qa, static_cast<const T*>(p.q) + b * p.q_bs, p.q_hs, kvh * p.group, p.group, lane);

  float o[ND][4];
#pragma unroll
  for (int n = 0; n < ND; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
  float m_a = -INFINITY, m_b = -INFINITY, l_a = 0.f, l_b = 0.f;  // rows r0 and r0 + 8

  const int32_t* table = p.tables + b * p.table_stride;
  const uint32_t ring = base_all + static_cast<uint32_t>(w) * kMmaStages * kStageBytes;
  uint32_t ok_bits = 0;  // per stage: its tile was loaded
  bool timed_out = false;

  auto issue = [&](int64_t i) {
    if (i >= n_mine) return;
    const int st = static_cast<int>(i % kMmaStages);
    if (lane == 0) {
      const int64_t t0 = (tile0 + w + i * kMmaWarps) * kMmaTile;
      const int64_t bi = t0 / p.block_size;
      const int blk = __ldg(table + bi);
      const bool ok = blk >= 0 && blk < p.num_blocks;
      if (!ok) flag(p.status, NIB_DEV_BAD_BLOCK);
      fence_proxy_async();  // this stage's generic zero-fill (if any) before the copies
      mbar_arrive_expect_tx(&bars[w][st], ok ? kStageBytes : 0u);
      if (ok) {
        const int off = static_cast<int>(t0 - bi * p.block_size);
        const uint32_t dst = ring + st * kStageBytes;
#pragma unroll
        for (int c = 0; c < D / 64; ++c) {  // one region per 64-element half
          tma_load_5d(dst + c * kMmaTile * 128, &kmap, 0, c, kvh, off, blk, &bars[w][st]);
          tma_load_5d(dst + kTileBytes + c * kMmaTile * 128, &vmap, 0, c, kvh, off, blk, &bars[w][st]);
        }
      }
      ok_bits = (ok_bits & ~(1u << st)) | (static_cast<uint32_t>(ok) << st);
    }
  };

#pragma unroll
  for (int i = 0; i < kMmaStages - 1; ++i) issue(i);
  for (int64_t i = 0; i < n_mine; ++i) {
    issue(i + kMmaStages - 1);
    const int st = static_cast<int>(i % kMmaStages);
    const bool done = mbar_wait(&bars[w][st], static_cast<uint32_t>((i / kMmaStages) & 1));
    if (!__all_sync(0xffffffffu, done)) {
      if (lane == 0) flag(p.status, kDevTimeout);
      // let the warp's other copies land (bounded) before leaving
      for (int64_t j = i + 1; j < i + kMmaStages && j < n_mine; ++j)
        (void)mbar_wait(&bars[w][j % kMmaStages], static_cast<uint32_t>((j / kMmaStages) & 1));
      timed_out = true;
      break;
    }
    const bool ok = (__shfl_sync(0xffffffffu, ok_bits, 0) >> st) & 1u;
    const int64_t t0 = (tile0 + w + i * kMmaWarps) * kMmaTile;
    const uint32_t kt = ring + st * kStageBytes;
    if (!ok) continue;  // bad block id: its tokens take no part
    // the tile's tokens in [t_begin, t_end), tile-relative (only the first and last tile are partial)
    const int lo = t_begin > t0 ? static_cast<int>(t_begin - t0) : 0;
    const int hi = t_end - t0 < kMmaTile ? static_cast<int>(t_end - t0) : kMmaTile;
    if (lo > 0 || hi < kMmaTile) zero_rows<D>(dsm + (kt - base_all), lo, hi, lane);
    mma_tile<T, D>(qa, kt, lo, hi, p.qscale, o, m_a, m_b, l_a, l_b, lane);
    __syncwarp();  // every lane has read the stage before it is refilled
  }

  // ---- per-row sums over the quad; merge the warps through shared memory
#pragma unroll
  for (int off = 1; off < 4; off <<= 1) {
    l_a += __shfl_xor_sync(0xffffffffu, l_a, off);
    l_b += __shfl_xor_sync(0xffffffffu, l_b, off);
  }
  if (__syncthreads_or(timed_out)) return;  // the rows are incomplete; the status bit says so
  constexpr int SW = D + 2;
  float* red = reinterpret_cast<float*>(dsm);  // [warps][16 rows][D + 2], over the rings
#pragma unroll
  for (int n = 0; n < ND; ++n) {
    const int d = n * 8 + cq;
    red[(w * 16 + r0) * SW + d] = o[n][0];
    red[(w * 16 + r0) * SW + d + 1] = o[n][1];
    red[(w * 16 + r0 + 8) * SW + d] = o[n][2];
    red[(w * 16 + r0 + 8) * SW + d + 1] = o[n][3];
  }
  if ((lane & 3) == 0) {
    red[(w * 16 + r0) * SW + D] = m_a;
    red[(w * 16 + r0) * SW + D + 1] = l_a;
    red[(w * 16 + r0 + 8) * SW + D] = m_b;
    red[(w * 16 + r0 + 8) * SW + D + 1] = l_b;
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < p.group * D; idx += blockDim.x) {
    const int r = idx / D, d = idx % D;
    float M = -INFINITY;
#pragma unroll
    for (int ww = 0; ww < kMmaWarps; ++ww) M = fmaxf(M, red[(ww * 16 + r) * SW + D]);
    float L = 0.f, A = 0.f;
    if (M != -INFINITY) {
#pragma unroll
      for (int ww = 0; ww < kMmaWarps; ++ww) {
        const float* rr = red + (ww * 16 + r) * SW;
        const float f = rr[D] == -INFINITY ? 0.f : ex2_fast(rr[D] - M);
        L += rr[D + 1] * f;
        A += rr[d] * f;
      }
    }
    const int h = kvh * p.group + r;
    if (p.splits == 1) {
      static_cast<T*>(p.out)[b * p.o_bs + h * p.o_hs + d] = Elem<T>::from_f(L > 0.f ? A / L : 0.f);
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

// ------------------------------------------------------------------ host side

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_tiled() {
  static std::once_flag once;
  static EncodeTiledFn fn = nullptr;
  std::call_once(once, [] {
    void* f = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault) == cudaSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(f);
  });
  return fn;
}

// whether the tensor-core kernel takes this call
bool decode_mma_eligible(const nib_decode_attention_args& a) {
  if (a.dtype != NIB_BF16 && a.dtype != NIB_F16) return false;
  if (a.head_dim != 64 && a.head_dim != 128) return false;
  if (a.num_heads / a.num_kv_heads > 16) return false;
  if (a.block_size % kMmaTile != 0 || a.block_size > 256 * 16) return false;
  const int64_t es = 2;
  // tensor-map rules: 16-byte aligned base and strides, extents below 2^32
  if (!aligned16(a.key_cache) || !aligned16(a.value_cache)) return false;
  for (int64_t s : {a.cache_block_stride, a.cache_slot_stride, a.cache_head_stride})
    if ((s * es) % 16 != 0 || s * es >= (int64_t{1} << 40)) return false;
  if (a.num_blocks >= (int64_t{1} << 31) || a.num_blocks < 1) return false;
  return encode_tiled() != nullptr;
}

static int make_cache_map(CUtensorMap* map, const nib_decode_attention_args& a, const void* cache) {
  const cuuint64_t dims[5] = {64, static_cast<cuuint64_t>(a.head_dim / 64), static_cast<cuuint64_t>(a.num_kv_heads),
                              static_cast<cuuint64_t>(a.block_size), static_cast<cuuint64_t>(a.num_blocks)};
  const cuuint64_t strides[4] = {128, static_cast<cuuint64_t>(a.cache_head_stride * 2),
                                 static_cast<cuuint64_t>(a.cache_slot_stride * 2),
                                 static_cast<cuuint64_t>(a.cache_block_stride * 2)};
  const cuuint32_t box[5] = {64, 1, 1, kMmaTile, 1};  // one 64-element half of the head per copy
  const cuuint32_t estr[5] = {1, 1, 1, 1, 1};
  const CUtensorMapDataType dt =
      a.dtype == NIB_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  const CUresult r = encode_tiled()(map, dt, 5, const_cast<void*>(cache), dims, strides, box, estr,
                                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("decode_attention: cuTensorMapEncodeTiled failed (%d)", static_cast<int>(r));
    return NIB_ERR_CUDA;
  }
  return NIB_OK;
}

size_t decode_mma_smem(int head_dim) {
  return static_cast<size_t>(kMmaWarps) * kMmaStages * 2 * kMmaTile * head_dim * 2 + 1024;
}

template <typename T, int D>
static int launch_mma(const nib_decode_attention_args& a, int splits, cudaStream_t st) {
  CUtensorMap kmap, vmap;
  int rc = make_cache_map(&kmap, a, a.key_cache);
  if (rc != NIB_OK) return rc;
  rc = make_cache_map(&vmap, a, a.value_cache);
  if (rc != NIB_OK) return rc;
  MmaDecodeParams p{};
  p.q = a.q;
  p.q_bs = a.q_batch_stride;
  p.q_hs = a.q_head_stride;
  p.tables = a.block_tables;
  p.table_stride = a.block_table_stride;
  p.max_blocks = a.max_blocks_per_seq;
  p.num_blocks = a.num_blocks;
  p.block_size = static_cast<int>(a.block_size);
  p.lens = a.context_lens;
  p.qscale = a.scale * 1.4426950408889634f;
  p.out = a.out;
  p.o_bs = a.out_batch_stride;
  p.o_hs = a.out_head_stride;
  p.ws = static_cast<float*>(a.workspace);
  p.num_heads = a.num_heads;
  p.num_kv_heads = a.num_kv_heads;
  p.group = a.num_heads / a.num_kv_heads;
  p.splits = splits;
  p.status = a.status;
  const size_t smem = decode_mma_smem(D);
  auto kernel = decode_attention_mma_kernel<T, D>;
  static int configured[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && configured[dev] < static_cast<int>(smem)) {
    const cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) {
      set_error("decode_attention: cannot reserve shared memory: %s", cudaGetErrorString(e));
      return NIB_ERR_CUDA;
    }
    configured[dev] = static_cast<int>(smem);
  }
  const dim3 grid(static_cast<unsigned>(a.batch * a.num_kv_heads), static_cast<unsigned>(splits));
  ::nib::launch_k(kernel, grid, kMmaWarps * 32, smem, st, kmap, vmap, p);
  return launch_status("decode_attention (tensor cores)");
}

int launch_decode_mma(const nib_decode_attention_args& a, int splits, cudaStream_t st) {
  if (a.dtype == NIB_BF16)
    return a.head_dim == 64 ? launch_mma<__nv_bfloat16, 64>(a, splits, st) : launch_mma<__nv_bfloat16, 128>(a, splits, st);
  return a.head_dim == 64 ? launch_mma<__half, 64>(a, splits, st) : launch_mma<__half, 128>(a, splits, st);
}

}  // namespace nib
