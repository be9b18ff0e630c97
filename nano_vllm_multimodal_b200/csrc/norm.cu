// RMSNorm and fused residual-add + RMSNorm (HBM-bound row kernels).
//
// Reference numerics (nanovllm/layers/layernorm.py:16-40,
// nanovllm/models/qwen3_vl.py:74-79,232-237):
//   s   = x (+ residual)            fp32 add; Qwen3-VL rounds s to the dtype first
//   var = mean(s^2)                 fp32
//   n   = dtype(s * (1/sqrt(var + eps)))
//   y   = dtype(n * w)              one more rounding
// The 1/sqrt is the IEEE sqrt followed by the IEEE divide; squares are rounded
// before they are summed, as `x.pow(2).mean()` does. The summation order is
// fixed (sumsq_tree per 16-byte vector, vectors in order per lane, lanes by
// xor butterfly, warps in order); PyTorch leaves its order unspecified.
//
// DeepStack fold (Qwen3-VL, DS = true, rounded-sum add only): a token t with
// index[t] = j >= 0 adds visual row j after the residual add and before the
// statistics, s = dtype(dtype(x + residual) + vis[j]), which is the order of
// the reference's layer output add (qwen3_vl.py:238), _add_deepstack_rows
// (qwen3_vl.py:332-344, called at :371-376) and the next input_layernorm.
//
// Layout: rows of n elements, each row read once with 16-byte vectors and
// written once. Rows of up to 256 vectors (2048 bf16) live in one warp's
// registers (G lanes x VPT vectors); longer rows use one CTA per row.
#include "dispatch.cuh"
#include "prologue_math.cuh"

namespace nib {

// DeepStack operands of the folded kernels (unused when DS = false)
struct DsArgs {
  const void* vis = nullptr;       // [vis_rows, n] visual embeddings
  int64_t vis_rs = 0;              // row stride in elements
  int64_t vis_rows = 0;
  const int32_t* index = nullptr;  // [rows]: visual row of each token or -1
  unsigned int* status = nullptr;
};

// visual row of token t (-1: none); an index outside [-1, vis_rows) is reported and ignored
__device__ __forceinline__ int64_t ds_row(const DsArgs& ds, int64_t t) {
  const int64_t j = __ldg(ds.index + t);
  if (j >= ds.vis_rows || j < -1) {
    flag(ds.status, NIB_DEV_BAD_INDEX);
    return -1;
  }
  return j;
}

template <typename T, typename W, int G, int VPT, int RB, bool DS = false, bool PW = false>
__global__ void __launch_bounds__(256, G < 32 ? 2 : 1)
rms_rows_warp(const T* __restrict__ x, int64_t x_ts, int64_t x_hs, const T* __restrict__ res,
              int64_t r_rs, const W* __restrict__ w, T* __restrict__ y, T* __restrict__ res_out,
              int64_t rows, int64_t heads, int n, float eps, int add, int round_sum, DsArgs ds) {
  ::nib::pdl_enter();
  // G lanes per row, VPT 16-byte vectors per lane, RB row batches per step
  // (all RB * VPT loads of a lane are issued before any math)
  constexpr int E = Elem<T>::kPerVec;
  constexpr int GPW = 32 / G;
  const int lane = threadIdx.x & 31;
  const int sub = lane / G;
  const int gl = lane % G;
  const int64_t warp = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  const int nv = n / E;
  const bool use_add = G == 32 && add != 0;  // short rows (G < 32) never carry a residual
  // A lane's weight vectors are the same for every row: short rows load them
  // once; full-warp rows do too when PW (small batches, where a weight load
  // after the row's reduction would add a memory round trip to every warp).
  constexpr bool kPreW = G < 32 || PW;
  float wfs[VPT][E];
  uint32_t wps[VPT][4];
  if constexpr (kPreW) {
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int vi = i * G + gl;
      if (vi < nv) {
        load_weights<T, W>(w, vi * E, wfs[i]);
        if constexpr (sizeof(T) == 2 && sizeof(W) == 2) from_u4(ld_vec(w + vi * E), wps[i]);
      }
    }
  }
  for (int64_t rb = warp * GPW * RB; rb < rows; rb += nwarps * GPW * RB) {
    uint4 xr[RB][VPT], rr[RB][VPT], dr[RB][DS ? VPT : 1];
    int64_t r[RB], dj[RB];
    bool active[RB];
    // token and head of this lane's row in batch 0; batch b is b * GPW rows
    // further on, so one division per step serves all RB batches
    int64_t tt = 0, hh = 0;
    if (heads != 1) {
      tt = (rb + sub) / heads;
      hh = rb + sub - tt * heads;
    }
#pragma unroll
    for (int b = 0; b < RB; ++b) {
      r[b] = rb + b * GPW + sub;
      active[b] = r[b] < rows;
      if (heads != 1 && b > 0) {
        hh += GPW;
        if (heads >= GPW) {
          if (hh >= heads) { hh -= heads; ++tt; }
        } else {  // fewer heads than rows per batch: several tokens on
          const int q = static_cast<int>(hh) / static_cast<int>(heads);
          tt += q;
          hh -= static_cast<int64_t>(q) * heads;
        }
      }
      int64_t t = 0, h = 0;
      if (active[b]) {
        t = heads == 1 ? r[b] : tt;
        h = heads == 1 ? 0 : hh;
      }
      if constexpr (DS) dj[b] = active[b] ? ds_row(ds, t) : -1;  // heads == 1
      const T* xp = x + t * x_ts + h * x_hs;
      const T* rp = use_add ? res + t * r_rs : nullptr;
#pragma unroll
      for (int i = 0; i < VPT; ++i) {
        const int vi = i * G + gl;
        const bool ok = active[b] && vi < nv;
        xr[b][i] = ok ? ld_stream(xp + vi * E) : zero_vec();
        rr[b][i] = (ok && use_add) ? ld_stream(rp + vi * E) : zero_vec();
      }
      if constexpr (DS) {
        const T* vp = static_cast<const T*>(ds.vis) + (dj[b] >= 0 ? dj[b] : 0) * ds.vis_rs;
#pragma unroll
        for (int i = 0; i < VPT; ++i) {
          const int vi = i * G + gl;
          dr[b][i] = (dj[b] >= 0 && vi < nv) ? ld_stream(vp + vi * E) : zero_vec();
        }
      }
    }
#pragma unroll
    for (int b = 0; b < RB; ++b) {
      float v[VPT][E];
      float ss = 0.f;
#pragma unroll
      for (int i = 0; i < VPT; ++i) {
        unpack<T>(xr[b][i], v[i]);
        if (use_add) {
          float rv[E];
          unpack<T>(rr[b][i], rv);
#pragma unroll
          for (int e = 0; e < E; ++e) {
            const float sv = __fadd_rn(v[i][e], rv[e]);
            v[i][e] = round_sum ? round_to<T>(sv) : sv;
          }
          if constexpr (DS) {
            if (dj[b] >= 0) {
              unpack<T>(dr[b][i], rv);
#pragma unroll
              for (int e = 0; e < E; ++e) v[i][e] = round_to<T>(__fadd_rn(v[i][e], rv[e]));
            }
          }
        }
        ss = __fadd_rn(ss, sumsq_tree<E>(v[i]));
      }
#pragma unroll
      for (int off = G / 2; off > 0; off >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, off));
      const float rs = inv_sqrt_rn(__fadd_rn(ss / static_cast<float>(n), eps));
#pragma unroll
      for (int i = 0; i < VPT; ++i) {
        const int vi = i * G + gl;
        if (!(active[b] && vi < nv)) continue;
        if (use_add) st_vec(res_out + r[b] * n + vi * E, pack<T>(v[i]));
        uint32_t words[4];
        if constexpr (kPreW) {
          normalize_vec<T, W>(v[i], words, rs, wfs[i], wps[i]);
        } else {
          float wf[E];
          uint32_t wp[4];
          load_weights<T, W>(w, vi * E, wf);
          if constexpr (sizeof(T) == 2 && sizeof(W) == 2) from_u4(ld_vec(w + vi * E), wp);
          normalize_vec<T, W>(v[i], words, rs, wf, wp);
        }
        st_vec(y + r[b] * n + vi * E, as_u4(words));
      }
    }
  }
}

// One CTA per row (rows longer than 256 vectors); VPT vectors per thread.
template <typename T, typename W, int VPT, bool DS = false>
__global__ void __launch_bounds__(1024)
rms_rows_block(const T* __restrict__ x, int64_t x_ts, int64_t x_hs, const T* __restrict__ res,
               int64_t r_rs, const W* __restrict__ w, T* __restrict__ y, T* __restrict__ res_out,
               int64_t rows, int64_t heads, int n, float eps, int add, int round_sum, DsArgs ds) {
  ::nib::pdl_enter();
  constexpr int E = Elem<T>::kPerVec;
  __shared__ float red[32];
  const int nv = n / E;
  const int nwarp = blockDim.x >> 5;
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
    const int64_t t = heads == 1 ? r : r / heads;
    const int64_t h = r - t * heads;
    const T* xp = x + t * x_ts + h * x_hs;
    const T* rp = add ? res + t * r_rs : nullptr;
    uint4 xr[VPT], rr[VPT], dr[DS ? VPT : 1];
    int64_t dj = -1;
    if constexpr (DS) dj = ds_row(ds, t);  // heads == 1
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int vi = i * blockDim.x + threadIdx.x;
      const bool ok = vi < nv;
      xr[i] = ok ? ld_stream(xp + vi * E) : zero_vec();
      rr[i] = (ok && add) ? ld_stream(rp + vi * E) : zero_vec();
    }
    if constexpr (DS) {
      const T* vp = static_cast<const T*>(ds.vis) + (dj >= 0 ? dj : 0) * ds.vis_rs;
#pragma unroll
      for (int i = 0; i < VPT; ++i) {
        const int vi = i * blockDim.x + threadIdx.x;
        dr[i] = (dj >= 0 && vi < nv) ? ld_stream(vp + vi * E) : zero_vec();
      }
    }
    float v[VPT][E];
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      unpack<T>(xr[i], v[i]);
      if (add) {
        float rv[E];
        unpack<T>(rr[i], rv);
#pragma unroll
        for (int e = 0; e < E; ++e) {
          const float s = __fadd_rn(v[i][e], rv[e]);
          v[i][e] = round_sum ? round_to<T>(s) : s;
        }
        if constexpr (DS) {
          if (dj >= 0) {
            unpack<T>(dr[i], rv);
#pragma unroll
            for (int e = 0; e < E; ++e) v[i][e] = round_to<T>(__fadd_rn(v[i][e], rv[e]));
          }
        }
      }
      ss = __fadd_rn(ss, sumsq_tree<E>(v[i]));
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, off));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    float tot = 0.f;
    for (int i = 0; i < nwarp; ++i) tot = __fadd_rn(tot, red[i]);
    __syncthreads();  // red is rewritten by the next row
    const float rs = inv_sqrt_rn(__fadd_rn(tot / static_cast<float>(n), eps));
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int vi = i * blockDim.x + threadIdx.x;
      if (vi >= nv) continue;
      if (add) st_vec(res_out + r * n + vi * E, pack<T>(v[i]));
      float wf[E];
      uint32_t wp[4], words[4];
      load_weights<T, W>(w, vi * E, wf);
      if constexpr (sizeof(T) == 2 && sizeof(W) == 2) from_u4(ld_vec(w + vi * E), wp);
      normalize_vec<T, W>(v[i], words, rs, wf, wp);
      st_vec(y + r * n + vi * E, as_u4(words));
    }
  }
}

template <typename T, typename W, int G, int VPT, int RB = 1, bool DS = false>
static void launch_warp(const void* x, int64_t x_ts, int64_t x_hs, const void* res, int64_t r_rs,
                        const void* w, void* y, void* res_out, int64_t rows, int64_t heads, int n,
                        float eps, int add, int round_sum, cudaStream_t st, const DsArgs& ds) {
  // Full-warp rows: 4-warp CTAs (graph-timed on B200 over separate input sets,
  // Qwen3-VL add + norm at H = 2048: 82.6 us vs 85.0 us with 8-warp CTAs at
  // 32,768 rows, 621.9 vs 625.2 us at 262,144). Few rows (decode batches):
  // narrower still, so that the rows spread over every SM instead of queueing
  // on a few of them.
  int threads = G == 32 ? 128 : 256;
  if (G == 32) {
    const int64_t per_sm = (rows + sm_count() - 1) / sm_count();
    if (per_sm < 4) threads = 32 * static_cast<int>(per_sm < 1 ? 1 : per_sm);
  }
  const int64_t rows_per_block = (threads / 32) * (32 / G) * RB;
  int64_t blocks = (rows + rows_per_block - 1) / rows_per_block;
  // Full-warp rows: one-shot CTAs (a retiring CTA's store drain overlaps the
  // next CTA's loads; measured 3% faster on B200 than 32 persistent CTAs per
  // SM). Short rows keep persistent warps, which load their weights once.
  const int64_t cap = G < 32 ? static_cast<int64_t>(sm_count()) * 32 : kMaxGrid;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  // a single wave of full-warp rows (decode batches) preloads the weights
  if (G == 32 && rows <= static_cast<int64_t>(sm_count()) * 4) {
    ::nib::launch_k(rms_rows_warp<T, W, G, VPT, RB, DS, true>, static_cast<unsigned>(blocks), threads, 0, st,
        static_cast<const T*>(x), x_ts, x_hs, static_cast<const T*>(res), r_rs,
        static_cast<const W*>(w), static_cast<T*>(y), static_cast<T*>(res_out), rows, heads, n, eps,
        add, round_sum, ds);
    return;
  }
  ::nib::launch_k(rms_rows_warp<T, W, G, VPT, RB, DS>, static_cast<unsigned>(blocks), threads, 0, st,
      static_cast<const T*>(x), x_ts, x_hs, static_cast<const T*>(res), r_rs,
      static_cast<const W*>(w), static_cast<T*>(y), static_cast<T*>(res_out), rows, heads, n, eps,
      add, round_sum, ds);
}

template <typename T, typename W, bool DS>
static int launch_rms(const void* x, int64_t x_ts, int64_t x_hs, const void* res, int64_t r_rs,
                      const void* w, void* y, void* res_out, int64_t rows, int64_t heads,
                      int64_t n64, float eps, int add, int round_sum, cudaStream_t st,
                      const DsArgs& ds) {
  constexpr int E = Elem<T>::kPerVec;
  const int n = static_cast<int>(n64);
  const int nv = n / E;
  if constexpr (!DS) if (nv <= 32 && !add) {
    // short rows (attention heads, q/k norm): G lanes x 2 vectors, lane g owns
    // vectors g and g + G - the rotate-half partners when a row is one head.
    // The fused attention prologue uses the same layout and summation order.
    const int half = (nv + 1) / 2;
    if (half <= 1) launch_warp<T, W, 1, 2, 8>(x, x_ts, x_hs, res, r_rs, w, y, res_out, rows, heads, n, eps, add, round_sum, st, ds);
    else if (half <= 2) launch_warp<T, W, 2, 2, 8>(x, x_ts, x_hs, res, r_rs, w, y, res_out, rows, heads, n, eps, add, round_sum, st, ds);
    else if (half <= 4) launch_warp<T, W, 4, 2, 8>(x, x_ts, x_hs, res, r_rs, w, y, res_out, rows, heads, n, eps, add, round_sum, st, ds);
    else if (half <= 8) launch_warp<T, W, 8, 2, 8>(x, x_ts, x_hs, res, r_rs, w, y, res_out, rows, heads, n, eps, add, round_sum, st, ds);
    else launch_warp<T, W, 16, 2, 8>(x, x_ts, x_hs, res, r_rs, w, y, res_out, rows, heads, n, eps, add, round_sum, st, ds);
    return launch_status("rms_norm");
  }
  if (nv <= 256) {
    const int vpt = (nv + 31) / 32;
    switch (vpt) {
#define NIB_RMS_VPT(V) \
      case V: launch_warp<T, W, 32, V, 1, DS>(x, x_ts, x_hs, res, r_rs, w, y, res_out, rows, heads, n, eps, add, round_sum, st, ds); break;
      NIB_RMS_VPT(1) NIB_RMS_VPT(2) NIB_RMS_VPT(3) NIB_RMS_VPT(4)
      NIB_RMS_VPT(5) NIB_RMS_VPT(6) NIB_RMS_VPT(7) NIB_RMS_VPT(8)
#undef NIB_RMS_VPT
    }
    return launch_status("rms_norm");
  }
  // long rows: one CTA per row, 4 vectors per thread
  int threads = ((nv + 3) / 4 + 31) / 32 * 32;
  NIB_SUPPORT(threads <= 1024, "rms_norm: row of %d elements is longer than this build supports", n);
  int64_t blocks = rows;
  const int64_t cap = static_cast<int64_t>(sm_count()) * (2048 / threads);
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  ::nib::launch_k(rms_rows_block<T, W, 4, DS>, static_cast<unsigned>(blocks), threads, 0, st,
      static_cast<const T*>(x), x_ts, x_hs, static_cast<const T*>(res), r_rs,
      static_cast<const W*>(w), static_cast<T*>(y), static_cast<T*>(res_out), rows, heads, n, eps,
      add, round_sum, ds);
  return launch_status("rms_norm");
}

template <typename T, bool DS = false>
static int dispatch_weight(int weight_dtype, int dtype, const void* x, int64_t x_ts, int64_t x_hs,
                           const void* res, int64_t r_rs, const void* w, void* y, void* res_out,
                           int64_t rows, int64_t heads, int64_t n, float eps, int add,
                           int round_sum, cudaStream_t st, const DsArgs& ds = DsArgs{}) {
  if (weight_dtype == dtype)
    return launch_rms<T, T, DS>(x, x_ts, x_hs, res, r_rs, w, y, res_out, rows, heads, n, eps, add, round_sum, st, ds);
  if (weight_dtype == NIB_F32)
    return launch_rms<T, float, DS>(x, x_ts, x_hs, res, r_rs, w, y, res_out, rows, heads, n, eps, add, round_sum, st, ds);
  set_error("rms_norm: weight dtype %d must equal the activation dtype %d or be float32", weight_dtype, dtype);
  return NIB_ERR_UNSUPPORTED;
}

static int check_vec_rows(int dtype, const void* p, int64_t s1, int64_t s2, int64_t n, const char* what) {
  const int E = 16 / elem_size(dtype);
  NIB_SUPPORT(aligned16(p), "%s: data pointer is not 16-byte aligned", what);
  NIB_SUPPORT(n % E == 0, "%s: row length %lld is not a multiple of %d elements", what, (long long)n, E);
  NIB_SUPPORT(s1 % E == 0 && s2 % E == 0, "%s: strides must be multiples of %d elements", what, E);
  return NIB_OK;
}

}  // namespace nib

using namespace nib;

extern "C" int nib_rms_norm(int dtype, const void* x, int64_t x_token_stride, int64_t x_head_stride,
                            int64_t tokens, int64_t heads, int64_t n, int weight_dtype,
                            const void* weight, float eps, void* out, void* stream) {
  NIB_REQUIRE(tokens >= 0 && heads >= 1 && n >= 1, "rms_norm: bad sizes");
  if (tokens == 0) return NIB_OK;
  NIB_REQUIRE(x && weight && out, "rms_norm: null pointer");
  int rc = check_vec_rows(dtype, x, x_token_stride, x_head_stride, n, "rms_norm input");
  if (rc) return rc;
  rc = check_vec_rows(dtype, out, 0, 0, n, "rms_norm output");
  if (rc) return rc;
  NIB_SUPPORT(aligned16(weight), "rms_norm: weight is not 16-byte aligned");
  NIB_SUPPORT(dtype != NIB_F32 || weight_dtype == NIB_F32, "rms_norm: float32 input needs float32 weight");
  NIB_DISPATCH(dtype, T,
               return dispatch_weight<T>(weight_dtype, dtype, x, x_token_stride, x_head_stride,
                                         nullptr, 0, weight, out, nullptr, tokens * heads, heads, n,
                                         eps, 0, 0, as_stream(stream)));
  return NIB_OK;
}

extern "C" int nib_add_rms_norm(int dtype, const void* x, int64_t x_row_stride, const void* residual,
                                int64_t residual_row_stride, int64_t rows, int64_t n,
                                int weight_dtype, const void* weight, float eps, int round_sum,
                                void* out, void* residual_out, void* stream) {
  NIB_REQUIRE(rows >= 0 && n >= 1, "add_rms_norm: bad sizes");
  if (rows == 0) return NIB_OK;
  NIB_REQUIRE(x && residual && weight && out && residual_out, "add_rms_norm: null pointer");
  int rc = check_vec_rows(dtype, x, x_row_stride, 0, n, "add_rms_norm input");
  if (rc) return rc;
  rc = check_vec_rows(dtype, residual, residual_row_stride, 0, n, "add_rms_norm residual");
  if (rc) return rc;
  rc = check_vec_rows(dtype, out, 0, 0, n, "add_rms_norm output");
  if (rc) return rc;
  rc = check_vec_rows(dtype, residual_out, 0, 0, n, "add_rms_norm residual output");
  if (rc) return rc;
  NIB_SUPPORT(aligned16(weight), "add_rms_norm: weight is not 16-byte aligned");
  NIB_SUPPORT(dtype != NIB_F32 || weight_dtype == NIB_F32, "add_rms_norm: float32 input needs float32 weight");
  NIB_DISPATCH(dtype, T,
               return dispatch_weight<T>(weight_dtype, dtype, x, x_row_stride, 0, residual,
                                         residual_row_stride, weight, out, residual_out, rows, 1, n,
                                         eps, 1, round_sum ? 1 : 0, as_stream(stream)));
  return NIB_OK;
}

extern "C" int nib_add_rms_norm_deepstack(int dtype, const void* x, int64_t x_row_stride,
                                          const void* residual, int64_t residual_row_stride,
                                          int64_t rows, int64_t n, int weight_dtype,
                                          const void* weight, float eps, const void* vis,
                                          int64_t vis_row_stride, int64_t vis_rows,
                                          const int32_t* index, void* out, void* residual_out,
                                          unsigned int* status, void* stream) {
  NIB_REQUIRE(rows >= 0 && n >= 1 && vis_rows >= 0, "add_rms_norm_deepstack: bad sizes");
  if (rows == 0) return NIB_OK;
  NIB_REQUIRE(x && residual && weight && out && residual_out && index,
              "add_rms_norm_deepstack: null pointer");
  NIB_REQUIRE(vis || vis_rows == 0, "add_rms_norm_deepstack: null visual embedding");
  int rc = check_vec_rows(dtype, x, x_row_stride, 0, n, "add_rms_norm_deepstack input");
  if (rc) return rc;
  rc = check_vec_rows(dtype, residual, residual_row_stride, 0, n, "add_rms_norm_deepstack residual");
  if (rc) return rc;
  rc = check_vec_rows(dtype, out, 0, 0, n, "add_rms_norm_deepstack output");
  if (rc) return rc;
  rc = check_vec_rows(dtype, residual_out, 0, 0, n, "add_rms_norm_deepstack residual output");
  if (rc) return rc;
  if (vis_rows > 0) {
    rc = check_vec_rows(dtype, vis, vis_row_stride, 0, n, "add_rms_norm_deepstack visual embedding");
    if (rc) return rc;
  }
  NIB_SUPPORT(aligned16(weight), "add_rms_norm_deepstack: weight is not 16-byte aligned");
  NIB_SUPPORT(dtype != NIB_F32 || weight_dtype == NIB_F32,
              "add_rms_norm_deepstack: float32 input needs float32 weight");
  DsArgs ds;
  ds.vis = vis;
  ds.vis_rs = vis_row_stride;
  ds.vis_rows = vis_rows;
  ds.index = index;
  ds.status = status;
  NIB_DISPATCH(dtype, T,
               return dispatch_weight<T, true>(weight_dtype, dtype, x, x_row_stride, 0, residual,
                                               residual_row_stride, weight, out, residual_out, rows,
                                               1, n, eps, 1, 1, as_stream(stream), ds));
  return NIB_OK;
}
