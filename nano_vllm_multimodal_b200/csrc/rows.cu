// Row gathers and row updates: embedding lookup, DeepStack add, row copy.
//
// embedding: nanovllm/layers/embed_head.py:34-42 (F.embedding row gather; the
//            tensor-parallel branch zeroes rows whose id is outside this
//            rank's vocab shard before the all-reduce).
// deepstack: nanovllm/models/qwen3_vl.py:332-344, hidden[rows[j]] += vis[j]
//            in the activation dtype (fp32 add, one rounding).
// One warp per row, 16-byte vectors where alignment allows.
#include "copy_rows.cuh"
#include "dispatch.cuh"

namespace nib {

template <int VW>
__global__ void __launch_bounds__(256)
embedding_kernel(const int64_t* __restrict__ ids, int64_t n_ids, const char* __restrict__ weight,
                 int64_t w_rs, int64_t vocab_rows, int64_t vstart, int64_t vend, int units,
                 int mask, char* __restrict__ out, int64_t row_bytes, unsigned int* status) {
  ::nib::pdl_enter();
  const int lane = threadIdx.x & 31;
  const int64_t warp = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  for (int64_t i = warp; i < n_ids; i += nwarps) {
    const int64_t id = __ldg(ids + i);
    char* dst = out + i * row_bytes;
    const int64_t row = id - vstart;
    const bool in_shard = id >= vstart && id < vend;
    if (!in_shard || row >= vocab_rows) {
      if (!mask || row >= vocab_rows || id < 0) {
        if (lane == 0) flag(status, NIB_DEV_BAD_INDEX);
      }
      warp_zero_row<VW>(dst, units, lane);
      continue;
    }
    warp_copy_row<VW>(dst, weight + row * w_rs, units, lane);
  }
}

// index[t] = -1 for every token, then index[rows[j]] = j (two launches on one stream)
__global__ void __launch_bounds__(256)
fill_index_kernel(int32_t* __restrict__ index, int64_t tokens) {
  ::nib::pdl_enter();
  for (int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; t < tokens;
       t += static_cast<int64_t>(gridDim.x) * blockDim.x)
    index[t] = -1;
}
__global__ void __launch_bounds__(256)
scatter_index_kernel(const int64_t* __restrict__ rows, int64_t n_rows, int64_t tokens,
                     int32_t* __restrict__ index, unsigned int* status) {
  ::nib::pdl_enter();
  for (int64_t j = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; j < n_rows;
       j += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = __ldg(rows + j);
    if (r < 0 || r >= tokens) {
      flag(status, NIB_DEV_BAD_INDEX);
      continue;
    }
    index[r] = static_cast<int32_t>(j);
  }
}

template <typename T>
__global__ void __launch_bounds__(256)
deepstack_add_kernel(T* __restrict__ h, int64_t h_rs, int64_t tokens, int n,
                     const int64_t* __restrict__ rows, int64_t n_rows, const T* __restrict__ vis,
                     int64_t v_rs, unsigned int* status) {
  ::nib::pdl_enter();
  constexpr int E = Elem<T>::kPerVec;
  const int lane = threadIdx.x & 31;
  const int nv = n / E;
  const int64_t warp = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  for (int64_t j = warp; j < n_rows; j += nwarps) {
    const int64_t r = __ldg(rows + j);
    if (r < 0 || r >= tokens) {
      if (lane == 0) flag(status, NIB_DEV_BAD_INDEX);
      continue;
    }
    T* hp = h + r * h_rs;
    const T* vp = vis + j * v_rs;
    for (int base = 0; base < nv; base += 128) {
      uint4 a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int u = base + i * 32 + lane;
        if (u < nv) {
          a[i] = ld_vec(hp + u * E);
          b[i] = ld_stream(vp + u * E);
        }
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int u = base + i * 32 + lane;
        if (u >= nv) continue;
        float x[E], y[E];
        unpack<T>(a[i], x);
        unpack<T>(b[i], y);
#pragma unroll
        for (int e = 0; e < E; ++e) x[e] = __fadd_rn(x[e], y[e]);
        st_vec(hp + u * E, pack<T>(x));
      }
    }
  }
}

template <int VW>
__global__ void __launch_bounds__(256)
copy_rows_kernel(const char* __restrict__ in, int64_t in_rs, int64_t rows, int units,
                 char* __restrict__ out, int64_t out_rs) {
  ::nib::pdl_enter();
  const int lane = threadIdx.x & 31;
  const int64_t warp = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  for (int64_t r = warp; r < rows; r += nwarps)
    warp_copy_row<VW>(out + r * out_rs, in + r * in_rs, units, lane);
}

static unsigned warp_grid(int64_t rows) {
  int64_t blocks = (rows + 7) / 8;
  const int64_t cap = static_cast<int64_t>(sm_count()) * 16;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  return static_cast<unsigned>(blocks);
}

}  // namespace nib

using namespace nib;

extern "C" int nib_embedding(int dtype, const int64_t* ids, int64_t n_ids, const void* weight,
                             int64_t weight_row_stride, int64_t vocab_rows, int64_t vocab_start,
                             int64_t vocab_end, int64_t hidden, int mask_out_of_range, void* out,
                             unsigned int* status, void* stream) {
  NIB_REQUIRE(n_ids >= 0 && hidden >= 1 && vocab_rows >= 0, "embedding: bad sizes");
  if (n_ids == 0) return NIB_OK;
  NIB_REQUIRE(ids && weight && out, "embedding: null pointer");
  NIB_REQUIRE(dtype == NIB_F32 || dtype == NIB_F16 || dtype == NIB_BF16, "embedding: bad dtype");
  const int es = elem_size(dtype);
  const int64_t row_bytes = hidden * es;
  const int vw = pick_vec_width({reinterpret_cast<uint64_t>(weight), reinterpret_cast<uint64_t>(out),
                                 static_cast<uint64_t>(weight_row_stride * es),
                                 static_cast<uint64_t>(row_bytes)});
  const int units = static_cast<int>(row_bytes / vw);
  const cudaStream_t st = as_stream(stream);
  NIB_VW_SWITCH(vw, VW,
                ::nib::launch_k(embedding_kernel<VW>, warp_grid(n_ids), 256, 0, st,
                    ids, n_ids, static_cast<const char*>(weight), weight_row_stride * es,
                    vocab_rows, vocab_start, vocab_end, units, mask_out_of_range,
                    static_cast<char*>(out), row_bytes, status));
  return launch_status("embedding");
}

extern "C" int nib_deepstack_add(int dtype, void* hidden, int64_t hidden_row_stride, int64_t tokens,
                                 int64_t n, const int64_t* rows, int64_t n_rows, const void* vis,
                                 int64_t vis_row_stride, unsigned int* status, void* stream) {
  NIB_REQUIRE(n_rows >= 0 && n >= 1 && tokens >= 0, "deepstack_add: bad sizes");
  if (n_rows == 0) return NIB_OK;
  NIB_REQUIRE(hidden && rows && vis, "deepstack_add: null pointer");
  const int E = 16 / elem_size(dtype);
  NIB_SUPPORT(aligned16(hidden) && aligned16(vis), "deepstack_add: pointers must be 16-byte aligned");
  NIB_SUPPORT(n % E == 0 && hidden_row_stride % E == 0 && vis_row_stride % E == 0,
              "deepstack_add: row length and strides must be multiples of %d elements", E);
  const cudaStream_t st = as_stream(stream);
  NIB_DISPATCH(dtype, T,
               ::nib::launch_k(deepstack_add_kernel<T>, warp_grid(n_rows), 256, 0, st,
                   static_cast<T*>(hidden), hidden_row_stride, tokens, static_cast<int>(n), rows,
                   n_rows, static_cast<const T*>(vis), vis_row_stride, status));
  return launch_status("deepstack_add");
}

extern "C" int nib_deepstack_row_index(const int64_t* rows, int64_t n_rows, int64_t tokens,
                                       int32_t* index, unsigned int* status, void* stream) {
  NIB_REQUIRE(n_rows >= 0 && tokens >= 0 && n_rows <= INT32_MAX, "deepstack_row_index: bad sizes");
  if (tokens == 0) return NIB_OK;
  NIB_REQUIRE(index && (rows || n_rows == 0), "deepstack_row_index: null pointer");
  const cudaStream_t st = as_stream(stream);
  int64_t blocks = (tokens + 255) / 256;
  if (blocks > kMaxGrid) blocks = kMaxGrid;
  ::nib::launch_k(fill_index_kernel, static_cast<unsigned>(blocks), 256, 0, st, index, tokens);
  if (n_rows > 0) {
    int64_t b2 = (n_rows + 255) / 256;
    if (b2 > kMaxGrid) b2 = kMaxGrid;
    ::nib::launch_k(scatter_index_kernel, static_cast<unsigned>(b2), 256, 0, st, rows, n_rows, tokens, index, status);
  }
  return launch_status("deepstack_row_index");
}

extern "C" int nib_copy_rows(int dtype, const void* in, int64_t in_row_stride, int64_t rows,
                             int64_t n, void* out, int64_t out_row_stride, void* stream) {
  NIB_REQUIRE(rows >= 0 && n >= 1, "copy_rows: bad sizes");
  if (rows == 0) return NIB_OK;
  NIB_REQUIRE(in && out, "copy_rows: null pointer");
  NIB_REQUIRE(dtype == NIB_F32 || dtype == NIB_F16 || dtype == NIB_BF16, "copy_rows: bad dtype");
  const int es = elem_size(dtype);
  const int64_t row_bytes = n * es;
  const int vw = pick_vec_width({reinterpret_cast<uint64_t>(in), reinterpret_cast<uint64_t>(out),
                                 static_cast<uint64_t>(in_row_stride * es),
                                 static_cast<uint64_t>(out_row_stride * es),
                                 static_cast<uint64_t>(row_bytes)});
  const int units = static_cast<int>(row_bytes / vw);
  const cudaStream_t st = as_stream(stream);
  NIB_VW_SWITCH(vw, VW,
                ::nib::launch_k(copy_rows_kernel<VW>, warp_grid(rows), 256, 0, st,
                    static_cast<const char*>(in), in_row_stride * es, rows, units,
                    static_cast<char*>(out), out_row_stride * es));
  return launch_status("copy_rows");
}
