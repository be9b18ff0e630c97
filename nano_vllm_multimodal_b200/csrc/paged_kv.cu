// Paged KV cache store / gather (byte-exact copies).
//
// store:  csrc/paged_kv/paged_kv_cuda.cu:21-59 semantics - token t with
//         slot s = slot_mapping[t] >= 0 overwrites flat slot s of the key and
//         value caches; s == -1 skips the token; other slots keep their bytes.
// gather: csrc/paged_kv/paged_kv_cuda.cu:61-94 semantics -
//         out[t] = cache[block_table[t / block_size], t % block_size].
//
// One warp per token row; rows move as 16-byte vectors whenever every
// address and stride is 16-byte aligned (else 8/4/2). Out-of-range slots and
// block ids are never dereferenced: they set a status bit (store skips the
// token, gather writes a zero row).
#include <cuda.h>

#include <mutex>

#include "copy_rows.cuh"
#include "dispatch.cuh"

namespace nib {

template <int VW>
__global__ void __launch_bounds__(256)
paged_store_kernel(const char* __restrict__ key, int64_t kts, const char* __restrict__ value,
                   int64_t vts, int64_t tokens, int units, char* __restrict__ kc,
                   char* __restrict__ vc, int64_t css, int64_t num_slots,
                   const int32_t* __restrict__ slots, unsigned int* status) {
  ::nib::pdl_enter();
  using V = typename VecOf<VW>::type;
  const int lane = threadIdx.x & 31;
  const int64_t warp = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  for (int64_t t = warp; t < tokens; t += nwarps) {
    const int32_t sv = __ldg(slots + t);
    if (sv < 0 || sv >= num_slots) {
      if (sv != -1 && lane == 0) flag(status, NIB_DEV_BAD_SLOT);
      continue;
    }
    const V* ks = reinterpret_cast<const V*>(key + t * kts);
    const V* vs = reinterpret_cast<const V*>(value + t * vts);
    V* kd = reinterpret_cast<V*>(kc + static_cast<int64_t>(sv) * css);
    V* vd = reinterpret_cast<V*>(vc + static_cast<int64_t>(sv) * css);
    for (int base = 0; base < units; base += 128) {
      V a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int u = base + i * 32 + lane;
        if (u < units) {
          a[i] = __ldg(ks + u);
          b[i] = __ldg(vs + u);
        }
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int u = base + i * 32 + lane;
        if (u < units) {
          kd[u] = a[i];
          vd[u] = b[i];
        }
      }
    }
  }
}

// blockIdx.y = sequence; warps of the x-grid stride over that sequence's tokens.
template <int VW>
__global__ void __launch_bounds__(256)
paged_gather_kernel(const char* __restrict__ cache, int64_t bst, int64_t sst, int64_t nblocks,
                    int64_t bs, int units, const int32_t* __restrict__ tables, int64_t table_stride,
                    const int32_t* __restrict__ seq_lens, const int64_t* __restrict__ cu,
                    int64_t fixed_len, char* __restrict__ out, int64_t row_bytes,
                    unsigned int* status) {
  ::nib::pdl_enter();
  const int lane = threadIdx.x & 31;
  const int64_t seq = blockIdx.y;
  const int64_t len = seq_lens ? static_cast<int64_t>(__ldg(seq_lens + seq)) : fixed_len;
  const int64_t obase = cu ? __ldg(cu + seq) : 0;
  const int32_t* tbl = tables + seq * table_stride;
  const int64_t warp = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  for (int64_t t = warp; t < len; t += nwarps) {
    const int64_t lb = t / bs;
    const int64_t off = t - lb * bs;
    const int32_t b = __ldg(tbl + lb);
    char* dst = out + (obase + t) * row_bytes;
    if (b < 0 || b >= nblocks) {
      if (lane == 0) flag(status, NIB_DEV_BAD_BLOCK);
      warp_zero_row<VW>(dst, units, lane);
      continue;
    }
    warp_copy_row<VW>(dst, cache + static_cast<int64_t>(b) * bst + off * sst, units, lane);
  }
}

// per_sm = 0: one CTA per warps_per_block rows (one-shot grid)
static unsigned grid_for_rows(int64_t rows, int warps_per_block, int per_sm) {
  int64_t blocks = (rows + warps_per_block - 1) / warps_per_block;
  const int64_t cap = per_sm > 0 ? static_cast<int64_t>(sm_count()) * per_sm : kMaxGrid;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  return static_cast<unsigned>(blocks);
}

static int gather_impl(int dtype, const void* cache, int64_t block_stride, int64_t slot_stride,
                       int64_t num_blocks, int64_t block_size, int64_t row_elems,
                       const int32_t* tables, int64_t table_stride, const int32_t* seq_lens,
                       const int64_t* cu, int64_t num_seqs, int64_t max_len, void* out,
                       unsigned int* status, cudaStream_t st) {
  const int es = elem_size(dtype);
  const int64_t row_bytes = row_elems * es;
  const int vw = pick_vec_width({reinterpret_cast<uint64_t>(cache), reinterpret_cast<uint64_t>(out),
                                 static_cast<uint64_t>(block_stride * es),
                                 static_cast<uint64_t>(slot_stride * es),
                                 static_cast<uint64_t>(row_bytes)});
  const int units = static_cast<int>(row_bytes / vw);
  NIB_SUPPORT(num_seqs <= 65535, "paged gather: at most 65535 sequences per launch");
  dim3 grid(grid_for_rows(max_len, 8, 16), static_cast<unsigned>(num_seqs));
  NIB_VW_SWITCH(vw, VW,
                ::nib::launch_k(paged_gather_kernel<VW>, grid, 256, 0, st,
                    static_cast<const char*>(cache), block_stride * es, slot_stride * es, num_blocks,
                    block_size, units, tables, table_stride, seq_lens, cu, max_len,
                    static_cast<char*>(out), row_bytes, status));
  return launch_status("paged_gather");
}

// ---------------------------------------------------------------- allocation-free variant
// Output offsets of nib_paged_gather_varlen_noalloc: a fixed array of this
// library's device module instead of a caller-allocated cu_seqlens buffer.
static __device__ __align__(256) int64_t g_gather_offsets[NIB_NOALLOC_MAX_SEQS + 1];

static std::mutex g_offsets_mu;

// Per device: the address of g_gather_offsets and the id of the CUDA context
// it was looked up in. A device reset destroys the context and unloads this
// module; the next context loads it again, possibly at another address, so a
// changed context id means the address is looked up again.
struct OffsetsEntry {
  unsigned long long ctx_id;
  int64_t* ptr;
};
static OffsetsEntry g_offsets_dev[64] = {};

using CtxGetCurrentFn = CUresult (*)(CUcontext*);
using CtxGetIdFn = CUresult (*)(CUcontext, unsigned long long*);

// Id of the calling thread's current context (0: none yet, or no driver entry
// point). The driver functions come through cudaGetDriverEntryPoint, so the
// library still links only the CUDA runtime.
static unsigned long long current_ctx_id() {
  static CtxGetCurrentFn get_current = nullptr;
  static CtxGetIdFn get_id = nullptr;
  static bool resolved = false;
  if (!resolved) {  // under g_offsets_mu
    void* f = nullptr;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &f, cudaEnableDefault) == cudaSuccess)
      get_current = reinterpret_cast<CtxGetCurrentFn>(f);
    f = nullptr;
    if (cudaGetDriverEntryPoint("cuCtxGetId", &f, cudaEnableDefault) == cudaSuccess)
      get_id = reinterpret_cast<CtxGetIdFn>(f);
    resolved = true;
  }
  CUcontext ctx = nullptr;
  unsigned long long id = 0;
  if (!get_current || !get_id || get_current(&ctx) != CUDA_SUCCESS || ctx == nullptr) return 0;
  if (get_id(ctx, &id) != CUDA_SUCCESS) return 0;
  return id;
}

// Device address of g_gather_offsets for the current device, looked up with
// that device current: on the first call on a device, and again whenever the
// device's context changed since (after cudaDeviceReset).
static int offsets_table(int64_t** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= 64) {
    set_error("paged_gather_varlen_noalloc: no usable current device (%s)", cudaGetErrorString(e));
    return NIB_ERR_CUDA;
  }
  std::lock_guard<std::mutex> lock(g_offsets_mu);
  OffsetsEntry& entry = g_offsets_dev[dev];
  unsigned long long ctx = current_ctx_id();
  if (entry.ptr == nullptr || ctx == 0 || ctx != entry.ctx_id) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_gather_offsets);
    if (e != cudaSuccess || p == nullptr) {
      set_error("paged_gather_varlen_noalloc: cudaGetSymbolAddress failed: %s", cudaGetErrorString(e));
      return NIB_ERR_CUDA;
    }
    if (ctx == 0) ctx = current_ctx_id();  // the lookup made the primary context current
    entry.ptr = static_cast<int64_t*>(p);
    entry.ctx_id = ctx;
  }
  *out = entry.ptr;
  return NIB_OK;
}

// Exclusive prefix sums of max(lens, 0) for n <= NIB_NOALLOC_MAX_SEQS, one CTA
// of 1024 threads with 4 entries each; writes offsets[0..n] (all of them, so
// nothing from an earlier call is ever read).
__global__ void __launch_bounds__(1024)
gather_offsets_kernel(const int32_t* __restrict__ lens, int n, int64_t* __restrict__ offsets) {
  ::nib::pdl_enter();
  __shared__ int64_t warp_total[32];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  int64_t v[4], local = 0;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int i = tid * 4 + k;
    const int32_t len = i < n ? __ldg(lens + i) : 0;
    v[k] = len > 0 ? len : 0;
    local += v[k];
  }
  int64_t incl = local;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const int64_t y = __shfl_up_sync(0xffffffffu, incl, off);
    if (lane >= off) incl += y;
  }
  if (lane == 31) warp_total[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    const int64_t w = warp_total[lane];
    int64_t wi = w;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int64_t y = __shfl_up_sync(0xffffffffu, wi, off);
      if (lane >= off) wi += y;
    }
    warp_total[lane] = wi - w;  // exclusive prefix of the warps
  }
  __syncthreads();
  int64_t base = warp_total[warp] + incl - local;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int i = tid * 4 + k;
    if (i < n) offsets[i] = base;
    base += v[k];
    if (i == n - 1) offsets[n] = base;
  }
  if (n == 0 && tid == 0) offsets[0] = 0;
}

}  // namespace nib

using namespace nib;

extern "C" int nib_paged_store(int dtype, const void* key, int64_t key_token_stride,
                               const void* value, int64_t value_token_stride, int64_t tokens,
                               int64_t row_elems, void* key_cache, void* value_cache,
                               int64_t cache_slot_stride, int64_t num_slots,
                               const int32_t* slot_mapping, unsigned int* status, void* stream) {
  NIB_REQUIRE(tokens >= 0 && row_elems >= 1 && num_slots >= 0, "paged_store: bad sizes");
  if (tokens == 0) return NIB_OK;
  NIB_REQUIRE(key && value && key_cache && value_cache && slot_mapping, "paged_store: null pointer");
  NIB_REQUIRE(dtype == NIB_F32 || dtype == NIB_F16 || dtype == NIB_BF16, "paged_store: bad dtype");
  const int es = elem_size(dtype);
  const int64_t row_bytes = row_elems * es;
  const int vw = pick_vec_width({reinterpret_cast<uint64_t>(key), reinterpret_cast<uint64_t>(value),
                                 reinterpret_cast<uint64_t>(key_cache),
                                 reinterpret_cast<uint64_t>(value_cache),
                                 static_cast<uint64_t>(key_token_stride * es),
                                 static_cast<uint64_t>(value_token_stride * es),
                                 static_cast<uint64_t>(cache_slot_stride * es),
                                 static_cast<uint64_t>(row_bytes)});
  const int units = static_cast<int>(row_bytes / vw);
  const cudaStream_t st = as_stream(stream);
  const unsigned grid = grid_for_rows(tokens, 8, 0);  // one-shot: 3% faster than 16 CTAs/SM
  NIB_VW_SWITCH(vw, VW,
                ::nib::launch_k(paged_store_kernel<VW>, grid, 256, 0, st,
                    static_cast<const char*>(key), key_token_stride * es,
                    static_cast<const char*>(value), value_token_stride * es, tokens, units,
                    static_cast<char*>(key_cache), static_cast<char*>(value_cache),
                    cache_slot_stride * es, num_slots, slot_mapping, status));
  return launch_status("paged_store");
}

extern "C" int nib_paged_gather(int dtype, const void* cache, int64_t block_stride,
                                int64_t slot_stride, int64_t num_blocks, int64_t block_size,
                                int64_t row_elems, const int32_t* block_table,
                                int64_t sequence_length, void* out, unsigned int* status,
                                void* stream) {
  NIB_REQUIRE(sequence_length >= 0 && row_elems >= 1 && block_size >= 1 && num_blocks >= 0,
              "paged_gather: bad sizes");
  if (sequence_length == 0) return NIB_OK;
  NIB_REQUIRE(cache && block_table && out, "paged_gather: null pointer");
  NIB_REQUIRE(dtype == NIB_F32 || dtype == NIB_F16 || dtype == NIB_BF16, "paged_gather: bad dtype");
  return gather_impl(dtype, cache, block_stride, slot_stride, num_blocks, block_size, row_elems,
                     block_table, 0, nullptr, nullptr, 1, sequence_length, out, status,
                     as_stream(stream));
}

extern "C" int nib_paged_gather_varlen(int dtype, const void* cache, int64_t block_stride,
                                       int64_t slot_stride, int64_t num_blocks, int64_t block_size,
                                       int64_t row_elems, const int32_t* block_tables,
                                       int64_t table_stride, const int32_t* seq_lens,
                                       const int64_t* cu_seqlens, int64_t num_seqs,
                                       int64_t max_seq_len, void* out, unsigned int* status,
                                       void* stream) {
  NIB_REQUIRE(num_seqs >= 0 && max_seq_len >= 0 && row_elems >= 1 && block_size >= 1,
              "paged_gather_varlen: bad sizes");
  if (num_seqs == 0 || max_seq_len == 0) return NIB_OK;
  NIB_REQUIRE(cache && block_tables && seq_lens && cu_seqlens && out,
              "paged_gather_varlen: null pointer");
  NIB_REQUIRE(dtype == NIB_F32 || dtype == NIB_F16 || dtype == NIB_BF16,
              "paged_gather_varlen: bad dtype");
  return gather_impl(dtype, cache, block_stride, slot_stride, num_blocks, block_size, row_elems,
                     block_tables, table_stride, seq_lens, cu_seqlens, num_seqs, max_seq_len, out,
                     status, as_stream(stream));
}

extern "C" int nib_paged_gather_varlen_noalloc(int dtype, const void* cache, int64_t block_stride,
                                               int64_t slot_stride, int64_t num_blocks,
                                               int64_t block_size, int64_t row_elems,
                                               const int32_t* block_tables, int64_t table_stride,
                                               const int32_t* seq_lens, int64_t num_seqs,
                                               int64_t max_seq_len, void* out, unsigned int* status,
                                               void* stream) {
  NIB_REQUIRE(num_seqs >= 0 && max_seq_len >= 0 && row_elems >= 1 && block_size >= 1,
              "paged_gather_varlen_noalloc: bad sizes");
  NIB_REQUIRE(num_seqs <= NIB_NOALLOC_MAX_SEQS,
              "paged_gather_varlen_noalloc: %lld sequences exceed the fixed offset table of %d; "
              "split the batch or use nib_paged_gather_varlen with caller-provided offsets",
              static_cast<long long>(num_seqs), NIB_NOALLOC_MAX_SEQS);
  if (num_seqs == 0 || max_seq_len == 0) return NIB_OK;
  NIB_REQUIRE(cache && block_tables && seq_lens && out, "paged_gather_varlen_noalloc: null pointer");
  NIB_REQUIRE(dtype == NIB_F32 || dtype == NIB_F16 || dtype == NIB_BF16,
              "paged_gather_varlen_noalloc: bad dtype");
  int64_t* offsets = nullptr;
  int rc = offsets_table(&offsets);
  if (rc != NIB_OK) return rc;
  const cudaStream_t st = as_stream(stream);
  ::nib::launch_k(gather_offsets_kernel, 1, 1024, 0, st, seq_lens, static_cast<int>(num_seqs), offsets);
  rc = launch_status("paged_gather_varlen_noalloc (offsets)");
  if (rc != NIB_OK) return rc;
  return gather_impl(dtype, cache, block_stride, slot_stride, num_blocks, block_size, row_elems,
                     block_tables, table_stride, seq_lens, offsets, num_seqs, max_seq_len, out, status,
                     st);
}
