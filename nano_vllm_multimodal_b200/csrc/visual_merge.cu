// Visual-embedding merge of a packed prefill batch
// (nanovllm/engine/model_runner.py:170-286, build_planned_visual_embeddings).
//
// The reference clones the token embeddings, then per feature key builds host
// index tensors, index_selects the feature rows (final and each DeepStack
// layer) and index_copies them into the clone and into one [R, H] payload per
// layer. Here the plan arrives as three device arrays (output row, source,
// feature row per replacement) plus a device table of the sources, and one
// launch writes every output row exactly once:
//   warps [0, tokens):       merged[t] = feature row (if t is planned) else token row
//   warps [tokens, tokens+R): deepstack[l][i] = source(i).deepstack[l][feature_row(i)]
// A token -> replacement map (int32, -1 for text rows) is built first by two
// small launches. Rows whose source dtype differs from the output dtype are
// converted element by element through fp32 (the reference's `.to(dtype)`:
// widening is exact, narrowing rounds to nearest even); equal dtypes copy bytes
// with the widest vector the row's addresses allow.
#include "copy_rows.cuh"
#include "dispatch.cuh"

static_assert(sizeof(nib_visual_source) == 32 + 16 * NIB_VISUAL_MAX_LAYERS,
              "nib_visual_source layout is part of the ABI");

namespace nib {

__device__ __forceinline__ float elem_as_float(const char* row, int dtype, int64_t e) {
  if (dtype == NIB_F32) return reinterpret_cast<const float*>(row)[e];
  if (dtype == NIB_BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(row)[e]);
  return __half2float(reinterpret_cast<const __half*>(row)[e]);
}

__device__ __forceinline__ void elem_from_float(char* row, int dtype, int64_t e, float v) {
  if (dtype == NIB_F32) reinterpret_cast<float*>(row)[e] = v;
  else if (dtype == NIB_BF16) reinterpret_cast<__nv_bfloat16*>(row)[e] = __float2bfloat16_rn(v);
  else reinterpret_cast<__half*>(row)[e] = __float2half_rn(v);
}

__device__ __forceinline__ int dtype_bytes(int dtype) { return dtype == NIB_F32 ? 4 : 2; }

// one warp: dst row (dtype dd) <- src row (dtype sd), n elements
__device__ __forceinline__ void warp_row(char* dst, int dd, const char* src, int sd, int64_t n, int lane) {
  if (sd == dd) {
    const int64_t bytes = n * dtype_bytes(dd);
    const uint64_t a = reinterpret_cast<uint64_t>(dst) | reinterpret_cast<uint64_t>(src) |
                       static_cast<uint64_t>(bytes);
    if ((a & 15u) == 0) warp_copy_row<16>(dst, src, static_cast<int>(bytes / 16), lane);
    else if ((a & 7u) == 0) warp_copy_row<8>(dst, src, static_cast<int>(bytes / 8), lane);
    else if ((a & 3u) == 0) warp_copy_row<4>(dst, src, static_cast<int>(bytes / 4), lane);
    else warp_copy_row<2>(dst, src, static_cast<int>(bytes / 2), lane);
    return;
  }
  for (int64_t e = lane; e < n; e += 32) elem_from_float(dst, dd, e, elem_as_float(src, sd, e));
}

__device__ __forceinline__ void warp_zero(char* dst, int64_t bytes, int lane) {
  for (int64_t b = lane; b < bytes / 2; b += 32) reinterpret_cast<uint16_t*>(dst)[b] = 0;
}

// source and feature row of replacement i; nullptr when either is out of range
__device__ __forceinline__ const nib_visual_source* resolve(const nib_visual_source* sources,
                                                            int64_t num_sources,
                                                            const int64_t* source_index,
                                                            const int64_t* feature_rows, int64_t i,
                                                            int64_t* f) {
  const int64_t k = __ldg(source_index + i);
  *f = __ldg(feature_rows + i);
  if (k < 0 || k >= num_sources) return nullptr;
  const nib_visual_source* s = sources + k;
  if (*f < 0 || *f >= s->final_count) return nullptr;
  return s;
}

__global__ void __launch_bounds__(256)
visual_row_map_fill(int32_t* __restrict__ row_map, int64_t tokens) {
  ::nib::pdl_enter();
  for (int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; t < tokens;
       t += static_cast<int64_t>(gridDim.x) * blockDim.x)
    row_map[t] = -1;
}

__global__ void __launch_bounds__(256)
visual_row_map_scatter(const int64_t* __restrict__ output_rows, int64_t n, int64_t tokens,
                       int32_t* __restrict__ row_map, unsigned int* status) {
  ::nib::pdl_enter();
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = __ldg(output_rows + i);
    if (r < 0 || r >= tokens) {
      flag(status, NIB_DEV_BAD_INDEX);
      continue;
    }
    row_map[r] = static_cast<int32_t>(i);
  }
}

__global__ void __launch_bounds__(256, 4)
visual_merge_kernel(const char* __restrict__ tok, int64_t tok_rs_bytes, int64_t tokens, int64_t n,
                    int dd, const nib_visual_source* __restrict__ sources, int64_t num_sources,
                    int layers, const int64_t* __restrict__ source_index,
                    const int64_t* __restrict__ feature_rows, int64_t R,
                    const int32_t* __restrict__ row_map, char* __restrict__ merged,
                    char* __restrict__ deepstack, unsigned int* status) {
  ::nib::pdl_enter();
  const int lane = threadIdx.x & 31;
  const int64_t row_bytes = n * dtype_bytes(dd);
  const int64_t warp = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  for (int64_t w = warp; w < tokens + R; w += nwarps) {
    // a merged-row warp writes one row, a DeepStack warp one row per layer
    const bool merged_row = w < tokens;
    int64_t i = merged_row ? __ldg(row_map + w) : w - tokens;
    const bool text = merged_row && i < 0;
    int64_t f = 0;
    const nib_visual_source* s = nullptr;
    if (!text) {
      s = resolve(sources, num_sources, source_index, feature_rows, i, &f);
      if (s == nullptr && lane == 0) flag(status, NIB_DEV_BAD_INDEX);
    }
    const int jobs = merged_row ? 1 : layers;
    for (int l = 0; l < jobs; ++l) {
      char* dst = merged_row ? merged + w * row_bytes : deepstack + (static_cast<int64_t>(l) * R + i) * row_bytes;
      const char* src = nullptr;
      int sd = dd;
      if (text) {
        src = tok + w * tok_rs_bytes;
      } else if (s != nullptr) {
        sd = s->dtype;
        const char* base = static_cast<const char*>(merged_row ? s->final_rows : s->deepstack[l]);
        const int64_t stride = merged_row ? s->final_row_stride : s->deepstack_row_stride[l];
        src = base + f * stride * dtype_bytes(sd);
      }
      if (src == nullptr) warp_zero(dst, row_bytes, lane);
      else warp_row(dst, dd, src, sd, n, lane);
    }
  }
}

}  // namespace nib

using namespace nib;

extern "C" int nib_visual_merge(int dtype, const void* token_embeddings, int64_t token_row_stride,
                                int64_t tokens, int64_t hidden, const nib_visual_source* sources,
                                int64_t num_sources, int num_layers, const int64_t* output_rows,
                                const int64_t* source_index, const int64_t* feature_rows,
                                int64_t num_replacements, int32_t* row_map, void* merged,
                                void* deepstack_out, unsigned int* status, void* stream) {
  NIB_REQUIRE(tokens >= 0 && hidden >= 1 && num_replacements >= 0 && num_sources >= 0,
              "visual_merge: bad sizes");
  NIB_REQUIRE(num_layers >= 0 && num_layers <= NIB_VISUAL_MAX_LAYERS,
              "visual_merge: at most %d DeepStack layers", NIB_VISUAL_MAX_LAYERS);
  NIB_REQUIRE(num_replacements <= INT32_MAX, "visual_merge: too many replacements");
  NIB_REQUIRE(dtype == NIB_F32 || dtype == NIB_F16 || dtype == NIB_BF16, "visual_merge: bad dtype");
  if (tokens == 0 && num_replacements == 0) return NIB_OK;
  NIB_REQUIRE((token_embeddings && merged && row_map) || tokens == 0, "visual_merge: null pointer");
  NIB_REQUIRE(num_replacements == 0 || (sources && output_rows && source_index && feature_rows),
              "visual_merge: null plan pointer");
  NIB_REQUIRE(num_layers == 0 || num_replacements == 0 || deepstack_out,
              "visual_merge: null DeepStack output");
  const cudaStream_t st = as_stream(stream);
  if (tokens > 0) {
    int64_t b = (tokens + 255) / 256;
    if (b > kMaxGrid) b = kMaxGrid;
    ::nib::launch_k(visual_row_map_fill, static_cast<unsigned>(b), 256, 0, st, row_map, tokens);
  }
  if (num_replacements > 0 && tokens > 0) {
    int64_t b = (num_replacements + 255) / 256;
    if (b > kMaxGrid) b = kMaxGrid;
    ::nib::launch_k(visual_row_map_scatter, static_cast<unsigned>(b), 256, 0, st, output_rows, num_replacements,
                                                                      tokens, row_map, status);
  }
  const int64_t R = num_layers > 0 ? num_replacements : 0;  // DeepStack warps only with layers
  const int64_t warps = tokens + R;
  if (warps > 0) {
    int64_t b = (warps + 7) / 8;  // one warp per output row, one-shot grid
    if (b > kMaxGrid) b = kMaxGrid;
    ::nib::launch_k(visual_merge_kernel, static_cast<unsigned>(b), 256, 0, st,
        static_cast<const char*>(token_embeddings), token_row_stride * elem_size(dtype), tokens,
        hidden, dtype, sources, num_sources, num_layers, source_index, feature_rows, R, row_map,
        static_cast<char*>(merged), static_cast<char*>(deepstack_out), status);
  }
  return launch_status("visual_merge");
}
