/*
 * nib_b200.h - C ABI of the B200 (sm_100a) per-token decoder elementwise path.
 *
 * Library: libnib_b200.so (built from nano_vllm_multimodal_b200/csrc/*.cu).
 * Every entry point takes plain device pointers, element counts and strides
 * (in ELEMENTS, not bytes), launches on the given CUDA stream (a cudaStream_t
 * passed as void*, NULL = legacy default stream) and returns a nib_status.
 * The entry points other than nib_paged_gather_varlen_noalloc neither
 * allocate, synchronise nor read device memory on the host, so they may be
 * captured in a CUDA graph. On a non-zero status, nib_last_error() returns a
 * message for the calling thread.
 *
 * Index errors (slot, position, block id, token id or row out of range) never
 * cause an out-of-bounds access: the offending row is skipped or written as
 * zeros, and if `status` is non-NULL the kernel ORs a NIB_DEV_* bit into that
 * device word, which the caller may read back after the stream completes.
 *
 * "Replaces" lines cite the NanoInfer interface each entry point stands in
 * for (file:line inside the NanoInfer project).
 */
#ifndef NIB_B200_H
#define NIB_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define NIB_ABI_VERSION 1

#if defined(__GNUC__)
#define NIB_API __attribute__((visibility("default")))
#else
#define NIB_API
#endif

typedef enum {
  NIB_OK = 0,
  NIB_ERR_INVALID = 1,     /* bad argument (null pointer, negative size, ...) */
  NIB_ERR_UNSUPPORTED = 2, /* valid request that this build has no kernel for
                              (dtype, head_dim, misaligned vector rows) */
  NIB_ERR_CUDA = 3         /* launch failed; message holds cudaGetErrorString */
} nib_status;

typedef enum { NIB_F32 = 0, NIB_F16 = 1, NIB_BF16 = 2 } nib_dtype;

/* device status bits (ORed into *status by kernels) */
#define NIB_DEV_BAD_SLOT 1u     /* slot_mapping value < -1 or >= num_slots */
#define NIB_DEV_BAD_POSITION 2u /* 1-D RoPE position outside the cos/sin table */
#define NIB_DEV_BAD_BLOCK 4u    /* block-table entry outside [0, num_blocks) */
#define NIB_DEV_BAD_INDEX 8u    /* token id / DeepStack row outside its range */

NIB_API int nib_abi_version(void);
NIB_API const char* nib_last_error(void);

/* ------------------------------------------------------------------ norms */

/* RMSNorm over rows of n elements, rows addressed as (token, head):
 *   x[t, h, :] = x + t*x_token_stride + h*x_head_stride,  rows = tokens*heads.
 * out is contiguous [tokens, heads, n]. weight has n elements of weight_dtype
 * (== dtype, or NIB_F32). Numerics: fp32 statistics, the normalised value is
 * rounded to dtype, then multiplied by the weight and rounded once more.
 * Replaces: RMSNorm.rms_forward           nanovllm/layers/layernorm.py:16-26
 *           Qwen3VLTextRMSNorm.forward     nanovllm/models/qwen3_vl.py:74-79
 *           (per-head q/k norm on strided views: nanovllm/models/qwen3.py:82-84) */
NIB_API int nib_rms_norm(int dtype, const void* x, int64_t x_token_stride, int64_t x_head_stride,
                 int64_t tokens, int64_t heads, int64_t n, int weight_dtype, const void* weight,
                 float eps, void* out, void* stream);

/* Fused residual add + RMSNorm over [rows, n] (row strides in elements).
 * round_sum = 0: RMSNorm.add_rms_forward (fp32 sum feeds the statistics,
 *                residual_out = sum rounded)  nanovllm/layers/layernorm.py:28-40
 * round_sum = 1: Qwen3-VL decoder (`h + residual` rounded to dtype first, then
 *                Qwen3VLTextRMSNorm)          nanovllm/models/qwen3_vl.py:232-237
 * out and residual_out are contiguous [rows, n]; either may alias x or
 * residual exactly (each element is read before it is written). */
NIB_API int nib_add_rms_norm(int dtype, const void* x, int64_t x_row_stride, const void* residual,
                     int64_t residual_row_stride, int64_t rows, int64_t n, int weight_dtype,
                     const void* weight, float eps, int round_sum, void* out, void* residual_out,
                     void* stream);

/* Qwen3-VL layer boundary with the DeepStack add folded in (one token per row):
 *   s = dtype(x + residual); if index[t] >= 0: s = dtype(s + vis[index[t]]);
 *   out = Qwen3VLTextRMSNorm(s); residual_out = s
 * in one pass over [rows, n]. index is int32 [rows] (nib_deepstack_row_index);
 * vis is [vis_rows, n] with row stride vis_row_stride. An index outside
 * [-1, vis_rows) sets NIB_DEV_BAD_INDEX in *status (when given) and the token
 * is treated as text. out/residual_out may alias x or residual as in
 * nib_add_rms_norm; vis must not alias them.
 * Replaces, in one kernel: the layer output add (nanovllm/models/qwen3_vl.py:238),
 * _add_deepstack_rows (qwen3_vl.py:332-344, called at :371-376) and the next
 * layer's input add + input_layernorm (qwen3_vl.py:232-235, 74-79). */
NIB_API int nib_add_rms_norm_deepstack(int dtype, const void* x, int64_t x_row_stride,
                               const void* residual, int64_t residual_row_stride, int64_t rows,
                               int64_t n, int weight_dtype, const void* weight, float eps,
                               const void* vis, int64_t vis_row_stride, int64_t vis_rows,
                               const int32_t* index, void* out, void* residual_out,
                               unsigned int* status, void* stream);

/* ------------------------------------------------------------------ visual merge */

#define NIB_VISUAL_MAX_LAYERS 8

/* One vision-feature source (one feature key of the reference's plan): its
 * final embedding rows and, per DeepStack layer, the rows of that layer (same
 * row count). Row strides in elements; dtype is a nib_dtype. Lives in device
 * memory (an array of these is read by the kernel). 160 bytes. */
typedef struct nib_visual_source {
  const void* final_rows;
  int64_t final_row_stride;
  int64_t final_count;
  int32_t dtype;
  int32_t reserved;
  const void* deepstack[NIB_VISUAL_MAX_LAYERS];
  int64_t deepstack_row_stride[NIB_VISUAL_MAX_LAYERS];
} nib_visual_source;

/* Packed-prefill visual merge. For replacement i < num_replacements (device
 * arrays): merged[output_rows[i]] = sources[source_index[i]].final_rows[feature_rows[i]],
 * and for every layer l < num_layers:
 * deepstack_out[l, i] = sources[source_index[i]].deepstack[l][feature_rows[i]].
 * Every other merged row is the token embedding row. merged is contiguous
 * [tokens, hidden] of `dtype`; deepstack_out contiguous [num_layers,
 * num_replacements, hidden]. Source rows of another dtype are converted (fp32
 * round trip, round to nearest). row_map: device scratch of `tokens` int32.
 * Out-of-range output rows, sources or feature rows set NIB_DEV_BAD_INDEX in
 * *status (when given); their rows are skipped (output rows) or zero-filled.
 * Three launches, no allocation, no synchronisation.
 * Replaces: build_planned_visual_embeddings / merge_planned_visual_embeddings
 * nanovllm/engine/model_runner.py:158-286 (per-key index_select/index_copy_) */
NIB_API int nib_visual_merge(int dtype, const void* token_embeddings, int64_t token_row_stride,
                     int64_t tokens, int64_t hidden, const nib_visual_source* sources,
                     int64_t num_sources, int num_layers, const int64_t* output_rows,
                     const int64_t* source_index, const int64_t* feature_rows,
                     int64_t num_replacements, int32_t* row_map, void* merged,
                     void* deepstack_out, unsigned int* status, void* stream);

/* ------------------------------------------------------------------ decode attention */

/* Paged decode attention: out[b, h] = softmax(q[b, h] . K^T * scale) V over the
 * first context_lens[b] tokens of request b's cache, token t at slot
 * t % block_size of block block_tables[b, t / block_size]; q head h reads kv
 * head h / (num_heads / num_kv_heads). Caches are [num_blocks, block_size,
 * num_kv_heads, head_dim] with the given strides (elements). dtype bf16 or
 * f16, head_dim 64 / 128 / 256, at most 16 q heads per kv head; arithmetic in
 * fp32, output rounded once. A context length outside [0, max_blocks_per_seq *
 * block_size] sets NIB_DEV_BAD_INDEX and is clamped; a block id outside
 * [0, num_blocks) sets NIB_DEV_BAD_BLOCK and its token is left out. An empty
 * context gives zeros. max_context_len (host upper bound, 0 = from the table
 * width) picks how many CTAs split a context; the partials then need
 * nib_decode_attention_workspace_bytes() bytes of device workspace.
 * Replaces: flash_attn_with_kvcache(q.unsqueeze(1), k_cache, v_cache,
 * cache_seqlens, block_table, softmax_scale, causal=True)
 * nanovllm/layers/attention.py:122-130 (numerics: the SDPA decode branch,
 * attention.py:286-300) */
typedef struct nib_decode_attention_args {
  int32_t struct_size; /* sizeof(nib_decode_attention_args) */
  int32_t dtype;
  int64_t batch;
  int32_t num_heads, num_kv_heads, head_dim;
  int32_t variant;     /* 0: tensor-core kernel where it applies (bf16/f16, head_dim 64/128,
                          <= 16 q heads per kv head, block_size % 16 == 0), else the CUDA-core
                          kernel; 1: CUDA-core kernel; 2: tensor-core kernel or NIB_ERR_UNSUPPORTED */
  const void* q;
  int64_t q_batch_stride, q_head_stride;
  const void* key_cache;
  const void* value_cache;
  int64_t cache_block_stride, cache_slot_stride, cache_head_stride;
  int64_t num_blocks, block_size;
  const int32_t* block_tables;
  int64_t block_table_stride, max_blocks_per_seq;
  const int32_t* context_lens;
  float scale;
  int32_t reserved2;
  void* out;
  int64_t out_batch_stride, out_head_stride;
  void* workspace;
  int64_t workspace_bytes;
  int64_t max_context_len;
  unsigned int* status;
} nib_decode_attention_args;

NIB_API int64_t nib_decode_attention_workspace_bytes(const nib_decode_attention_args* args);
NIB_API int nib_decode_attention(const nib_decode_attention_args* args, void* stream);

/* ------------------------------------------------------------------ activation */

/* y[t, :] = silu(x[t, :I]) * x[t, I:2I], computed in fp32, rounded once.
 * x row stride in elements; y contiguous [rows, I].
 * Replaces: SiluAndMul.forward  nanovllm/layers/activation.py:8-11 */
NIB_API int nib_silu_and_mul(int dtype, const void* x, int64_t x_row_stride, int64_t rows,
                     int64_t inter, void* y, void* stream);

/* ------------------------------------------------------------------ attention prologue */

typedef enum {
  NIB_ROPE_NONE = 0,
  NIB_ROPE_TABLE = 1,       /* 1-D neox RoPE from the fp32 cos|sin table */
  NIB_ROPE_MROPE_CHUNKED = 2,    /* Qwen2.5-VL multimodal RoPE */
  NIB_ROPE_MROPE_INTERLEAVED = 3 /* Qwen3-VL multimodal RoPE */
} nib_rope_mode;

typedef struct {
  int32_t struct_size; /* sizeof(nib_qk_prologue_args) */
  int32_t dtype;       /* activations: q, k, v, outputs, caches */
  int64_t tokens;
  int32_t num_heads, num_kv_heads, head_dim;
  /* inputs: [tokens, heads, head_dim] with arbitrary token/head strides,
     innermost dim contiguous */
  const void* q; int64_t q_token_stride, q_head_stride;
  const void* k; int64_t k_token_stride, k_head_stride;
  const void* v; int64_t v_token_stride, v_head_stride; /* only read when storing */
  /* outputs: contiguous [tokens, num_heads, head_dim], [tokens, num_kv_heads, head_dim];
     k_out may be NULL when storing: rotated k then goes to the key cache only
     (decode and chunked-prefill attention read k from the cache) */
  void* q_out;
  void* k_out;
  /* per-head RMSNorm (0 = off) */
  int32_t norm;
  int32_t weight_dtype;
  const void* q_weight;
  const void* k_weight;
  float eps;
  /* rotary */
  int32_t rope_mode;   /* nib_rope_mode */
  const int64_t* positions; /* TABLE: [tokens]; MROPE: [3, tokens] */
  int64_t positions_axis_stride, positions_token_stride;
  const float* cos_sin_table; int64_t table_rows; /* TABLE: [table_rows, head_dim] fp32 */
  const float* inv_freq;                          /* MROPE: [head_dim/2] fp32 */
  int32_t sections[3];
  /* paged store (NULL key_cache = off): flat slot s of a cache holds
     num_kv_heads*head_dim elements at cache + s*cache_slot_stride */
  void* key_cache;
  void* value_cache;
  const int32_t* slot_mapping; /* [tokens], -1 = skip */
  int64_t num_slots, cache_slot_stride;
  unsigned int* status;
  /* 0 = choose automatically (rotary alone, no norm and no store: a warp-per-token
     rotary kernel; otherwise one of the two below); 1 = register-staged kernel (any
     strides); 2 = bulk-copy pipelined kernel (q/k/v consecutive head ranges of one row) */
  int32_t variant;
} nib_qk_prologue_args;

/* Per token: optional per-head RMSNorm of q and k, rotary embedding of the
 * normalised q and k, rotated q/k written to q_out/k_out, and (when
 * key_cache != NULL and slot >= 0) rotated k and raw v written to the paged
 * caches. head_dim must be 64, 128 or 256. All kernel variants compute
 * bit-identical results.
 * Replaces, fused, the sequence
 *   q_norm / k_norm        nanovllm/models/qwen3.py:82-84, qwen3_vl.py:170-171
 *   RotaryEmbedding.forward  nanovllm/layers/rotary_embedding.py:37-48
 *   MultimodalRotaryEmbedding.forward  nanovllm/layers/multimodal_rotary_embedding.py:103-117
 *   store_kvcache / PagedKVBackend.store  nanovllm/layers/attention.py:10-33,87-93
 * Each stage is also reachable alone (norm = 0, rope_mode = NONE, key_cache = NULL). */
NIB_API int nib_qk_prologue(const nib_qk_prologue_args* args, void* stream);

/* apply_multimodal_rotary_emb with caller-supplied cos/sin [3, tokens, head_dim]
 * (contiguous, cos_dtype). x: [tokens, heads, head_dim] strided, x_dtype; out
 * contiguous. Any even head_dim. interleaved = 0: fp32 math; 1: arithmetic in
 * the promoted dtype of x and cos, each product and the sum rounded.
 * Replaces: apply_multimodal_rotary_emb  nanovllm/layers/multimodal_rotary_embedding.py:12-45 */
NIB_API int nib_mrope_apply(int x_dtype, const void* x, int64_t x_token_stride, int64_t x_head_stride,
                    int64_t tokens, int64_t heads, int64_t head_dim, int cos_dtype,
                    const void* cos, const void* sin, const int32_t sections[3], int interleaved,
                    void* out, void* stream);

/* cos/sin [3, tokens, head_dim] of positions[axis, t] * inv_freq (fp32 math,
 * rounded to out_dtype), second half of head_dim repeating the first.
 * Replaces: MultimodalRotaryEmbedding.cos_sin  nanovllm/layers/multimodal_rotary_embedding.py:89-101 */
NIB_API int nib_mrope_cos_sin(const int64_t* positions, int64_t positions_axis_stride,
                      int64_t positions_token_stride, int64_t tokens, const float* inv_freq,
                      int64_t head_dim, int out_dtype, void* cos, void* sin, void* stream);

/* ------------------------------------------------------------------ paged KV */

/* For token t with slot = slot_mapping[t] >= 0: copy row_elems elements of
 * key[t] / value[t] to key_cache / value_cache at slot*cache_slot_stride.
 * slot == -1 skips the token; every other slot keeps its bytes.
 * Replaces: nanovllm_paged_kv::store   csrc/paged_kv/paged_kv.cpp:199-201,
 *           store_kernel/store_cuda    csrc/paged_kv/paged_kv_cuda.cu:21-59,96-131 */
NIB_API int nib_paged_store(int dtype, const void* key, int64_t key_token_stride, const void* value,
                    int64_t value_token_stride, int64_t tokens, int64_t row_elems,
                    void* key_cache, void* value_cache, int64_t cache_slot_stride,
                    int64_t num_slots, const int32_t* slot_mapping, unsigned int* status,
                    void* stream);

/* out[t] = cache[block_table[t / block_size]][t % block_size] for
 * t < sequence_length; out contiguous [sequence_length, row_elems].
 * cache row (block b, offset o) at b*block_stride + o*slot_stride.
 * Replaces: nanovllm_paged_kv::gather  csrc/paged_kv/paged_kv.cpp:202,
 *           gather_kernel/gather_cuda  csrc/paged_kv/paged_kv_cuda.cu:61-94,133-164 */
NIB_API int nib_paged_gather(int dtype, const void* cache, int64_t block_stride, int64_t slot_stride,
                     int64_t num_blocks, int64_t block_size, int64_t row_elems,
                     const int32_t* block_table, int64_t sequence_length, void* out,
                     unsigned int* status, void* stream);

/* Many sequences in one launch: sequence s (s < num_seqs) gathers seq_lens[s]
 * rows through block_tables[s, :] (row stride table_stride) into
 * out[cu_seqlens[s] : cu_seqlens[s] + seq_lens[s]]. max_seq_len bounds the grid.
 * Replaces the per-request loop of SDPAAttention._gather_cache
 * nanovllm/layers/attention.py:206-216,285-292. */
NIB_API int nib_paged_gather_varlen(int dtype, const void* cache, int64_t block_stride,
                            int64_t slot_stride, int64_t num_blocks, int64_t block_size,
                            int64_t row_elems, const int32_t* block_tables, int64_t table_stride,
                            const int32_t* seq_lens, const int64_t* cu_seqlens, int64_t num_seqs,
                            int64_t max_seq_len, void* out, unsigned int* status, void* stream);

/* Same gather as nib_paged_gather_varlen, for callers that cannot allocate
 * device memory: hosts whose memory planner reserves the GPU up front and hands
 * a library only the buffers it asked for, or runtimes that forbid allocation
 * on the serving path because cudaMalloc/cudaFree synchronise the device. The
 * per-sequence output offsets that nib_paged_gather_varlen takes from its
 * caller (cu_seqlens) are computed here, from seq_lens, into a fixed device
 * array that is part of this library: every GPU that loads the library holds
 * NIB_NOALLOC_MAX_SEQS + 1 int64 offsets (32 KiB) until the process exits.
 * No counterpart in the reference (it always has PyTorch allocate).
 * - num_seqs above NIB_NOALLOC_MAX_SEQS is rejected with NIB_ERR_INVALID.
 * - The first call on a device looks the array up (cudaGetSymbolAddress) with
 *   that device current; make that first call before any stream capture. The
 *   address is kept per device together with the id of the CUDA context it
 *   belongs to; after cudaDeviceReset the next call (again outside a capture)
 *   sees the new context and looks the array up again.
 * - All calls on a device share the one array and each call rewrites it:
 *   calls whose kernels overlap on the GPU (different streams without ordering)
 *   race on it. Order them, e.g. issue them on one stream.
 * out receives sum(max(seq_lens[s], 0)) rows, sequence after sequence. */
#define NIB_NOALLOC_MAX_SEQS 4096
NIB_API int nib_paged_gather_varlen_noalloc(int dtype, const void* cache, int64_t block_stride,
                                            int64_t slot_stride, int64_t num_blocks, int64_t block_size,
                                            int64_t row_elems, const int32_t* block_tables,
                                            int64_t table_stride, const int32_t* seq_lens,
                                            int64_t num_seqs, int64_t max_seq_len, void* out,
                                            unsigned int* status, void* stream);

/* ------------------------------------------------------------------ rows */

/* out[i] = weight[ids[i] - vocab_start] when vocab_start <= ids[i] < vocab_end,
 * else a row of zeros (the tensor-parallel mask; ids outside [0, vocab) at
 * tp = 1 also set NIB_DEV_BAD_INDEX). weight row stride in elements; out
 * contiguous [n_ids, hidden].
 * Replaces: VocabParallelEmbedding.forward  nanovllm/layers/embed_head.py:34-42 */
NIB_API int nib_embedding(int dtype, const int64_t* ids, int64_t n_ids, const void* weight,
                  int64_t weight_row_stride, int64_t vocab_rows, int64_t vocab_start,
                  int64_t vocab_end, int64_t hidden, int mask_out_of_range, void* out,
                  unsigned int* status, void* stream);

/* In place: hidden[rows[j]] = hidden[rows[j]] + vis[j] (dtype add, one
 * rounding), j < n_rows; rows must be distinct and inside [0, tokens).
 * Replaces (in place): Qwen3VLLanguageModel._add_deepstack_rows
 * nanovllm/models/qwen3_vl.py:332-344 */
NIB_API int nib_deepstack_add(int dtype, void* hidden, int64_t hidden_row_stride, int64_t tokens,
                      int64_t n, const int64_t* rows, int64_t n_rows, const void* vis,
                      int64_t vis_row_stride, unsigned int* status, void* stream);

/* index[t] = j for t = rows[j] (j < n_rows), -1 for every other t < tokens:
 * the token -> visual-row map nib_add_rms_norm_deepstack reads. rows are the
 * sorted distinct visual token rows of _add_deepstack_rows; a row outside
 * [0, tokens) sets NIB_DEV_BAD_INDEX in *status (when given) and is skipped.
 * Two launches (fill, scatter) on `stream`; no allocation, no synchronisation.
 * Replaces: the row selection of _add_deepstack_rows
 * nanovllm/models/qwen3_vl.py:332-344 (built once per forward, used by the
 * three DeepStack layers) */
NIB_API int nib_deepstack_row_index(const int64_t* rows, int64_t n_rows, int64_t tokens,
                            int32_t* index, unsigned int* status, void* stream);

/* out[r] = in[r] for r < rows (n elements per row): the out-of-place half of
 * _add_deepstack_rows (the clone at nanovllm/models/qwen3_vl.py:342). */
NIB_API int nib_copy_rows(int dtype, const void* in, int64_t in_row_stride, int64_t rows, int64_t n,
                  void* out, int64_t out_row_stride, void* stream);

/* ------------------------------------------------------------------ diagnostics */

/* Status bit a kernel ORs into *status when one of its bounded bulk-copy
 * waits (an mbarrier phase) gave up: the warp then waited, again bounded, for
 * its other copies in flight and returned; its rows were not written. */
#define NIB_DEV_TIMEOUT 16u

/* Makes the library's bounded bulk-copy wait run out on purpose and returns:
 * one warp arms an mbarrier for 32 bytes, lets a bulk copy bring 16 of them
 * from src, waits at most limit_ns (1 us .. 2 s) of wall time, then sets
 * NIB_DEV_TIMEOUT in *status, waits for its second (complete) 16-byte copy
 * from src + 16 and writes *drained = 1 when that copy landed. This is the
 * control flow of the pipelined attention prologue after a wait that gave up.
 * src: 32 readable, 16-byte-aligned device bytes; status, drained: device words.
 * No counterpart in the reference (it has no bounded device waits). */
NIB_API int nib_selftest_bounded_wait(const void* src, int64_t limit_ns, unsigned int* status,
                                      int* drained, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* NIB_B200_H */
