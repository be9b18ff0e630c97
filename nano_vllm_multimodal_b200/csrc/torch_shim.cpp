// Thin PyTorch binding over the C ABI (libnib_b200.so).
//
// Registers
//  * the reference's own paged-KV interface, unchanged, so
//    nanovllm/layers/paged_kv/cuda_backend.py keeps working:
//      nanovllm_paged_kv::store / ::gather      (csrc/paged_kv/paged_kv.cpp:199-203)
//      torch.classes.nanovllm_paged_kv.PagedKVCache (csrc/paged_kv/paged_kv.cpp:41-197)
//  * the rest of the hot path under nanoinfer_b200::*.
// Only the CUDA dispatch key is implemented: CPU tensors raise, there is no
// fallback. Outputs are allocated with at::empty on the input's device (the
// caching allocator, so every op stays CUDA-graph capturable); the kernels
// run on the current stream.
#include <ATen/ATen.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <cuda_runtime_api.h>
#include <torch/custom_class.h>
#include <torch/library.h>

#include <algorithm>
#include <array>
#include <cstring>
#include <functional>
#include <limits>
#include <string>
#include <vector>

#include "nib_b200.h"

namespace nib_torch {

using at::Tensor;
using c10::optional;

int code_of(at::ScalarType t) {
  switch (t) {
    case at::kFloat: return NIB_F32;
    case at::kHalf: return NIB_F16;
    case at::kBFloat16: return NIB_BF16;
    default: TORCH_CHECK(false, "nanoinfer_b200: unsupported dtype ", t);
  }
  return -1;
}

void* stream_of(const Tensor& t) {
  return c10::cuda::getCurrentCUDAStream(t.device().index()).stream();
}

void check(int rc, const char* what) {
  TORCH_CHECK(rc == NIB_OK, what, " failed (status ", rc, "): ", nib_last_error());
}

unsigned int* status_ptr(const optional<Tensor>& s) {
  if (!s.has_value()) return nullptr;
  TORCH_CHECK(s->is_cuda() && s->scalar_type() == at::kInt && s->numel() >= 1,
              "status must be a CUDA int32 tensor");
  return reinterpret_cast<unsigned int*>(s->data_ptr());
}

// Every tensor handed to a kernel must live on the launching device: a host or
// foreign-device pointer would be dereferenced by the GPU.
void on_device(const Tensor& ref, const Tensor& t, const char* what) {
  TORCH_CHECK(t.is_cuda() && t.device() == ref.device(), what, " must be on ", ref.device(),
              " (got ", t.device(), ")");
}

#define NIB_CUDA_CHECK(expr)                                                         \
  do {                                                                               \
    const cudaError_t err_ = (expr);                                                 \
    TORCH_CHECK(err_ == cudaSuccess, #expr, " failed with CUDA error ",              \
                static_cast<int>(err_), ": ", cudaGetErrorString(err_));             \
  } while (false)

// ------------------------------------------------------------------ norms

// x: [..., n] with a contiguous last dim. 2-D and 3-D inputs keep their
// strides (the q/k views of a fused qkv row); other ranks must be viewable as
// [-1, n].
Tensor rms_norm(const Tensor& x, const Tensor& weight, double eps) {
  TORCH_CHECK(x.dim() >= 1 && x.stride(-1) == 1, "rms_norm: last dim must be contiguous");
  const int64_t n = x.size(-1);
  TORCH_CHECK(weight.numel() == n, "rms_norm: weight has ", weight.numel(), " elements, expected ", n);
  on_device(x, weight, "rms_norm weight");
  c10::cuda::CUDAGuard guard(x.device());
  Tensor out = at::empty(x.sizes(), x.options().memory_format(at::MemoryFormat::Contiguous));
  if (x.numel() == 0) return out;
  int64_t tokens, heads, ts, hs;
  const void* xp = x.data_ptr();
  if (x.dim() == 3) {
    tokens = x.size(0); heads = x.size(1); ts = x.stride(0); hs = x.stride(1);
  } else if (x.dim() == 2) {
    tokens = x.size(0); heads = 1; ts = x.stride(0); hs = 0;
  } else {
    TORCH_CHECK(x.is_contiguous(), "rms_norm: inputs of rank ", x.dim(), " must be contiguous");
    tokens = x.numel() / n; heads = 1; ts = n; hs = 0;
  }
  Tensor w = weight.contiguous();
  check(nib_rms_norm(code_of(x.scalar_type()), xp, ts, hs, tokens, heads, n,
                     code_of(w.scalar_type()), w.data_ptr(), static_cast<float>(eps),
                     out.data_ptr(), stream_of(x)),
        "nanoinfer_b200::rms_norm");
  return out;
}

std::tuple<Tensor, Tensor> add_rms_norm(const Tensor& x, const Tensor& residual,
                                        const Tensor& weight, double eps, bool round_sum) {
  TORCH_CHECK(x.sizes() == residual.sizes(), "add_rms_norm: x and residual shapes differ");
  TORCH_CHECK(x.scalar_type() == residual.scalar_type(), "add_rms_norm: x and residual dtypes differ");
  TORCH_CHECK(x.dim() >= 1 && x.stride(-1) == 1 && residual.stride(-1) == 1,
              "add_rms_norm: last dim must be contiguous");
  const int64_t n = x.size(-1);
  TORCH_CHECK(weight.numel() == n, "add_rms_norm: weight size mismatch");
  on_device(x, residual, "add_rms_norm residual");
  on_device(x, weight, "add_rms_norm weight");
  c10::cuda::CUDAGuard guard(x.device());
  Tensor y = at::empty(x.sizes(), x.options().memory_format(at::MemoryFormat::Contiguous));
  Tensor r = at::empty(x.sizes(), x.options().memory_format(at::MemoryFormat::Contiguous));
  if (x.numel() == 0) return {y, r};
  Tensor xx = x.dim() == 2 ? x : x.contiguous().view({-1, n});
  Tensor rr = residual.dim() == 2 ? residual : residual.contiguous().view({-1, n});
  Tensor w = weight.contiguous();
  check(nib_add_rms_norm(code_of(x.scalar_type()), xx.data_ptr(), xx.stride(0), rr.data_ptr(),
                         rr.stride(0), xx.size(0), n, code_of(w.scalar_type()), w.data_ptr(),
                         static_cast<float>(eps), round_sum ? 1 : 0, y.data_ptr(), r.data_ptr(),
                         stream_of(x)),
        "nanoinfer_b200::add_rms_norm");
  return {y, r};
}

// ------------------------------------------------------------------ activation

Tensor silu_and_mul(const Tensor& x) {
  TORCH_CHECK(x.dim() >= 1 && x.size(-1) % 2 == 0, "silu_and_mul: last dim must be even");
  TORCH_CHECK(x.stride(-1) == 1, "silu_and_mul: last dim must be contiguous");
  const int64_t inter = x.size(-1) / 2;
  std::vector<int64_t> osz(x.sizes().begin(), x.sizes().end());
  osz.back() = inter;
  c10::cuda::CUDAGuard guard(x.device());
  Tensor y = at::empty(osz, x.options().memory_format(at::MemoryFormat::Contiguous));
  if (y.numel() == 0) return y;
  Tensor xx = x.dim() == 2 ? x : x.contiguous().view({-1, 2 * inter});
  check(nib_silu_and_mul(code_of(x.scalar_type()), xx.data_ptr(), xx.stride(0), xx.size(0), inter,
                         y.data_ptr(), stream_of(x)),
        "nanoinfer_b200::silu_and_mul");
  return y;
}

// ------------------------------------------------------------------ attention prologue

std::tuple<Tensor, Tensor> qk_prologue(const Tensor& q, const Tensor& k, const optional<Tensor>& v,
                                       const optional<Tensor>& positions,
                                       const optional<Tensor>& q_weight,
                                       const optional<Tensor>& k_weight, double eps,
                                       int64_t rope_mode, const optional<Tensor>& cos_sin_table,
                                       const optional<Tensor>& inv_freq, at::IntArrayRef sections,
                                       const optional<Tensor>& key_cache,
                                       const optional<Tensor>& value_cache,
                                       const optional<Tensor>& slot_mapping,
                                       const optional<Tensor>& status, int64_t variant, bool emit_k) {
  TORCH_CHECK(q.dim() == 3 && k.dim() == 3, "qk_prologue: q and k must be [tokens, heads, head_dim]");
  TORCH_CHECK(q.size(0) == k.size(0) && q.size(2) == k.size(2), "qk_prologue: q/k shape mismatch");
  TORCH_CHECK(q.scalar_type() == k.scalar_type(), "qk_prologue: q and k dtypes differ");
  TORCH_CHECK(q.stride(2) == 1 && k.stride(2) == 1, "qk_prologue: head_dim must be contiguous");
  on_device(q, k, "qk_prologue key");
  for (const auto* t : {&v, &positions, &q_weight, &k_weight, &cos_sin_table, &inv_freq, &key_cache,
                        &value_cache, &slot_mapping, &status})
    if (t->has_value()) on_device(q, **t, "qk_prologue argument");
  c10::cuda::CUDAGuard guard(q.device());
  Tensor qo = at::empty(q.sizes(), q.options().memory_format(at::MemoryFormat::Contiguous));
  TORCH_CHECK(emit_k || key_cache.has_value(), "qk_prologue: emit_k=False needs the caches (rotated k goes only there)");
  // emit_k=False: rotated k is written to the key cache only (decode and
  // chunked prefill read k from the cache); the second result is then empty
  Tensor ko = emit_k ? at::empty(k.sizes(), k.options().memory_format(at::MemoryFormat::Contiguous))
                     : at::empty({0}, k.options());
  if (q.size(0) == 0) return {qo, ko};
  nib_qk_prologue_args a{};
  a.struct_size = sizeof(nib_qk_prologue_args);
  a.dtype = code_of(q.scalar_type());
  a.tokens = q.size(0);
  a.num_heads = static_cast<int32_t>(q.size(1));
  a.num_kv_heads = static_cast<int32_t>(k.size(1));
  a.head_dim = static_cast<int32_t>(q.size(2));
  a.q = q.data_ptr(); a.q_token_stride = q.stride(0); a.q_head_stride = q.stride(1);
  a.k = k.data_ptr(); a.k_token_stride = k.stride(0); a.k_head_stride = k.stride(1);
  a.q_out = qo.data_ptr();
  a.k_out = emit_k ? ko.data_ptr() : nullptr;
  Tensor qw, kw;
  if (q_weight.has_value()) {
    TORCH_CHECK(k_weight.has_value(), "qk_prologue: q_weight without k_weight");
    qw = q_weight->contiguous();
    kw = k_weight->contiguous();
    TORCH_CHECK(qw.scalar_type() == kw.scalar_type(), "qk_prologue: q/k weight dtypes differ");
    TORCH_CHECK(qw.numel() == a.head_dim && kw.numel() == a.head_dim, "qk_prologue: norm weight size");
    a.norm = 1;
    a.weight_dtype = code_of(qw.scalar_type());
    a.q_weight = qw.data_ptr();
    a.k_weight = kw.data_ptr();
    a.eps = static_cast<float>(eps);
  }
  a.rope_mode = static_cast<int32_t>(rope_mode);
  Tensor table, inv;
  if (rope_mode != NIB_ROPE_NONE) {
    TORCH_CHECK(positions.has_value(), "qk_prologue: rope needs positions");
    const Tensor& p = *positions;
    TORCH_CHECK(p.scalar_type() == at::kLong, "qk_prologue: positions must be int64");
    a.positions = p.data_ptr<int64_t>();
    if (rope_mode == NIB_ROPE_TABLE) {
      TORCH_CHECK(p.dim() == 1 && p.size(0) == a.tokens, "qk_prologue: positions must be [tokens]");
      a.positions_token_stride = p.stride(0);
      TORCH_CHECK(cos_sin_table.has_value(), "qk_prologue: table rope needs cos_sin_cache");
      table = cos_sin_table->contiguous();
      TORCH_CHECK(table.scalar_type() == at::kFloat && table.numel() % a.head_dim == 0,
                  "qk_prologue: cos_sin_cache must be float32 [max_position, 1, head_dim]");
      a.cos_sin_table = table.data_ptr<float>();
      a.table_rows = table.numel() / a.head_dim;
    } else {
      TORCH_CHECK(p.dim() == 2 && p.size(0) == 3 && p.size(1) == a.tokens,
                  "qk_prologue: positions must be [3, tokens]");
      a.positions_axis_stride = p.stride(0);
      a.positions_token_stride = p.stride(1);
      TORCH_CHECK(inv_freq.has_value() && sections.size() == 3, "qk_prologue: M-RoPE needs inv_freq and 3 sections");
      inv = inv_freq->contiguous();
      TORCH_CHECK(inv.scalar_type() == at::kFloat && inv.numel() == a.head_dim / 2,
                  "qk_prologue: inv_freq must be float32 [head_dim/2]");
      a.inv_freq = inv.data_ptr<float>();
      for (int i = 0; i < 3; ++i) a.sections[i] = static_cast<int32_t>(sections[i]);
    }
  }
  if (key_cache.has_value()) {
    TORCH_CHECK(value_cache.has_value() && slot_mapping.has_value() && v.has_value(),
                "qk_prologue: store needs v, value_cache and slot_mapping");
    const Tensor& kc = *key_cache;
    const Tensor& vc = *value_cache;
    const Tensor& vv = *v;
    const Tensor& sm = *slot_mapping;
    TORCH_CHECK(kc.is_contiguous() && vc.is_contiguous() && kc.sizes() == vc.sizes() && kc.dim() == 4,
                "qk_prologue: caches must be contiguous [blocks, block_size, kv_heads, head_dim]");
    TORCH_CHECK(kc.size(2) == a.num_kv_heads && kc.size(3) == a.head_dim, "qk_prologue: cache shape");
    TORCH_CHECK(kc.scalar_type() == q.scalar_type() && vc.scalar_type() == q.scalar_type() &&
                    vv.scalar_type() == q.scalar_type(), "qk_prologue: cache/value dtype mismatch");
    TORCH_CHECK(vv.dim() == 3 && vv.sizes() == k.sizes() && vv.stride(2) == 1, "qk_prologue: v shape");
    TORCH_CHECK(sm.scalar_type() == at::kInt && sm.dim() == 1 && sm.is_contiguous() &&
                    sm.size(0) == a.tokens, "qk_prologue: slot_mapping must be contiguous int32 [tokens]");
    a.v = vv.data_ptr(); a.v_token_stride = vv.stride(0); a.v_head_stride = vv.stride(1);
    a.key_cache = kc.data_ptr();
    a.value_cache = vc.data_ptr();
    a.slot_mapping = sm.data_ptr<int32_t>();
    a.num_slots = kc.size(0) * kc.size(1);
    a.cache_slot_stride = kc.stride(1);
  }
  a.status = status_ptr(status);
  a.variant = static_cast<int32_t>(variant);
  check(nib_qk_prologue(&a, stream_of(q)), "nanoinfer_b200::qk_prologue");
  return {qo, ko};
}

Tensor mrope_apply(const Tensor& x, const Tensor& cos, const Tensor& sin, at::IntArrayRef sections,
                   bool interleaved) {
  TORCH_CHECK(x.dim() == 3 && x.stride(2) == 1, "mrope_apply: x must be [tokens, heads, head_dim]");
  TORCH_CHECK(sections.size() == 3, "mrope_apply: three sections");
  on_device(x, cos, "mrope_apply cos");
  on_device(x, sin, "mrope_apply sin");
  TORCH_CHECK(cos.dim() == 3 && cos.size(0) == 3 && cos.size(1) == x.size(0) && cos.size(2) == x.size(2) &&
                  sin.sizes() == cos.sizes(), "mrope_apply: cos/sin must be [3, tokens, head_dim]");
  c10::cuda::CUDAGuard guard(x.device());
  Tensor out = at::empty(x.sizes(), x.options().memory_format(at::MemoryFormat::Contiguous));
  if (x.numel() == 0) return out;
  Tensor c = cos.contiguous(), s = sin.to(cos.scalar_type()).contiguous();
  int32_t sec[3] = {static_cast<int32_t>(sections[0]), static_cast<int32_t>(sections[1]),
                    static_cast<int32_t>(sections[2])};
  check(nib_mrope_apply(code_of(x.scalar_type()), x.data_ptr(), x.stride(0), x.stride(1), x.size(0),
                        x.size(1), x.size(2), code_of(c.scalar_type()), c.data_ptr(), s.data_ptr(),
                        sec, interleaved ? 1 : 0, out.data_ptr(), stream_of(x)),
        "nanoinfer_b200::mrope_apply");
  return out;
}

std::tuple<Tensor, Tensor> mrope_cos_sin(const Tensor& positions, const Tensor& inv_freq,
                                         at::ScalarType dtype) {
  TORCH_CHECK(positions.dim() == 2 && positions.size(0) == 3 && positions.scalar_type() == at::kLong,
              "mrope_cos_sin: positions must be int64 [3, tokens]");
  on_device(positions, inv_freq, "mrope_cos_sin inv_freq");
  Tensor inv = inv_freq.contiguous();
  TORCH_CHECK(inv.scalar_type() == at::kFloat, "mrope_cos_sin: inv_freq must be float32");
  c10::cuda::CUDAGuard guard(positions.device());
  const int64_t T = positions.size(1), D = inv.numel() * 2;
  Tensor c = at::empty({3, T, D}, positions.options().dtype(dtype));
  Tensor s = at::empty({3, T, D}, positions.options().dtype(dtype));
  if (T == 0) return {c, s};
  check(nib_mrope_cos_sin(positions.data_ptr<int64_t>(), positions.stride(0), positions.stride(1), T,
                          inv.data_ptr<float>(), D, code_of(dtype), c.data_ptr(), s.data_ptr(),
                          stream_of(positions)),
        "nanoinfer_b200::mrope_cos_sin");
  return {c, s};
}

// ------------------------------------------------------------------ paged KV

void paged_store(const Tensor& key, const Tensor& value, Tensor key_cache, Tensor value_cache,
                 const Tensor& slot_mapping) {
  TORCH_CHECK(key.is_cuda() && value.is_cuda() && key_cache.is_cuda() && value_cache.is_cuda() &&
                  slot_mapping.is_cuda(),
              "Paged KV CUDA Store requires CUDA tensors");
  TORCH_CHECK(key.scalar_type() == value.scalar_type() &&
                  key.scalar_type() == key_cache.scalar_type() &&
                  key.scalar_type() == value_cache.scalar_type(),
              "Paged KV CUDA Store dtype mismatch");
  TORCH_CHECK(key.dim() == 3 && value.dim() == 3 && key.sizes() == value.sizes(),
              "Paged KV CUDA Store: key/value must be [tokens, kv_heads, head_dim]");
  TORCH_CHECK(key.stride(2) == 1 && value.stride(2) == 1 && key.stride(1) == key.size(2) &&
                  value.stride(1) == value.size(2),
              "Paged KV CUDA Store: each token's [kv_heads, head_dim] must be contiguous");
  TORCH_CHECK(key_cache.dim() == 4 && key_cache.sizes() == value_cache.sizes(),
              "Paged KV CUDA Store: cache shape");
  TORCH_CHECK(key_cache.is_contiguous() && value_cache.is_contiguous(),
              "Paged KV CUDA Store: caches must be contiguous");
  TORCH_CHECK(slot_mapping.scalar_type() == at::kInt && slot_mapping.is_contiguous(),
              "Paged KV CUDA Store: slot_mapping must be contiguous int32");
  for (const Tensor* t : std::initializer_list<const Tensor*>{&value, &key_cache, &value_cache, &slot_mapping}) on_device(key, *t, "Paged KV CUDA Store tensor");
  TORCH_CHECK(slot_mapping.dim() == 1 && slot_mapping.size(0) == key.size(0),
              "Paged KV CUDA Store: slot_mapping length must equal the number of tokens");
  const int64_t tokens = key.size(0);
  if (tokens == 0) return;
  c10::cuda::CUDAGuard guard(key.device());
  const int64_t row = key.size(1) * key.size(2);
  TORCH_CHECK(key_cache.size(2) * key_cache.size(3) == row, "Paged KV CUDA Store: cache row size");
  check(nib_paged_store(code_of(key.scalar_type()), key.data_ptr(), key.stride(0), value.data_ptr(),
                        value.stride(0), tokens, row, key_cache.data_ptr(), value_cache.data_ptr(),
                        key_cache.stride(1), key_cache.size(0) * key_cache.size(1),
                        slot_mapping.data_ptr<int32_t>(), nullptr, stream_of(key)),
        "nanovllm_paged_kv::store");
}

Tensor paged_gather(const Tensor& cache, const Tensor& block_table, int64_t sequence_length) {
  TORCH_CHECK(cache.is_cuda() && block_table.is_cuda(), "Paged KV CUDA Gather requires CUDA tensors");
  TORCH_CHECK(cache.dim() == 4, "Paged KV CUDA Gather: cache must be [blocks, block, kv_heads, head_dim]");
  TORCH_CHECK(cache.stride(3) == 1 && cache.stride(2) == cache.size(3),
              "Paged KV CUDA Gather: each slot's [kv_heads, head_dim] must be contiguous");
  TORCH_CHECK(block_table.scalar_type() == at::kInt && block_table.is_contiguous(),
              "Paged KV CUDA Gather: block_table must be contiguous int32");
  TORCH_CHECK(sequence_length >= 0, "Paged KV CUDA Gather: negative sequence length");
  on_device(cache, block_table, "Paged KV CUDA Gather block_table");
  TORCH_CHECK(block_table.numel() * cache.size(1) >= sequence_length,
              "Paged KV CUDA Gather: block_table does not cover the requested sequence length");
  c10::cuda::CUDAGuard guard(cache.device());
  Tensor out = at::empty({sequence_length, cache.size(2), cache.size(3)}, cache.options());
  if (sequence_length == 0) return out;
  check(nib_paged_gather(code_of(cache.scalar_type()), cache.data_ptr(), cache.stride(0),
                         cache.stride(1), cache.size(0), cache.size(1), cache.size(2) * cache.size(3),
                         block_table.data_ptr<int32_t>(), sequence_length, out.data_ptr(), nullptr,
                         stream_of(cache)),
        "nanovllm_paged_kv::gather");
  return out;
}

Tensor paged_gather_varlen(const Tensor& cache, const Tensor& block_tables, const Tensor& seq_lens,
                           const Tensor& cu_seqlens, int64_t total_tokens, int64_t max_seq_len,
                           const optional<Tensor>& status) {
  TORCH_CHECK(cache.dim() == 4 && cache.stride(3) == 1 && cache.stride(2) == cache.size(3),
              "paged_gather_varlen: cache must be [blocks, block, kv_heads, head_dim] with contiguous slots");
  TORCH_CHECK(block_tables.dim() == 2 && block_tables.scalar_type() == at::kInt && block_tables.stride(1) == 1,
              "paged_gather_varlen: block_tables must be int32 [num_seqs, max_blocks]");
  TORCH_CHECK(seq_lens.scalar_type() == at::kInt && seq_lens.is_contiguous(), "paged_gather_varlen: seq_lens int32");
  TORCH_CHECK(cu_seqlens.scalar_type() == at::kLong && cu_seqlens.is_contiguous(), "paged_gather_varlen: cu_seqlens int64");
  for (const Tensor* t : std::initializer_list<const Tensor*>{&block_tables, &seq_lens, &cu_seqlens}) on_device(cache, *t, "paged_gather_varlen tensor");
  TORCH_CHECK(seq_lens.numel() == block_tables.size(0) && cu_seqlens.numel() >= block_tables.size(0),
              "paged_gather_varlen: one seq_len and one cu_seqlens entry per sequence");
  c10::cuda::CUDAGuard guard(cache.device());
  Tensor out = at::empty({total_tokens, cache.size(2), cache.size(3)}, cache.options());
  if (total_tokens == 0) return out;
  check(nib_paged_gather_varlen(code_of(cache.scalar_type()), cache.data_ptr(), cache.stride(0),
                                cache.stride(1), cache.size(0), cache.size(1),
                                cache.size(2) * cache.size(3), block_tables.data_ptr<int32_t>(),
                                block_tables.stride(0), seq_lens.data_ptr<int32_t>(),
                                cu_seqlens.data_ptr<int64_t>(), block_tables.size(0), max_seq_len,
                                out.data_ptr(), status_ptr(status), stream_of(cache)),
        "nanoinfer_b200::paged_gather_varlen");
  return out;
}

// ------------------------------------------------------------------ rows

Tensor embedding(const Tensor& ids, const Tensor& weight, int64_t vocab_start, int64_t vocab_end,
                 bool mask, const optional<Tensor>& status) {
  TORCH_CHECK(ids.scalar_type() == at::kLong, "embedding: ids must be int64");
  TORCH_CHECK(weight.dim() == 2 && weight.stride(1) == 1, "embedding: weight must be [vocab, hidden]");
  on_device(weight, ids, "embedding ids");
  c10::cuda::CUDAGuard guard(weight.device());
  Tensor idc = ids.contiguous();
  std::vector<int64_t> osz(ids.sizes().begin(), ids.sizes().end());
  osz.push_back(weight.size(1));
  Tensor out = at::empty(osz, weight.options());
  if (idc.numel() == 0) return out;
  check(nib_embedding(code_of(weight.scalar_type()), idc.data_ptr<int64_t>(), idc.numel(),
                      weight.data_ptr(), weight.stride(0), weight.size(0), vocab_start, vocab_end,
                      weight.size(1), mask ? 1 : 0, out.data_ptr(), status_ptr(status),
                      stream_of(weight)),
        "nanoinfer_b200::embedding");
  return out;
}

void deepstack_add_(Tensor hidden, const Tensor& rows, const Tensor& vis, const optional<Tensor>& status) {
  TORCH_CHECK(hidden.dim() == 2 && hidden.stride(1) == 1, "deepstack_add_: hidden must be [tokens, hidden]");
  TORCH_CHECK(rows.scalar_type() == at::kLong && rows.dim() == 1, "deepstack_add_: rows must be int64 [n]");
  TORCH_CHECK(vis.dim() == 2 && vis.size(0) == rows.size(0) && vis.size(1) == hidden.size(1) &&
                  vis.stride(1) == 1 && vis.scalar_type() == hidden.scalar_type(),
              "deepstack_add_: visual embedding must be [n, hidden] of the hidden dtype");
  if (rows.numel() == 0) return;
  on_device(hidden, rows, "deepstack_add_ rows");
  on_device(hidden, vis, "deepstack_add_ visual embedding");
  c10::cuda::CUDAGuard guard(hidden.device());
  Tensor rc = rows.contiguous();
  check(nib_deepstack_add(code_of(hidden.scalar_type()), hidden.data_ptr(), hidden.stride(0),
                          hidden.size(0), hidden.size(1), rc.data_ptr<int64_t>(), rc.numel(),
                          vis.data_ptr(), vis.stride(0), status_ptr(status), stream_of(hidden)),
        "nanoinfer_b200::deepstack_add_");
}

Tensor decode_attention(const Tensor& q, const Tensor& k_cache, const Tensor& v_cache,
                        const Tensor& context_lens, const Tensor& block_tables, double scale,
                        int64_t max_context_len, const optional<Tensor>& status, int64_t variant) {
  TORCH_CHECK(q.dim() == 3 && q.stride(2) == 1, "decode_attention: q must be [batch, heads, head_dim]");
  TORCH_CHECK(k_cache.dim() == 4 && v_cache.sizes() == k_cache.sizes() && k_cache.stride(3) == 1 &&
                  v_cache.strides() == k_cache.strides(),
              "decode_attention: caches must be [blocks, block_size, kv_heads, head_dim] of one layout");
  TORCH_CHECK(q.scalar_type() == k_cache.scalar_type() && v_cache.scalar_type() == q.scalar_type(),
              "decode_attention: q and caches must share a dtype");
  TORCH_CHECK(q.size(2) == k_cache.size(3), "decode_attention: head_dim mismatch");
  TORCH_CHECK(context_lens.scalar_type() == at::kInt && context_lens.dim() == 1 && context_lens.size(0) == q.size(0),
              "decode_attention: context_lens must be int32 [batch]");
  TORCH_CHECK(block_tables.scalar_type() == at::kInt && block_tables.dim() == 2 &&
                  block_tables.size(0) == q.size(0) && block_tables.stride(1) == 1,
              "decode_attention: block_tables must be int32 [batch, max_blocks]");
  on_device(q, k_cache, "decode_attention key cache");
  on_device(q, v_cache, "decode_attention value cache");
  on_device(q, context_lens, "decode_attention context_lens");
  on_device(q, block_tables, "decode_attention block_tables");
  c10::cuda::CUDAGuard guard(q.device());
  Tensor out = at::empty(q.sizes(), q.options().memory_format(at::MemoryFormat::Contiguous));
  if (q.size(0) == 0) return out;
  Tensor lens = context_lens.contiguous();
  nib_decode_attention_args a{};
  a.struct_size = sizeof(a);
  a.dtype = code_of(q.scalar_type());
  a.batch = q.size(0);
  a.num_heads = static_cast<int32_t>(q.size(1));
  a.num_kv_heads = static_cast<int32_t>(k_cache.size(2));
  a.head_dim = static_cast<int32_t>(q.size(2));
  a.q = q.data_ptr();
  a.q_batch_stride = q.stride(0);
  a.q_head_stride = q.stride(1);
  a.key_cache = k_cache.data_ptr();
  a.value_cache = v_cache.data_ptr();
  a.cache_block_stride = k_cache.stride(0);
  a.cache_slot_stride = k_cache.stride(1);
  a.cache_head_stride = k_cache.stride(2);
  a.num_blocks = k_cache.size(0);
  a.block_size = k_cache.size(1);
  a.block_tables = block_tables.data_ptr<int32_t>();
  a.block_table_stride = block_tables.stride(0);
  a.max_blocks_per_seq = block_tables.size(1);
  a.context_lens = lens.data_ptr<int32_t>();
  a.scale = static_cast<float>(scale);
  a.out = out.data_ptr();
  a.out_batch_stride = out.stride(0);
  a.out_head_stride = out.stride(1);
  a.max_context_len = max_context_len;
  a.variant = static_cast<int32_t>(variant);
  a.status = status_ptr(status);
  const int64_t need = nib_decode_attention_workspace_bytes(&a);
  TORCH_CHECK(need >= 0, "decode_attention: unsupported configuration (head_dim ", a.head_dim, ", heads ",
              a.num_heads, "/", a.num_kv_heads, ", dtype ", q.scalar_type(), ")");
  Tensor ws;
  if (need > 0) {
    ws = at::empty({need}, q.options().dtype(at::kByte));
    a.workspace = ws.data_ptr();
    a.workspace_bytes = need;
  }
  check(nib_decode_attention(&a, stream_of(q)), "nanoinfer_b200::decode_attention");
  return out;
}

Tensor deepstack_row_index(const Tensor& rows, int64_t tokens, const optional<Tensor>& status) {
  TORCH_CHECK(rows.scalar_type() == at::kLong && rows.dim() == 1, "deepstack_row_index: rows must be int64 [n]");
  TORCH_CHECK(tokens >= 0, "deepstack_row_index: tokens must be >= 0");
  c10::cuda::CUDAGuard guard(rows.device());
  Tensor index = at::empty({tokens}, rows.options().dtype(at::kInt));
  if (tokens == 0) return index;
  Tensor rc = rows.contiguous();
  check(nib_deepstack_row_index(rc.data_ptr<int64_t>(), rc.numel(), tokens, index.data_ptr<int32_t>(),
                                status_ptr(status), stream_of(rows)),
        "nanoinfer_b200::deepstack_row_index");
  return index;
}

std::tuple<Tensor, Tensor> add_rms_norm_deepstack(const Tensor& x, const Tensor& residual,
                                                  const Tensor& weight, double eps, const Tensor& vis,
                                                  const Tensor& index, const optional<Tensor>& status) {
  TORCH_CHECK(x.dim() == 2 && x.sizes() == residual.sizes(),
              "add_rms_norm_deepstack: x and residual must be [tokens, hidden] of one shape");
  TORCH_CHECK(x.scalar_type() == residual.scalar_type() && vis.scalar_type() == x.scalar_type(),
              "add_rms_norm_deepstack: x, residual and the visual embedding must share a dtype");
  TORCH_CHECK(x.stride(1) == 1 && residual.stride(1) == 1, "add_rms_norm_deepstack: last dim must be contiguous");
  const int64_t n = x.size(1);
  TORCH_CHECK(vis.dim() == 2 && vis.size(1) == n && (vis.size(0) == 0 || vis.stride(1) == 1),
              "add_rms_norm_deepstack: visual embedding must be [rows, hidden]");
  TORCH_CHECK(index.scalar_type() == at::kInt && index.dim() == 1 && index.size(0) == x.size(0),
              "add_rms_norm_deepstack: index must be int32 [tokens]");
  TORCH_CHECK(weight.numel() == n, "add_rms_norm_deepstack: weight size mismatch");
  on_device(x, residual, "add_rms_norm_deepstack residual");
  on_device(x, weight, "add_rms_norm_deepstack weight");
  on_device(x, vis, "add_rms_norm_deepstack visual embedding");
  on_device(x, index, "add_rms_norm_deepstack index");
  c10::cuda::CUDAGuard guard(x.device());
  Tensor y = at::empty(x.sizes(), x.options().memory_format(at::MemoryFormat::Contiguous));
  Tensor r = at::empty(x.sizes(), x.options().memory_format(at::MemoryFormat::Contiguous));
  if (x.numel() == 0) return {y, r};
  Tensor w = weight.contiguous();
  Tensor ic = index.contiguous();
  check(nib_add_rms_norm_deepstack(code_of(x.scalar_type()), x.data_ptr(), x.stride(0), residual.data_ptr(),
                                   residual.stride(0), x.size(0), n, code_of(w.scalar_type()), w.data_ptr(),
                                   static_cast<float>(eps), vis.numel() ? vis.data_ptr() : nullptr,
                                   vis.numel() ? vis.stride(0) : n, vis.size(0), ic.data_ptr<int32_t>(),
                                   y.data_ptr(), r.data_ptr(), status_ptr(status), stream_of(x)),
        "nanoinfer_b200::add_rms_norm_deepstack");
  return {y, r};
}

// plan: int64 [3 * R] on the device (output rows | source index | feature rows);
// table: int64 [K, sizeof(nib_visual_source) / 8] on the device
std::tuple<Tensor, Tensor> visual_merge(const Tensor& tokens, const Tensor& table, int64_t num_layers,
                                        const Tensor& plan, int64_t num_replacements,
                                        const optional<Tensor>& status) {
  TORCH_CHECK(tokens.dim() == 2 && (tokens.size(0) == 0 || tokens.stride(1) == 1),
              "visual_merge: token embeddings must be [tokens, hidden] with a contiguous last dim");
  TORCH_CHECK(table.scalar_type() == at::kLong && table.dim() == 2 &&
                  table.size(1) * 8 == static_cast<int64_t>(sizeof(nib_visual_source)) && table.is_contiguous(),
              "visual_merge: bad source table");
  TORCH_CHECK(plan.scalar_type() == at::kLong && plan.is_contiguous() && plan.numel() >= 3 * num_replacements,
              "visual_merge: bad plan");
  TORCH_CHECK(num_layers >= 0 && num_layers <= NIB_VISUAL_MAX_LAYERS, "visual_merge: too many DeepStack layers");
  on_device(tokens, table, "visual_merge source table");
  on_device(tokens, plan, "visual_merge plan");
  c10::cuda::CUDAGuard guard(tokens.device());
  const int64_t T = tokens.size(0), H = tokens.size(1), R = num_replacements;
  Tensor merged = at::empty({T, H}, tokens.options());
  Tensor ds = at::empty({num_layers, R, H}, tokens.options());
  Tensor row_map = at::empty({T}, tokens.options().dtype(at::kInt));
  const int64_t* pp = plan.data_ptr<int64_t>();
  check(nib_visual_merge(code_of(tokens.scalar_type()), tokens.data_ptr(), T ? tokens.stride(0) : H, T, H,
                         reinterpret_cast<const nib_visual_source*>(table.data_ptr<int64_t>()), table.size(0),
                         static_cast<int>(num_layers), pp, pp + R, pp + 2 * R, R, row_map.data_ptr<int32_t>(),
                         merged.data_ptr(), ds.data_ptr(), status_ptr(status), stream_of(tokens)),
        "nanoinfer_b200::visual_merge");
  return {merged, ds};
}

Tensor deepstack_add(const Tensor& hidden, const Tensor& rows, const Tensor& vis,
                     const optional<Tensor>& status) {
  TORCH_CHECK(hidden.dim() == 2 && hidden.stride(1) == 1, "deepstack_add: hidden must be [tokens, hidden]");
  c10::cuda::CUDAGuard guard(hidden.device());
  Tensor out = at::empty(hidden.sizes(), hidden.options().memory_format(at::MemoryFormat::Contiguous));
  if (hidden.numel() == 0) return out;
  check(nib_copy_rows(code_of(hidden.scalar_type()), hidden.data_ptr(), hidden.stride(0),
                      hidden.size(0), hidden.size(1), out.data_ptr(), out.stride(0), stream_of(hidden)),
        "nanoinfer_b200::deepstack_add (copy)");
  deepstack_add_(out, rows, vis, status);
  return out;
}

// ------------------------------------------------------------------ PagedKVCache

at::ScalarType parse_dtype(const std::string& name) {
  if (name == "float16") return at::kHalf;
  if (name == "bfloat16") return at::kBFloat16;
  if (name == "float32") return at::kFloat;
  TORCH_CHECK(false, "PagedKVCache does not support dtype ", name);
}

// Owns one cudaMalloc'd cache allocation and the device buffer that receives
// each step's slot mapping (the interface of the reference's runtime owner,
// csrc/paged_kv/paged_kv.cpp:41-179: tensor(), copy_slots_async(),
// pending_host_copy_count(); the same checks and messages).
//
// The slot mapping is copied on the caller's current stream. The reference
// copies on a private transfer stream and orders it with two events each step
// (the transfer waits for the compute stream, the compute stream waits for the
// transfer), so nothing overlaps anyway; one copy in stream order gives the
// same ordering with no cross-stream events: the previous step's kernels on
// this stream finish reading the buffer before it is refilled, and this
// step's kernels start after the copy landed.
//
// The pinned source must stay alive until its copy has run. Each call records
// one event of a fixed ring (created once, here in the constructor) behind its
// copy and keeps the source in that ring entry; entries whose event has
// completed are released at the start of the next call. A full ring (the host
// more than kRing steps ahead of the GPU) waits for its oldest copy.
class PagedKVCache : public torch::CustomClassHolder {
 public:
  static constexpr int kRing = 16;

  PagedKVCache(std::vector<int64_t> sizes, std::string dtype_name, int64_t device_index)
      : device_(device_index) {
    TORCH_CHECK(device_ >= 0, "CUDA device index must be non-negative");
    TORCH_CHECK(!sizes.empty(), "PagedKVCache shape must not be empty");
    const at::ScalarType dtype = parse_dtype(dtype_name);
    int64_t numel = 1;
    for (int64_t s : sizes) {
      TORCH_CHECK(s > 0, "PagedKVCache dimensions must be positive");
      TORCH_CHECK(numel <= std::numeric_limits<int64_t>::max() / s, "PagedKVCache shape overflows int64");
      numel *= s;
    }
    c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(device_));
    cache_ = owned_device_tensor(static_cast<size_t>(numel) * c10::elementSize(dtype), sizes, dtype);
    for (Pending& p : ring_) NIB_CUDA_CHECK(cudaEventCreateWithFlags(&p.copied, cudaEventDisableTiming));
  }

  ~PagedKVCache() override {
    c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(device_));
    for (Pending& p : ring_) {
      if (p.source.defined()) cudaEventSynchronize(p.copied);  // a source must outlive its copy
      p.source.reset();
      if (p.copied) cudaEventDestroy(p.copied);
    }
  }

  Tensor tensor() const { return cache_; }

  int64_t pending_host_copy_count() const { return live_; }

  Tensor copy_slots_async(const Tensor& host) {
    TORCH_CHECK(host.device().is_cpu(), "slot mapping source must be a CPU tensor");
    TORCH_CHECK(host.scalar_type() == at::kInt, "slot mapping source must be int32");
    TORCH_CHECK(host.dim() == 1 && host.is_contiguous(), "slot mapping source must be contiguous and one-dimensional");
    c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(device_));
    release_landed();
    const int64_t n = host.numel();
    if (n == 0) return at::empty({0}, at::TensorOptions().dtype(at::kInt).device(at::kCUDA, device_));
    TORCH_CHECK(host.is_pinned(), "slot mapping source must use pinned CPU memory");
    if (slots_.numel() < n) {
      // grown only when a step has more tokens than any before; the old buffer
      // is freed by its deleter once no tensor refers to it
      slots_ = owned_device_tensor(static_cast<size_t>(n) * sizeof(int32_t), {n}, at::kInt);
    }
    Pending& p = ring_[next_];
    if (p.source.defined()) {  // ring full: the oldest copy must land before its entry is reused
      NIB_CUDA_CHECK(cudaEventSynchronize(p.copied));
      p.source.reset();
      --live_;
    }
    const cudaStream_t stream = c10::cuda::getCurrentCUDAStream(static_cast<c10::DeviceIndex>(device_)).stream();
    NIB_CUDA_CHECK(cudaMemcpyAsync(slots_.data_ptr(), host.data_ptr(), static_cast<size_t>(n) * sizeof(int32_t),
                                   cudaMemcpyHostToDevice, stream));
    NIB_CUDA_CHECK(cudaEventRecord(p.copied, stream));
    p.source = host;
    ++live_;
    next_ = (next_ + 1) % kRing;
    return slots_.narrow(0, 0, n);
  }

 private:
  struct Pending {
    Tensor source;            // the pinned host tensor, kept until `copied` completes
    cudaEvent_t copied = nullptr;
  };

  Tensor owned_device_tensor(size_t bytes, at::IntArrayRef sizes, at::ScalarType dtype) const {
    void* p = nullptr;
    NIB_CUDA_CHECK(cudaMalloc(&p, bytes));
    const int64_t dev = device_;
    return at::from_blob(p, sizes, [dev](void* q) {
      if (q == nullptr) return;
      c10::cuda::CUDAGuard g(static_cast<c10::DeviceIndex>(dev));
      cudaFree(q);
    }, at::TensorOptions().dtype(dtype).device(at::kCUDA, device_));
  }

  // release, oldest first, every source whose copy has landed
  void release_landed() {
    for (int i = 0; i < kRing && live_ > 0; ++i) {
      Pending& p = ring_[(next_ + kRing - live_) % kRing];
      const cudaError_t st = cudaEventQuery(p.copied);
      if (st == cudaErrorNotReady) return;
      NIB_CUDA_CHECK(st);
      p.source.reset();
      --live_;
    }
  }

  int64_t device_;
  Tensor cache_;
  Tensor slots_;
  std::array<Pending, kRing> ring_{};
  int next_ = 0;   // ring entry of the next copy
  int live_ = 0;   // entries holding a source: the oldest is next_ - live_
};

// A step's host inputs (token ids, positions, slot mapping, cu_seqlens, ...;
// nanovllm/engine/model_runner.py:700-725,823-870 builds one pinned tensor and
// one copy per array) staged through ONE pinned buffer and ONE host-to-device
// copy: stage() writes every CPU tensor into the next slot of a small ring of
// pinned buffers (16-byte aligned offsets), copies the slot into one fresh
// device allocation on the current stream and returns typed views of it. A
// slot is rewritten only after the copy that last read it has completed (its
// event), so the host can prepare up to `slots` steps ahead.
class StepInputStager : public torch::CustomClassHolder {
 public:
  StepInputStager(int64_t device_index, int64_t slots, int64_t initial_bytes) : device_(device_index) {
    TORCH_CHECK(device_ >= 0, "CUDA device index must be non-negative");
    TORCH_CHECK(slots >= 1 && slots <= 64, "StepInputStager: slots must be in [1, 64]");
    TORCH_CHECK(initial_bytes >= 0, "StepInputStager: initial_bytes must be >= 0");
    c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(device_));
    ring_.resize(static_cast<size_t>(slots));
    for (Slot& s : ring_) {
      NIB_CUDA_CHECK(cudaEventCreateWithFlags(&s.done, cudaEventDisableTiming));
      grow(s, static_cast<size_t>(initial_bytes));
    }
  }

  ~StepInputStager() override {
    c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(device_));
    for (Slot& s : ring_) {
      if (s.pending) cudaEventSynchronize(s.done);
      if (s.host) cudaFreeHost(s.host);
      if (s.done) cudaEventDestroy(s.done);
    }
  }

  std::vector<Tensor> stage(std::vector<Tensor> host) {
    std::vector<size_t> offs;
    size_t total = 0;
    for (const Tensor& t : host) {
      TORCH_CHECK(t.device().is_cpu() && t.is_contiguous(), "StepInputStager: inputs must be contiguous CPU tensors");
      offs.push_back(total);
      total += (t.nbytes() + 15u) / 16u * 16u;
    }
    c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(device_));
    const auto opts = at::TensorOptions().dtype(at::kByte).device(at::kCUDA, device_);
    Tensor dev = at::empty({static_cast<int64_t>(total)}, opts);
    if (total > 0) {
      Slot& s = ring_[next_];
      next_ = (next_ + 1) % ring_.size();
      if (s.pending) {  // the copy that last read this slot must have landed
        NIB_CUDA_CHECK(cudaEventSynchronize(s.done));
        s.pending = false;
      }
      grow(s, total);
      for (size_t i = 0; i < host.size(); ++i)
        if (host[i].nbytes()) std::memcpy(static_cast<char*>(s.host) + offs[i], host[i].data_ptr(), host[i].nbytes());
      cudaStream_t st = c10::cuda::getCurrentCUDAStream(static_cast<c10::DeviceIndex>(device_)).stream();
      NIB_CUDA_CHECK(cudaMemcpyAsync(dev.data_ptr(), s.host, total, cudaMemcpyHostToDevice, st));
      NIB_CUDA_CHECK(cudaEventRecord(s.done, st));
      s.pending = true;
    }
    std::vector<Tensor> out;
    out.reserve(host.size());
    for (size_t i = 0; i < host.size(); ++i) {
      const Tensor& t = host[i];
      Tensor v = dev.narrow(0, static_cast<int64_t>(offs[i]), static_cast<int64_t>(t.nbytes()));
      out.push_back(v.view(t.scalar_type()).view(t.sizes()));
    }
    return out;
  }

  int64_t slots() const { return static_cast<int64_t>(ring_.size()); }
  int64_t slot_bytes(int64_t i) const {
    TORCH_CHECK(i >= 0 && i < slots(), "StepInputStager: slot index out of range");
    return static_cast<int64_t>(ring_[static_cast<size_t>(i)].bytes);
  }

 private:
  struct Slot {
    void* host = nullptr;
    size_t bytes = 0;
    cudaEvent_t done = nullptr;
    bool pending = false;
  };

  static void grow(Slot& s, size_t bytes) {
    if (s.bytes >= bytes) return;
    const size_t want = std::max<size_t>(bytes, 2 * s.bytes);  // amortised growth
    if (s.pending) {
      NIB_CUDA_CHECK(cudaEventSynchronize(s.done));
      s.pending = false;
    }
    if (s.host) NIB_CUDA_CHECK(cudaFreeHost(s.host));
    s.host = nullptr;
    s.bytes = 0;
    NIB_CUDA_CHECK(cudaHostAlloc(&s.host, want, cudaHostAllocDefault));
    s.bytes = want;
  }

  int64_t device_;
  std::vector<Slot> ring_;
  size_t next_ = 0;
};

int64_t abi_version() { return nib_abi_version(); }

}  // namespace nib_torch

static auto step_input_stager_class =
    torch::class_<nib_torch::StepInputStager>("nanoinfer_b200", "StepInputStager")
        .def(torch::init<int64_t, int64_t, int64_t>())
        .def("stage", &nib_torch::StepInputStager::stage)
        .def("slots", &nib_torch::StepInputStager::slots)
        .def("slot_bytes", &nib_torch::StepInputStager::slot_bytes);

static auto paged_kv_cache_class =
    torch::class_<nib_torch::PagedKVCache>("nanovllm_paged_kv", "PagedKVCache")
        .def(torch::init<std::vector<int64_t>, std::string, int64_t>())
        .def("tensor", &nib_torch::PagedKVCache::tensor)
        .def("pending_host_copy_count", &nib_torch::PagedKVCache::pending_host_copy_count)
        .def("copy_slots_async", &nib_torch::PagedKVCache::copy_slots_async);

TORCH_LIBRARY(nanovllm_paged_kv, m) {
  m.def("store(Tensor key, Tensor value, Tensor(a!) key_cache, Tensor(b!) value_cache, "
        "Tensor slot_mapping) -> ()");
  m.def("gather(Tensor cache, Tensor block_table, int sequence_length) -> Tensor");
}

TORCH_LIBRARY_IMPL(nanovllm_paged_kv, CUDA, m) {
  m.impl("store", TORCH_FN(nib_torch::paged_store));
  m.impl("gather", TORCH_FN(nib_torch::paged_gather));
}

TORCH_LIBRARY(nanoinfer_b200, m) {
  m.def("abi_version() -> int", &nib_torch::abi_version);
  m.def("rms_norm(Tensor x, Tensor weight, float eps) -> Tensor");
  m.def("add_rms_norm(Tensor x, Tensor residual, Tensor weight, float eps, bool round_sum) -> (Tensor, Tensor)");
  m.def("silu_and_mul(Tensor x) -> Tensor");
  m.def("qk_prologue(Tensor q, Tensor k, Tensor? v, Tensor? positions, Tensor? q_weight, "
        "Tensor? k_weight, float eps, int rope_mode, Tensor? cos_sin_cache, Tensor? inv_freq, "
        "int[] sections, Tensor(a!)? key_cache, Tensor(b!)? value_cache, Tensor? slot_mapping, "
        "Tensor(c!)? status, int variant=0, bool emit_k=True) -> (Tensor, Tensor)");
  m.def("mrope_apply(Tensor x, Tensor cos, Tensor sin, int[] sections, bool interleaved) -> Tensor");
  m.def("mrope_cos_sin(Tensor positions, Tensor inv_freq, ScalarType dtype) -> (Tensor, Tensor)");
  m.def("paged_gather_varlen(Tensor cache, Tensor block_tables, Tensor seq_lens, Tensor cu_seqlens, "
        "int total_tokens, int max_seq_len, Tensor(a!)? status) -> Tensor");
  m.def("embedding(Tensor ids, Tensor weight, int vocab_start, int vocab_end, bool mask, "
        "Tensor(a!)? status) -> Tensor");
  m.def("deepstack_add(Tensor hidden, Tensor rows, Tensor vis, Tensor(a!)? status) -> Tensor");
  m.def("deepstack_row_index(Tensor rows, int tokens, Tensor(a!)? status) -> Tensor");
  m.def("decode_attention(Tensor q, Tensor k_cache, Tensor v_cache, Tensor context_lens, Tensor block_tables, "
        "float scale, int max_context_len, Tensor(a!)? status, int variant=0) -> Tensor");
  m.def("visual_merge(Tensor tokens, Tensor table, int num_layers, Tensor plan, int num_replacements, "
        "Tensor(a!)? status) -> (Tensor, Tensor)");
  m.def("add_rms_norm_deepstack(Tensor x, Tensor residual, Tensor weight, float eps, Tensor vis, "
        "Tensor index, Tensor(a!)? status) -> (Tensor, Tensor)");
  m.def("deepstack_add_(Tensor(a!) hidden, Tensor rows, Tensor vis, Tensor(b!)? status) -> ()");
}

TORCH_LIBRARY_IMPL(nanoinfer_b200, CUDA, m) {
  m.impl("rms_norm", TORCH_FN(nib_torch::rms_norm));
  m.impl("add_rms_norm", TORCH_FN(nib_torch::add_rms_norm));
  m.impl("silu_and_mul", TORCH_FN(nib_torch::silu_and_mul));
  m.impl("qk_prologue", TORCH_FN(nib_torch::qk_prologue));
  m.impl("mrope_apply", TORCH_FN(nib_torch::mrope_apply));
  m.impl("mrope_cos_sin", TORCH_FN(nib_torch::mrope_cos_sin));
  m.impl("paged_gather_varlen", TORCH_FN(nib_torch::paged_gather_varlen));
  m.impl("embedding", TORCH_FN(nib_torch::embedding));
  m.impl("deepstack_add", TORCH_FN(nib_torch::deepstack_add));
  m.impl("deepstack_add_", TORCH_FN(nib_torch::deepstack_add_));
  m.impl("deepstack_row_index", TORCH_FN(nib_torch::deepstack_row_index));
  m.impl("decode_attention", TORCH_FN(nib_torch::decode_attention));
  m.impl("visual_merge", TORCH_FN(nib_torch::visual_merge));
  m.impl("add_rms_norm_deepstack", TORCH_FN(nib_torch::add_rms_norm_deepstack));
}
