"""CPU restatement of NanoInfer's per-token decoder elementwise path.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``): the checker for the CUDA
kernels, never the product path.

Every floating-point function below spells out the rounding order of the
reference's eager PyTorch code with CPU tensor arithmetic (fp32 math, explicit
bf16/fp16 rounding points). Byte and index work (paged-KV store/gather,
embedding rows, DeepStack row selection) is restated in numpy on integer views
of the tensors, so it is bit-exact by construction. Citations are
``file:line`` inside the NanoInfer project.
"""

from __future__ import annotations

import numpy as np
import torch
import torch.nn.functional as F

__all__ = [
    "add_rms_norm",
    "rms_norm",
    "text_rms_norm",
    "add_text_rms_norm",
    "add_text_rms_norm_deepstack",
    "planned_visual_embeddings",
    "paged_decode_attention",
    "paged_decode_attention_abs",
    "silu_and_mul",
    "silu_and_mul_fp32",
    "rope_cos_sin_cache",
    "apply_rope",
    "mrope_inv_freq",
    "mrope_cos_sin",
    "mrope_select",
    "apply_mrope",
    "mrope_forward",
    "paged_store",
    "paged_store_",
    "paged_gather",
    "embedding",
    "add_deepstack_rows",
    "qk_norm_rope_store",
    "qwen3_vl_fused_layer",
]


def _round(t: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    return t.to(dtype)


# --------------------------------------------------------------------------- norms
#
# ``order`` selects how the fp32 statistics mean(x^2) and 1/sqrt(var + eps) are
# evaluated. "torch" runs the reference's own ops (``x.pow(2).mean()`` and
# ``torch.rsqrt``) as this CPU build executes them. "kernel" evaluates the SAME
# formula with an explicit order: squares rounded to fp32; the squares of each
# 16-byte vector summed as a pairwise tree ((s0+s1)+(s2+s3))+((s4+s5)+(s6+s7));
# a lane adds its vectors' sums in order; lanes combined by an xor butterfly
# (and, for rows longer than 256 vectors, warps summed in order); then IEEE
# ``sum / n``, ``+ eps``, ``sqrt`` and ``1 / .`` - the order the CUDA kernels
# use. Any fp32 summation order is a valid evaluation of ``mean``; fixing one
# makes the kernels checkable bit-for-bit. Everything after the statistics is
# identical.


def _vec_elems(dtype):
    return 16 // torch.empty((), dtype=dtype).element_size()


def _vector_sums(sq, vec):
    """Pairwise-tree sum of the squares inside each 16-byte vector -> [rows, n/vec]."""
    v = sq.reshape(sq.shape[0], -1, vec)
    while v.shape[-1] > 1:
        v = (v[..., 0::2] + v[..., 1::2]).astype(np.float32)
    return v[..., 0]


def _lanes_sumsq(sq, nv, vec, lanes, vpt):
    rows = sq.shape[0]
    vs = _vector_sums(sq, vec)
    acc = np.zeros((rows, lanes), np.float32)
    lane = np.arange(lanes)
    for i in range(vpt):
        vi = i * lanes + lane
        ok = vi < nv
        acc[:, ok] = acc[:, ok] + vs[:, vi[ok]]
    off = lanes // 2
    while off >= 1:
        acc = acc + acc[:, lane ^ off]
        off //= 2
    return acc[:, 0]


def _block_sumsq(sq, nv, vec, threads, vpt=4):
    rows = sq.shape[0]
    vs = _vector_sums(sq, vec)
    acc = np.zeros((rows, threads), np.float32)
    th = np.arange(threads)
    for i in range(vpt):
        vi = i * threads + th
        ok = vi < nv
        acc[:, ok] = acc[:, ok] + vs[:, vi[ok]]
    off = 16
    while off >= 1:
        acc = acc + acc[:, th ^ off]
        off //= 2
    tot = np.zeros(rows, np.float32)
    for w in range(threads // 32):
        tot = tot + acc[:, w * 32]
    return tot


def kernel_sumsq(s32, vec, add):
    """Sum of squares of each row of ``s32`` ([rows, n] fp32 numpy) in the
    kernels' order (``nano_vllm_multimodal_b200/csrc/norm.cu`` launch rules:
    <= 32 vectors and no residual -> a power-of-two group of lanes holding 2
    vectors each (the fused attention prologue uses the same per-head layout);
    <= 256 vectors -> 32 lanes; longer rows -> one CTA, 4 vectors per thread)."""
    rows, n = s32.shape
    nv = n // vec
    sq = (s32 * s32).astype(np.float32)
    if nv <= 32 and not add:
        # short rows (attention heads): a lane owns vectors l and l + lanes, i.e.
        # for a head the two rotate-half partners of the same frequencies
        lanes = 1
        while lanes < -(-nv // 2):
            lanes *= 2
        return _lanes_sumsq(sq, nv, vec, lanes, 2)
    if nv <= 256:
        return _lanes_sumsq(sq, nv, vec, 32, -(-nv // 32))
    threads = -(-(-(-nv // 4)) // 32) * 32
    return _block_sumsq(sq, nv, vec, threads)


def _inv_rms(s, eps, order, dtype, add=False):
    """1/sqrt(mean(s^2) + eps) for fp32 ``s`` [..., n], keepdim."""
    if order == "torch":
        return torch.rsqrt(s.pow(2).mean(dim=-1, keepdim=True) + eps)
    n = s.shape[-1]
    rows = s.reshape(-1, n).contiguous().numpy()
    ss = kernel_sumsq(rows, _vec_elems(dtype), add)
    r = np.float32(1.0) / np.sqrt(ss / np.float32(n) + np.float32(eps))
    return torch.from_numpy(r.astype(np.float32)).reshape(*s.shape[:-1], 1)


def add_rms_norm(x, residual, weight, eps, order="torch"):
    """Fused residual add + RMSNorm.

    Follows ``nanovllm/layers/layernorm.py:28-40`` (``add_rms_forward``): the sum
    is kept in fp32 for the statistics, the new residual is that sum rounded to
    the activation dtype, the normalised value is rounded before the weight
    multiply, and the weight multiply rounds once more (``mul_`` on the
    rounded tensor).
    """
    dtype = x.dtype
    s = x.float() + residual.float()
    res_out = _round(s, dtype)
    n = _round(s * _inv_rms(s, eps, order, dtype, add=True), dtype)
    y = _round(n.float() * weight.float(), dtype)
    return y, res_out


def rms_norm(x, weight, eps, order="torch"):
    """RMSNorm without residual: ``nanovllm/layers/layernorm.py:16-26``.

    Output is a new tensor (``x.float()`` copies), laid out contiguously.
    """
    dtype = x.dtype
    xf = x.float()
    n = _round(xf * _inv_rms(xf, eps, order, dtype), dtype)
    return _round(n.float() * weight.float(), dtype).contiguous()


def text_rms_norm(x, weight, eps, order="torch"):
    """``Qwen3VLTextRMSNorm.forward``: ``nanovllm/models/qwen3_vl.py:74-79``.

    ``weight * normalized.to(input_dtype)``: the product is taken in the
    promoted dtype of the weight and the activation (bf16 x bf16 -> bf16,
    fp32 weight -> fp32 output).
    """
    dtype = x.dtype
    xf = x.float()
    n = _round(xf * _inv_rms(xf, eps, order, dtype), dtype)
    out_dtype = torch.promote_types(weight.dtype, dtype)
    return _round(weight.float() * n.float(), out_dtype).contiguous()


def add_text_rms_norm(x, residual, weight, eps, order="torch"):
    """Qwen3-VL residual add then text RMSNorm.

    ``nanovllm/models/qwen3_vl.py:232-237``: ``hidden_states + residual`` is a
    plain activation-dtype add (one rounding) and the norm then runs on the
    rounded sum, unlike ``add_rms_norm`` which normalises the fp32 sum.
    Returns ``(normed, rounded_sum)``.
    """
    s = _round(x.float() + residual.float(), x.dtype)
    if order == "torch":
        return text_rms_norm(s, weight, eps), s
    sf = s.float()
    n = _round(sf * _inv_rms(sf, eps, order, x.dtype, add=True), x.dtype)
    out_dtype = torch.promote_types(weight.dtype, x.dtype)
    return _round(weight.float() * n.float(), out_dtype).contiguous(), s


# --------------------------------------------------------------------------- activation


def silu_and_mul(x):
    """``SiluAndMul.forward`` as eager PyTorch runs it.

    ``nanovllm/layers/activation.py:8-11``: ``silu`` rounds to the activation
    dtype, the product rounds again.
    """
    gate, up = x.chunk(2, -1)
    return F.silu(gate) * up


def silu_and_mul_fp32(x):
    """Single-rounding form: ``silu(gate) * up`` in fp32, rounded once.

    This is what the reference's ``@torch.compile``d ``SiluAndMul`` computes on
    GPU (inductor upcasts the fused expression to fp32).
    """
    gate, up = x.chunk(2, -1)
    return _round(F.silu(gate.float()) * up.float(), x.dtype)


# --------------------------------------------------------------------------- rotary


def rope_cos_sin_cache(head_size, max_position, base):
    """``RotaryEmbedding.__init__`` table: ``nanovllm/layers/rotary_embedding.py:29-35``.

    Shape ``[max_position, 1, head_size]`` fp32: cos of the first half, sin of
    the second half of the last dimension.
    """
    inv_freq = 1.0 / (base ** (torch.arange(0, head_size, 2, dtype=torch.float) / head_size))
    t = torch.arange(max_position, dtype=torch.float)
    freqs = torch.einsum("i,j -> ij", t, inv_freq)
    return torch.cat((freqs.cos(), freqs.sin()), dim=-1).unsqueeze_(1)


def _rotate_neox_fp32(x, cos, sin):
    # nanovllm/layers/rotary_embedding.py:6-14: fp32 math, one rounding at the end
    half = x.shape[-1] // 2
    xf = x.float()
    x1, x2 = xf[..., :half], xf[..., half:]
    y1 = x1 * cos - x2 * sin
    y2 = x2 * cos + x1 * sin
    return _round(torch.cat((y1, y2), dim=-1), x.dtype)


def apply_rope(positions, query, key, cos_sin_cache):
    """``RotaryEmbedding.forward``: ``nanovllm/layers/rotary_embedding.py:37-48``."""
    cos_sin = cos_sin_cache[positions.long()]
    half = cos_sin.shape[-1] // 2
    cos, sin = cos_sin[..., :half], cos_sin[..., half:]
    return _rotate_neox_fp32(query, cos, sin), _rotate_neox_fp32(key, cos, sin)


def mrope_inv_freq(head_dim, base):
    """``MultimodalRotaryEmbedding.__init__`` inverse frequencies.

    ``nanovllm/layers/multimodal_rotary_embedding.py:70-86`` (built in fp32).
    """
    return 1.0 / (base ** (torch.arange(0, head_dim, 2, dtype=torch.float32) / head_dim))


def mrope_cos_sin(positions, inv_freq, dtype):
    """``MultimodalRotaryEmbedding.cos_sin``: ``multimodal_rotary_embedding.py:89-101``.

    fp32 ``position * inv_freq``, duplicated to the full head dim, cos/sin in
    fp32, then rounded to ``dtype``. Returns two ``[3, T, head_dim]`` tensors.
    """
    freqs = positions.to(torch.float32).unsqueeze(-1) * inv_freq.view(1, 1, -1)
    emb = torch.cat((freqs, freqs), dim=-1)
    return _round(emb.cos(), dtype), _round(emb.sin(), dtype)


def mrope_select(values, sections, strategy):
    """``_select_frequency_layout``: ``multimodal_rotary_embedding.py:120-147``.

    ``values`` is ``[3, T, D]``; the result is ``[T, 1, D]``.

    * ``chunked`` (Qwen2.5-VL): split the last dim into ``sections+sections``;
      chunk ``i`` takes its values from axis ``i % 3``.
    * ``interleaved`` (Qwen3-VL): on the first half, frequency ``j`` reads axis
      1 when ``j % 3 == 1 and j < 3*sections[1]``, axis 2 when
      ``j % 3 == 2 and j < 3*sections[2]``, else axis 0; the second half
      repeats the first.
    """
    d = values.shape[-1]
    if strategy == "chunked":
        bounds = np.cumsum((0,) + tuple(sections) + tuple(sections))
        parts = [values[i % 3, ..., bounds[i]:bounds[i + 1]] for i in range(6)]
        selected = torch.cat(parts, dim=-1)
    elif strategy == "interleaved":
        half = d // 2
        sel = values[0, ..., :half].clone()
        for axis, offset in ((1, 1), (2, 2)):
            idx = list(range(offset, sections[axis] * 3, 3))
            sel[..., idx] = values[axis, ..., :half][..., idx]
        selected = torch.cat((sel, sel), dim=-1)
    else:
        raise ValueError("multimodal rotary strategy must be 'chunked' or 'interleaved'")
    return selected.unsqueeze(1)


def _rotate_half(x):
    half = x.shape[-1] // 2
    return torch.cat((-x[..., half:], x[..., :half]), dim=-1)


def apply_mrope(query, key, cos, sin, sections, strategy="chunked"):
    """``apply_multimodal_rotary_emb``: ``multimodal_rotary_embedding.py:12-45``.

    ``chunked``: fp32 math on the (already rounded) cos/sin, rounded once.
    ``interleaved``: arithmetic in the tensors' own dtype, i.e. for bf16
    ``round(round(q*c) + round(rotate_half(q)*s))``.
    """
    sc = mrope_select(cos, sections, strategy)
    ss = mrope_select(sin, sections, strategy)
    qd, kd = query.dtype, key.dtype
    if strategy == "chunked":
        q, k, sc, ss = query.float(), key.float(), sc.float(), ss.float()
    else:
        q, k = query, key
    q_out = q * sc + _rotate_half(q) * ss
    k_out = k * sc + _rotate_half(k) * ss
    return _round(q_out, qd), _round(k_out, kd)


def mrope_forward(positions, query, key, inv_freq, sections, strategy):
    """``MultimodalRotaryEmbedding.forward``: ``multimodal_rotary_embedding.py:103-117``."""
    cos, sin = mrope_cos_sin(positions, inv_freq, query.dtype)
    return apply_mrope(query, key, cos, sin, sections, strategy)


# --------------------------------------------------------------------------- byte / index work


def _as_int_view(t: torch.Tensor) -> np.ndarray:
    """Integer view of a CPU tensor's bytes (bit-exact copy semantics)."""
    itype = {1: torch.int8, 2: torch.int16, 4: torch.int32, 8: torch.int64}[t.element_size()]
    return t.contiguous().view(itype).numpy()


def _from_int_view(a: np.ndarray, dtype: torch.dtype) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a)).view(dtype)


def paged_store(key, value, key_cache, value_cache, slot_mapping):
    """Paged-KV store: ``nanovllm/layers/paged_kv/pytorch_backend.py:26-38``.

    For token ``i`` with ``slot_mapping[i] >= 0``, row ``i`` of key/value
    (``kv_heads*head_dim`` elements) overwrites flat slot ``slot_mapping[i]`` of
    the caches; ``-1`` skips the token, and every other slot keeps its bytes.
    Returns new ``(key_cache, value_cache)`` tensors (inputs untouched).
    """
    nb, bs, h, d = key_cache.shape
    slots = slot_mapping.numpy().astype(np.int64)
    valid = slots >= 0
    out = []
    for src, cache in ((key, key_cache), (value, value_cache)):
        c = _as_int_view(cache).reshape(nb * bs, h * d).copy()
        s = _as_int_view(src).reshape(src.shape[0], h * d)
        c[slots[valid]] = s[valid]
        out.append(_from_int_view(c.reshape(nb, bs, h, d), cache.dtype))
    return out[0], out[1]


def paged_store_(key, value, key_cache, value_cache, slot_mapping):
    """In-place form of the same store, as the reference's PyTorch backend runs
    it (``pytorch_backend.py:34-38``: ``index_copy_`` of the valid rows into the
    flattened caches). Used where the caches are too large to copy."""
    valid = slot_mapping >= 0
    slots = slot_mapping[valid].to(dtype=torch.long)
    key_cache.flatten(0, 1).index_copy_(0, slots, key[valid])
    value_cache.flatten(0, 1).index_copy_(0, slots, value[valid])


def paged_gather(cache, block_table, sequence_length):
    """Paged-KV gather: ``nanovllm/layers/paged_kv/pytorch_backend.py:40-50``.

    ``out[t] = cache[block_table[t // block_size], t % block_size]`` for
    ``t < sequence_length``; result ``[sequence_length, kv_heads, head_dim]``.
    """
    nb, bs, h, d = cache.shape
    req = (sequence_length + bs - 1) // bs
    if req == 0:
        return torch.empty((0, h, d), dtype=cache.dtype)
    c = _as_int_view(cache)
    ids = block_table.numpy()[:req].astype(np.int64)
    rows = c[ids].reshape(req * bs, h, d)[:sequence_length]
    return _from_int_view(rows, cache.dtype)


def paged_decode_attention(q, k_cache, v_cache, context_lens, block_tables, scale):
    """Decode attention over a paged cache, the reference's SDPA decode branch
    (``nanovllm/layers/attention.py:286-300``; gather ``:163-178``, SDPA with
    grouped-query heads ``:180-204``) evaluated in float64.

    Per request ``b``: K, V = the first ``context_lens[b]`` cached tokens
    (``paged_gather``); q head ``h`` uses kv head ``h // (heads / kv_heads)``;
    ``out = softmax(q . K^T * scale) V`` rounded once to q's dtype. An empty
    context gives zeros. q is ``[batch, heads, head_dim]``.
    """
    batch, heads, dim = q.shape
    group = heads // k_cache.shape[2]
    out = torch.zeros(batch, heads, dim, dtype=q.dtype)
    for b in range(batch):
        n = int(context_lens[b])
        if n == 0:
            continue
        k = paged_gather(k_cache, block_tables[b], n).double()
        v = paged_gather(v_cache, block_tables[b], n).double()
        for h in range(heads):
            p = torch.softmax((k[:, h // group] @ q[b, h].double()) * scale, dim=0)
            out[b, h] = (p @ v[:, h // group]).to(q.dtype)
    return out


def paged_decode_attention_abs(q, k_cache, v_cache, context_lens, block_tables, scale):
    """The softmax-weighted mean of ``|v|`` for each output element of
    :func:`paged_decode_attention` (float64, ``[batch, heads, head_dim]``):
    ``sum_t p_t |v_t| / sum_t p_t``. A kernel that rounds the probabilities
    ``p_t`` to bf16/fp16 before ``P V`` (as flash-attn's decode kernel and the
    tensor-core kernel here do) errs by at most ``2^-8`` times this amount."""
    batch, heads, dim = q.shape
    group = heads // k_cache.shape[2]
    out = torch.zeros(batch, heads, dim, dtype=torch.float64)
    for b in range(batch):
        n = int(context_lens[b])
        if n == 0:
            continue
        k = paged_gather(k_cache, block_tables[b], n).double()
        v = paged_gather(v_cache, block_tables[b], n).double().abs()
        for h in range(heads):
            p = torch.softmax((k[:, h // group] @ q[b, h].double()) * scale, dim=0)
            out[b, h] = p @ v[:, h // group]
    return out


def embedding(ids, weight):
    """``VocabParallelEmbedding.forward`` at tp=1: ``nanovllm/layers/embed_head.py:34-42``.

    Row gather ``weight[ids]``.
    """
    w = _as_int_view(weight)
    return _from_int_view(w[ids.numpy().astype(np.int64)], weight.dtype)


def add_deepstack_rows(hidden_states, visual_token_rows, visual_embedding):
    """``Qwen3VLLanguageModel._add_deepstack_rows``: ``nanovllm/models/qwen3_vl.py:332-344``.

    Returns the input object itself when there are no rows; otherwise a new
    tensor equal to the input except ``out[rows[j]] = h[rows[j]] + vis[j]``
    (one activation-dtype rounding).
    """
    if visual_token_rows.numel() == 0:
        return hidden_states
    rows = visual_token_rows.long()
    updated = hidden_states.index_select(0, rows) + visual_embedding
    out = hidden_states.clone()
    out.index_copy_(0, rows, updated)
    return out


# --------------------------------------------------------------------------- visual merge


def planned_visual_embeddings(token_embeddings, replacements, features):
    """``build_planned_visual_embeddings``: ``nanovllm/engine/model_runner.py:170-286``.

    ``replacements``: ``(output_row, feature_key, feature_row)`` in plan order;
    ``features``: key -> ``(final, (deepstack_0, ...))``. The merged tensor is a
    copy of the token embeddings with row ``output_row`` taken from
    ``final[feature_row]``; DeepStack payload ``l`` holds
    ``deepstack_l[feature_row]`` at the replacement's plan index. Feature rows
    are converted to the token dtype (``.to(dtype)``). Returns
    ``(merged, payloads, visual_rows)``.
    """
    merged = token_embeddings.clone()
    layers = len(next(iter(features.values()))[1]) if replacements else 0
    payloads = tuple(torch.empty(len(replacements), merged.shape[1], dtype=merged.dtype)
                     for _ in range(layers))
    for i, (out_row, key, feat_row) in enumerate(replacements):
        final, deepstack = features[key]
        merged[out_row] = final[feat_row].to(merged.dtype)
        for l in range(layers):
            payloads[l][i] = deepstack[l][feat_row].to(merged.dtype)
    rows = torch.tensor([r[0] for r in replacements], dtype=torch.int64)
    return merged, payloads, rows


# --------------------------------------------------------------------------- compositions


def add_text_rms_norm_deepstack(x, residual, weight, eps, visual_token_rows, visual_embedding,
                                order="torch"):
    """Qwen3-VL layer boundary with a DeepStack layer in between.

    The layer's output add ``mlp_residual + mlp(h)`` (``nanovllm/models/qwen3_vl.py:238``,
    one dtype rounding), then ``_add_deepstack_rows`` on that output
    (``:332-344``, called at ``:371-376``), then the next layer's
    ``input_layernorm`` (``:234``, ``Qwen3VLTextRMSNorm`` ``:74-79``), whose
    ``attention_residual`` is the DeepStack-updated sum. Returns
    ``(normed, updated_sum)``.
    """
    s = _round(x.float() + residual.float(), x.dtype)
    s = add_deepstack_rows(s, visual_token_rows, visual_embedding)
    if order == "torch":
        return text_rms_norm(s, weight, eps), s
    sf = s.float()
    n = _round(sf * _inv_rms(sf, eps, order, x.dtype, add=True), x.dtype)
    out_dtype = torch.promote_types(weight.dtype, x.dtype)
    return _round(weight.float() * n.float(), out_dtype).contiguous(), s



def qk_norm_rope_store(
    qkv,
    num_heads,
    num_kv_heads,
    head_dim,
    *,
    positions,
    rope,
    q_weight=None,
    k_weight=None,
    eps=1e-6,
    norm="rms",
    key_cache=None,
    value_cache=None,
    slot_mapping=None,
    inplace=False,
    order="torch",
):
    """The attention prologue that the fused kernel replaces.

    Composition, per model:

    * Qwen3 (``nanovllm/models/qwen3.py:77-86``): split ``qkv``, per-head
      ``RMSNorm.rms_forward`` on q and k, 1-D ``RotaryEmbedding``, store.
    * Qwen3-VL (``nanovllm/models/qwen3_vl.py:161-172``): per-head
      ``Qwen3VLTextRMSNorm``, interleaved M-RoPE, store.
    * Qwen2.5-VL (``nanovllm/models/qwen25_vl.py:66-76``): no q/k norm, chunked
      M-RoPE, store.

    ``rope`` is ``("table", cos_sin_cache)`` or
    ``("mrope", inv_freq, sections, strategy)``; ``norm`` is ``"rms"``
    (RMSNorm), ``"text"`` (Qwen3VLTextRMSNorm) or ``None``. The store writes
    the rotated k and the raw v (``nanovllm/layers/attention.py:87-93``).
    Returns ``(q, k, key_cache, value_cache)`` (caches are new tensors, or
    ``None`` when not given; with ``inplace=True`` the given caches are
    updated and returned).
    """
    q_size = num_heads * head_dim
    kv_size = num_kv_heads * head_dim
    q, k, v = qkv.split([q_size, kv_size, kv_size], dim=-1)
    q = q.reshape(-1, num_heads, head_dim)
    k = k.reshape(-1, num_kv_heads, head_dim)
    v = v.reshape(-1, num_kv_heads, head_dim)
    if norm == "rms":
        q, k = rms_norm(q, q_weight, eps, order), rms_norm(k, k_weight, eps, order)
    elif norm == "text":
        q, k = text_rms_norm(q, q_weight, eps, order), text_rms_norm(k, k_weight, eps, order)
    if rope[0] == "table":
        q, k = apply_rope(positions, q, k, rope[1])
    else:
        _, inv_freq, sections, strategy = rope
        q, k = mrope_forward(positions, q, k, inv_freq, sections, strategy)
    kc = vc = None
    if key_cache is not None:
        if inplace:
            paged_store_(k, v, key_cache, value_cache, slot_mapping)
            kc, vc = key_cache, value_cache
        else:
            kc, vc = paged_store(k, v, key_cache, value_cache, slot_mapping)
    return q, k, kc, vc


def qwen3_vl_fused_layer(
    hidden,
    residual,
    qkv,
    attn_out,
    gate_up,
    *,
    positions,
    inv_freq,
    sections,
    w_in,
    w_post,
    q_weight,
    k_weight,
    eps,
    num_heads,
    num_kv_heads,
    head_dim,
    key_cache,
    value_cache,
    slot_mapping,
    inplace=False,
):
    """One decoder layer's elementwise work with the GEMM outputs supplied.

    ``nanovllm/models/qwen3_vl.py:226-240``: residual add + input norm, the
    attention prologue (q/k norm, interleaved M-RoPE, paged store), residual add
    + post-attention norm, and ``SiluAndMul`` on the gate/up projection. The
    projections themselves (qkv, o_proj, gate_up) are inputs here.
    Returns ``(normed_in, h1, q, k, key_cache, value_cache, normed_post, h2, act)``.
    """
    y1, h1 = add_text_rms_norm(hidden, residual, w_in, eps)
    q, k, kc, vc = qk_norm_rope_store(
        qkv, num_heads, num_kv_heads, head_dim,
        positions=positions, rope=("mrope", inv_freq, sections, "interleaved"),
        q_weight=q_weight, k_weight=k_weight, eps=eps, norm="text",
        key_cache=key_cache, value_cache=value_cache, slot_mapping=slot_mapping, inplace=inplace,
    )
    y2, h2 = add_text_rms_norm(attn_out, h1, w_post, eps)
    act = silu_and_mul(gate_up)
    return y1, h1, q, k, kc, vc, y2, h2, act
