"""Attention-side pieces of the hot path: the paged KV store, the fused
attention prologue and the paged decode attention that reads the cache.

``store_kvcache`` keeps the signature of ``nanovllm/layers/attention.py:10-33``.
``attention_prologue`` replaces, in one kernel launch, the sequence the
decoder layers run between the qkv projection and the attention kernel:

* Qwen3       ``nanovllm/models/qwen3.py:77-86``       split, q/k RMSNorm, 1-D RoPE, store
* Qwen3-VL    ``nanovllm/models/qwen3_vl.py:161-172``  split, q/k text norm, interleaved M-RoPE, store
* Qwen2.5-VL  ``nanovllm/models/qwen25_vl.py:66-76``   split, chunked M-RoPE, store

It returns the rotated q and k (prefill attention without a block table reads
them directly, ``attention.py:99-116``) and the v view; the caches are already
written, so the caller's attention must skip its own store.
"""

from __future__ import annotations

import sys

import torch
from torch import nn

from nano_vllm_multimodal_b200 import ops
from nano_vllm_multimodal_b200.layers.paged_kv.base import validate_store_inputs


def store_kvcache(key, value, k_cache, v_cache, slot_mapping) -> None:
    """Write this step's K/V rows into the paged caches (slot -1 = skip)."""
    validate_store_inputs(key, value, k_cache, v_cache, slot_mapping)
    ops.paged_store(key, value, k_cache, v_cache, slot_mapping)


def _step_context():
    """The runner's per-step ``Context`` (``nanovllm/utils/context.py``): the
    model runner sets it before every forward, so attention reads the slot
    mapping, sequence boundaries and block tables from there."""
    from nanovllm.utils.context import get_context
    return get_context()


def _attention_kernels():
    """The prefill / decode attention functions as ``nanovllm.layers.attention``
    binds them now (``install()`` rebinds the decode one to this package's
    kernel; tests of the reference may patch either)."""
    ref = sys.modules.get("nanovllm.layers.attention")
    varlen = getattr(ref, "flash_attn_varlen_func", None)
    decode = getattr(ref, "flash_attn_with_kvcache", None)
    if varlen is None:
        from flash_attn import flash_attn_varlen_func as varlen
    if decode is None:
        decode = flash_attn_with_kvcache
    return varlen, decode


class Attention(nn.Module):
    """Drop-in for ``nanovllm.layers.attention.Attention`` (``attention.py:36-132``).

    Same constructor, the same ``k_cache``/``v_cache``/``paged_kv_backend``
    attributes that ``ModelRunner.allocate_kv_cache`` assigns
    (``model_runner.py:681-690``), and the same ``forward(q, k, v)``: store this
    step's K/V (through the runner's backend when it set one, else this
    package's store), then prefill attention over the packed sequences or
    decode attention over the paged cache.

    ``forward_stored(q, k, v)`` is the same step for callers whose fused
    prologue has already written K/V into the caches.
    """

    def __init__(self, num_heads, head_dim, scale, num_kv_heads):
        super().__init__()
        self.num_heads = num_heads
        self.head_dim = head_dim
        self.scale = scale
        self.num_kv_heads = num_kv_heads
        self.k_cache = self.v_cache = torch.tensor([])
        self.paged_kv_backend = None

    def forward(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor):
        k_cache, v_cache = self.k_cache, self.v_cache
        if k_cache.numel() and v_cache.numel():
            slots = _step_context().slot_mapping
            if self.paged_kv_backend is None:
                store_kvcache(k, v, k_cache, v_cache, slots)
            else:
                self.paged_kv_backend.store(k, v, k_cache, v_cache, slots)
        return self.forward_stored(q, k, v)

    def forward_stored(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor):
        ctx = _step_context()
        varlen, decode = _attention_kernels()
        if ctx.is_prefill:
            if ctx.block_tables is not None:  # prefix cache / chunked prefill: read history from the cache
                k, v = self.k_cache, self.v_cache
            return varlen(q, k, v, max_seqlen_q=ctx.max_seqlen_q, cu_seqlens_q=ctx.cu_seqlens_q,
                          max_seqlen_k=ctx.max_seqlen_k, cu_seqlens_k=ctx.cu_seqlens_k,
                          softmax_scale=self.scale, causal=True, block_table=ctx.block_tables)
        return decode(q.unsqueeze(1), self.k_cache, self.v_cache, cache_seqlens=ctx.context_lens,
                      block_table=ctx.block_tables, softmax_scale=self.scale, causal=True)


def _rope_args(rotary_emb):
    if hasattr(rotary_emb, "cos_sin_cache"):
        return dict(rope_mode=ops.ROPE_TABLE, cos_sin_cache=rotary_emb.cos_sin_cache)
    if hasattr(rotary_emb, "inv_freq") and hasattr(rotary_emb, "sections"):
        mode = (ops.ROPE_MROPE_INTERLEAVED if rotary_emb.strategy == "interleaved"
                else ops.ROPE_MROPE_CHUNKED)
        return dict(rope_mode=mode, inv_freq=rotary_emb.inv_freq, sections=tuple(rotary_emb.sections))
    raise TypeError(f"unsupported rotary embedding module {type(rotary_emb).__name__}")


def attention_prologue(qkv: torch.Tensor, *, num_heads: int, num_kv_heads: int, head_dim: int,
                       positions: torch.Tensor, rotary_emb, q_norm=None, k_norm=None,
                       k_cache: torch.Tensor | None = None, v_cache: torch.Tensor | None = None,
                       slot_mapping: torch.Tensor | None = None, emit_k: bool = True):
    """Fused q/k norm + rotary + paged store -> ``(q, k, v)``.

    ``q_norm``/``k_norm`` are RMSNorm-like modules (``weight``, ``eps``) or
    ``None``; ``rotary_emb`` is a ``RotaryEmbedding`` (table) or a
    ``MultimodalRotaryEmbedding``. The store runs when both caches are
    non-empty, as in ``Attention.forward`` (``attention.py:87-93``).
    ``emit_k=False`` with a store: rotated k goes to the key cache only and
    the returned ``k`` is ``None`` (for attention that reads the cache).
    """
    q_size, kv_size = num_heads * head_dim, num_kv_heads * head_dim
    q, k, v = qkv.split([q_size, kv_size, kv_size], dim=-1)
    q = q.view(-1, num_heads, head_dim)
    k = k.view(-1, num_kv_heads, head_dim)
    v = v.view(-1, num_kv_heads, head_dim)
    store = k_cache is not None and v_cache is not None and k_cache.numel() and v_cache.numel()
    if store:
        validate_store_inputs(k, v, k_cache, v_cache, slot_mapping)
    if (q_norm is None) != (k_norm is None):
        raise ValueError("q_norm and k_norm must be given together")
    emit_k = emit_k or not store
    if not ops.prologue_supported(q, k, v if store else None):
        # unusual head size / layout: the same stages as separate kernels
        if q_norm is not None:
            q, k = q_norm(q), k_norm(k)
        q, k = rotary_emb(positions, q, k)
        if store:
            ops.paged_store(k, v, k_cache, v_cache, slot_mapping)
        return q, k, v
    if positions.dtype != torch.long:
        positions = positions.long()
    norm = {}
    if q_norm is not None:
        norm = dict(q_weight=q_norm.weight, k_weight=k_norm.weight, eps=q_norm.eps)
    cache = {}
    if store:
        cache = dict(v=v, key_cache=k_cache, value_cache=v_cache, slot_mapping=slot_mapping)
    q_rot, k_rot = ops.qk_prologue(q, k, positions=positions, **norm, **_rope_args(rotary_emb), **cache,
                                   emit_k=emit_k)
    return q_rot, k_rot, v


def paged_decode_attention(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                           context_lens: torch.Tensor, block_tables: torch.Tensor, scale: float,
                           max_context_len: int = 0) -> torch.Tensor:
    """One query token per request against its paged cache -> ``[batch, heads, head_dim]``
    (the reference's SDPA decode branch, ``nanovllm/layers/attention.py:286-300``)."""
    if context_lens.dtype != torch.int32:
        context_lens = context_lens.to(torch.int32)
    if block_tables.dtype != torch.int32:
        block_tables = block_tables.to(torch.int32)
    return ops.decode_attention(q, k_cache, v_cache, context_lens, block_tables, scale, max_context_len)


_FA_DEFAULTS = {"softcap": 0.0, "rotary_interleaved": True, "return_softmax_lse": False}


def flash_attn_with_kvcache(q, k_cache, v_cache, k=None, v=None, rotary_cos=None, rotary_sin=None,
                            cache_seqlens=None, cache_batch_idx=None, cache_leftpad=None,
                            block_table=None, softmax_scale=None, causal=False, **kwargs):
    """Drop-in for the decode call ``flash_attn_with_kvcache(q.unsqueeze(1), k_cache, v_cache,
    cache_seqlens=..., block_table=..., softmax_scale=..., causal=True)``
    (``nanovllm/layers/attention.py:122-130``): q ``[batch, 1, heads, head_dim]`` ->
    ``[batch, 1, heads, head_dim]``. With one query token per request, causal and
    non-causal attention are the same. Features that call does not use (appending
    k/v, rotary, batch indices, left padding, windows, softcap, ...) are refused."""
    unused = dict(k=k, v=v, rotary_cos=rotary_cos, rotary_sin=rotary_sin,
                  cache_batch_idx=cache_batch_idx, cache_leftpad=cache_leftpad)
    given = [name for name, val in unused.items() if val is not None]
    for name, val in kwargs.items():
        if name == "num_splits":  # a scheduling hint of flash-attn; the split count is chosen here
            continue
        if name == "window_size":
            if tuple(val) != (-1, -1):
                given.append(name)
        elif name == "alibi_slopes":
            if val is not None:
                given.append(name)
        elif name in _FA_DEFAULTS:
            if val != _FA_DEFAULTS[name]:
                given.append(name)
        else:
            given.append(name)
    if given:
        raise NotImplementedError(f"flash_attn_with_kvcache: unsupported arguments {given}")
    if q.dim() != 4 or q.shape[1] != 1:
        raise NotImplementedError("flash_attn_with_kvcache: one query token per request is supported")
    if cache_seqlens is None or block_table is None:
        raise NotImplementedError("flash_attn_with_kvcache: a paged cache (block_table, cache_seqlens) is required")
    scale = softmax_scale if softmax_scale is not None else q.shape[-1] ** -0.5
    lens = cache_seqlens
    if isinstance(lens, int):
        lens = torch.full((q.shape[0],), lens, dtype=torch.int32, device=q.device)
    out = paged_decode_attention(q[:, 0], k_cache, v_cache, lens, block_table, scale,
                                 block_table.shape[1] * k_cache.shape[1])
    return out.unsqueeze(1)
