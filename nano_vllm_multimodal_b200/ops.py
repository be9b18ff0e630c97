"""Python entry points of the sm_100a hot path (``torch.ops.nanoinfer_b200``).

Every function here launches hand-written CUDA from ``libnib_b200.so`` on the
current stream; CPU tensors raise (``NotImplementedError`` from the dispatcher
or ``ValueError`` below). Nothing synchronises unless index validation is
switched on with ``NANOINFER_B200_VALIDATE=1`` (or the reference's
``NANOVLLM_PAGED_KV_VALIDATE_INDICES=1``): then each op hands the kernels a
per-device status word and, after the launch, reads it back and raises on a
bad slot / position / block id / row. Validation mode synchronises, so it
cannot be captured in a CUDA graph (same contract as the reference's opt-in
host checks, ``nanovllm/layers/paged_kv/base.py:68-72``).
"""

from __future__ import annotations

import os

import torch

from nano_vllm_multimodal_b200._lib import load_ops

ROPE_NONE = 0
ROPE_TABLE = 1
ROPE_MROPE_CHUNKED = 2
ROPE_MROPE_INTERLEAVED = 3

DEV_BAD_SLOT = 1
DEV_BAD_POSITION = 2
DEV_BAD_BLOCK = 4
DEV_BAD_INDEX = 8

_VALIDATE_ENV = ("NANOINFER_B200_VALIDATE", "NANOVLLM_PAGED_KV_VALIDATE_INDICES")
_STATUS: dict[int, torch.Tensor] = {}


def _ops():
    load_ops()
    return torch.ops.nanoinfer_b200


def validation_enabled() -> bool:
    for name in _VALIDATE_ENV:
        if os.environ.get(name, "0").strip().lower() in {"1", "true", "yes", "on"}:
            return True
    return False


def _status_for(t: torch.Tensor):
    if not validation_enabled() or not t.is_cuda:
        return None
    idx = t.device.index if t.device.index is not None else torch.cuda.current_device()
    st = _STATUS.get(idx)
    if st is None:
        st = torch.zeros(1, dtype=torch.int32, device=t.device)
        _STATUS[idx] = st
    return st


def _check_status(st, what: str) -> None:
    if st is None:
        return
    bits = int(st.item())
    if not bits:
        return
    st.zero_()
    names = []
    if bits & DEV_BAD_SLOT:
        names.append("slot_mapping contains a slot outside [-1, num_slots)")
    if bits & DEV_BAD_POSITION:
        names.append("a position is outside the rotary cos/sin table")
    if bits & DEV_BAD_BLOCK:
        names.append("block_table contains an invalid physical block")
    if bits & DEV_BAD_INDEX:
        names.append("an index (token id or row) is out of range")
    raise ValueError(f"{what}: " + "; ".join(names))


# ---------------------------------------------------------------- norms / activation


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    """RMSNorm of the last dim (``nanovllm/layers/layernorm.py:16-26``)."""
    return _ops().rms_norm(x, weight, float(eps))


def add_rms_norm(x, residual, weight, eps, round_sum: bool = False):
    """Residual add + RMSNorm -> ``(normed, new_residual)``.

    ``round_sum=False``: ``RMSNorm.add_rms_forward`` (``layernorm.py:28-40``);
    ``round_sum=True``: Qwen3-VL's rounded add then text norm
    (``nanovllm/models/qwen3_vl.py:232-237``).
    """
    return _ops().add_rms_norm(x, residual, weight, float(eps), bool(round_sum))


def silu_and_mul(x: torch.Tensor) -> torch.Tensor:
    """``silu(x[..., :I]) * x[..., I:]`` (``nanovllm/layers/activation.py:8-11``)."""
    return _ops().silu_and_mul(x)


# ---------------------------------------------------------------- attention prologue


def prologue_supported(*tensors) -> bool:
    """Whether the fused prologue kernel takes these ``[T, heads, D]`` tensors
    directly: head_dim 64/128/256, 16-byte aligned rows and strides. Other
    layouts go through the generic rotation kernel."""
    t0 = tensors[0]
    d = t0.shape[-1]
    per_vec = 16 // t0.element_size()
    if d not in (64, 128, 256):
        return False
    for t in tensors:
        if t is None:
            continue
        if t.dim() != 3 or t.stride(-1) != 1 or t.data_ptr() % 16:
            return False
        if t.stride(0) % per_vec or t.stride(1) % per_vec:
            return False
    return True



def qk_prologue(q, k, *, v=None, positions=None, q_weight=None, k_weight=None, eps=1e-6,
                rope_mode=ROPE_NONE, cos_sin_cache=None, inv_freq=None, sections=(),
                key_cache=None, value_cache=None, slot_mapping=None, variant=0, emit_k=True):
    """Per-head norm + RoPE/M-RoPE + paged store in one kernel -> ``(q_rot, k_rot)``.

    ``variant``: 0 picks automatically, 1 forces the register-staged kernel,
    2 the bulk-copy pipelined kernel (q/k/v consecutive ranges of one row).
    Both give bit-identical results.

    ``emit_k=False`` (only with the caches): rotated k is written to the key
    cache alone and ``k_rot`` is ``None``; decode and prefill over a block
    table read k from the cache, so the contiguous copy would go unread."""
    st = _status_for(q)
    q_rot, k_rot = _ops().qk_prologue(q, k, v, positions, q_weight, k_weight, float(eps), int(rope_mode),
                                      cos_sin_cache, inv_freq, list(sections), key_cache, value_cache,
                                      slot_mapping, st, int(variant), bool(emit_k))
    _check_status(st, "qk_prologue")
    return q_rot, (k_rot if emit_k else None)


def rope(positions, q, k, cos_sin_cache):
    """1-D neox RoPE (``nanovllm/layers/rotary_embedding.py:37-48``)."""
    return qk_prologue(q, k, positions=positions, rope_mode=ROPE_TABLE, cos_sin_cache=cos_sin_cache)


def mrope(positions, q, k, inv_freq, sections, strategy):
    """Multimodal RoPE (``nanovllm/layers/multimodal_rotary_embedding.py:103-117``)."""
    mode = ROPE_MROPE_INTERLEAVED if strategy == "interleaved" else ROPE_MROPE_CHUNKED
    return qk_prologue(q, k, positions=positions, rope_mode=mode, inv_freq=inv_freq, sections=sections)


def mrope_apply(x, cos, sin, sections, interleaved: bool):
    """Rotate ``x`` with caller-given ``[3, T, D]`` cos/sin (any even D)."""
    return _ops().mrope_apply(x, cos, sin, list(sections), bool(interleaved))


def mrope_cos_sin(positions, inv_freq, dtype):
    return _ops().mrope_cos_sin(positions, inv_freq, dtype)


# ---------------------------------------------------------------- paged KV


def paged_store(key, value, key_cache, value_cache, slot_mapping) -> None:
    load_ops()
    torch.ops.nanovllm_paged_kv.store(key, value, key_cache, value_cache, slot_mapping)


def paged_gather(cache, block_table, sequence_length: int) -> torch.Tensor:
    load_ops()
    return torch.ops.nanovllm_paged_kv.gather(cache, block_table, int(sequence_length))


def paged_gather_varlen(cache, block_tables, seq_lens, cu_seqlens, total_tokens: int,
                        max_seq_len: int) -> torch.Tensor:
    """Gather many sequences in one launch into one packed ``[total, kv_heads, D]``.

    ``seq_lens`` (int32) and ``cu_seqlens`` (int64 exclusive prefix sums) live on
    the device; ``total_tokens``/``max_seq_len`` are host ints (no sync).
    """
    st = _status_for(cache)
    out = _ops().paged_gather_varlen(cache, block_tables, seq_lens, cu_seqlens, int(total_tokens),
                                     int(max_seq_len), st)
    _check_status(st, "paged_gather_varlen")
    return out


# ---------------------------------------------------------------- rows


def embedding(ids, weight, vocab_start: int = 0, vocab_end: int | None = None, mask: bool = False):
    """Row gather ``weight[ids - vocab_start]``; ids outside the shard give zero rows."""
    if vocab_end is None:
        vocab_end = vocab_start + weight.shape[0]
    st = _status_for(weight)
    out = _ops().embedding(ids, weight, int(vocab_start), int(vocab_end), bool(mask), st)
    _check_status(st, "embedding")
    return out


def deepstack_add(hidden, rows, vis) -> torch.Tensor:
    """Out of place: copy of ``hidden`` with ``vis`` added at ``rows``."""
    st = _status_for(hidden)
    out = _ops().deepstack_add(hidden, rows, vis, st)
    _check_status(st, "deepstack_add")
    return out


def deepstack_add_(hidden, rows, vis) -> torch.Tensor:
    """In place: ``hidden[rows] += vis`` (one activation-dtype rounding)."""
    st = _status_for(hidden)
    _ops().deepstack_add_(hidden, rows, vis, st)
    _check_status(st, "deepstack_add_")
    return hidden


def visual_merge(token_embeddings, table, num_layers: int, plan, num_replacements: int):
    """Packed-prefill visual merge (``nib_visual_merge``) -> ``(merged, deepstack)``,
    ``deepstack`` being ``[num_layers, num_replacements, hidden]``. ``table`` and
    ``plan`` are the device int64 buffers that
    ``layers.visual_merge.build_planned_visual_embeddings`` packs."""
    st = _status_for(token_embeddings)
    out = _ops().visual_merge(token_embeddings, table, int(num_layers), plan, int(num_replacements), st)
    _check_status(st, "visual_merge")
    return out


DECODE_AUTO, DECODE_CUDA_CORES, DECODE_TENSOR_CORES = 0, 1, 2


def decode_attention(q, k_cache, v_cache, context_lens, block_tables, scale: float,
                     max_context_len: int = 0, variant: int = DECODE_AUTO) -> torch.Tensor:
    """Paged decode attention -> ``[batch, heads, head_dim]`` (``nib_decode_attention``).
    ``max_context_len`` is an optional host upper bound of ``context_lens`` (0: the
    block-table width times the block size); it only chooses how a context is split.
    ``variant``: the tensor-core kernel where it applies (default), or force the
    CUDA-core (1) or tensor-core (2) kernel."""
    st = _status_for(q)
    out = _ops().decode_attention(q, k_cache, v_cache, context_lens, block_tables, float(scale),
                                  int(max_context_len), st, int(variant))
    _check_status(st, "decode_attention")
    return out


def deepstack_row_index(rows, tokens: int) -> torch.Tensor:
    """int32 ``[tokens]``: ``j`` at ``rows[j]``, ``-1`` elsewhere (the map the
    folded add + norm + DeepStack kernel reads; build once per forward)."""
    st = _status_for(rows)
    out = _ops().deepstack_row_index(rows, int(tokens), st)
    _check_status(st, "deepstack_row_index")
    return out


def add_rms_norm_deepstack(x, residual, weight, eps, vis, row_index):
    """Qwen3-VL layer boundary in one pass -> ``(normed, new_residual)``:
    ``s = dtype(x + residual)``; tokens with ``row_index[t] >= 0`` add
    ``vis[row_index[t]]`` (one more rounding); ``normed = Qwen3VLTextRMSNorm(s)``.
    Equals ``add_rms_norm(..., round_sum=True)`` after ``deepstack_add_`` on the sum
    (``nanovllm/models/qwen3_vl.py:238,332-344,371-376`` then ``:232-235``)."""
    st = _status_for(x)
    out = _ops().add_rms_norm_deepstack(x, residual, weight, float(eps), vis, row_index, st)
    _check_status(st, "add_rms_norm_deepstack")
    return out
