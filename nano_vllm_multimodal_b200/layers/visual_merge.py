"""Packed-prefill visual-embedding merge (the input side of the decoder path).

Interface of ``nanovllm/engine/model_runner.py:105-111,158-286``:
``build_planned_visual_embeddings(token_embeddings, plan, features)`` returns the
token embeddings with every planned row replaced by its vision-feature row, one
``[R, hidden]`` DeepStack payload per layer in plan order, and the planned
output rows; ``merge_planned_visual_embeddings`` returns only the first. The
plan (``replacements`` with ``output_row``, ``feature_key``, ``feature_row``)
and the features (tensors or bundles with ``final_embedding`` and a tuple of
``deepstack_embeddings``) are the reference's objects, read by attribute.

Validation runs on the host first, in the reference's order and with its
messages. The plan is then packed into one pinned int64 buffer (output rows,
source index and feature row per replacement, followed by a table of the
sources' device pointers and strides), copied to the device asynchronously,
and one kernel launch writes every output row once (``nib_visual_merge``).
"""

from __future__ import annotations

import operator
from dataclasses import dataclass

import numpy as np
import torch

from nano_vllm_multimodal_b200 import ops

MAX_LAYERS = 8                          # NIB_VISUAL_MAX_LAYERS
_TABLE_WORDS = 4 + 2 * MAX_LAYERS       # sizeof(nib_visual_source) / 8
_DTYPE_CODE = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}


@dataclass(frozen=True, slots=True)
class PlannedVisualEmbeddings:
    """Same fields as the reference's ``PlannedVisualEmbeddings`` (model_runner.py:105-111)."""

    final_embedding: torch.Tensor
    deepstack_embeddings: tuple[torch.Tensor, ...]
    visual_rows: torch.Tensor


def _feature_parts(key: str, feature):
    if isinstance(feature, torch.Tensor):
        # the reference wraps a bare tensor in VisionFeatureBundle, which checks its rank
        if feature.ndim != 2:
            raise ValueError("final vision embedding must be rank-2")
        return feature, ()
    final = getattr(feature, "final_embedding", None)
    deepstack = getattr(feature, "deepstack_embeddings", None)
    if not isinstance(final, torch.Tensor) or not isinstance(deepstack, tuple):
        raise TypeError(f"visual feature must be a bundle: {key}")
    return final, deepstack


def _on_device(t: torch.Tensor, device, dtype) -> torch.Tensor:
    """A kernel-readable view: on `device`, a dtype the kernel converts from,
    unit stride along the hidden dimension."""
    if t.dtype not in _DTYPE_CODE:
        t = t.to(dtype)
    if t.device != device:
        t = t.to(device)
    if t.shape[0] > 1 and t.stride(1) != 1 or t.shape[0] <= 1 and not t.is_contiguous():
        t = t.contiguous()
    return t


def build_planned_visual_embeddings(token_embeddings: torch.Tensor, plan, features,
                                    *, result_type=PlannedVisualEmbeddings):
    """See the module docstring; ``result_type`` lets an integration return the
    reference's own dataclass."""
    if token_embeddings.ndim != 2:
        raise ValueError("token embeddings must have shape [tokens, hidden_size]")
    device = token_embeddings.device
    if not plan.replacements:
        return result_type(final_embedding=token_embeddings, deepstack_embeddings=(),
                           visual_rows=torch.empty(0, dtype=torch.int64, device=device))
    token_count, hidden_size = token_embeddings.shape
    reps = plan.replacements
    n = len(reps)
    # the plan's fields, extracted without a per-replacement Python loop body
    out_rows = np.fromiter(map(operator.attrgetter("output_row"), reps), dtype=np.int64, count=n)
    feat_rows = np.fromiter(map(operator.attrgetter("feature_row"), reps), dtype=np.int64, count=n)
    keys = list(map(operator.attrgetter("feature_key"), reps))
    key_index = {k: j for j, k in enumerate(dict.fromkeys(keys))}
    source_index = np.fromiter(map(key_index.__getitem__, keys), dtype=np.int64, count=n)
    _, first_seen = np.unique(source_index, return_index=True)  # first plan index of each key

    # Validation with the reference's messages, raising the error its sequential
    # loop (model_runner.py:190-235) meets first: the checks of a key run at that
    # key's first replacement, before that replacement's row checks.
    sources: list[tuple[torch.Tensor, tuple[torch.Tensor, ...]]] = []
    layer_count = None
    key_error, key_error_at = None, n
    for key, j in key_index.items():
        try:
            feature = features.get(key)
            if feature is None:
                raise KeyError(f"missing visual feature: {key}")
            final, deepstack = _feature_parts(key, feature)
            if final.shape[1] != hidden_size:
                raise ValueError("visual feature hidden size mismatch: "
                                 f"feature={tuple(final.shape)}, hidden_size={hidden_size}")
            if layer_count is None:
                layer_count = len(deepstack)
            elif layer_count != len(deepstack):
                raise ValueError("visual features must have the same deepstack layer count")
        except (KeyError, TypeError, ValueError) as e:
            key_error, key_error_at = e, int(first_seen[j])
            break
        sources.append((final, deepstack))
    counts = np.array([f.shape[0] for f, _ in sources] + [np.iinfo(np.int64).max] * (len(key_index) - len(sources)),
                      dtype=np.int64)
    bad_out = (out_rows < 0) | (out_rows >= token_count)
    bad_feat = (feat_rows < 0) | (feat_rows >= counts[source_index])
    bad = bad_out | bad_feat
    row_error_at = int(np.argmax(bad)) if bad.any() else n
    if key_error is not None and key_error_at <= row_error_at:
        raise key_error
    if row_error_at < n:
        r = reps[row_error_at]
        if bad_out[row_error_at]:
            raise IndexError(f"visual output row is out of range: {r.output_row}")
        raise IndexError("visual feature row is out of range: "
                         f"key={r.feature_key}, row={r.feature_row}")
    layers = layer_count or 0
    if layers > MAX_LAYERS:
        raise NotImplementedError(f"at most {MAX_LAYERS} DeepStack layers are supported, got {layers}")

    tokens = _on_device(token_embeddings, device, token_embeddings.dtype)
    table = torch.zeros(len(sources), _TABLE_WORDS, dtype=torch.int64)
    keep = []  # device copies made here stay referenced until the launch is queued
    for k, (final, deepstack) in enumerate(sources):
        f = _on_device(final, device, tokens.dtype)
        ds = [_on_device(d, device, tokens.dtype) for d in deepstack]
        ds = [d if d.dtype == f.dtype else d.to(f.dtype) for d in ds]  # one dtype per source
        keep.extend([f, *ds])
        table[k, 0] = f.data_ptr()
        table[k, 1] = f.stride(0) if f.shape[0] > 1 else hidden_size
        table[k, 2] = f.shape[0]
        table[k, 3] = _DTYPE_CODE[f.dtype]
        for l, d in enumerate(ds):
            table[k, 4 + l] = d.data_ptr()
            table[k, 4 + MAX_LAYERS + l] = d.stride(0) if d.shape[0] > 1 else hidden_size
    host = torch.from_numpy(np.concatenate((out_rows, source_index, feat_rows, table.view(-1).numpy())))
    if device.type == "cuda":
        host = host.pin_memory()
    packed = host.to(device, non_blocking=True)
    merged, deepstack = ops.visual_merge(tokens, packed[3 * n:].view(len(sources), _TABLE_WORDS),
                                         layers, packed, n)
    del keep
    return result_type(final_embedding=merged,
                       deepstack_embeddings=tuple(deepstack[l] for l in range(layers)),
                       visual_rows=packed[:n])


def merge_planned_visual_embeddings(token_embeddings: torch.Tensor, plan, features) -> torch.Tensor:
    return build_planned_visual_embeddings(token_embeddings, plan, features).final_embedding
