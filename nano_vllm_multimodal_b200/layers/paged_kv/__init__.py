"""Paged-KV backend layer (interface of ``nanovllm/layers/paged_kv/__init__.py``).

Only the ``cuda`` backend is provided here: it is the one this package
replaces. ``pytorch`` and ``triton`` remain the reference's own.
"""

from __future__ import annotations

from nano_vllm_multimodal_b200.layers.paged_kv.base import (
    GatherDimensions,
    PagedKVAllocation,
    PagedKVBackend,
    StoreDimensions,
    index_value_validation_enabled,
    resolve_paged_kv_backend_name,
    validate_gather_inputs,
    validate_store_inputs,
)


def create_paged_kv_backend(name: str) -> PagedKVBackend:
    if name == "cuda":
        from nano_vllm_multimodal_b200.layers.paged_kv.cuda_backend import CUDAPagedKVBackend

        return CUDAPagedKVBackend()
    raise ValueError(f"unknown paged KV backend: {name} (this package provides only 'cuda')")


__all__ = [
    "GatherDimensions",
    "index_value_validation_enabled",
    "PagedKVAllocation",
    "PagedKVBackend",
    "StoreDimensions",
    "create_paged_kv_backend",
    "resolve_paged_kv_backend_name",
    "validate_gather_inputs",
    "validate_store_inputs",
]
