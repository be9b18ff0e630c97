"""The ``cuda`` paged-KV backend, backed by the sm_100a kernels.

Interface of ``nanovllm/layers/paged_kv/cuda_backend.py:30-104``: allocation
through the ``torch.classes.nanovllm_paged_kv.PagedKVCache`` owner,
``copy_slots_async`` through its pinned transfer stream, and
``torch.ops.nanovllm_paged_kv.store/gather`` for the data path. Adds
``gather_varlen`` (every sequence of a batch in one launch).
"""

from __future__ import annotations

from typing import Sequence

import torch

from nano_vllm_multimodal_b200 import ops
from nano_vllm_multimodal_b200._lib import load_ops
from nano_vllm_multimodal_b200.layers.paged_kv.base import (
    PagedKVAllocation,
    validate_gather_inputs,
    validate_store_inputs,
)

_DTYPE_NAMES = {torch.float16: "float16", torch.bfloat16: "bfloat16", torch.float32: "float32"}


class CUDAPagedKVBackend:
    name = "cuda"

    @staticmethod
    def _load() -> None:
        load_ops()

    def allocate(self, shape: Sequence[int], *, dtype: torch.dtype,
                 device: torch.device | str) -> PagedKVAllocation:
        resolved = torch.device(device)
        if resolved.type != "cuda":
            raise ValueError("CUDA Paged KV allocation requires a CUDA device")
        if dtype not in _DTYPE_NAMES:
            raise ValueError(f"CUDA Paged KV allocation does not support dtype {dtype}")
        self._load()
        index = torch.cuda.current_device() if resolved.index is None else resolved.index
        owner = torch.classes.nanovllm_paged_kv.PagedKVCache(list(shape), _DTYPE_NAMES[dtype], index)
        return PagedKVAllocation(owner.tensor(), owner)

    def copy_slots_async(self, allocation: PagedKVAllocation, host_slots: torch.Tensor) -> torch.Tensor:
        if allocation.owner is None:
            raise ValueError("CUDA Paged KV allocation has no native owner")
        return allocation.owner.copy_slots_async(host_slots)

    def store(self, key, value, key_cache, value_cache, slot_mapping) -> None:
        validate_store_inputs(key, value, key_cache, value_cache, slot_mapping)
        if not key.is_cuda:
            raise ValueError("CUDA Paged KV Store requires CUDA tensors")
        ops.paged_store(key, value, key_cache, value_cache, slot_mapping)

    def gather(self, cache, block_table, sequence_length: int) -> torch.Tensor:
        validate_gather_inputs(cache, block_table, sequence_length)
        if not cache.is_cuda:
            raise ValueError("CUDA Paged KV Gather requires CUDA tensors")
        return ops.paged_gather(cache, block_table, sequence_length)

    def gather_varlen(self, cache, block_tables, seq_lens, cu_seqlens, total_tokens: int,
                      max_seq_len: int) -> torch.Tensor:
        """All sequences of a batch in one launch -> packed ``[total_tokens, kv_heads, D]``."""
        if not cache.is_cuda:
            raise ValueError("CUDA Paged KV Gather requires CUDA tensors")
        return ops.paged_gather_varlen(cache, block_tables, seq_lens, cu_seqlens, total_tokens,
                                       max_seq_len)
