"""A step's host -> device inputs in one pinned staging copy.

The reference builds each per-step input array as its own pinned tensor and
copies it with its own non-blocking ``.cuda()``
(``nanovllm/engine/model_runner.py:700-725,823-870`` for prefill: token ids,
positions, cu_seqlens_q/k, slot mapping, context lengths, query starts, block
tables; ``model_runner.py:892-935`` for decode: token ids, positions, slot
mapping, context lengths, block tables).
:class:`StepInputStager` converts the arrays once into contiguous host arrays,
writes them into one slot of a small ring of pinned buffers and moves the slot
with one ``cudaMemcpyAsync`` into one device allocation; the returned tensors
are views of it, with the dtypes and shapes the reference's tensors have.
The native part is ``torch.classes.nanoinfer_b200.StepInputStager``.
"""

from __future__ import annotations

import array

import numpy as np
import torch

from nano_vllm_multimodal_b200._lib import load_ops

_NP = {torch.int64: np.int64, torch.int32: np.int32, torch.float32: np.float32}
_CODE = {torch.int64: "q", torch.int32: "i", torch.float32: "f"}  # array module type codes


def host_array(values, dtype: torch.dtype) -> torch.Tensor:
    """A contiguous CPU tensor of `dtype` from a list or tuple (of equal-length
    lists or tuples for 2-D, e.g. the decode position rows of
    model_runner.py:326-337), a numpy array or a tensor. Python sequences go
    through the ``array`` module, which converts ints about 1.6x faster than
    numpy."""
    if isinstance(values, torch.Tensor):
        return values.to(dtype=dtype, device="cpu").contiguous()
    if isinstance(values, (list, tuple)) and values:
        if isinstance(values[0], (list, tuple)):
            n = len(values[0])
            if n and all(len(r) == n for r in values):
                out = np.empty((len(values), n), dtype=_NP[dtype])
                for i, r in enumerate(values):  # per-row arrays: the list fast path
                    out[i] = np.frombuffer(array.array(_CODE[dtype], r), dtype=_NP[dtype])
                return torch.from_numpy(out)
        elif not isinstance(values[0], (list, tuple)):
            return torch.frombuffer(array.array(_CODE[dtype], values), dtype=dtype)
    return torch.from_numpy(np.ascontiguousarray(np.asarray(values, dtype=_NP[dtype])))


class StepInputStager:
    def __init__(self, device=None, slots: int = 3, initial_bytes: int = 1 << 20) -> None:
        load_ops()
        dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        if dev.index is None:
            dev = torch.device("cuda", torch.cuda.current_device())
        self.device = dev
        self._native = torch.classes.nanoinfer_b200.StepInputStager(dev.index, int(slots), int(initial_bytes))

    def stage(self, *arrays) -> list[torch.Tensor]:
        """Device tensors with the same values, dtypes and shapes as the given CPU
        tensors (or ``(values, dtype)`` pairs), from one pinned staging copy on the
        current stream."""
        host = [host_array(a[0], a[1]) if isinstance(a, tuple) else a for a in arrays]
        return list(self._native.stage(host))

    def slot_bytes(self) -> list[int]:
        return [self._native.slot_bytes(i) for i in range(self._native.slots())]

    def prefill_inputs(self, input_ids, position_rows, cu_seqlens_q, cu_seqlens_k, slot_mapping,
                       full_context_lens, query_start_lens, block_tables=None, position_axes: int = 1):
        """The tensors ``ModelRunner.prepare_prefill`` creates (model_runner.py:823-870),
        staged together: a dict with ``input_ids`` (int64 [T]), ``positions`` (int64
        [T] when ``position_axes == 1`` else [axes, T]), ``cu_seqlens_q``,
        ``cu_seqlens_k``, ``slot_mapping``, ``full_context_lens``,
        ``query_start_lens`` (int32) and ``block_tables`` (int32 [B, max], rows
        padded with -1 as model_runner.py:700-705, or None)."""
        names = ["input_ids", "positions", "cu_seqlens_q", "cu_seqlens_k", "slot_mapping",
                 "full_context_lens", "query_start_lens"]
        arrays = [(input_ids, torch.int64), (position_rows, torch.int64), (cu_seqlens_q, torch.int32),
                  (cu_seqlens_k, torch.int32), (slot_mapping, torch.int32), (full_context_lens, torch.int32),
                  (query_start_lens, torch.int32)]
        if block_tables is not None:
            names.append("block_tables")
            arrays.append((_padded_tables(block_tables), torch.int32))
        out = dict(zip(names, self.stage(*arrays)))
        if position_axes == 1 and out["positions"].dim() == 2:
            out["positions"] = out["positions"][0]
        out.setdefault("block_tables", None)
        return out

    def decode_inputs(self, input_ids, position_rows, slot_mapping, context_lens, block_tables,
                      position_axes: int = 1):
        """The tensors ``ModelRunner.prepare_decode`` creates (model_runner.py:892-935),
        one token per sequence, staged together: a dict with ``input_ids`` (int64 [B]),
        ``positions`` (int64 [B] when ``position_axes == 1`` else [axes, B]),
        ``slot_mapping`` and ``context_lens`` (int32 [B]) and ``block_tables`` (int32
        [B, max], rows padded with -1 as model_runner.py:696-707). The reference makes
        five pinned tensors and five copies for these every decode step."""
        names = ["input_ids", "positions", "slot_mapping", "context_lens", "block_tables"]
        arrays = [(input_ids, torch.int64), (position_rows, torch.int64), (slot_mapping, torch.int32),
                  (context_lens, torch.int32), (_padded_tables(block_tables), torch.int32)]
        out = dict(zip(names, self.stage(*arrays)))
        if position_axes == 1 and out["positions"].dim() == 2:
            out["positions"] = out["positions"][0]
        return out


def _padded_tables(block_tables) -> np.ndarray:
    """Block tables as one int32 [B, max] array, rows padded with -1
    (model_runner.py:696-707)."""
    width = max((len(b) for b in block_tables), default=0)
    padded = np.full((len(block_tables), width), -1, dtype=np.int32)
    for i, b in enumerate(block_tables):
        padded[i, :len(b)] = b
    return padded
