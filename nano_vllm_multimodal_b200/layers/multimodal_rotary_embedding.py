"""Multimodal RoPE with the interface of ``nanovllm/layers/multimodal_rotary_embedding.py``.

Both frequency layouts are supported: ``chunked`` (Qwen2.5-VL, sections
``[t, h, w]`` as contiguous chunks of each half head) and ``interleaved``
(Qwen3-VL, frequency ``j`` takes H when ``j % 3 == 1`` and W when
``j % 3 == 2`` inside their section ranges, T elsewhere). Error messages are
the reference's, so callers that match on them keep working.
"""

from __future__ import annotations

import torch
from torch import nn

from nano_vllm_multimodal_b200 import ops

_STRATEGY_ERROR = "multimodal rotary strategy must be 'chunked' or 'interleaved'"


def rotate_half(x: torch.Tensor) -> torch.Tensor:
    first, second = x.chunk(2, dim=-1)
    return torch.cat((-second, first), dim=-1)


def apply_multimodal_rotary_emb(query, key, cos, sin, sections, strategy: str = "chunked"):
    """Rotate ``query``/``key`` by caller-supplied ``cos``/``sin`` ``[3, T, D]``.

    Validation mirrors ``multimodal_rotary_embedding.py:20-31``; the rotation
    runs the generic M-RoPE kernel (any even head dim, any float dtypes):
    chunked in fp32, interleaved in the promoted dtype of the tensor and cos,
    rounding every product and the sum as eager PyTorch does.
    """
    if query.ndim != 3 or key.ndim != 3:
        raise ValueError("query and key must have shape [num_tokens, num_heads, head_dim]")
    if cos.ndim != 3 or sin.ndim != 3 or cos.shape != sin.shape:
        raise ValueError("cos and sin must have equal shape [3, num_tokens, head_dim]")
    if cos.shape[0] != 3 or cos.shape[1] != query.shape[0]:
        raise ValueError("rotary positions must match the query token count")
    if query.shape[-1] != key.shape[-1] or query.shape[-1] != cos.shape[-1]:
        raise ValueError("query, key, cos, and sin must use the same head dimension")
    sections = tuple(sections)
    if 2 * sum(sections) != query.shape[-1]:
        raise ValueError("multimodal rotary sections must cover the head dimension")
    if strategy not in {"chunked", "interleaved"}:
        raise ValueError(_STRATEGY_ERROR)
    inter = strategy == "interleaved"
    return (ops.mrope_apply(query, cos, sin, sections, inter),
            ops.mrope_apply(key, cos, sin, sections, inter))


class MultimodalRotaryEmbedding(nn.Module):
    """3-axis rotary embedding; ``forward`` is one fused kernel launch.

    ``inv_freq`` is built with the reference's recipe
    (``multimodal_rotary_embedding.py:70-86``): fp32 ``1 / base**(2i/D)``,
    computed on the CPU for the interleaved layout and on the default device
    for the chunked one, then moved to the default device.
    """

    def __init__(self, *, head_dim: int, base: float, sections: tuple[int, int, int],
                 strategy: str = "chunked") -> None:
        super().__init__()
        if head_dim <= 0 or head_dim % 2:
            raise ValueError("head_dim must be a positive even number")
        if len(sections) != 3 or any(section <= 0 for section in sections):
            raise ValueError("sections must contain three positive dimensions")
        if sum(sections) != head_dim // 2:
            raise ValueError("multimodal rotary sections must sum to half the head dimension")
        if strategy not in {"chunked", "interleaved"}:
            raise ValueError(_STRATEGY_ERROR)
        self.head_dim = head_dim
        self.sections = tuple(sections)
        self.strategy = strategy
        frequency_device = torch.get_default_device()
        construction_device = "cpu" if strategy == "interleaved" else frequency_device
        inv_freq = 1.0 / (base ** (torch.arange(0, head_dim, 2, dtype=torch.float32,
                                                device=construction_device) / head_dim))
        if inv_freq.device != frequency_device:
            inv_freq = inv_freq.to(frequency_device)
        self.register_buffer("inv_freq", inv_freq, persistent=False)

    @staticmethod
    def _int_positions(positions: torch.Tensor) -> torch.Tensor:
        if positions.dtype == torch.long:
            return positions
        if positions.is_floating_point():
            raise ValueError("positions must be an integer tensor")
        return positions.long()

    @torch.no_grad()
    def cos_sin(self, positions: torch.Tensor, dtype: torch.dtype):
        if positions.ndim != 2 or positions.shape[0] != 3:
            raise ValueError("positions must have shape [3, num_tokens]")
        pos = self._int_positions(positions).to(self.inv_freq.device)
        return ops.mrope_cos_sin(pos, self.inv_freq, dtype)

    def forward(self, positions: torch.Tensor, query: torch.Tensor, key: torch.Tensor):
        if positions.ndim != 2 or positions.shape[0] != 3:
            raise ValueError("positions must have shape [3, num_tokens]")
        if query.ndim != 3 or key.ndim != 3:
            raise ValueError("query and key must have shape [num_tokens, num_heads, head_dim]")
        if positions.shape[1] != query.shape[0]:
            raise ValueError("rotary positions must match the query token count")
        if query.shape[-1] != key.shape[-1] or query.shape[-1] != self.head_dim:
            raise ValueError("query, key, cos, and sin must use the same head dimension")
        pos = self._int_positions(positions)
        if ops.prologue_supported(query, key):
            return ops.mrope(pos, query, key, self.inv_freq, self.sections, self.strategy)
        # unusual head size / layout: materialise cos/sin, generic rotation kernel
        cos, sin = self.cos_sin(pos, query.dtype)
        return apply_multimodal_rotary_emb(query, key, cos, sin, self.sections, self.strategy)
