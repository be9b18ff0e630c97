"""1-D rotary embedding with the interface of ``nanovllm/layers/rotary_embedding.py``."""

from functools import lru_cache

import torch
from torch import nn

from nano_vllm_multimodal_b200 import ops


def apply_rotary_emb(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """Neox rotate-half of ``x [T, heads, D]`` by ``cos/sin [T, 1, D/2]`` (fp32 math).

    Same contract as ``rotary_embedding.py:6-14``: fp32 products and sums,
    one rounding to ``x.dtype``. Runs the generic rotation kernel with the
    three rotary axes all equal to the given table.
    """
    if x.dim() != 3 or cos.dim() != 3 or cos.shape != sin.shape or cos.shape[1] != 1:
        raise ValueError("apply_rotary_emb expects x [tokens, heads, head_dim] and cos/sin [tokens, 1, head_dim/2]")
    half = x.shape[-1] // 2
    if cos.shape[0] != x.shape[0] or cos.shape[-1] != half:
        raise ValueError("cos/sin must match the token count and half the head dimension")
    full_cos = torch.cat((cos, cos), dim=-1).squeeze(1).float().expand(3, -1, -1)
    full_sin = torch.cat((sin, sin), dim=-1).squeeze(1).float().expand(3, -1, -1)
    return ops.mrope_apply(x, full_cos, full_sin, (half, 0, 0), interleaved=False)


class RotaryEmbedding(nn.Module):
    """Neox RoPE from the fp32 ``cos_sin_cache`` table ``[max_position, 1, D]``.

    The table is built exactly as ``rotary_embedding.py:29-35`` builds it
    (cos of the first half, sin of the second); ``forward`` runs the fused
    prologue kernel in table mode, which reads the row of each position.
    """

    def __init__(self, head_size: int, rotary_dim: int, max_position_embeddings: int, base: float) -> None:
        super().__init__()
        self.head_size = head_size
        assert rotary_dim == head_size
        inv_freq = 1.0 / (base ** (torch.arange(0, rotary_dim, 2, dtype=torch.float) / rotary_dim))
        t = torch.arange(max_position_embeddings, dtype=torch.float)
        freqs = torch.einsum("i,j -> ij", t, inv_freq)
        cache = torch.cat((freqs.cos(), freqs.sin()), dim=-1).unsqueeze_(1)
        self.register_buffer("cos_sin_cache", cache, persistent=False)

    def forward(self, positions: torch.Tensor, query: torch.Tensor, key: torch.Tensor):
        if positions.dtype != torch.long:
            positions = positions.long()
        if ops.prologue_supported(query, key):
            return ops.rope(positions, query, key, self.cos_sin_cache)
        # unusual head size / layout: gather the table rows, generic rotation kernel
        cos_sin = self.cos_sin_cache[positions]
        cos, sin = cos_sin.chunk(2, dim=-1)
        return apply_rotary_emb(query, cos, sin), apply_rotary_emb(key, cos, sin)


@lru_cache(1)
def get_rope(head_size: int, rotary_dim: int, max_position: int, base: float):
    return RotaryEmbedding(head_size, rotary_dim, max_position, base)
