"""Qwen3-VL pieces of the hot path: the text RMSNorm and the DeepStack add.

Interfaces of ``nanovllm/models/qwen3_vl.py:68-79`` (``Qwen3VLTextRMSNorm``)
and ``:332-344`` (``Qwen3VLLanguageModel._add_deepstack_rows``).
"""

import torch
from torch import nn

from nano_vllm_multimodal_b200 import ops


class Qwen3VLTextRMSNorm(nn.Module):
    """``weight * normalize(x).to(dtype)``; numerically the same kernel as RMSNorm.

    ``forward(x, residual)`` (an addition to the reference interface) folds the
    Qwen3-VL decoder's separate ``hidden + residual`` (one dtype rounding,
    ``qwen3_vl.py:232-237``) into the same pass and returns
    ``(normed, hidden + residual)``.

    ``forward(x, residual, deepstack=(visual_embedding, row_index))`` also folds
    the DeepStack add that the reference applies to the previous layer's output
    (``qwen3_vl.py:371-376``): tokens with ``row_index[t] >= 0`` add
    ``visual_embedding[row_index[t]]`` to the rounded sum before the norm.
    ``row_index`` comes from :func:`deepstack_row_index`.
    """

    def __init__(self, hidden_size: int, eps: float = 1e-6) -> None:
        super().__init__()
        self.weight = nn.Parameter(torch.ones(hidden_size))
        self.eps = eps

    def _check_dtype(self, x: torch.Tensor) -> None:
        if self.weight.dtype != x.dtype:
            raise TypeError("Qwen3VLTextRMSNorm: weight dtype must match the activations "
                            f"({self.weight.dtype} vs {x.dtype})")

    def forward(self, hidden_states: torch.Tensor, residual: torch.Tensor | None = None,
                deepstack: tuple[torch.Tensor, torch.Tensor] | None = None):
        self._check_dtype(hidden_states)
        if deepstack is not None:
            if residual is None:
                raise ValueError("Qwen3VLTextRMSNorm: the DeepStack fold needs the residual")
            visual_embedding, row_index = deepstack
            return ops.add_rms_norm_deepstack(hidden_states, residual, self.weight, self.eps,
                                              visual_embedding, row_index)
        if residual is None:
            return ops.rms_norm(hidden_states, self.weight, self.eps)
        return ops.add_rms_norm(hidden_states, residual, self.weight, self.eps, round_sum=True)


def deepstack_row_index(visual_token_rows: torch.Tensor, num_tokens: int) -> torch.Tensor:
    """Token -> visual-row map (int32 ``[num_tokens]``, ``-1`` for text tokens) for
    ``Qwen3VLTextRMSNorm.forward(..., deepstack=...)``. The rows are the same for
    the three DeepStack layers, so one map serves all of them."""
    return ops.deepstack_row_index(visual_token_rows, num_tokens)


def add_deepstack_rows(hidden_states: torch.Tensor, visual_token_rows: torch.Tensor,
                       visual_embedding: torch.Tensor) -> torch.Tensor:
    """Out of place, like the reference: no rows -> the input object itself;
    otherwise a new tensor with ``visual_embedding[j]`` added at row
    ``visual_token_rows[j]`` (one dtype rounding). The input is not modified."""
    if visual_token_rows.numel() == 0:
        return hidden_states
    return ops.deepstack_add(hidden_states, visual_token_rows, visual_embedding)


def add_deepstack_rows_(hidden_states: torch.Tensor, visual_token_rows: torch.Tensor,
                        visual_embedding: torch.Tensor) -> torch.Tensor:
    """In place on a hidden-state tensor the caller owns (moves only the
    visual rows: 6 bytes x hidden per row for bf16); returns it."""
    if visual_token_rows.numel() == 0:
        return hidden_states
    return ops.deepstack_add_(hidden_states, visual_token_rows, visual_embedding)
