"""``RMSNorm`` with the interface of ``nanovllm/layers/layernorm.py:6-50``."""

import torch
from torch import nn

from nano_vllm_multimodal_b200 import ops


class RMSNorm(nn.Module):
    """RMSNorm over the last dim, optionally fused with the residual add.

    ``forward(x)`` -> normed ``x`` (``rms_forward``, layernorm.py:16-26);
    ``forward(x, residual)`` -> ``(normed(x + residual), x + residual)``
    (``add_rms_forward``, layernorm.py:28-40). Inputs are never modified.
    """

    def __init__(self, hidden_size: int, eps: float = 1e-6) -> None:
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(hidden_size))

    def rms_forward(self, x: torch.Tensor) -> torch.Tensor:
        return ops.rms_norm(x, self.weight, self.eps)

    def add_rms_forward(self, x: torch.Tensor, residual: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        return ops.add_rms_norm(x, residual, self.weight, self.eps, round_sum=False)

    def forward(self, x: torch.Tensor, residual: torch.Tensor | None = None):
        if residual is None:
            return self.rms_forward(x)
        return self.add_rms_forward(x, residual)
