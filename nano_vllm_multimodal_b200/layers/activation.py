"""``SiluAndMul`` with the interface of ``nanovllm/layers/activation.py:6-11``."""

import torch
from torch import nn

from nano_vllm_multimodal_b200 import ops


class SiluAndMul(nn.Module):
    """``silu(x[..., :I]) * x[..., I:]``, fp32 math rounded once."""

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return ops.silu_and_mul(x)
