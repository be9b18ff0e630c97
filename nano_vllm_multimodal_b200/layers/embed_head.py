"""``VocabParallelEmbedding`` with the interface of ``nanovllm/layers/embed_head.py:9-42``."""

import torch
import torch.distributed as dist
from torch import nn

from nano_vllm_multimodal_b200 import ops


class VocabParallelEmbedding(nn.Module):
    """Token-id row gather; at tensor-parallel size > 1 each rank gathers the
    ids of its vocab shard (other ids give zero rows in the same kernel) and
    the partial rows are summed with ``all_reduce`` (``embed_head.py:34-42``)."""

    def __init__(self, num_embeddings: int, embedding_dim: int):
        super().__init__()
        self.tp_rank = dist.get_rank()
        self.tp_size = dist.get_world_size()
        assert num_embeddings % self.tp_size == 0
        self.num_embeddings = num_embeddings
        self.num_embeddings_per_partition = self.num_embeddings // self.tp_size
        self.vocab_start_idx = self.num_embeddings_per_partition * self.tp_rank
        self.vocab_end_idx = self.vocab_start_idx + self.num_embeddings_per_partition
        self.weight = nn.Parameter(torch.empty(self.num_embeddings_per_partition, embedding_dim))
        self.weight.weight_loader = self.weight_loader

    def weight_loader(self, param: nn.Parameter, loaded_weight: torch.Tensor):
        param_data = param.data
        shard_size = param_data.size(0)
        start_idx = self.tp_rank * shard_size
        param_data.copy_(loaded_weight.narrow(0, start_idx, shard_size))

    def forward(self, x: torch.Tensor):
        y = ops.embedding(x if x.dtype == torch.long else x.long(), self.weight,
                          self.vocab_start_idx, self.vocab_end_idx, mask=self.tp_size > 1)
        if self.tp_size > 1:
            dist.all_reduce(y)
        return y
