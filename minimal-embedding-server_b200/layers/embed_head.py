"""``VocabParallelEmbedding`` (``layers/embed_head.py:7-52``).

The reference shards the vocabulary and all-reduces the masked lookups (one ``[T, H]``
all-reduce per forward).  Here every rank keeps the whole table (1.24 GB at bf16 for the
largest model, small next to 180 GB of HBM), so the lookup is a local gather with an
identical result and no collective.
"""
from __future__ import annotations

import torch
import torch.distributed as dist
from torch import nn

from .. import _C


class VocabParallelEmbedding(nn.Module):

    def __init__(self, num_embeddings: int, embedding_dim: int):
        super().__init__()
        if dist.is_available() and dist.is_initialized():
            self.tp_rank, self.tp_size = dist.get_rank(), dist.get_world_size()
        else:
            self.tp_rank, self.tp_size = 0, 1
        self.num_embeddings = num_embeddings
        self.embedding_dim = embedding_dim
        self.weight = nn.Parameter(torch.zeros(num_embeddings, embedding_dim,
                                               dtype=torch.bfloat16), requires_grad=False)
        self.weight.weight_loader = self.weight_loader

    def weight_loader(self, param: nn.Parameter, loaded_weight: torch.Tensor, *args):
        param.data.copy_(loaded_weight.to(param.dtype))

    def forward(self, x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        return _C.embedding(x, self.weight, out)

    def forward_f32(self, x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        """The lookup widened to fp32: the first value of the fp32 residual stream."""
        return _C.embedding_f32(x, self.weight, out)
