"""Attention backend interface and factory (``layers/attention/base.py:9-74``).

``create_attention`` keeps the reference's backend names.  The reference's two backends
call third-party kernels (sgl-kernel FlashAttention, FlashInfer); in this package every
name resolves to :class:`B200Attention`, the sm_100a tcgen05 kernel, so an existing
``MESConfig(attn_backend="flash_attn")`` works unchanged.
"""
from __future__ import annotations

from abc import ABC, abstractmethod

import torch
from torch import nn

BACKENDS = ("b200", "flash_attn", "flash_infer")


class BaseAttention(nn.Module, ABC):

    def __init__(self, num_heads: int, head_dim: int, scale: float, num_kv_heads: int):
        super().__init__()
        self.num_heads = num_heads
        self.head_dim = head_dim
        self.scale = scale
        self.num_kv_heads = num_kv_heads

    @abstractmethod
    def forward(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                positions: torch.Tensor) -> torch.Tensor:
        """``q [T, Hq*D]``, ``k``/``v [T, Hkv*D]`` of a packed batch whose sequences start
        where ``positions`` does not continue by +1 -> ``[T, Hq*D]``."""


def create_attention(num_heads: int, head_dim: int, scale: float, num_kv_heads: int,
                     attn_backend: str = "b200") -> BaseAttention:
    if attn_backend not in BACKENDS:
        raise ValueError(f"Unknown attention backend: {attn_backend}")
    from .b200 import B200Attention
    return B200Attention(num_heads, head_dim, scale, num_kv_heads)
