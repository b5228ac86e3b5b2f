"""NeoX rotary embedding with the reference's interface (``layers/rotary_embedding.py``).

``RotaryEmbedding`` builds the same fp32 ``cos_sin_cache [max_position, head_size]``
(``:29-37``; ``model.to(bf16)`` turns it into the bf16 cache the reference's GPU path
reads, and the kernel accepts either).  ``forward(positions, query, key)`` rotates
``query`` and ``key`` in place and returns them (``:39-55``); ``forward_fused`` applies the
Qwen3 per-head q/k RMSNorm and the rotation in one kernel over the packed QKV buffer.
``get_rope`` keeps the reference's one-instance cache (``:58-68``).
"""
from __future__ import annotations

from functools import lru_cache

import torch
from torch import nn

from .. import _C


class RotaryEmbedding(nn.Module):

    def __init__(self, head_size: int, rotary_dim: int, max_position_embeddings: int,
                 base: float) -> None:
        super().__init__()
        self.head_size = head_size
        assert rotary_dim == head_size
        inv_freq = 1.0 / (base ** (torch.arange(0, rotary_dim, 2, dtype=torch.float) / rotary_dim))
        t = torch.arange(max_position_embeddings, dtype=torch.float)
        freqs = torch.einsum("i,j -> ij", t, inv_freq)
        cache = torch.cat((freqs.cos(), freqs.sin()), dim=-1)
        self.register_buffer("cos_sin_cache", cache, persistent=False)

    def _rotate(self, x: torch.Tensor, positions: torch.Tensor, nq: int, nk: int,
                q_weight=None, k_weight=None, eps: float = 1e-6):
        return _C.qknorm_rope(x, positions, self.cos_sin_cache.contiguous(), nq, nk,
                              self.head_size, q_weight, k_weight, eps)

    def forward(self, positions: torch.Tensor, query: torch.Tensor, key: torch.Tensor):
        D = self.head_size
        T = positions.shape[0]
        q2 = query.view(T, -1)
        k2 = key.view(T, -1)
        nq, nk = q2.shape[1] // D, k2.shape[1] // D
        if (q2.stride(0) == k2.stride(0) and q2.stride(1) == 1 and k2.stride(1) == 1
                and k2.data_ptr() == q2.data_ptr() + nq * D * q2.element_size()):
            self._rotate(q2, positions, nq, nk)  # q and k are adjacent views of one buffer
        else:
            self._rotate(q2, positions, nq, 0)
            self._rotate(k2, positions, 0, nk)
        return query, key

    def forward_fused(self, positions: torch.Tensor, qkv: torch.Tensor, num_heads: int,
                      num_kv_heads: int, q_norm=None, k_norm=None) -> torch.Tensor:
        """In place on the packed ``[T, (Hq + 2 Hkv) * D]`` QKV buffer: optional per-head
        RMSNorm (``q_norm``/``k_norm`` modules) then RoPE of the q and k heads."""
        eps = q_norm.eps if q_norm is not None else 1e-6
        return self._rotate(qkv, positions, num_heads, num_kv_heads,
                            None if q_norm is None else q_norm.weight,
                            None if k_norm is None else k_norm.weight, eps)


@lru_cache(1)
def get_rope(head_size: int, rotary_dim: int, max_position: int, base: float,
             rope_scaling: dict | None = None):
    assert rope_scaling is None
    return RotaryEmbedding(head_size, rotary_dim, max_position, base)
