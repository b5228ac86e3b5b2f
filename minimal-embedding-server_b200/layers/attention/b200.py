"""Varlen causal GQA prefill attention backend on sm_100a (``mes_varlen_attention``).

Replaces ``FlashAttention.forward`` (``layers/attention/flashattention.py:19-48``) and
``FlashInferAttention.forward`` (``layers/attention/flashinfer.py:55-101``).  The
reference derives ``cu_seqlens`` from position jumps on the host, with one ``.item()``
synchronisation per sequence boundary, in every layer.  Here ``mes_varlen_schedule`` does
it on the device once per forward: the model opens a :func:`batch_schedule` context and
every layer reuses the same workspace; called outside such a context the layer schedules
its own batch.
"""
from __future__ import annotations

import contextlib
import threading

import torch

from ... import _C
from .base import BaseAttention

_state = threading.local()


@contextlib.contextmanager
def batch_schedule(positions: torch.Tensor):
    """Schedule one packed batch on the device and share it with every attention layer
    called inside the ``with`` block for this ``positions`` tensor.  Contexts nest, so the
    micro-batches of one forward can each hold their own schedule."""
    prev = getattr(_state, "current", ())
    entry = (positions, _C.varlen_schedule(positions))
    _state.current = prev + (entry,)
    try:
        yield entry[1]
    finally:
        _state.current = prev


def _workspace_for(positions: torch.Tensor) -> torch.Tensor:
    for pos, ws in reversed(getattr(_state, "current", ())):
        if pos is positions:
            return ws
    return _C.varlen_schedule(positions)


class B200Attention(BaseAttention):

    def forward(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                positions: torch.Tensor) -> torch.Tensor:
        T = positions.shape[0]
        D = self.head_dim
        q2, k2, v2 = q.view(T, -1), k.view(T, -1), v.view(T, -1)
        esz = q2.element_size()
        packed = (q2.stride(1) == 1 and q2.stride(0) == k2.stride(0) == v2.stride(0)
                  and k2.data_ptr() == q2.data_ptr() + self.num_heads * D * esz
                  and v2.data_ptr() == k2.data_ptr() + self.num_kv_heads * D * esz
                  and q2.data_ptr() % 16 == 0 and q2.stride(0) % 8 == 0)
        if packed:
            qkv = q2.as_strided((T, (self.num_heads + 2 * self.num_kv_heads) * D),
                                (q2.stride(0), 1))
        else:
            qkv = torch.cat([q2, k2, v2], dim=1)
        return _C.varlen_attention(qkv, _workspace_for(positions), self.num_heads,
                                   self.num_kv_heads, D, self.scale)

    def forward_packed(self, qkv: torch.Tensor, positions: torch.Tensor,
                       out: torch.Tensor | None = None) -> torch.Tensor:
        """Attention straight from the packed ``[T, (Hq + 2 Hkv) * D]`` QKV buffer."""
        return _C.varlen_attention(qkv, _workspace_for(positions), self.num_heads,
                                   self.num_kv_heads, self.head_dim, self.scale, out)
