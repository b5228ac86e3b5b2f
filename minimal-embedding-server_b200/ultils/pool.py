"""Last-token pooling (``ultils/pool.py:4-9`` of the reference) and the fused pooled L2
normalisation the GPU worker's post-process runs (``core/gpu_worker.py:252-261``).

``last_token_pool`` keeps the reference's signature for one sequence's hidden states.
``last_token_l2`` pools a whole packed batch at once: it gathers the row of each
sequence's last token and divides it by ``max(||x||_2, 1e-12)`` in one sm_100a kernel
(``mes_last_token_l2``), producing fp32 on the device.
"""
from __future__ import annotations

import torch

from .. import _C


def last_token_pool(hidden_states: torch.Tensor, seq_len: int) -> torch.Tensor:
    """The hidden state of the last of ``seq_len`` tokens (``pool.py:4-9``)."""
    return hidden_states[seq_len - 1]


def last_token_l2(hidden_states: torch.Tensor, last_token_indices: torch.Tensor,
                  out: torch.Tensor | None = None) -> torch.Tensor:
    """fp32 ``[B, H]``: ``F.normalize(hidden_states[last_token_indices], p=2, dim=1)`` for a
    packed bf16 ``[T, H]`` batch and int64 device indices ``[B]``."""
    return _C.last_token_l2(hidden_states, last_token_indices, out)
