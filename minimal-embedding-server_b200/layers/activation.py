"""``SiluAndMul`` (``layers/activation.py:6-14``): ``silu(x[..., :I]) * x[..., I:]`` in fp32,
rounded once to bf16, as one sm_100a kernel."""
from __future__ import annotations

import torch
from torch import nn

from .. import _C


class SiluAndMul(nn.Module):

    def forward(self, x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        return _C.silu_mul(x, out)
