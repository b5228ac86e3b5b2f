"""RMSNorm with the reference's interface (``layers/layernorm.py:7-51``).

``forward(x)`` computes ``bf16(bf16(x * rsqrt(mean(x^2) + eps)) * w)`` with fp32
statistics (``rms_forward:18-27``); ``forward(x, residual)`` first forms the fp32 sum
``s = x + residual``, returns ``bf16(s)`` as the new residual and normalises ``s``
(``add_rms_forward:30-41``).  Both run as one fused sm_100a kernel.  Inputs are not
modified unless the caller passes ``out=`` / ``residual_out=`` buffers that alias them.

``residual_norm`` serves the model's fp32 residual stream: it normalises the fp32
residual (optionally adding a bf16 delta to it first, in place) and returns bf16.
"""
from __future__ import annotations

import torch
from torch import nn

from .. import _C


class RMSNorm(nn.Module):

    def __init__(self, hidden_size: int, eps: float = 1e-6) -> None:
        super().__init__()
        self.hidden_size = hidden_size
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(hidden_size, dtype=torch.bfloat16),
                                   requires_grad=False)

    def rms_forward(self, x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        shape = x.shape
        y = _C.rmsnorm(x.reshape(-1, shape[-1]), self.weight,
                       self.eps, None if out is None else out.view(-1, shape[-1]))
        return y.view(shape)

    def add_rms_forward(self, x: torch.Tensor, residual: torch.Tensor,
                        out: torch.Tensor | None = None,
                        residual_out: torch.Tensor | None = None):
        return _C.add_rmsnorm(x, residual, self.weight, self.eps, out, residual_out)

    def residual_norm(self, residual: torch.Tensor, delta: torch.Tensor | None = None,
                      out: torch.Tensor | None = None) -> torch.Tensor:
        """bf16 RMSNorm of the fp32 ``residual`` (after ``residual += delta`` if given)."""
        if delta is None:
            return _C.rmsnorm(residual, self.weight, self.eps, out)
        return _C.add_rmsnorm_f32res(delta, residual, self.weight, self.eps, out)

    def forward(self, x: torch.Tensor, residual: torch.Tensor | None = None, *,
                out: torch.Tensor | None = None, residual_out: torch.Tensor | None = None):
        if residual is None:
            return self.rms_forward(x, out)
        return self.add_rms_forward(x, residual, out, residual_out)
