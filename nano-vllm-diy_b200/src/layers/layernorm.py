"""RMSNorm on the sm_100a kernel (reference: src/layers/layernorm.py:4-39).

forward(x) -> bf16(w * x / sqrt(mean(x^2) + eps))
forward(x, residual) -> (norm(x + residual), bf16(x + residual)), the sum
taken in fp32 as in RMSNorm.residual_forward.
"""
from __future__ import annotations

import torch
from torch import nn

from src import b200


class RMSNorm(nn.Module):

    def __init__(self, dim: int, eps: float = 1e-8) -> None:
        super().__init__()
        self.weight = nn.Parameter(torch.ones(dim), requires_grad=False)
        self.eps = eps

    def forward(self, x: torch.Tensor, residual: torch.Tensor | None = None):
        if residual is None:
            return b200.rms_norm(x, self.weight, self.eps)
        return b200.rms_norm(x, self.weight, self.eps, residual=residual)
