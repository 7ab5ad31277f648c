"""SiLU-and-mul (reference: src/layers/activation.py:6-10)."""
import torch
from torch import nn

from src import b200


class SiluAndMul(nn.Module):

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return b200.silu_and_mul(x)
