"""Token selection from logits [B, V].

Sampler keeps the reference's temperature sampling (src/layers/sampler.py:4-17:
softmax(logits / T) divided by Exp(1) noise, argmax -- the Gumbel-max form) in
torch; `greedy` is the argmax kernel used by the greedy decode benchmark.
"""
import torch
from torch import nn

from src import b200


class Sampler(nn.Module):

    def forward(self, logits: torch.Tensor, temperatures: torch.Tensor) -> torch.Tensor:
        scaled = logits.float().div_(temperatures.unsqueeze(dim=1))
        probs = torch.softmax(scaled, dim=-1)
        noise = torch.empty_like(probs).exponential_(1).clamp_min_(1e-10)
        return probs.div_(noise).argmax(dim=-1)


def greedy(logits: torch.Tensor) -> torch.Tensor:
    return b200.argmax(logits)
