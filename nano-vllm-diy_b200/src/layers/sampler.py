"""Token selection from logits [B, V] (reference: src/layers/sampler.py:4-17).

Sampler keeps the reference's interface -- Sampler()(logits, temperatures)
on the logits ParallelLMHead returns -- and its arithmetic in the Gumbel-max
form: argmax_j softmax(l / T)_j / E_j = argmax_j (l_j / T - ln E_j) with
E ~ Exp(1) (softmax's normaliser is common to the row).  One kernel per
call: the Exp(1) draws come from Philox-4x32-10 inside the kernel (a fresh
offset per call), or from `noise` when the caller passes the draws (the
reference draws them with `exponential_`), which reproduces the reference's
choice for those draws.  `greedy` is the argmax kernel.
"""
import torch
from torch import nn

from src import b200


class Sampler(nn.Module):

    def __init__(self, seed: int | None = None):
        super().__init__()
        self.seed = int(torch.randint(0, 2 ** 62, (1,)).item()) if seed is None else int(seed)
        self.calls = 0

    def forward(self, logits: torch.Tensor, temperatures: torch.Tensor,
                noise: torch.Tensor | None = None) -> torch.Tensor:
        temperatures = temperatures.to(torch.float32)
        keys = b200.select_tokens(logits, 0, temperatures, noise, self.seed, self.calls)
        self.calls += 1
        return b200.tokens_from_keys(keys)


def greedy(logits: torch.Tensor) -> torch.Tensor:
    return b200.argmax(logits)
