"""Vocab-parallel embedding and LM head (reference: src/layers/llm_head.py:1-69).

VocabParallelEmbedding keeps rows [rank * V/tp, (rank + 1) * V/tp) of the
table; forward gathers them on the GPU (rows of other shards are zero) and,
at tp > 1, sums over ranks with torch.distributed.all_reduce.
ParallelLMHead takes the last token of every sequence in prefill, multiplies
by its vocab shard on the tcgen05 GEMM, and at tp > 1 gathers the shards to
rank 0 and concatenates them (other ranks return None).
"""
from __future__ import annotations

import torch
import torch.distributed as dist
from torch import nn

from src import b200
from src.utils.context import Context
from src.utils.math import divide


class VocabParallelEmbedding(nn.Module):

    def __init__(self, num_embeddings: int, embedding_dim: int, tp: tuple[int, int] = (0, 1)):
        super().__init__()
        self.num_embeddings = num_embeddings
        self.embedding_dim = embedding_dim
        self.tp_rank, self.tp_world_size = tp
        self.num_embeddings_per_partition = divide(num_embeddings, self.tp_world_size)
        self.vocab_start_idx = self.tp_rank * self.num_embeddings_per_partition
        self.vocab_end_idx = self.vocab_start_idx + self.num_embeddings_per_partition
        self.weight = nn.Parameter(torch.empty(self.num_embeddings_per_partition, embedding_dim),
                                   requires_grad=False)
        self.weight.weight_loader = self.weight_loader

    def weight_loader(self, param: nn.Parameter, loaded_weight: torch.Tensor):
        assert loaded_weight.shape[0] == self.num_embeddings, (
            f"Expected weight shape[0] {self.num_embeddings}, but got {loaded_weight.shape[0]}")
        assert loaded_weight.shape[1] == self.embedding_dim, (
            f"Expected weight shape[1] {self.embedding_dim}, but got {loaded_weight.shape[1]}")
        n = self.num_embeddings_per_partition
        param.data.copy_(loaded_weight.narrow(0, self.tp_rank * n, n))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        y = b200.embedding(x, self.weight, self.vocab_start_idx, self.vocab_end_idx)
        if self.tp_world_size > 1:
            dist.all_reduce(y)
        return y


class ParallelLMHead(VocabParallelEmbedding):

    def __init__(self, num_embeddings: int, embedding_dim: int, tp: tuple[int, int] = (0, 1)):
        super().__init__(num_embeddings, embedding_dim, tp)

    def forward(self, x: torch.Tensor, ctx: Context) -> torch.Tensor | None:
        if ctx.is_prefill:
            x = x[ctx.cu_seqlens_q[1:] - 1].contiguous()
        logits = b200.linear(x, self.weight)
        if self.tp_world_size > 1:
            parts = ([torch.empty_like(logits) for _ in range(self.tp_world_size)]
                     if self.tp_rank == 0 else None)
            dist.gather(logits, parts, 0)
            logits = torch.cat(parts, -1) if self.tp_rank == 0 else None
        return logits
