"""Vocab-parallel embedding and LM head (reference: src/layers/llm_head.py:1-69).

VocabParallelEmbedding keeps rows [rank * V/tp, (rank + 1) * V/tp) of the
table.  At tp 1 forward is the lookup kernel.  At tp > 1 the reference's
masked lookup + all_reduce is one exchange kernel over NVLink (the rank that
owns a token's row writes it into every rank's output) when the process has
the fused communicator and the batch fits its buffers, else the lookup +
torch.distributed.all_reduce.
ParallelLMHead takes the last token of every sequence in prefill and
multiplies by its vocab shard on the tcgen05 GEMM.  forward keeps the
reference's result (at tp > 1 the shards gathered to rank 0 and
concatenated; other ranks return None); select_tokens instead picks each
sequence's token on every rank from the local shards (greedy, or the
reference sampler's temperature sampling in its Gumbel-max form), so only
an 8-byte key per sequence crosses NVLink.
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
        if self.tp_world_size > 1:
            from src.layers import tp_comm
            comm = tp_comm.ensure(x.device, self.embedding_dim)
            if comm is not None and comm.can_exchange(x.numel(), self.embedding_dim):
                y = comm.embedding(x.reshape(-1), self.weight, self.vocab_start_idx,
                                   self.vocab_end_idx, self.num_embeddings)
                return y.view(*x.shape, self.embedding_dim)
        y = b200.embedding(x, self.weight, self.vocab_start_idx, self.vocab_end_idx)
        if self.tp_world_size > 1:
            dist.all_reduce(y)
        return y


class ParallelLMHead(VocabParallelEmbedding):

    def __init__(self, num_embeddings: int, embedding_dim: int, tp: tuple[int, int] = (0, 1)):
        super().__init__(num_embeddings, embedding_dim, tp)

    def select_tokens(self, x: torch.Tensor, ctx: Context, temperatures: torch.Tensor | None = None,
                      noise: torch.Tensor | None = None, seed: int = 0,
                      offset: int = 0) -> torch.Tensor:
        """int64 [B] tokens on every rank: the argmax (greedy, no
        temperatures) or the sample of src/layers/sampler.py:4-17 over the
        full vocabulary, computed from this rank's logits shard.  `noise`
        ([B, V/tp] fp32 Exp(1) draws of this shard) replaces the in-kernel
        Philox draws keyed by (seed, offset)."""
        if ctx.is_prefill:
            x = x[ctx.cu_seqlens_q[1:] - 1].contiguous()
        logits = b200.linear(x, self.weight)
        if self.tp_world_size == 1:
            if temperatures is None and noise is None:
                return b200.argmax(logits)
            return b200.tokens_from_keys(b200.select_tokens(logits, 0, temperatures, noise, seed,
                                                            offset))
        from src.layers import tp_comm
        comm = tp_comm.get()
        if comm is not None and comm.can_exchange(logits.shape[0]):
            return comm.select_tokens(logits, self.vocab_start_idx, temperatures, noise, seed, offset)
        keys = b200.select_tokens(logits, self.vocab_start_idx, temperatures, noise, seed, offset)
        dist.all_reduce(keys, op=dist.ReduceOp.MAX)
        return b200.tokens_from_keys(keys)

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
