"""Paged varlen attention and the KV-cache scatter (reference:
src/layers/attention.py:1-104).

store_kvcache(key, value, k_cache, v_cache, slot_mapping) writes each token's
K/V row to cache.view(-1, Hkv * d)[slot] with 16-byte vector stores and skips
slot -1.  Attention.forward(q, k, v, ctx) scatters when the cache is
allocated, then attends causally (bottom-right aligned) with GQA, reading K/V
from the paged cache through ctx.block_tables when they are set and from the
per-token k / v otherwise -- flash_attn_varlen_func's contract at
attention.py:93-104, on the sm_100a kernels.
"""
from __future__ import annotations

import torch
from torch import nn

from src import b200
from src.utils.context import Context


def store_kvcache(key: torch.Tensor, value: torch.Tensor, k_cache: torch.Tensor,
                  v_cache: torch.Tensor, slot_mapping: torch.Tensor) -> None:
    # key/value: (batch_seq_len, num_kv_heads, head_dim)
    # k_cache/v_cache: (num_blocks, block_size, num_kv_heads, head_dim)
    b200.store_kvcache(key, value, k_cache, v_cache, slot_mapping)


def attend(q: torch.Tensor, k: torch.Tensor | None, v: torch.Tensor | None,
           k_cache: torch.Tensor, v_cache: torch.Tensor, ctx: Context, scale: float,
           out: torch.Tensor | None = None) -> torch.Tensor:
    """Attention over the batch described by ctx (no cache write)."""
    if ctx.block_tables is not None:
        return b200.paged_attention(q, None, None, k_cache, v_cache, ctx.cu_seqlens_q,
                                    ctx.cu_seqlens_k, ctx.max_seqlen_q, ctx.max_seqlen_k, scale,
                                    ctx.block_tables, out=out)
    return b200.paged_attention(q, k, v, None, None, ctx.cu_seqlens_q, ctx.cu_seqlens_k,
                                ctx.max_seqlen_q, ctx.max_seqlen_k, scale, None, out=out)


class Attention(nn.Module):

    def __init__(self, head_dim: int, num_heads: int, num_kv_heads: int, scale: float = None):
        super().__init__()
        self.head_dim = head_dim
        self.num_heads = num_heads
        self.num_kv_heads = num_kv_heads
        self.scale = scale if scale is not None else head_dim ** -0.5
        # ModelRunner.allocate_kv_cache assigns views of its cache to every
        # module that has both attributes; empty until then.
        self.k_cache = torch.tensor([])
        self.v_cache = torch.tensor([])

    def forward(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, ctx: Context):
        k_cache, v_cache = self.k_cache, self.v_cache
        if k_cache.numel() and v_cache.numel():
            store_kvcache(k, v, k_cache, v_cache, ctx.slot_mapping)
        return attend(q, k, v, k_cache, v_cache, ctx, self.scale)
