"""Neox rotary embedding (reference: src/layers/pos_embedding.py:1-52).

The fp32 [max_seq_len, 1, head_dim] table of [cos | sin] is built with the
same arithmetic as build_rope_cos_sin and shared by every layer that asks for
the same (max_seq_len, head_dim, base); forward() rotates q and k on the GPU.
"""
from __future__ import annotations

from functools import lru_cache

import torch
from torch import nn

from src import b200


@lru_cache(maxsize=4)
def _table_cpu(max_seq_len: int, head_dim: int, base: float) -> torch.Tensor:
    exps = torch.arange(0, head_dim, 2, device="cpu").float() / head_dim
    inv_freq = 1.0 / (base ** exps)
    angles = torch.outer(torch.arange(max_seq_len, dtype=torch.float, device="cpu"), inv_freq)
    return torch.cat((angles.cos(), angles.sin()), dim=-1).unsqueeze_(1)


_tables: dict = {}


def build_rope_cos_sin(max_seq_len: int, head_dim: int, base: float = 10000) -> torch.Tensor:
    """The table is computed on the CPU (so every device gets the same bits)
    and one copy per (shape, base, device) is shared by all layers."""
    device = torch.get_default_device()
    key = (max_seq_len, head_dim, float(base), str(device))
    t = _tables.get(key)
    if t is None:
        t = _table_cpu(max_seq_len, head_dim, float(base)).to(device)
        _tables[key] = t
    return t


class RoPE(nn.Module):

    def __init__(self, max_seq_len: int, head_dim: int, base: float = 1000000) -> None:
        super().__init__()
        self.head_dim = head_dim
        self.register_buffer("cos_sin", build_rope_cos_sin(max_seq_len, head_dim, base),
                             persistent=False)

    def forward(self, q: torch.Tensor, k: torch.Tensor, positions: torch.Tensor):
        T = positions.shape[0]
        q3 = q.view(T, -1, self.head_dim)
        k3 = k.view(T, -1, self.head_dim)
        qo, ko, _ = b200.qk_norm_rope_store(q3, k3, None, None, None, 0.0, self.cos_sin,
                                            positions, need_kv_out=True)
        return qo.view_as(q), ko.view_as(k)
