"""Tensor-parallel linear layers on the tcgen05 GEMM.

Same classes, constructor arguments, parameter shapes and `weight_loader`
protocol as src/layers/linear.py of nano-vllm-diy, so checkpoints load through
the reference loader unchanged.  forward() runs libb200ops' GEMM;
RowParallelLinear at tp > 1 runs the GEMM and the sum over ranks as one fused
kernel through the process's tensor-parallel communicator (src.layers.tp_comm,
created on first use), and otherwise the GEMM followed by torch.distributed.all_reduce.
"""
from __future__ import annotations

import torch
import torch.distributed as dist
from torch import nn

from src import b200
from src.utils.math import divide


def _take_shard(loaded: torch.Tensor, parts: int, index: int, dim: int) -> torch.Tensor:
    """Shard `index` of `parts` equal slices of `loaded` along `dim`."""
    size = divide(loaded.shape[dim], parts)
    return loaded.narrow(dim, index * size, size)


class LinearBase(nn.Module):
    """Holds weight [out, in] (and bias [out]) with a `.weight_loader` attribute
    (reference: src/layers/linear.py:7-29)."""

    def __init__(self, in_features: int, out_features: int, bias: bool = False,
                 tp: tuple[int, int] = (0, 1)):
        super().__init__()
        self.in_features = in_features
        self.out_features = out_features
        self.tp_rank, self.tp_world_size = tp
        self.weight = nn.Parameter(torch.empty(out_features, in_features), requires_grad=False)
        self.weight.weight_loader = self.weight_loader
        if bias:
            self.bias = nn.Parameter(torch.empty(out_features), requires_grad=False)
            self.bias.weight_loader = self.weight_loader
        else:
            self.register_parameter("bias", None)

    def weight_loader(self, param: nn.Parameter, loaded_weight: torch.Tensor, *args):
        raise NotImplementedError

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        raise NotImplementedError


class Linear(LinearBase):
    """Unsharded linear (reference: src/layers/linear.py:31-50)."""

    def weight_loader(self, param: nn.Parameter, loaded_weight: torch.Tensor):
        assert loaded_weight.shape == param.shape, (
            f"Expected weight shape {param.shape}, but got {loaded_weight.shape}")
        param.data.copy_(loaded_weight)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return b200.linear(x, self.weight, self.bias)


class ColumnParallelLinear(LinearBase):
    """Output features split over ranks (reference: src/layers/linear.py:52-75)."""

    def __init__(self, in_features: int, out_features: int, bias: bool = False,
                 tp: tuple[int, int] = (0, 1)):
        assert out_features % tp[1] == 0, "out_features must be divisible by tp_world_size"
        super().__init__(in_features, divide(out_features, tp[1]), bias, tp)

    def weight_loader(self, param: nn.Parameter, loaded_weight: torch.Tensor):
        full_out = self.out_features * self.tp_world_size
        assert loaded_weight.shape[0] == full_out, (
            f"Expected weight shape ({full_out}, {self.in_features}), but got {loaded_weight.shape}")
        if loaded_weight.ndim == 2:
            assert loaded_weight.shape[1] == self.in_features, (
                f"Expected weight shape ({full_out}, {self.in_features}), but got {loaded_weight.shape}")
        param.data.copy_(_take_shard(loaded_weight, self.tp_world_size, self.tp_rank, 0))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return b200.linear(x, self.weight, self.bias)


class MergedColumnParallelLinear(ColumnParallelLinear):
    """Several column-parallel projections stacked row-wise per rank, e.g.
    gate_up = [gate_shard ; up_shard] (reference: src/layers/linear.py:77-102)."""

    def __init__(self, in_features: int, out_features_list: list[int], bias: bool = False,
                 tp: tuple[int, int] = (0, 1)):
        assert all(o % tp[1] == 0 for o in out_features_list), (
            "out_features must be divisible by tp_world_size")
        super().__init__(in_features, sum(out_features_list), bias, tp)
        self.out_features_list = out_features_list

    def weight_loader(self, param: nn.Parameter, loaded_weight: torch.Tensor, loaded_shard_id: int):
        rows = self.out_features_list[loaded_shard_id]
        assert loaded_weight.shape[0] == rows, (
            f"Expected weight shape ({rows}, {self.in_features}), but got {loaded_weight.shape}")
        if loaded_weight.ndim == 2:
            assert loaded_weight.shape[1] == self.in_features, (
                f"Expected weight shape ({rows}, {self.in_features}), but got {loaded_weight.shape}")
        offset = divide(sum(self.out_features_list[:loaded_shard_id]), self.tp_world_size)
        dst = param.data.narrow(0, offset, divide(rows, self.tp_world_size))
        dst.copy_(_take_shard(loaded_weight, self.tp_world_size, self.tp_rank, 0))


class QKVParallelLinear(ColumnParallelLinear):
    """Fused q/k/v projection; per rank the rows are [q | k | v] of this rank's
    heads (reference: src/layers/linear.py:104-142)."""

    def __init__(self, model_dim: int, head_dim: int, num_heads: int, num_kv_heads: int,
                 bias: bool = False, tp: tuple[int, int] = (0, 1)):
        assert num_heads % tp[1] == 0, "num_heads must be divisible by tp_world_size"
        assert num_kv_heads % tp[1] == 0, "num_kv_heads must be divisible by tp_world_size"
        super().__init__(model_dim, (num_heads + 2 * num_kv_heads) * head_dim, bias, tp)
        self.head_dim = head_dim
        self.num_heads = num_heads
        self.num_kv_heads = num_kv_heads

    def _shard_rows(self, shard_id: str) -> tuple[int, int]:
        """(start row in the full [q|k|v] layout, rows) of q, k or v."""
        q = self.num_heads * self.head_dim
        kv = self.num_kv_heads * self.head_dim
        return {"q": (0, q), "k": (q, kv), "v": (q + kv, kv)}[shard_id]

    def weight_loader(self, param: nn.Parameter, loaded_weight: torch.Tensor, loaded_shard_id: str):
        assert loaded_shard_id in ("q", "k", "v"), (
            f"Expected loaded_shard_id to be one of ['q', 'k', 'v'], but got {loaded_shard_id}")
        if loaded_weight.ndim == 2:
            assert loaded_weight.shape[1] == self.in_features, (
                f"Expected weight shape ({self.out_features}, {self.in_features}), but got {loaded_weight.shape}")
        start, rows = self._shard_rows(loaded_shard_id)
        assert loaded_weight.shape[0] == rows, (
            f"Expected weight shape ({rows}, {self.in_features}), but got {loaded_weight.shape}")
        dst = param.data.narrow(0, divide(start, self.tp_world_size), divide(rows, self.tp_world_size))
        dst.copy_(_take_shard(loaded_weight, self.tp_world_size, self.tp_rank, 0))


class RowParallelLinear(LinearBase):
    """Input features split over ranks; the per-rank partial products are
    summed over ranks, bias added once by rank 0
    (reference: src/layers/linear.py:144-173)."""

    def __init__(self, in_features: int, out_features: int, bias: bool = False,
                 tp: tuple[int, int] = (0, 1)):
        assert in_features % tp[1] == 0, "in_features must be divisible by tp_world_size"
        super().__init__(divide(in_features, tp[1]), out_features, bias, tp)

    def weight_loader(self, param: nn.Parameter, loaded_weight: torch.Tensor):
        if loaded_weight.ndim == 2:
            full_in = self.in_features * self.tp_world_size
            assert loaded_weight.shape[0] == self.out_features, (
                f"Expected weight shape ({self.out_features}, {self.in_features}), but got {loaded_weight.shape}")
            assert loaded_weight.shape[1] == full_in, (
                f"Expected weight shape ({self.out_features}, {full_in}), but got {loaded_weight.shape}")
            param.data.copy_(_take_shard(loaded_weight, self.tp_world_size, self.tp_rank, 1))
        else:
            assert loaded_weight.shape[0] == self.out_features, (
                f"Expected weight shape ({self.out_features},), but got {loaded_weight.shape}")
            param.data.copy_(loaded_weight)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        bias = self.bias if self.tp_rank == 0 else None
        if self.tp_world_size == 1:
            return b200.linear(x, self.weight, bias)
        from src.layers import tp_comm
        comm = tp_comm.ensure(x.device, self.out_features)
        if comm is not None:
            return comm.linear_allreduce(x, self.weight, bias)
        y = b200.linear(x, self.weight, bias)
        dist.all_reduce(y)
        return y
