"""Process-wide tensor-parallel communicator used by RowParallelLinear.

`get()` returns the fused GEMM + all-reduce communicator of this process, or
None when none is set up.  `ensure(device, hidden)` creates one on the first
row-parallel call at tp > 1 so that an engine which only initialises the
default process group (src/engine/model_runner.py:30 in the reference) gets
the fused path without any change: the reference's ModelRunner runs an eager
warm-up forward (model_runner.py:122-136) before it captures CUDA graphs, and
that first forward is where every rank creates the communicator, at the same
point of the program (the creation is a collective).

With no communicator -- tp == 1, creation disabled by B200_FUSED_ALLREDUCE=0,
or the first call happening inside a CUDA-graph capture -- RowParallelLinear
runs its GEMM and then torch.distributed.all_reduce, the reference's code path.
"""
from __future__ import annotations

import os

import torch

_comm = None
_disabled = os.environ.get("B200_FUSED_ALLREDUCE", "1") == "0"


def get():
    return _comm


def set_comm(comm) -> None:
    global _comm
    _comm = comm


def ensure(device: torch.device, hidden: int):
    """The communicator, created collectively on first use (None when it
    cannot be: disabled, or inside a graph capture)."""
    global _comm
    if _comm is not None or _disabled:
        return _comm
    if torch.cuda.is_current_stream_capturing():
        return None
    from src.layers.tp_allreduce import FusedRowParallel
    _comm = FusedRowParallel(device, max_tokens=512, max_hidden=max(hidden, 8))
    return _comm


def set_enabled(flag: bool) -> None:
    """Allow (True) or forbid (False) `ensure` to create a communicator."""
    global _disabled
    _disabled = not flag


def clear() -> None:
    global _comm
    if _comm is not None and hasattr(_comm, "close"):
        _comm.close()
    _comm = None
