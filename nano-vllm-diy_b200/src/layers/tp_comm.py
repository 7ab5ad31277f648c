"""Process-wide tensor-parallel communicator used by RowParallelLinear.

`get()` returns the fused GEMM + all-reduce communicator of this process, or
None when none has been set up (tp == 1, or before `setup()` is called after
torch.distributed.init_process_group).  With None, RowParallelLinear falls
back to torch.distributed.all_reduce after its GEMM.
"""
from __future__ import annotations

_comm = None


def get():
    return _comm


def set_comm(comm) -> None:
    global _comm
    _comm = comm


def clear() -> None:
    global _comm
    if _comm is not None and hasattr(_comm, "close"):
        _comm.close()
    _comm = None
