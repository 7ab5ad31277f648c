"""Bounded device waits run out cleanly (one GPU, no fault).

Every spin of the kernels (mbarriers, peer flags, merge counters) gives up
after 1 s of %globaltimer, records a bit in the device error word and lets
the kernel finish, so the CUDA context stays usable and the host learns of
the failure from b200_device_error.  Here the fused GEMM + all-reduce runs as
rank 0 of a two-rank job whose "peer" buffers are a second local allocation
that no other rank ever signals: rank 0's wait on its own flag (which only
the absent peer would raise) must run out, set the peer-timeout bit and
return.  The next kernels on the same context must then run and be right.
"""
import time

import pytest
import torch

from oracle import layers as L

pytestmark = pytest.mark.gpu

PEER_TIMEOUT = 0x2  # B200_DEVERR_PEER_TIMEOUT


@torch.inference_mode()
def test_peer_flag_wait_runs_out_and_reports():
    from src import b200
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    assert b200.device_error(clear=True) == 0
    g = torch.Generator(device=dev).manual_seed(5)
    T, N, K = 64, 512, 256
    x = torch.randn(T, K, device=dev, generator=g).to(torch.bfloat16)
    w = (torch.randn(N, K, device=dev, generator=g) * 0.02).to(torch.bfloat16)
    world, rows, ldo, positions = 2, T, N, 4096

    def sym():
        # one rank's symmetric buffers for the one-shot exchange
        return dict(stage=torch.zeros(2 * world * rows * ldo, dtype=torch.bfloat16, device=dev),
                    out=torch.zeros(rows * ldo, dtype=torch.bfloat16, device=dev),
                    flags=torch.zeros(2 * positions, dtype=torch.int32, device=dev),
                    done=torch.zeros(positions, dtype=torch.int32, device=dev))

    me, ghost = sym(), sym()
    addrs = {k: [me[k].data_ptr(), ghost[k].data_ptr()] for k in me}
    assert b200.linear_allreduce_supported(T, N, K, world, rows, ldo, positions)
    t0 = time.perf_counter()
    rc = b200.linear_allreduce(x, w, None, 0, world, addrs["stage"], addrs["out"], addrs["flags"],
                               addrs["done"], rows, ldo, positions, one_shot=True)
    assert rc == 0
    torch.cuda.synchronize()
    waited = time.perf_counter() - t0
    err = b200.device_error(clear=True)
    assert err & PEER_TIMEOUT, err
    assert waited >= 0.9, waited  # the wait ran its 1 s course, then returned
    # the partial was still pushed to the ghost's staging area, and the flag
    # the ghost would have waited on was raised
    assert int(ghost["flags"].count_nonzero()) > 0
    # the context is intact: the plain GEMM runs and is right
    y = b200.linear(x, w)
    torch.cuda.synchronize()
    assert b200.device_error(clear=True) == 0
    assert L.rel_err(y.cpu(), L.linear(x.cpu(), w.cpu())) <= 1e-2
