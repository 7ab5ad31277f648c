"""The allocation-free decode attention entry point
(b200_paged_decode_attention_static) against the workspace entry point and
the oracle.

Callers that cannot allocate device memory -- a host that reaches the
library through an FFI boundary while another allocator owns the GPU's
memory, or a serving loop that must never call cudaMalloc because it can
synchronise the device -- use this variant, whose scratch is a fixed array
inside the library.  It must give the same attention output as
b200_paged_attention, call after call (the array keeps the previous call's
contents, so the counters it relies on have to be cleared by each call), and
within the attention tolerance of the oracle's restatement of
flash_attn_varlen_func.

Collected last on purpose (file name), so a run that stops at the first
failure has already run every other test.
"""
import ctypes

import pytest
import torch

from oracle import layers as L

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _case(lens_k, Hq, Hkv, seed, page=256):
    g = torch.Generator().manual_seed(seed)
    B = len(lens_k)
    nblocks = sum((n + page - 1) // page for n in lens_k) + 2
    perm = torch.randperm(nblocks, generator=g).tolist()
    width = max((n + page - 1) // page for n in lens_k)
    bt = torch.full((B, width), -1, dtype=torch.int32)
    for b, n in enumerate(lens_k):
        for j in range((n + page - 1) // page):
            bt[b, j] = perm.pop()
    kc = torch.randn(nblocks, page, Hkv, 128, generator=g).to(torch.bfloat16)
    vc = torch.randn(nblocks, page, Hkv, 128, generator=g).to(torch.bfloat16)
    q = torch.randn(B, Hq, 128, generator=g).to(torch.bfloat16)
    cu_q = torch.arange(B + 1, dtype=torch.int32)
    cu_k = torch.tensor([0] + torch.tensor(lens_k).cumsum(0).tolist(), dtype=torch.int32)
    return [t.to(DEV) for t in (q, kc, vc, bt, cu_q, cu_k)]


def _static_call(q, kc, vc, bt, cu_q, cu_k, max_k, out):
    from src import b200
    lib = b200.load_library()
    B, Hq, _ = q.shape
    page, Hkv = kc.shape[1], kc.shape[2]
    rc = lib.b200_paged_decode_attention_static(
        ctypes.c_void_p(q.data_ptr()), q.stride(0), q.shape[0],
        ctypes.c_void_p(kc.data_ptr()), ctypes.c_void_p(vc.data_ptr()), kc.shape[0] * page,
        ctypes.c_void_p(bt.data_ptr()), bt.stride(0), bt.shape[1],
        ctypes.c_void_p(cu_q.data_ptr()), ctypes.c_void_p(cu_k.data_ptr()), B, max_k, Hq, Hkv, page,
        128 ** -0.5, ctypes.c_void_p(out.data_ptr()), out.stride(0),
        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    return rc


def _oracle(q, kc, vc, bt, cu_q, cu_k):
    return L.varlen_attention(q.cpu(), None, None, cu_q.cpu(), cu_k.cpu(), 128 ** -0.5,
                              kc.cpu(), vc.cpu(), bt.cpu())


def test_static_decode_matches_workspace_entry_two_calls_in_a_row():
    from src import b200
    lens_k = [5000, 1, 257, 4096, 33, 700, 256]
    q, kc, vc, bt, cu_q, cu_k = _case(lens_k, 32, 8, seed=71)
    ref = b200.paged_attention(q, None, None, kc, vc, cu_q, cu_k, 1, max(lens_k), 128 ** -0.5, bt)
    want = _oracle(q, kc, vc, bt, cu_q, cu_k)
    torch.cuda.synchronize()
    for call in range(2):
        out = torch.full_like(q, float("nan"))
        rc = _static_call(q, kc, vc, bt, cu_q, cu_k, max(lens_k), out)
        assert rc == 0, b200.load_library().b200_last_error()
        torch.cuda.synchronize()
        # the same kernel on the same inputs: bit-identical to the workspace
        # entry point, and within the attention tolerance of the oracle
        assert torch.equal(out, ref), call
        assert L.rel_err(out.cpu(), want) <= 1e-2, call
    assert b200.device_error(clear=True) == 0


def test_static_decode_allocates_nothing():
    """After a first call (which looks up the array's address on this device),
    a call changes neither torch's allocations nor the device's free memory."""
    from src import b200
    lens_k = [900, 3000, 17]
    q, kc, vc, bt, cu_q, cu_k = _case(lens_k, 16, 8, seed=73)
    out = torch.empty_like(q)
    assert _static_call(q, kc, vc, bt, cu_q, cu_k, max(lens_k), out) == 0
    torch.cuda.synchronize()
    alloc0 = torch.cuda.memory_allocated()
    free0, _ = torch.cuda.mem_get_info()
    assert _static_call(q, kc, vc, bt, cu_q, cu_k, max(lens_k), out) == 0
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert torch.cuda.memory_allocated() == alloc0
    assert free1 == free0
    assert L.rel_err(out.cpu(), _oracle(q, kc, vc, bt, cu_q, cu_k)) <= 1e-2


def test_static_decode_rejects_problems_beyond_its_array():
    from src import b200
    q, kc, vc, bt, cu_q, cu_k = _case([300, 300], 32, 8, seed=72)
    out = torch.empty_like(q)
    # two sequences of up to 32 Mi keys would need far more than 32 MiB
    rc = _static_call(q, kc, vc, bt, cu_q, cu_k, 32768 * 1024, out)
    assert rc == -4  # B200_ERR_WORKSPACE
    assert b"scratch" in b200.load_library().b200_last_error()
    # a refused call leaves nothing behind: the next good call is exact
    rc = _static_call(q, kc, vc, bt, cu_q, cu_k, 300, out)
    assert rc == 0, b200.load_library().b200_last_error()
    ref = b200.paged_attention(q, None, None, kc, vc, cu_q, cu_k, 1, 300, 128 ** -0.5, bt)
    torch.cuda.synchronize()
    assert torch.equal(out, ref)
    assert b200.device_error(clear=True) == 0
