"""RMSNorm (+ residual) handed to the projection that consumes it
(b200_rmsnorm_linear), through the C-ABI, against the oracle: the decoder
layer's input_layernorm -> qkv_proj and post_attention_layernorm -> gate_up
(src/models/qwen3.py:162-168).  With B200_FUSE_NORM=1 the norm rows run
inside the persistent SM-pair GEMM's launch (a grid barrier before the
activation loads); by default, and wherever the GEMM is another kernel, the
rms_norm kernel runs first.  Both paths must give the same products within
the GEMM tolerance and the residual sum bit-exactly."""
import pytest
import torch

from oracle import layers as L

pytestmark = pytest.mark.gpu

DEV = "cuda"


@pytest.fixture(autouse=True)
def _clean_error_word():
    from src import b200
    b200.device_error(clear=True)
    yield
    assert b200.device_error(clear=True) == 0, "device error word set"


def randn(*s, std=1.0, seed=0):
    return (torch.randn(*s, generator=torch.Generator().manual_seed(seed)) * std).to(torch.bfloat16)


# (T, N, K, silu): Qwen3-8B's qkv and gate_up at the decode batch (SM-pair
# kernel: cluster split-K and grouped schedules, norm fused), a prefill-sized
# batch, and small batches on the single-SM kernel (norm launched first)
SHAPES = [(256, 6144, 4096, False), (256, 24576, 4096, True), (300, 4096, 4096, False),
          (7, 1536, 1024, False), (64, 6144, 2048, True), (512, 2048, 1024, True)]


@pytest.mark.parametrize("with_residual", [False, True], ids=["plain", "residual"])
@pytest.mark.parametrize("T,N,K,silu", SHAPES)
def test_rmsnorm_linear_matches_oracle(T, N, K, silu, with_residual, monkeypatch):
    from src import b200
    x = randn(T, K, seed=1)
    r = randn(T, K, seed=2) if with_residual else None
    nw = randn(K, std=0.2, seed=3) + 1
    w = randn(N, K, std=0.02, seed=4)
    if with_residual:
        n, s = L.rms_norm_residual(x, r, nw, 1e-6)
    else:
        n, s = L.rms_norm(x, nw, 1e-6), None
    ref = n.float() @ w.float().t()
    if silu:
        ref = L.silu_and_mul(ref.to(torch.bfloat16))
    outs = {}
    for fuse in ("1", "0"):
        monkeypatch.setenv("B200_FUSE_NORM", fuse)
        before = b200.load_library().b200_launch_count()
        got = b200.rmsnorm_linear(x.to(DEV), nw.to(DEV), 1e-6, w.to(DEV),
                                  residual=r.to(DEV) if with_residual else None, silu=silu)
        torch.cuda.synchronize()
        launches = b200.load_library().b200_launch_count() - before
        y, res = got if with_residual else (got, None)
        assert L.rel_err(y.cpu(), ref) <= (2e-2 if silu else 1e-2), (fuse, L.rel_err(y.cpu(), ref))
        if with_residual:
            assert torch.equal(res.cpu(), s)  # x + residual rounds once: bit-exact
        outs[fuse] = (y.cpu(), launches)
    assert outs["0"][1] == 2, outs["0"][1]          # rms_norm kernel, then the GEMM
    assert outs["1"][1] in (1, 2), outs["1"][1]      # one launch where the GEMM is the pair kernel
    assert L.rel_err(outs["1"][0], outs["0"][0].float()) <= 1e-2


def test_rmsnorm_linear_fuses_at_the_decode_batch(monkeypatch):
    """At the decode batch (T = 256) both of Qwen3-8B's norm-fed projections
    run on the SM-pair kernel and, with B200_FUSE_NORM=1, take the norm in
    the same launch; 20 calls in a row (the grid barrier's generation keeps
    advancing) give identical results."""
    from src import b200
    monkeypatch.setenv("B200_FUSE_NORM", "1")
    lib = b200.load_library()
    x = randn(256, 4096, seed=5).to(DEV)
    r = randn(256, 4096, seed=6).to(DEV)
    nw = (randn(4096, std=0.2, seed=7) + 1).to(DEV)
    for N, silu in ((6144, False), (24576, True)):
        w = randn(N, 4096, std=0.02, seed=8).to(DEV)
        before = lib.b200_launch_count()
        y0, r0 = b200.rmsnorm_linear(x, nw, 1e-6, w, residual=r, silu=silu)
        torch.cuda.synchronize()
        assert lib.b200_launch_count() - before == 1
        for _ in range(20):
            y, rr = b200.rmsnorm_linear(x, nw, 1e-6, w, residual=r, silu=silu)
        torch.cuda.synchronize()
        assert torch.equal(y, y0) and torch.equal(rr, r0)
