"""Parity of each sm_100a kernel (called through the C-ABI) with the oracle.

Integer / byte work (KV scatter, embedding rows, argmax, cache slots) must be
bit-exact; floating-point kernels are held to max|gpu - ref| / max|ref| <=
2e-2 against an fp32-accumulated reference (1e-2 for plain GEMMs).
"""
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


def _g(seed):
    return torch.Generator().manual_seed(seed)


def randn(*s, std=1.0, seed=0):
    return (torch.randn(*s, generator=_g(seed)) * std).to(torch.bfloat16)


# --------------------------------------------------------------------------- GEMM
GEMM_SHAPES = [
    (1, 128, 64), (7, 384, 1024), (32, 4096, 4096), (100, 1000, 512), (256, 6144, 4096),
    (256, 4096, 12288), (300, 1024, 4096), (1000, 2048, 1024), (64, 18992, 256), (129, 256, 4104),
    (256, 1536, 4096), (256, 768, 4096),  # qkv per rank at tp 4 / 8: cluster split-K
]


@pytest.mark.parametrize("T,N,K", GEMM_SHAPES)
def test_linear(T, N, K):
    from src import b200
    x = randn(T, K, seed=1)
    w = randn(N, K, std=0.02, seed=2)
    ref = x.float() @ w.float().t()
    y = b200.linear(x.to(DEV), w.to(DEV))
    torch.cuda.synchronize()
    assert y.shape == (T, N)
    err = L.rel_err(y.cpu(), ref)
    assert err <= 1e-2, err


@pytest.mark.parametrize("kernel,pairs", [("grouped", ""), ("grouped", "1"), ("grouped", "3"),
                                          ("grouped", "17"), ("streamk", ""), ("streamk", "3"),
                                          ("streamk", "17"), ("cluster", ""), ("single", "")])
@pytest.mark.parametrize("T,N,K", [(256, 4096, 4096), (77, 1280, 2048), (513, 768, 1024),
                                   (256, 24576, 1024), (256, 6144, 4096)])
def test_linear_kernels_and_splits(T, N, K, kernel, pairs, monkeypatch):
    """Every GEMM schedule gives the same product within tolerance: the
    SM-pair kernel (tcgen05.mma.cta_group::2) with its grouped split-K
    schedule (whole tiles only, split tiles only, both) and with its
    stream-K schedule (whole tiles, contributor / finisher segments),
    whatever number of pairs shares the work, the same kernel's cluster
    split-K mode (plain GEMM; the SiLU call takes the default path), and the
    single-SM kernel."""
    from src import b200
    monkeypatch.setenv("B200_GEMM_PAIR", {"single": "0", "cluster": "3"}.get(kernel, "2"))
    monkeypatch.setenv("B200_GEMM_SCHED", "streamk" if kernel == "streamk" else "")
    monkeypatch.setenv("B200_GEMM_PAIRS", pairs)
    x = randn(T, K, seed=11)
    w = randn(N, K, std=0.02, seed=12)
    ref = x.float() @ w.float().t()
    y = b200.linear(x.to(DEV), w.to(DEV))
    g = b200.linear_silu_and_mul(x.to(DEV), w.to(DEV))
    torch.cuda.synchronize()
    assert L.rel_err(y.cpu(), ref) <= 1e-2
    assert L.rel_err(g.cpu(), L.silu_and_mul(ref.to(torch.bfloat16))) <= 2e-2
    assert b200.device_error(clear=True) == 0


@pytest.mark.parametrize("C,NP", [(2, 192), (2, 256), (3, 256), (3, 128), (4, 256), (4, 96), (3, 64)])
@pytest.mark.parametrize("T,N,K", [(256, 4096, 4096), (256, 6144, 4096), (200, 1000, 1024),
                                   (512, 768, 12288), (256, 4096, 12288)])
def test_linear_cluster_split_k(T, N, K, C, NP, monkeypatch):
    """The SM-pair kernel's cluster split-K mode with clusters of C pairs (2C
    CTAs, K split C ways) and NP weight rows per tile, forced: every member
    pushes the 32-wide chunks the others own into their rings (NP = 96 at
    C = 4 and NP = 64 at C = 3 leave a member owning nothing)."""
    from src import b200
    monkeypatch.setenv("B200_GEMM_PAIR", "3")
    monkeypatch.setenv("B200_GEMM_CSK", f"{C},{NP}")
    x = randn(T, K, seed=13)
    w = randn(N, K, std=0.02, seed=14)
    ref = x.float() @ w.float().t()
    y = b200.linear(x.to(DEV), w.to(DEV))
    torch.cuda.synchronize()
    assert L.rel_err(y.cpu(), ref) <= 1e-2
    # the same call again: the rings and barriers start clean every launch
    y2 = b200.linear(x.to(DEV), w.to(DEV))
    torch.cuda.synchronize()
    assert torch.equal(y, y2)


@pytest.mark.parametrize("kernel,T", [("default", 48), ("grouped", 200), ("streamk", 200), ("cluster", 200)])
@pytest.mark.parametrize("col0", [0, 1])
def test_linear_bias_and_strided_out(kernel, T, col0, monkeypatch):
    """Bias and an output view with a row stride wider than N; col0 = 1 makes
    the rows 2-byte aligned only, so the kernels store without TMA."""
    from src import b200
    monkeypatch.setenv("B200_GEMM_PAIR", {"default": "1", "cluster": "3"}.get(kernel, "2"))
    monkeypatch.setenv("B200_GEMM_SCHED", "streamk" if kernel == "streamk" else "")
    N, K = 640, 1024
    x = randn(T, K, seed=3)
    w = randn(N, K, std=0.02, seed=4)
    b = randn(N, std=0.5, seed=5)
    ref = x.float() @ w.float().t() + b.float()
    out = torch.zeros(T, N + 64, dtype=torch.bfloat16, device=DEV)
    b200.linear(x.to(DEV), w.to(DEV), b.to(DEV), out=out[:, col0:col0 + N])
    torch.cuda.synchronize()
    assert L.rel_err(out[:, col0:col0 + N].cpu(), ref) <= 1e-2
    assert torch.count_nonzero(out[:, :col0]) == 0
    assert torch.count_nonzero(out[:, col0 + N:]) == 0
    assert b200.device_error(clear=True) == 0


@pytest.mark.parametrize("T,I,K", [(1, 64, 256), (40, 1536, 1024), (256, 3072, 1024), (256, 1536, 4096), (300, 512, 2048), (16, 96, 512)])
def test_linear_silu_and_mul(T, I, K):
    from src import b200
    x = randn(T, K, seed=6)
    w = randn(2 * I, K, std=0.02, seed=7)
    ref = L.silu_and_mul(L.linear(x, w))
    y = b200.linear_silu_and_mul(x.to(DEV), w.to(DEV))
    torch.cuda.synchronize()
    assert y.shape == (T, I)
    assert L.rel_err(y.cpu(), ref) <= 2e-2


# --------------------------------------------------------------------------- norms
@pytest.mark.parametrize("rows,dim", [(1, 128), (37, 1024), (256, 4096), (5, 5120), (3, 8192)])
def test_rms_norm(rows, dim):
    from src import b200
    x = randn(rows, dim, seed=8)
    w = randn(dim, std=0.3, seed=9) + 1
    r = randn(rows, dim, seed=10)
    ref = L.rms_norm(x, w, 1e-6)
    y = b200.rms_norm(x.to(DEV), w.to(DEV), 1e-6)
    ref2, res2 = L.rms_norm_residual(x, r, w, 1e-6)
    y2, yr = b200.rms_norm(x.to(DEV), w.to(DEV), 1e-6, residual=r.to(DEV))
    torch.cuda.synchronize()
    assert L.rel_err(y.cpu(), ref) <= 2e-2
    assert L.rel_err(y2.cpu(), ref2) <= 2e-2
    assert torch.equal(yr.cpu(), res2)  # x + residual rounds once: bit-exact


# --------------------------------------------------------------------------- qk norm + rope + store
@pytest.mark.parametrize("T,Hq,Hkv", [(1, 16, 8), (70, 32, 8), (256, 8, 1)])
def test_qk_norm_rope_store(T, Hq, Hkv):
    from src import b200
    d = 128
    qkv = randn(T, (Hq + 2 * Hkv) * d, seed=11)
    qw = randn(d, std=0.2, seed=12) + 1
    kw = randn(d, std=0.2, seed=13) + 1
    pos = torch.randint(0, 4000, (T,), generator=_g(14))
    cs = L.rope_cos_sin(4096, d, 1e6)
    nblk, page = 4, 256
    perm = torch.randperm(nblk * page, generator=_g(15))[:T].to(torch.int32)
    slots = perm.clone()
    slots[::5] = -1
    q, k, v = qkv.split([Hq * d, Hkv * d, Hkv * d], -1)
    q, k, v = q.reshape(T, Hq, d), k.reshape(T, Hkv, d), v.reshape(T, Hkv, d)
    rq, rk = L.rope(L.rms_norm(q, qw, 1e-6), L.rms_norm(k, kw, 1e-6), pos, cs)
    kc = torch.zeros(nblk, page, Hkv, d, dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    L.store_kvcache(rk, v, kc, vc, slots)

    dq = qkv.to(DEV)
    gq, gk, gv = dq.split([Hq * d, Hkv * d, Hkv * d], -1)
    gq, gk, gv = gq.view(T, Hq, d), gk.view(T, Hkv, d), gv.view(T, Hkv, d)
    gkc = torch.zeros(nblk, page, Hkv, d, dtype=torch.bfloat16, device=DEV)
    gvc = torch.zeros_like(gkc)
    oq, ok, ov = b200.qk_norm_rope_store(gq, gk, gv, qw.to(DEV), kw.to(DEV), 1e-6,
                                         cs.to(DEV).view(4096, d), pos.to(DEV), slots.to(DEV),
                                         gkc, gvc)
    torch.cuda.synchronize()
    assert L.rel_err(oq.cpu(), rq) <= 2e-2
    assert L.rel_err(ok.cpu(), rk) <= 2e-2
    assert torch.equal(ov.cpu(), v)
    assert torch.equal(gvc.cpu(), vc)  # v rows land in exactly the same slots
    assert L.rel_err(gkc.cpu(), kc) <= 2e-2
    # same slots written, nothing else touched
    assert torch.equal((gkc.cpu() != 0).any(-1).any(-1), (kc != 0).any(-1).any(-1))
    # most elements are bit-identical (the only differences come from the
    # fp32 summation order inside the norm)
    same = (oq.cpu() == rq).float().mean().item()
    assert same > 0.97, same


# --------------------------------------------------------------------------- scatter
@pytest.mark.parametrize("T,Hkv", [(1, 8), (256, 8), (300, 1), (17, 4)])
def test_store_kvcache_bit_exact(T, Hkv):
    from src import b200
    d = 128
    nblk, page = 3, 256
    k = randn(T, Hkv, d, seed=16)
    v = randn(T, Hkv, d, seed=17)
    slots = torch.randperm(nblk * page, generator=_g(18))[:T].to(torch.int32)
    slots[1::3] = -1
    kc = randn(nblk, page, Hkv, d, seed=19)
    vc = randn(nblk, page, Hkv, d, seed=20)
    gkc, gvc = kc.to(DEV), vc.to(DEV)
    L.store_kvcache(k, v, kc, vc, slots)
    b200.store_kvcache(k.to(DEV), v.to(DEV), gkc, gvc, slots.to(DEV))
    torch.cuda.synchronize()
    assert torch.equal(gkc.cpu(), kc)
    assert torch.equal(gvc.cpu(), vc)


def test_store_kvcache_strided_key_view():
    """k/v as views into a fused qkv row (stride(0) > D), as Qwen3Attention passes them."""
    from src import b200
    T, Hq, Hkv, d = 33, 4, 2, 128
    qkv = randn(T, (Hq + 2 * Hkv) * d, seed=21)
    _, k, v = qkv.split([Hq * d, Hkv * d, Hkv * d], -1)
    k, v = k.view(T, Hkv, d), v.view(T, Hkv, d)
    slots = torch.arange(T, dtype=torch.int32) * 3
    kc = torch.zeros(1, 256, Hkv, d, dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    L.store_kvcache(k, v, kc, vc, slots)
    gq = qkv.to(DEV)
    _, gk, gv = gq.split([Hq * d, Hkv * d, Hkv * d], -1)
    gkc, gvc = torch.zeros_like(kc, device=DEV), torch.zeros_like(vc, device=DEV)
    b200.store_kvcache(gk.view(T, Hkv, d), gv.view(T, Hkv, d), gkc, gvc, slots.to(DEV))
    torch.cuda.synchronize()
    assert torch.equal(gkc.cpu(), kc) and torch.equal(gvc.cpu(), vc)


def test_store_kvcache_out_of_range_slot_flags_error():
    from src import b200
    T, Hkv, d = 4, 2, 128
    k = randn(T, Hkv, d, seed=22)
    kc = torch.zeros(1, 256, Hkv, d, dtype=torch.bfloat16, device=DEV)
    vc = torch.zeros_like(kc)
    slots = torch.tensor([0, 256, -1, 5], dtype=torch.int32, device=DEV)  # 256 is past the cache
    b200.store_kvcache(k.to(DEV), k.to(DEV), kc, vc, slots)
    torch.cuda.synchronize()
    assert b200.device_error(clear=True) & 4
    assert torch.equal(kc[0, 0].cpu(), k[0]) and torch.equal(kc[0, 5].cpu(), k[3])
    assert torch.count_nonzero(kc[0, 1:5]) == 0


# --------------------------------------------------------------------------- misc
def test_silu_and_mul():
    from src import b200
    x = randn(77, 2 * 3072, seed=23)
    y = b200.silu_and_mul(x.to(DEV))
    torch.cuda.synchronize()
    assert L.rel_err(y.cpu(), L.silu_and_mul(x)) <= 2e-2


@pytest.mark.parametrize("start,end", [(0, 1000), (250, 500)])
def test_embedding_exact(start, end):
    from src import b200
    V, H = 1000, 1024
    w = randn(end - start, H, seed=24)
    ids = torch.randint(0, V, (65,), generator=_g(25))
    y = b200.embedding(ids.to(DEV), w.to(DEV), start, end)
    torch.cuda.synchronize()
    assert torch.equal(y.cpu(), L.vocab_embedding(ids, w, start, end))


def test_argmax_exact():
    from src import b200
    x = randn(9, 151936, seed=26)
    x[3, 100] = 50.0
    x[3, 90000] = 50.0  # tie -> first index
    y = b200.argmax(x.to(DEV))
    torch.cuda.synchronize()
    assert torch.equal(y.cpu(), torch.argmax(x, -1))
    assert y[3].item() == 100


@pytest.mark.parametrize("rows,V,pad", [(5, 1001, 0), (3, 37, 0), (4, 4100, 4), (2, 16, 0)])
def test_argmax_ragged_rows(rows, V, pad):
    """Rows whose start is not 16-byte aligned (scalar loads), lengths that
    are not a multiple of 8 (scalar tail after the 16-byte loads), ties."""
    from src import b200
    x = randn(rows, V + pad, seed=27)
    x[0, V - 1] = 40.0  # maximum in the tail
    x[rows - 1, 1] = 40.0
    x[rows - 1, V - 2] = 40.0  # tie -> first index
    xd = x.to(DEV)[:, :V]
    y = b200.argmax(xd)
    torch.cuda.synchronize()
    assert torch.equal(y.cpu(), torch.argmax(x[:, :V], -1))


# --------------------------------------------------------------------------- attention
def _paged_case(lens_q, lens_k, Hq, Hkv, page=256, seed=30, extra_blocks=3):
    g = _g(seed)
    B = len(lens_q)
    d = 128
    nblocks = sum((lk + page - 1) // page for lk in lens_k) + extra_blocks
    perm = torch.randperm(nblocks, generator=g).tolist()
    width = max((lk + page - 1) // page for lk in lens_k)
    bt = torch.full((B, width), -1, dtype=torch.int32)
    for b, lk in enumerate(lens_k):
        for j in range((lk + page - 1) // page):
            bt[b, j] = perm.pop()
    kc = (torch.randn(nblocks, page, Hkv, d, generator=g)).to(torch.bfloat16)
    vc = (torch.randn(nblocks, page, Hkv, d, generator=g)).to(torch.bfloat16)
    cu_q = torch.tensor([0] + list(torch.tensor(lens_q).clamp(min=0).cumsum(0).tolist()), dtype=torch.int32)
    cu_k = torch.tensor([0] + list(torch.tensor(lens_k).cumsum(0).tolist()), dtype=torch.int32)
    T = int(cu_q[-1])
    q = torch.randn(T, Hq, d, generator=g).to(torch.bfloat16)
    return q, kc, vc, bt, cu_q, cu_k


@pytest.mark.parametrize("Hq,Hkv", [(32, 8), (16, 8), (8, 1), (64, 8)])
def test_decode_attention_paged(Hq, Hkv):
    from src import b200
    lens_k = [1, 128, 129, 255, 256, 257, 1000, 4096, 3000, 77]
    lens_q = [1] * len(lens_k)
    q, kc, vc, bt, cu_q, cu_k = _paged_case(lens_q, lens_k, Hq, Hkv)
    scale = 128 ** -0.5
    ref = L.varlen_attention(q, None, None, cu_q, cu_k, scale, kc, vc, bt)
    out = b200.paged_attention(q.to(DEV), None, None, kc.to(DEV), vc.to(DEV), cu_q.to(DEV),
                               cu_k.to(DEV), 1, max(lens_k), scale, bt.to(DEV))
    torch.cuda.synchronize()
    assert L.rel_err(out.cpu(), ref) <= 2e-2


def test_decode_attention_long_and_repeated():
    """Sequences of > 32 items (the merge loops in rounds) and two calls in a
    row (the scheduler counters of the merge phase must reset)."""
    from src import b200
    lens_k = [9000, 8193, 256, 511, 33]
    q, kc, vc, bt, cu_q, cu_k = _paged_case([1] * 5, lens_k, 32, 8, seed=31)
    scale = 128 ** -0.5
    ref = L.varlen_attention(q, None, None, cu_q, cu_k, scale, kc, vc, bt)
    args = (q.to(DEV), None, None, kc.to(DEV), vc.to(DEV), cu_q.to(DEV), cu_k.to(DEV), 1,
            max(lens_k), scale, bt.to(DEV))
    out1 = b200.paged_attention(*args)
    out2 = b200.paged_attention(*args)
    torch.cuda.synchronize()
    assert L.rel_err(out1.cpu(), ref) <= 2e-2
    assert torch.equal(out1, out2)


def test_decode_attention_mix_alternating_batches():
    """A serving-like mix (about 100 sequences of 100-2100 keys: most are split
    into 2-5 items and merged) on 512-key pages, three calls alternating two
    batches in one workspace: the per-(sequence, kv head) completion counters
    and both queues must come back to zero after every call."""
    import random
    from src import b200
    rng = random.Random(7)
    scale = 128 ** -0.5
    cases = []
    for seed in (41, 42):
        lens_k = [rng.randint(100, 2100) for _ in range(120 if seed == 41 else 97)]
        q, kc, vc, bt, cu_q, cu_k = _paged_case([1] * len(lens_k), lens_k, 32, 8, page=512, seed=seed)
        ref = L.varlen_attention(q, None, None, cu_q, cu_k, scale, kc, vc, bt)
        args = (q.to(DEV), None, None, kc.to(DEV), vc.to(DEV), cu_q.to(DEV), cu_k.to(DEV), 1,
                max(lens_k), scale, bt.to(DEV))
        cases.append((args, ref))
    for i in (0, 1, 0):
        args, ref = cases[i]
        out = b200.paged_attention(*args)
        torch.cuda.synchronize()
        assert L.rel_err(out.cpu(), ref) <= 2e-2, i
    assert b200.device_error(clear=True) == 0


def test_decode_attention_graph_padding():
    """CUDA-graph replay pads cu_seqlens with 0 and block tables with -1
    (src/engine/model_runner.py:248-257): padded rows must be skipped."""
    from src import b200
    lens_k = [300, 5, 1024]
    q, kc, vc, bt, cu_q, cu_k = _paged_case([1, 1, 1], lens_k, 32, 8)
    pad = 5
    cu_qp = torch.cat([cu_q, torch.zeros(pad, dtype=torch.int32)])
    cu_kp = torch.cat([cu_k, torch.zeros(pad, dtype=torch.int32)])
    btp = torch.cat([bt, torch.full((pad, bt.shape[1]), -1, dtype=torch.int32)])
    qp = torch.cat([q, torch.randn(pad, 32, 128).to(torch.bfloat16)])
    scale = 128 ** -0.5
    ref = L.varlen_attention(q, None, None, cu_q, cu_k, scale, kc, vc, bt)
    out = b200.paged_attention(qp.to(DEV), None, None, kc.to(DEV), vc.to(DEV), cu_qp.to(DEV),
                               cu_kp.to(DEV), 1, 8192, scale, btp.to(DEV))
    torch.cuda.synchronize()
    assert L.rel_err(out[:3].cpu(), ref) <= 2e-2


@pytest.mark.parametrize("Hq,Hkv", [(32, 8), (16, 8), (4, 4)])
def test_prefill_attention_fresh(Hq, Hkv):
    from src import b200
    g = _g(40)
    lens = [1, 63, 64, 65, 200, 513]
    cu = torch.tensor([0] + torch.tensor(lens).cumsum(0).tolist(), dtype=torch.int32)
    T = int(cu[-1])
    q = torch.randn(T, Hq, 128, generator=g).to(torch.bfloat16)
    k = torch.randn(T, Hkv, 128, generator=g).to(torch.bfloat16)
    v = torch.randn(T, Hkv, 128, generator=g).to(torch.bfloat16)
    scale = 128 ** -0.5
    ref = L.varlen_attention(q, k, v, cu, cu, scale)
    out = b200.paged_attention(q.to(DEV), k.to(DEV), v.to(DEV), None, None, cu.to(DEV), cu.to(DEV),
                               max(lens), max(lens), scale, None)
    torch.cuda.synchronize()
    assert L.rel_err(out.cpu(), ref) <= 2e-2


def test_prefill_attention_paged_prefix_and_chunks():
    """Prefix-cache hits, chunked prefill and decode rows in one batch
    (block_tables set, Lk > Lq)."""
    from src import b200
    lens_q = [512, 1, 37, 200, 1]
    lens_k = [1024, 600, 37, 900, 1]
    q, kc, vc, bt, cu_q, cu_k = _paged_case(lens_q, lens_k, 32, 8, seed=41)
    scale = 128 ** -0.5
    ref = L.varlen_attention(q, None, None, cu_q, cu_k, scale, kc, vc, bt)
    out = b200.paged_attention(q.to(DEV), None, None, kc.to(DEV), vc.to(DEV), cu_q.to(DEV),
                               cu_k.to(DEV), max(lens_q), max(lens_k), scale, bt.to(DEV))
    torch.cuda.synchronize()
    assert L.rel_err(out.cpu(), ref) <= 2e-2


@pytest.mark.parametrize("kernel", ["tcgen05", "legacy"])
@pytest.mark.parametrize("Hq,Hkv,page", [(32, 8, 256), (16, 8, 512), (8, 1, 256), (4, 4, 256)])
def test_prefill_attention_kernels_paged_with_stale_pages(kernel, Hq, Hkv, page, monkeypatch):
    """Both prefill kernels (tcgen05 / TMEM / TMA, and the mma.sync one
    selected by B200_PREFILL=legacy) on chunks, prefix hits, fresh prompts and
    decode rows, with the unused tail of every last page holding NaN (stale
    cache bits that P = 0 must not turn into NaN outputs)."""
    from src import b200
    monkeypatch.setenv("B200_PREFILL", "legacy" if kernel == "legacy" else "")
    lens_q = [128, 1, 300, 129, 700, 1, 64]
    lens_k = [128, 513, 300, 1000, 1400, 2, 2000]
    q, kc, vc, bt, cu_q, cu_k = _paged_case(lens_q, lens_k, Hq, Hkv, page=page, seed=43)
    for b, lk in enumerate(lens_k):
        last = int(bt[b, (lk - 1) // page])
        used = lk - ((lk - 1) // page) * page
        kc[last, used:] = float("nan")
        vc[last, used:] = float("nan")
    scale = 128 ** -0.5
    ref = L.varlen_attention(q, None, None, cu_q, cu_k, scale, kc, vc, bt)
    out = b200.paged_attention(q.to(DEV), None, None, kc.to(DEV), vc.to(DEV), cu_q.to(DEV),
                               cu_k.to(DEV), max(lens_q), max(lens_k), scale, bt.to(DEV))
    torch.cuda.synchronize()
    assert torch.isfinite(out.float()).all()
    assert L.rel_err(out.cpu(), ref) <= 2e-2


@pytest.mark.parametrize("kernel", ["tcgen05", "legacy"])
def test_prefill_attention_kernels_fresh_long(kernel, monkeypatch):
    """Fresh varlen prefill (per-token K / V), sequences up to 3000 tokens."""
    from src import b200
    monkeypatch.setenv("B200_PREFILL", "legacy" if kernel == "legacy" else "")
    g = _g(44)
    lens = [3000, 1, 127, 128, 129, 900]
    Hq, Hkv = 16, 4
    cu = torch.tensor([0] + torch.tensor(lens).cumsum(0).tolist(), dtype=torch.int32)
    T = int(cu[-1])
    q = torch.randn(T, Hq, 128, generator=g).to(torch.bfloat16)
    k = torch.randn(T, Hkv, 128, generator=g).to(torch.bfloat16)
    v = torch.randn(T, Hkv, 128, generator=g).to(torch.bfloat16)
    scale = 128 ** -0.5
    ref = L.varlen_attention(q, k, v, cu, cu, scale)
    out = b200.paged_attention(q.to(DEV), k.to(DEV), v.to(DEV), None, None, cu.to(DEV), cu.to(DEV),
                               max(lens), max(lens), scale, None)
    torch.cuda.synchronize()
    assert L.rel_err(out.cpu(), ref) <= 2e-2
