"""Tensor parallelism on 2, 4 and 8 GPUs (NCCL process group, one process
per GPU; each case is skipped when the machine shows fewer GPUs).

* the fused RowParallelLinear (GEMM + all-reduce over NVLink peer memory),
  both exchange patterns, against the oracle's restatement of
  src/layers/linear.py:169-173 -- sum over ranks of each rank's bf16 partial
  product, rounded once; every rank must hold the bit-identical result;
* fifty calls in a row (the handshake flags reset themselves);
* BASELINE config 1 (x [512, 1536], W [1024, 1536] per rank, world 2, seed
  0) on the fused kernel against the golden rows of the reference's own
  RowParallelLinear under gloo;
* the vocabulary-parallel embedding as one NVLink exchange, bit-exact
  against the oracle's lookup of the full table (src/layers/llm_head.py:38-49);
* token selection over the ranks' vocabulary shards (greedy, and the
  reference sampler with given Exp(1) draws), the same token on every rank
  and equal to the oracle's choice over the full logits
  (src/layers/llm_head.py:60-69, src/layers/sampler.py:4-17);
* the Qwen3 model at tp = world against the oracle's tp = world forward,
  prefill and CUDA-graph decode steps.
"""
import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _init(rank, world, port):
    import datetime
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, device_id=torch.device("cuda", rank),
                            timeout=datetime.timedelta(seconds=60))
    return torch.device("cuda", rank)


def _fused_worker(rank, world, port, one_shot):
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    sys.path[:0] = [os.path.dirname(here), os.path.join(os.path.dirname(here), "nano-vllm-diy_b200")]
    import torch.distributed as dist
    from oracle import layers as L
    from src import b200
    from src.layers.tp_allreduce import FusedRowParallel
    dev = _init(rank, world, port)
    comm = FusedRowParallel(dev, max_tokens=512, max_hidden=4096, one_shot=one_shot)
    try:
        N, K = 4096, 2048
        for T in (1, 7, 64, 256, 300, 512):
            gen = torch.Generator().manual_seed(T)
            x = torch.randn(T, K, generator=gen).to(torch.bfloat16)
            w = (torch.randn(N, K, generator=gen) * 0.02).to(torch.bfloat16)
            xs, ws = x.chunk(world, -1), w.chunk(world, 1)
            ref = sum(L.linear(xs[r], ws[r]).float() for r in range(world)).to(torch.bfloat16)
            y = comm.linear_allreduce(xs[rank].contiguous().to(dev), ws[rank].contiguous().to(dev))
            torch.cuda.synchronize()
            assert comm.fallback_calls == 0, f"fused path not taken (T={T}): {comm.fallback_reason}"
            err = L.rel_err(y.cpu(), ref)
            assert err <= 1e-2, (T, err)
            parts = [torch.empty_like(y) for _ in range(world)]
            dist.all_gather(parts, y.contiguous())
            for p in parts:
                assert torch.equal(p, parts[0]), "ranks disagree"
        # fifty calls in a row on one shape
        gen = torch.Generator().manual_seed(99)
        x = torch.randn(256, K, generator=gen).to(torch.bfloat16)
        w = (torch.randn(N, K, generator=gen) * 0.02).to(torch.bfloat16)
        xd, wd = x.chunk(world, -1)[rank].contiguous().to(dev), w.chunk(world, 1)[rank].contiguous().to(dev)
        first = comm.linear_allreduce(xd, wd).clone()
        for _ in range(50):
            y = comm.linear_allreduce(xd, wd)
        torch.cuda.synchronize()
        assert torch.equal(y, first)
        assert b200.device_error(clear=True) == 0
    finally:
        comm.close()
        dist.destroy_process_group()


def _config1_worker(rank, world, port, one_shot):
    """BASELINE config 1 on the fused kernel: the reference's RowParallelLinear
    (F.linear per rank + all_reduce) gave the golden rows under gloo."""
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    sys.path[:0] = [os.path.dirname(here), os.path.join(os.path.dirname(here), "nano-vllm-diy_b200")]
    import torch.distributed as dist
    from oracle import layers as L
    from oracle import model as OM
    from src import b200
    from src.layers.tp_allreduce import FusedRowParallel
    dev = _init(rank, world, port)
    comm = FusedRowParallel(dev, max_tokens=512, max_hidden=1024, one_shot=one_shot)
    try:
        golden = torch.load(os.path.join(here, "golden", "row_parallel_c1.pt"))
        gen = torch.Generator().manual_seed(0)
        x = torch.randn(512, 3072, generator=gen).to(torch.bfloat16)
        w = (torch.randn(1024, 3072, generator=gen) * 0.02).to(torch.bfloat16)
        xs, ws = x.chunk(world, -1), w.chunk(world, 1)
        y = comm.linear_allreduce(xs[rank].contiguous().to(dev), ws[rank].contiguous().to(dev))
        torch.cuda.synchronize()
        assert comm.fallback_calls == 0, comm.fallback_reason
        yc = y.cpu()
        assert L.rel_err(yc[::64], golden["rows"]) <= 1e-2
        assert L.rel_err(yc, OM._row_parallel(x, w, world)) <= 1e-2
        ref32 = x.float() @ w.float().t()
        assert L.rel_err(yc, ref32) <= 1e-2
        parts = [torch.empty_like(y) for _ in range(world)]
        dist.all_gather(parts, y.contiguous())
        for p in parts:
            assert torch.equal(p, parts[0]), "ranks disagree"
        assert b200.device_error(clear=True) == 0
    finally:
        comm.close()
        dist.destroy_process_group()


def _exchange_worker(rank, world, port):
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    sys.path[:0] = [os.path.dirname(here), os.path.join(os.path.dirname(here), "nano-vllm-diy_b200")]
    import torch.distributed as dist
    from oracle import layers as L
    from src import b200
    from src.layers.tp_allreduce import FusedRowParallel
    dev = _init(rank, world, port)
    comm = FusedRowParallel(dev, max_tokens=512, max_hidden=1024)
    try:
        V, H, T, B = 151936, 1024, 300, 256
        Vs = V // world
        start = rank * Vs
        g = torch.Generator().manual_seed(5)
        table = torch.randn(V, H, generator=g).to(torch.bfloat16)
        shard = table[start:start + Vs].contiguous().to(dev)
        for rep in range(3):
            ids = torch.randint(-2, V + 2, (T,), generator=g)
            y = comm.embedding(ids.to(dev), shard, start, start + Vs, V)
            torch.cuda.synchronize()
            assert torch.equal(y.cpu(), L.vocab_embedding(ids, table, 0, V)), rep
        logits = (torch.randn(B, V, generator=g) * 2).to(torch.bfloat16)
        logits[::5, 7] = logits[::5, V - 3] = logits.max() + 1  # ties: the lower index wins
        local = logits[:, start:start + Vs].contiguous().to(dev)
        for rep in range(3):
            tok = comm.select_tokens(local, start)
            torch.cuda.synchronize()
            assert torch.equal(tok.cpu(), logits.float().argmax(-1)), rep
        temps = (torch.rand(B, generator=g) + 0.2).float()
        noise = torch.empty(B, V).exponential_(1, generator=g)
        tok = comm.select_tokens(local, start, temps.to(dev), noise[:, start:start + Vs].contiguous().to(dev))
        torch.cuda.synchronize()
        assert torch.equal(tok.cpu(), L.sample(logits, temps, noise))
        assert b200.device_error(clear=True) == 0
    finally:
        comm.close()
        dist.destroy_process_group()


def _model_worker(rank, world, port):
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    sys.path[:0] = [os.path.dirname(here), os.path.join(os.path.dirname(here), "nano-vllm-diy_b200")]
    import torch.distributed as dist
    from oracle import layers as L
    from oracle import model as OM
    from oracle.metadata import SeqState, prepare_seqs
    from oracle.weights import Qwen3Shape, random_weights
    from src import b200
    from src.engine.model_runner import ModelRunner
    from src.layers import tp_comm
    from src.layers.pos_embedding import _table_cpu
    from src.layers.tp_allreduce import FusedRowParallel
    dev = _init(rank, world, port)
    # 8 kv heads and 16 q heads: one kv head per rank at tp 8
    shape = Qwen3Shape(hidden=1024, layers=2, heads=16, kv_heads=8, head_dim=128, inter=2048,
                       vocab=4096, max_pos=4096)
    tp_comm.set_comm(FusedRowParallel(dev, max_tokens=512, max_hidden=shape.hidden))
    try:
        W = random_weights(shape, seed=21)
        runner = ModelRunner(shape.hf_config(), rank=rank, world_size=world, max_num_seqs=8,
                             max_seq_len=4096, device=dev)
        runner.load_weights(W.items())
        runner.allocate_kv_cache(8)
        runner.kv_cache.zero_()
        okv = OM.OracleKV(shape, 8, 256)
        cs = _table_cpu(shape.max_pos, shape.head_dim, float(shape.theta))
        g = torch.Generator().manual_seed(22)
        seqs = [SeqState(torch.randint(0, 4096, (n,), generator=g).tolist(), 0, n, [2 * i, 2 * i + 1])
                for i, n in enumerate((9, 300, 77))]
        runner.capture_cudagraph([4])
        for step in range(3):
            meta = prepare_seqs(seqs, 256)
            octx = {k: meta[k] for k in ("cu_seqlens_q", "cu_seqlens_k", "slot_mapping",
                                         "block_tables", "is_prefill")}
            ref = OM.compute_logits(shape, W, OM.forward(shape, W, meta["input_ids"], meta["positions"],
                                                         octx, okv, tp=world, cos_sin=cs), octx)
            ids, pos, ctx = runner.prepare(seqs)
            logits = runner.run_model(ids, pos, ctx)
            torch.cuda.synchronize()
            if rank == 0:
                err = L.rel_err(logits.cpu(), ref)
                assert err <= 2e-2, (step, err)
            # the same step again, tokens selected on the vocabulary shards:
            # every rank holds rank 0's argmax of the gathered logits
            toks = runner.step_tokens(seqs)
            every = [None] * world
            dist.all_gather_object(every, toks)
            assert all(t == every[0] for t in every), every
            if rank == 0:
                assert toks == logits.float().argmax(-1).tolist()
            for s, t in zip(seqs, ref.float().argmax(-1).tolist()):
                s.num_cached_tokens = len(s.token_ids)
                s.token_ids.append(int(t))
                s.num_scheduled_tokens = 1
        assert tp_comm.get().fused_calls > 0
        assert b200.device_error(clear=True) == 0
        runner.release_graphs()
    finally:
        tp_comm.clear()
        dist.destroy_process_group()


def _need(world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")


@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("one_shot", [True, False], ids=["one-shot", "two-shot"])
def test_fused_row_parallel_allreduce(world, one_shot):
    _need(world)
    import torch.multiprocessing as mp
    mp.spawn(_fused_worker, args=(world, _free_port(), one_shot), nprocs=world, join=True)


@pytest.mark.parametrize("one_shot", [True, False], ids=["one-shot", "two-shot"])
def test_fused_allreduce_config1_matches_reference_golden(one_shot):
    _need(2)
    import torch.multiprocessing as mp
    mp.spawn(_config1_worker, args=(2, _free_port(), one_shot), nprocs=2, join=True)


@pytest.mark.parametrize("world", [2, 4, 8])
def test_embedding_and_token_selection_exchanges(world):
    _need(world)
    import torch.multiprocessing as mp
    mp.spawn(_exchange_worker, args=(world, _free_port()), nprocs=world, join=True)


@pytest.mark.parametrize("world", [2, 4, 8])
def test_qwen3_tp_matches_oracle(world):
    _need(world)
    import torch.multiprocessing as mp
    mp.spawn(_model_worker, args=(world, _free_port()), nprocs=world, join=True)
