"""The reference engine's call sequence, over this build's modules, on the GPU.

The reference's src/engine cannot be shipped to the GPU machine, so this
test restates, step for step, what its ModelRunner does to the model
(src/engine/model_runner.py), and checks the logits against the oracle:
  * the model is built under bf16 / cuda defaults with tp = (0, 1) and
    loaded from a safetensors checkpoint through Qwen3ForCausalLM.load
    (model_runner.py:31-36, src/utils/loader.py:12-28);
  * warmup_model: one eager forward of max_batched_seq_len // max_seq_len
    sequences of max_seq_len zeros with no block tables -- 2 x 8192 tokens,
    more than a CUDA-graph batch (model_runner.py:122-136);
  * allocate_kv_cache: one [2, L, blocks, 256, Hkv, d] tensor whose views are
    assigned to every module with k_cache and v_cache (model_runner.py:158-165);
  * capture_cudagraph: graph_vars zero-filled, batch sizes [1, 2, 4, 8, 16]
    captured largest first, each after an eager warm-up, with Context(
    is_prefill=True, max_seqlen_q=1, max_seqlen_k=max_seq_len=8192)
    (model_runner.py:269-315);
  * run_model: prefill eagerly, decode by replaying the smallest graph >= bs
    after filling graph_vars with -1 / 0 padding, then compute_logits
    (model_runner.py:241-259); prepare_seqs as restated by the oracle
    (model_runner.py:174-233, pinned to the reference's own output);
  * the Sampler (model_runner.py:262-266) on the logits with given Exp(1)
    draws, against the oracle's restatement of src/layers/sampler.py.
"""
import os
import tempfile

import pytest
import torch

from oracle import layers as L
from oracle import model as OM
from oracle.metadata import SeqState, prepare_seqs
from oracle.weights import Qwen3Shape, random_weights

pytestmark = pytest.mark.gpu

BLOCK = 256
MAX_SEQ_LEN = 8192            # RunnerConfig._max_seq_len (runner_config.py:9)
MAX_BATCHED = 16384           # RunnerConfig.max_batched_seq_len (runner_config.py:7)
MAX_NUM_SEQS = 16
SHAPE = Qwen3Shape(hidden=256, layers=2, heads=4, kv_heads=2, head_dim=128, inter=512, vocab=1000,
                   max_pos=MAX_SEQ_LEN)


def _ctx_dev(meta, dev):
    from src.utils.context import Context
    t = lambda x: None if x is None else x.to(dev)
    return Context(is_prefill=meta["is_prefill"], cu_seqlens_q=t(meta["cu_seqlens_q"]),
                   cu_seqlens_k=t(meta["cu_seqlens_k"]), max_seqlen_q=meta["max_seqlen_q"],
                   max_seqlen_k=meta["max_seqlen_k"], slot_mapping=t(meta["slot_mapping"]),
                   context_lens=t(meta["context_lens"]), block_tables=t(meta["block_tables"]))


@torch.inference_mode()
def test_reference_runner_sequence_over_this_build():
    from safetensors.torch import save_file
    from src.layers.sampler import Sampler
    from src.models.qwen3 import Qwen3ForCausalLM
    from src.utils.context import Context
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    W = random_weights(SHAPE, seed=61)
    ckpt = tempfile.mkdtemp()
    save_file({k: v.contiguous() for k, v in W.items()}, os.path.join(ckpt, "model.safetensors"))

    # model_runner.py:31-36
    prev_dtype, prev_dev = torch.get_default_dtype(), torch.get_default_device()
    torch.set_default_dtype(torch.bfloat16)
    torch.set_default_device("cuda")
    try:
        model = Qwen3ForCausalLM(SHAPE.hf_config(), tp=(0, 1))
        model.load(ckpt)
        sampler = Sampler()

        def run_model(input_ids, positions, is_prefill, ctx):  # model_runner.py:241-259
            if is_prefill or input_ids.size(0) > 512 or not graphs:
                return model.compute_logits(model(input_ids, positions, ctx), ctx)
            bs = input_ids.size(0)
            graph = graphs[next(x for x in graph_bs if x >= bs)]
            gv = graph_vars
            gv["input_ids"][:bs] = input_ids
            gv["positions"][:bs] = positions
            gv["slot_mapping"].fill_(-1)
            gv["slot_mapping"][:bs] = ctx.slot_mapping
            gv["cu_seqlens_q"].zero_()
            gv["cu_seqlens_q"][:bs + 1] = ctx.cu_seqlens_q
            gv["cu_seqlens_k"].zero_()
            gv["cu_seqlens_k"][:bs + 1] = ctx.cu_seqlens_k
            gv["block_tables"].fill_(-1)
            gv["block_tables"][:bs, :ctx.block_tables.size(1)] = ctx.block_tables
            graph.replay()
            return model.compute_logits(gv["outputs"][:bs], ctx)

        def run(seqs):  # model_runner.py:261-266 (logits; sampling below)
            meta = prepare_seqs(seqs, BLOCK)
            ctx = _ctx_dev(meta, dev)
            return run_model(meta["input_ids"].to(dev), meta["positions"].to(dev), meta["is_prefill"], ctx)

        graphs = {}
        graph_bs = []
        graph_vars = {}
        # warmup_model (model_runner.py:122-136)
        seq_len = min(MAX_BATCHED, MAX_SEQ_LEN)
        num_seqs = min(MAX_BATCHED // seq_len, MAX_NUM_SEQS)
        warm = [SeqState([0] * seq_len, 0, seq_len, []) for _ in range(num_seqs)]
        wl = run(warm)
        assert wl.shape == (num_seqs, SHAPE.vocab) and torch.isfinite(wl.float()).all()
        # allocate_kv_cache (model_runner.py:158-165)
        nblk = 16
        kv_cache = torch.zeros(2, SHAPE.layers, nblk, BLOCK, SHAPE.kv_heads, SHAPE.head_dim)
        layer_id = 0
        for module in model.modules():
            if hasattr(module, "k_cache") and hasattr(module, "v_cache"):
                module.k_cache = kv_cache[0, layer_id]
                module.v_cache = kv_cache[1, layer_id]
                layer_id += 1
        assert layer_id == SHAPE.layers
        # capture_cudagraph (model_runner.py:269-315)
        max_bs = min(MAX_NUM_SEQS, 512)
        max_num_blocks = (MAX_SEQ_LEN + BLOCK - 1) // BLOCK
        input_ids = torch.zeros(max_bs, dtype=torch.int64)
        positions = torch.zeros(max_bs, dtype=torch.int64)
        cu_seqlens_q = torch.zeros(max_bs + 1, dtype=torch.int32)
        cu_seqlens_k = torch.zeros(max_bs + 1, dtype=torch.int32)
        slot_mapping = torch.zeros(max_bs, dtype=torch.int32)
        block_tables = torch.zeros(max_bs, max_num_blocks, dtype=torch.int32)
        outputs = torch.zeros(max_bs, SHAPE.hidden)
        graph_bs = [1, 2, 4, 8] + list(range(16, max_bs + 1, 16))
        graph_pool = None
        for bs in reversed(graph_bs):
            graph = torch.cuda.CUDAGraph()
            ctx = Context(is_prefill=True, cu_seqlens_q=cu_seqlens_q[:bs + 1],
                          cu_seqlens_k=cu_seqlens_k[:bs + 1], max_seqlen_q=1, max_seqlen_k=MAX_SEQ_LEN,
                          slot_mapping=slot_mapping[:bs], block_tables=block_tables[:bs])
            outputs[:bs] = model(input_ids[:bs], positions[:bs], ctx)  # warmup
            with torch.cuda.graph(graph, graph_pool):
                outputs[:bs] = model(input_ids[:bs], positions[:bs], ctx)  # capture
            if graph_pool is None:
                graph_pool = graph.pool()
            graphs[bs] = graph
            torch.cuda.synchronize()
        graph_vars = dict(input_ids=input_ids, positions=positions, cu_seqlens_q=cu_seqlens_q,
                          cu_seqlens_k=cu_seqlens_k, slot_mapping=slot_mapping, block_tables=block_tables,
                          outputs=outputs)
        # the capture warm-ups wrote slot 0 (graph_vars start at zero, as in the
        # reference); the requests below use blocks from 1 on
    finally:
        torch.set_default_device(prev_dev)
        torch.set_default_dtype(prev_dtype)

    g = torch.Generator().manual_seed(62)
    seqs = [SeqState(torch.randint(0, SHAPE.vocab, (n,), generator=g).tolist(), 0, n,
                     [1 + 4 * i + j for j in range(4)]) for i, n in enumerate((37, 300, 5))]
    okv = OM.OracleKV(SHAPE, nblk, BLOCK)
    cs = L.rope_cos_sin(SHAPE.max_pos, SHAPE.head_dim, SHAPE.theta)
    from src import b200
    for step in range(4):  # prefill (eager), then three decode steps (graph of batch 4)
        meta = prepare_seqs(seqs, BLOCK)
        octx = {k: meta[k] for k in ("cu_seqlens_q", "cu_seqlens_k", "slot_mapping", "block_tables",
                                     "is_prefill")}
        ref = OM.compute_logits(SHAPE, W, OM.forward(SHAPE, W, meta["input_ids"], meta["positions"], octx,
                                                     okv, cos_sin=cs), octx)
        with torch.inference_mode():
            logits = run(seqs)
        torch.cuda.synchronize()
        assert L.rel_err(logits.cpu(), ref) <= 2e-2, step
        # the Sampler the runner calls, on given Exp(1) draws
        temps = torch.full((len(seqs),), 0.7)
        noise = torch.empty(len(seqs), SHAPE.vocab).exponential_(1, generator=g)
        toks = sampler(logits, temps.to(dev), noise=noise.to(dev)).tolist()
        assert toks == L.sample(logits.cpu(), temps, noise).tolist()
        for s, t in zip(seqs, toks):
            s.num_cached_tokens = len(s.token_ids)
            s.token_ids.append(int(t))
            s.num_scheduled_tokens = 1
    assert b200.device_error(clear=True) == 0
    graphs.clear()
