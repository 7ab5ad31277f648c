"""The oracle against golden vectors produced by the reference's own code
(tests/golden/make_golden.py, run on CPU).  CPU only.

Integer / byte work is bit-exact (KV scatter through the reference's Triton
kernel, ModelRunner.prepare_seqs metadata, weight-loader shards); bf16
floating point is bit-exact where the oracle evaluates the same fp32
expressions as the reference module (RMSNorm, RoPE, residual add) and held to
the stated relative tolerance elsewhere.
"""
import os

import pytest
import torch

from oracle import layers as L
from oracle import model as OM
from oracle.metadata import SeqState, prepare_seqs
from oracle.weights import Qwen3Shape, random_weights

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def load(name):
    return torch.load(os.path.join(GOLD, name), weights_only=False)


@pytest.mark.parametrize("dim", [1024, 128])
def test_rmsnorm_bit_exact(dim):
    d = load("layers.pt")[f"rmsnorm{dim}"]
    assert torch.equal(L.rms_norm(d["x"], d["w"], 1e-6), d["y"])
    y, r = L.rms_norm_residual(d["x"], d["r"], d["w"], 1e-6)
    assert torch.equal(y, d["y_res"])
    assert torch.equal(r, d["r_out"])


def test_rope_bit_exact():
    d = load("layers.pt")["rope"]
    cs = L.rope_cos_sin(d["max_pos"], 128, d["base"])
    q, k = L.rope(d["q"], d["k"], d["pos"], cs)
    assert torch.equal(q, d["q_out"])
    assert torch.equal(k, d["k_out"])


def test_silu_and_mul():
    d = load("layers.pt")["silu"]
    y = L.silu_and_mul(d["x"])
    # exp implementations may differ in the last fp32 bit -> at most one bf16 ulp
    assert L.rel_err(y, d["y"]) <= 8e-3
    assert (y == d["y"]).float().mean() > 0.99


def test_column_linear():
    d = load("layers.pt")["column"]
    assert L.rel_err(L.linear(d["x"], d["w"]), d["y"]) <= 1e-2


def test_weight_loader_shards_bit_exact():
    """The product's loaders (src.layers.linear) shard exactly like the reference's."""
    from src.layers.linear import (ColumnParallelLinear, MergedColumnParallelLinear,
                                   QKVParallelLinear, RowParallelLinear)
    shards = load("layers.pt")["shards"]
    src = shards["inputs"]
    bf = torch.bfloat16
    for rank in range(2):
        c = ColumnParallelLinear(128, 192, tp=(rank, 2))
        c.weight.data = c.weight.data.to(bf)
        c.weight.weight_loader(c.weight, src["w"])
        assert torch.equal(c.weight.data, shards[f"column_r{rank}"])
        m = MergedColumnParallelLinear(128, [192, 192], tp=(rank, 2))
        m.weight.data = m.weight.data.to(bf)
        m.weight.weight_loader(m.weight, src["w"], 0)
        m.weight.weight_loader(m.weight, src["up"], 1)
        assert torch.equal(m.weight.data, shards[f"merged_r{rank}"])
        q = QKVParallelLinear(128, 128, 4, 2, tp=(rank, 2))
        q.weight.data = q.weight.data.to(bf)
        q.weight.weight_loader(q.weight, src["q"], "q")
        q.weight.weight_loader(q.weight, src["k"], "k")
        q.weight.weight_loader(q.weight, src["v"], "v")
        assert torch.equal(q.weight.data, shards[f"qkv_r{rank}"])
        r = RowParallelLinear(192, 128, tp=(rank, 2))
        r.weight.data = r.weight.data.to(bf)
        r.weight.weight_loader(r.weight, src["row"])
        assert torch.equal(r.weight.data, shards[f"row_r{rank}"])


def test_store_kvcache_matches_reference_triton_kernel():
    d = load("kvcache.pt")
    kc, vc = d["k_cache_in"].clone(), d["v_cache_in"].clone()
    L.store_kvcache(d["k"], d["v"], kc, vc, d["slots"])
    assert torch.equal(kc, d["k_cache"])
    assert torch.equal(vc, d["v_cache"])


@pytest.mark.parametrize("case", ["fresh", "paged"])
def test_attention_against_sdpa(case):
    d = load("attention.pt")[case]
    scale = 128 ** -0.5
    if case == "fresh":
        out = L.varlen_attention(d["q"], d["k"], d["v"], d["cu_q"], d["cu_k"], scale)
    else:
        out = L.varlen_attention(d["q"], None, None, d["cu_q"], d["cu_k"], scale, d["k_cache"],
                                 d["v_cache"], d["block_table"])
    assert L.rel_err(out, d["out"]) <= 1e-2


def test_prepare_seqs_bit_exact():
    for batch in load("metadata.pt"):
        seqs = [SeqState(s["token_ids"], s["num_cached_tokens"], s["num_scheduled_tokens"],
                         s["block_table"]) for s in batch["seqs"]]
        m = prepare_seqs(seqs, 256)
        for key in ("input_ids", "positions", "cu_seqlens_q", "cu_seqlens_k", "context_lens",
                    "slot_mapping"):
            assert torch.equal(m[key], batch[key].to(m[key].dtype)), key
        if batch["block_tables"] is None:
            assert m["block_tables"] is None
        else:
            assert torch.equal(m["block_tables"], batch["block_tables"])
        assert m["max_seqlen_q"] == batch["max_seqlen_q"]
        assert m["max_seqlen_k"] == batch["max_seqlen_k"]
        assert m["is_prefill"] == batch["is_prefill"]


def test_row_parallel_config1():
    """BASELINE config 1 (gloo, world_size 2): the reference's ranks agree
    bit for bit, its error against fp32 is small, and the oracle's TP
    restatement reproduces the reference output within bf16 tolerance."""
    d = load("row_parallel_c1.pt")
    assert d["ranks_identical"]
    assert d["fp32_rel_err"] < 1e-2
    gen = torch.Generator().manual_seed(0)
    x = torch.randn(512, 3072, generator=gen).to(torch.bfloat16)
    w = (torch.randn(1024, 3072, generator=gen) * 0.02).to(torch.bfloat16)
    y = OM._row_parallel(x, w, 2)
    assert L.rel_err(y[::64], d["rows"]) <= 1e-2


def test_tiny_qwen3_model():
    """The oracle's Qwen3 forward (prefill + 3 paged decode steps) against the
    reference model's logits."""
    d = load("qwen3_tiny.pt")
    shape = Qwen3Shape(**d["shape"])
    W = random_weights(shape, seed=d["seed"])
    kv = OM.OracleKV(shape, 4, 256)
    cs = L.rope_cos_sin(shape.max_pos, shape.head_dim, shape.theta)
    for st in d["steps"]:
        ctx = dict(cu_seqlens_q=st["cu_seqlens_q"], cu_seqlens_k=st["cu_seqlens_k"],
                   slot_mapping=st["slot_mapping"], block_tables=st["block_tables"],
                   is_prefill=st["is_prefill"])
        h = OM.forward(shape, W, st["input_ids"], st["positions"], ctx, kv, cos_sin=cs)
        logits = OM.compute_logits(shape, W, h, ctx)
        assert L.rel_err(logits, st["logits"]) <= 2e-2
