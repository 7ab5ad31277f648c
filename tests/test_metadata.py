"""Host metadata (src.engine.metadata.build) vs the oracle's restatement of
ModelRunner.prepare_seqs: integer work, bit-exact (CPU only)."""
import random

import numpy as np
import pytest
import torch

from oracle.metadata import SeqState, prepare_seqs


def _random_batch(rng: random.Random, block_size: int, allow_warmup: bool):
    seqs = []
    next_block = 0
    for _ in range(rng.randint(1, 12)):
        n = rng.randint(1, 3000)
        toks = [rng.randint(0, 151935) for _ in range(n)]
        mode = rng.choice(["fresh", "decode", "chunk", "prefix"] + (["warmup"] if allow_warmup else []))
        if mode == "fresh":
            cached, sched = 0, n
        elif mode == "decode":
            cached, sched = n - 1, 1
        elif mode == "chunk":
            cached = rng.randint(0, n - 1) // block_size * block_size
            sched = rng.randint(1, n - cached)
        elif mode == "prefix":
            cached = rng.randint(0, (n - 1) // block_size) * block_size
            sched = n - cached
        else:
            cached, sched = 0, n
        nblocks = (cached + sched + block_size - 1) // block_size
        table = [] if mode == "warmup" else list(range(next_block, next_block + nblocks))
        rng.shuffle(table)
        next_block += nblocks
        seqs.append(SeqState(toks, cached, sched, table))
    if allow_warmup:
        for s in seqs:
            s.block_table = []
            s.num_cached_tokens = 0
            s.num_scheduled_tokens = len(s)
    return seqs


@pytest.mark.parametrize("seed", range(12))
@pytest.mark.parametrize("block_size", [256, 512])
def test_build_matches_prepare_seqs(seed, block_size):
    from src.engine.metadata import build
    rng = random.Random(seed)
    seqs = _random_batch(rng, block_size, allow_warmup=(seed == 0))
    ref = prepare_seqs(seqs, block_size)
    got = build(seqs, block_size)
    assert np.array_equal(got.input_ids, ref["input_ids"].numpy())
    assert np.array_equal(got.positions, ref["positions"].numpy())
    assert np.array_equal(got.cu_seqlens_q, ref["cu_seqlens_q"].numpy())
    assert np.array_equal(got.cu_seqlens_k, ref["cu_seqlens_k"].numpy())
    assert np.array_equal(got.context_lens, ref["context_lens"].numpy())
    assert np.array_equal(got.slot_mapping, ref["slot_mapping"].numpy())
    assert got.max_seqlen_q == ref["max_seqlen_q"] and got.max_seqlen_k == ref["max_seqlen_k"]
    assert got.is_prefill == ref["is_prefill"]
    if ref["block_tables"] is None:
        assert got.block_tables is None
    else:
        assert np.array_equal(got.block_tables, ref["block_tables"].numpy())


def test_decode_batch_properties():
    """Pure decode: one token per sequence at position len-1, no prefill flag."""
    from src.engine.metadata import build
    seqs = [SeqState(list(range(n)), n - 1, 1, [i * 20 + j for j in range((n + 255) // 256)])
            for i, n in enumerate([1, 2, 256, 257, 1000])]
    m = build(seqs, 256)
    assert not m.is_prefill
    assert m.positions.tolist() == [0, 1, 255, 256, 999]
    assert m.slot_mapping.tolist() == [0 * 256 + 0, 20 * 256 + 1, 40 * 256 + 255,
                                       61 * 256 + 0, 83 * 256 + 999 % 256]
    assert m.block_tables is not None and m.block_tables.shape == (5, 4)
    assert m.block_tables[0].tolist() == [0, -1, -1, -1]


@pytest.mark.gpu
@pytest.mark.parametrize("seed", range(12))
@pytest.mark.parametrize("block_size", [256, 512])
def test_device_builder_matches_prepare_seqs(seed, block_size):
    """The device-side expansion (b200_step_metadata) against the oracle's
    restatement of prepare_seqs, bit-exact, warm-up batches included."""
    from src.engine.metadata import build_on_device
    rng = random.Random(seed)
    seqs = _random_batch(rng, block_size, allow_warmup=(seed == 0))
    ref = prepare_seqs(seqs, block_size)
    ids, pos, ctx = build_on_device(seqs, block_size, torch.device("cuda", 0))
    torch.cuda.synchronize()
    assert torch.equal(ids.cpu(), ref["input_ids"])
    assert torch.equal(pos.cpu(), ref["positions"])
    assert torch.equal(ctx.cu_seqlens_q.cpu(), ref["cu_seqlens_q"])
    assert torch.equal(ctx.cu_seqlens_k.cpu(), ref["cu_seqlens_k"])
    assert torch.equal(ctx.context_lens.cpu(), ref["context_lens"])
    assert torch.equal(ctx.slot_mapping.cpu(), ref["slot_mapping"])
    assert ctx.max_seqlen_q == ref["max_seqlen_q"] and ctx.max_seqlen_k == ref["max_seqlen_k"]
    assert ctx.is_prefill == ref["is_prefill"]
    if ref["block_tables"] is None:
        assert ctx.block_tables is None
    else:
        assert torch.equal(ctx.block_tables.cpu(), ref["block_tables"])
    from src import b200
    assert b200.device_error(clear=True) == 0


@pytest.mark.gpu
def test_device_builder_against_reference_goldens():
    """The batches the reference's own prepare_seqs ran on (tests/golden/metadata.pt)."""
    from src.engine.metadata import build_on_device
    import os
    batches = torch.load(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "metadata.pt"))
    for batch in batches:
        seqs = [SeqState(s["token_ids"], s["num_cached_tokens"], s["num_scheduled_tokens"],
                         s["block_table"]) for s in batch["seqs"]]
        ids, pos, ctx = build_on_device(seqs, 256, torch.device("cuda", 0))
        torch.cuda.synchronize()
        got = {"input_ids": ids, "positions": pos, "cu_seqlens_q": ctx.cu_seqlens_q,
               "cu_seqlens_k": ctx.cu_seqlens_k, "context_lens": ctx.context_lens,
               "slot_mapping": ctx.slot_mapping}
        for key, t in got.items():
            assert torch.equal(t.cpu(), batch[key].to(t.dtype)), key
        if batch["block_tables"] is None:
            assert ctx.block_tables is None
        else:
            assert torch.equal(ctx.block_tables.cpu(), batch["block_tables"])
        assert ctx.max_seqlen_q == batch["max_seqlen_q"] and ctx.max_seqlen_k == batch["max_seqlen_k"]
        assert ctx.is_prefill == batch["is_prefill"]
