"""Delta-encoded step messages to the worker ranks (src.engine.rpc), CPU only.

The reference pickles every scheduled Sequence whole into a 1 MiB shared
block for every step (src/engine/model_runner.py:99-120).  Here rank 0
sends deltas; the worker's mirrors must equal rank 0's sequences after every
step -- token lists, cached / scheduled counts, block tables, temperatures --
so prepare_seqs (the oracle's restatement of model_runner.py:174-233) gives
the worker the same step metadata, through prefill chunks, decode appends,
block-table growth and replacement, preemption (a table cleared and
re-grown), sequences leaving and coming back, and dropped state.
"""
import hashlib
import multiprocessing as mp
import pickle
import random
import uuid
from dataclasses import dataclass, field

import numpy as np
import torch

from oracle.metadata import prepare_seqs

BLOCK = 256


@dataclass
class FakeSeq:
    seq_id: int
    token_ids: list
    num_cached_tokens: int = 0
    num_scheduled_tokens: int = 0
    block_table: list = field(default_factory=list)
    temperature: float = 1.0

    def __len__(self):
        return len(self.token_ids)

    def __getitem__(self, k):
        return self.token_ids[k]


def _evolve(rng, live, next_id, next_block):
    """One scheduler-like step over the live sequences; returns the batch."""
    if rng.random() < 0.3 or not live:
        n = rng.randint(1, 1500)
        live.append(FakeSeq(next_id[0], [rng.randint(0, 151935) for _ in range(n)],
                            temperature=rng.choice([0.6, 1.0, 1.3])))
        next_id[0] += 1
    batch = []
    for s in list(live):
        r = rng.random()
        if r < 0.05:
            live.remove(s)           # finished
            continue
        if r < 0.15:
            continue                 # not scheduled this step
        if r < 0.18:
            s.block_table = []       # preempted: blocks freed
            s.num_cached_tokens = 0
        if s.num_cached_tokens < len(s) - 1:   # prefill, possibly chunked
            s.num_scheduled_tokens = min(len(s) - s.num_cached_tokens, rng.choice([512, 10 ** 6]))
        else:
            s.num_scheduled_tokens = 1
        need = (s.num_cached_tokens + s.num_scheduled_tokens + BLOCK - 1) // BLOCK
        while len(s.block_table) < need:
            s.block_table.append(next_block[0])
            next_block[0] += 1
        if r > 0.97 and s.block_table:
            s.block_table[0] = next_block[0]   # a table entry replaced
            next_block[0] += 1
        batch.append(s)
    return batch


def _advance(batch, rng):
    for s in batch:
        s.num_cached_tokens += s.num_scheduled_tokens
        if s.num_cached_tokens >= len(s):
            s.token_ids.append(rng.randint(0, 151935))


def _same(a, b):
    return (a.token_ids == b.token_ids and a.num_cached_tokens == b.num_cached_tokens
            and a.num_scheduled_tokens == b.num_scheduled_tokens and a.block_table == b.block_table
            and abs(a.temperature - b.temperature) < 1e-6)


def test_mirrors_follow_the_sequences():
    from src.engine.rpc import StepDecoder, StepEncoder
    rng = random.Random(0)
    enc, dec = StepEncoder(keep_steps=5), StepDecoder()
    live, next_id, next_block = [], [0], [0]
    for step in range(300):
        batch = _evolve(rng, live, next_id, next_block)
        method, got = dec.decode(enc.encode("run", batch))
        assert method == "run" and len(got) == len(batch)
        for a, b in zip(got, batch):
            assert a.seq_id == b.seq_id and _same(a, b), (step, b.seq_id)
        if batch:
            ma, mb = prepare_seqs(got, BLOCK), prepare_seqs(batch, BLOCK)
            for k in ("input_ids", "positions", "cu_seqlens_q", "cu_seqlens_k", "slot_mapping"):
                assert torch.equal(ma[k], mb[k]), (step, k)
        _advance(batch, rng)
    # state for sequences gone longer than keep_steps was dropped on both sides
    assert set(dec.seqs) == set(enc.sent)


def test_decode_step_bytes():
    """256 sequences of ~1k tokens in decode: deltas of ~30 bytes per
    sequence against pickling every Sequence whole."""
    from src.engine.rpc import StepDecoder, StepEncoder
    rng = random.Random(1)
    seqs = [FakeSeq(i, [rng.randint(0, 151935) for _ in range(rng.randint(100, 2048))],
                    block_table=[]) for i in range(256)]
    for s in seqs:
        s.num_cached_tokens = len(s) - 1
        s.num_scheduled_tokens = 1
        s.block_table = list(range(1000 * s.seq_id, 1000 * s.seq_id + (len(s) + BLOCK - 1) // BLOCK))
    enc, dec = StepEncoder(), StepDecoder()
    first = enc.encode("run", seqs)          # the whole state once
    dec.decode(first)
    for s in seqs:
        s.token_ids.append(7)
        s.num_cached_tokens += 1
    step = enc.encode("run", seqs)
    _, got = dec.decode(step)
    assert all(_same(a, b) for a, b in zip(got, seqs))
    full = len(pickle.dumps(["run", seqs]))
    assert len(step) <= 40 * 256 + 16, len(step)
    assert full > 100 * len(step), (full, len(step))


def _receiver(name, ev, done, q, steps):
    from src.engine.rpc import ShmChannel, StepDecoder
    ch = ShmChannel(name)
    dec = StepDecoder()
    for _ in range(steps):
        ev.wait()
        ev.clear()
        method, seqs = dec.decode(ch.read())
        h = hashlib.sha256()
        for s in seqs:
            h.update(np.asarray(s.token_ids + s.block_table + [s.num_cached_tokens, s.num_scheduled_tokens],
                                dtype=np.int64).tobytes())
        q.put(h.hexdigest())
        done.set()
    ch.close()


def test_two_processes_over_shared_memory():
    """Rank 0 writes, a spawned worker reads; one message outgrows the 64 KiB
    block and moves the channel to a larger one."""
    import sys
    from src.engine.rpc import ShmChannel, StepEncoder
    ctx = mp.get_context("spawn")
    name = "b200rpc_" + uuid.uuid4().hex[:12]
    ch = ShmChannel(name, size=1 << 16, create=True)
    ev, done, q = ctx.Event(), ctx.Event(), ctx.Queue()
    steps = 40
    p = ctx.Process(target=_receiver, args=(name, ev, done, q, steps))
    p.start()
    try:
        rng = random.Random(2)
        enc = StepEncoder()
        live, next_id, next_block = [], [0], [0]
        for step in range(steps):
            batch = _evolve(rng, live, next_id, next_block)
            if step == 20:  # a large prefill batch: several hundred KiB
                for i in range(40):
                    big = FakeSeq(next_id[0], [rng.randint(0, 151935) for _ in range(4000)])
                    next_id[0] += 1
                    big.num_scheduled_tokens = 4000
                    big.block_table = list(range(next_block[0], next_block[0] + 16))
                    next_block[0] += 16
                    live.append(big)
                    batch.append(big)
            ch.write(enc.encode("run", batch))
            done.clear()
            ev.set()
            h = hashlib.sha256()
            for s in batch:
                h.update(np.asarray(s.token_ids + s.block_table + [s.num_cached_tokens,
                                                                   s.num_scheduled_tokens],
                                    dtype=np.int64).tobytes())
            assert q.get(timeout=60) == h.hexdigest(), step
            assert done.wait(timeout=60)
            _advance(batch, rng)
        assert ch.generation >= 1
    finally:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
        ch.close()
    assert p.exitcode == 0
