"""Step messages from rank 0 to the other tensor-parallel ranks, as deltas.

The reference's ModelRunner sends every call to the worker ranks as
pickle([method, *args]) through a 1 MiB shared-memory block
(src/engine/model_runner.py:99-120): each `run(seqs)` pickles every
scheduled Sequence whole -- its full token list included -- so a decode step
of 256 sequences of ~1k tokens moves megabytes (and overflows the 1 MiB
block).  Here rank 0 keeps, per sequence id, what it last sent and encodes a
step as
  header  u32 magic, u32 method id, u32 sequences, u32 dropped ids
  dropped ids (u64 each): sequences the receiver should forget
  per sequence: u64 seq_id, u32 flags, u32 num_cached_tokens,
                u32 num_scheduled_tokens, f32 temperature,
                u32 new tokens + the token ids appended since the last send
                (int32 each; all of them when FULL_TOKENS),
                u32 new block entries + the entries (int32; the whole table
                when FULL_BLOCKS)
so a decode step costs ~30 bytes per sequence.  The receiver (StepDecoder)
holds a mirror of every live sequence and returns Sequence-like objects with
the fields ModelRunner.prepare_seqs and the sampler read (token_ids,
num_cached_tokens, num_scheduled_tokens, block_table, temperature, len,
indexing).  Whatever changes in a way a delta cannot express (a token list
that shrank, a block table whose sent prefix changed, a sequence the
receiver forgot) is sent whole, so the mirror is always exact.  Sequences
absent from `keep_steps` consecutive messages are dropped on both sides.

ShmChannel carries the bytes: a shared-memory block with a u32 length prefix
(grown by re-creating the block under a new name when a message does not
fit), signalled with one multiprocessing Event per receiving rank, as the
reference does.
"""
from __future__ import annotations

import struct
from dataclasses import dataclass, field
from multiprocessing.shared_memory import SharedMemory

import numpy as np

MAGIC = 0xB200D17A
FULL_TOKENS = 1
FULL_BLOCKS = 2
METHODS = ["run", "exit", "call"]


@dataclass
class SeqMirror:
    """The receiver's copy of one sequence (the fields the runner reads)."""
    seq_id: int
    token_ids: list = field(default_factory=list)
    num_cached_tokens: int = 0
    num_scheduled_tokens: int = 0
    block_table: list = field(default_factory=list)
    temperature: float = 1.0

    def __len__(self) -> int:
        return len(self.token_ids)

    def __getitem__(self, key):
        return self.token_ids[key]


class StepEncoder:
    """Rank 0 side: encodes (method, seqs) as deltas against what it sent."""

    def __init__(self, keep_steps: int = 64):
        self.keep_steps = keep_steps
        self.sent: dict[int, tuple[int, int, tuple]] = {}  # seq_id -> (tokens, block entries, block prefix)
        self.last_seen: dict[int, int] = {}
        self.step = 0

    def encode(self, method: str, seqs=()) -> bytes:
        self.step += 1
        dropped = [sid for sid, st in self.last_seen.items()
                   if self.step - st > self.keep_steps and sid not in {s.seq_id for s in seqs}]
        for sid in dropped:
            self.sent.pop(sid, None)
            self.last_seen.pop(sid, None)
        parts = [struct.pack("<IIII", MAGIC, METHODS.index(method), len(seqs), len(dropped))]
        if dropped:
            parts.append(np.asarray(dropped, dtype=np.uint64).tobytes())
        for s in seqs:
            sid = s.seq_id
            toks = s.token_ids
            table = s.block_table
            prev = self.sent.get(sid)
            flags = 0
            if prev is None or prev[0] > len(toks):
                flags |= FULL_TOKENS
                new_toks = toks
            else:
                new_toks = toks[prev[0]:]
            if prev is None or prev[1] > len(table) or tuple(table[:prev[1]]) != prev[2]:
                flags |= FULL_BLOCKS
                new_blocks = table
            else:
                new_blocks = table[prev[1]:]
            parts.append(struct.pack("<QIIIfI", sid, flags, s.num_cached_tokens, s.num_scheduled_tokens,
                                     float(getattr(s, "temperature", 1.0)), len(new_toks)))
            parts.append(np.asarray(new_toks, dtype=np.int32).tobytes())
            parts.append(struct.pack("<I", len(new_blocks)))
            parts.append(np.asarray(new_blocks, dtype=np.int32).tobytes())
            self.sent[sid] = (len(toks), len(table), tuple(table))
            self.last_seen[sid] = self.step
        return b"".join(parts)


class StepDecoder:
    """Worker side: applies messages to its mirrors; returns (method, seqs)."""

    def __init__(self):
        self.seqs: dict[int, SeqMirror] = {}

    def decode(self, buf) -> tuple[str, list[SeqMirror]]:
        mv = memoryview(buf)
        magic, method, n, ndrop = struct.unpack_from("<IIII", mv, 0)
        if magic != MAGIC:
            raise ValueError("not a step message")
        off = 16
        if ndrop:
            for sid in np.frombuffer(mv, dtype=np.uint64, count=ndrop, offset=off).tolist():
                self.seqs.pop(int(sid), None)
            off += 8 * ndrop
        out = []
        for _ in range(n):
            sid, flags, cached, sched, temp, ntok = struct.unpack_from("<QIIIfI", mv, off)
            off += struct.calcsize("<QIIIfI")
            toks = np.frombuffer(mv, dtype=np.int32, count=ntok, offset=off).tolist()
            off += 4 * ntok
            (nblk,) = struct.unpack_from("<I", mv, off)
            off += 4
            blocks = np.frombuffer(mv, dtype=np.int32, count=nblk, offset=off).tolist()
            off += 4 * nblk
            m = self.seqs.get(sid)
            if m is None:
                if not (flags & FULL_TOKENS and flags & FULL_BLOCKS):
                    raise ValueError(f"delta for unknown sequence {sid}")
                m = self.seqs[sid] = SeqMirror(sid)
            if flags & FULL_TOKENS:
                m.token_ids = toks
            else:
                m.token_ids.extend(toks)
            if flags & FULL_BLOCKS:
                m.block_table = blocks
            else:
                m.block_table.extend(blocks)
            m.num_cached_tokens = cached
            m.num_scheduled_tokens = sched
            m.temperature = temp
            out.append(m)
        return METHODS[method], out


class ShmChannel:
    """One writer (rank 0), any number of readers, one message in flight."""

    HEADER = 8  # u32 length, u32 generation (bumped when the block is re-created)

    def __init__(self, name: str, size: int = 1 << 20, create: bool = False):
        self.base = name
        self.generation = 0
        self.create = create
        self.shm = SharedMemory(name=self._name(0), create=create, size=size if create else 0)

    def _name(self, gen: int) -> str:
        return self.base if gen == 0 else f"{self.base}_{gen}"

    def write(self, data: bytes) -> None:
        need = self.HEADER + len(data)
        if need > self.shm.size:
            # grow: a new block under the next name; readers follow the
            # generation number left in the old block's header
            old = self.shm
            self.generation += 1
            self.shm = SharedMemory(name=self._name(self.generation), create=True, size=max(need, 2 * old.size))
            struct.pack_into("<II", old.buf, 0, 0xFFFFFFFF, self.generation)
            old.close()
            self._retired = getattr(self, "_retired", []) + [old]
        self.shm.buf[self.HEADER:need] = data
        struct.pack_into("<II", self.shm.buf, 0, len(data), self.generation)

    def read(self) -> bytes:
        n, gen = struct.unpack_from("<II", self.shm.buf, 0)
        while n == 0xFFFFFFFF:  # the writer moved to a larger block
            self.shm.close()
            self.generation = gen
            self.shm = SharedMemory(name=self._name(gen))
            n, gen = struct.unpack_from("<II", self.shm.buf, 0)
        return bytes(self.shm.buf[self.HEADER:self.HEADER + n])

    def close(self) -> None:
        self.shm.close()
        if self.create:
            for old in getattr(self, "_retired", []):
                old.unlink()
            self.shm.unlink()
