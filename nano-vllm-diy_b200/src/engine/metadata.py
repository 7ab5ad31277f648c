"""Attention metadata of one forward step, built on the host with numpy.

Same result as the reference's ModelRunner.prepare_seqs
(src/engine/model_runner.py:174-233): for each sequence, start =
min(num_cached_tokens, len - 1), end = start + num_scheduled_tokens; tokens and
positions [start, end); cu_seqlens_q / cu_seqlens_k prefix sums of (end -
start) / end; slot(p) = block_table[p // block_size] * block_size +
p % block_size; -1-padded block tables only when some sequence attends to
cached keys; is_prefill unless every query length is 1.

Two builders with the same result:
  * build + to_device: every array on the host (numpy), six pinned copies;
  * build_on_device: the host prepares only per-sequence values (start,
    query length, block-table length: O(B)), the block tables and the token
    ids; one kernel (b200_step_metadata) expands positions, slot mapping and
    the prefix sums on the GPU.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

from src.utils.context import Context


@dataclass
class StepMeta:
    input_ids: np.ndarray      # int64 [T]
    positions: np.ndarray      # int64 [T]
    cu_seqlens_q: np.ndarray   # int32 [B + 1]
    cu_seqlens_k: np.ndarray   # int32 [B + 1]
    context_lens: np.ndarray   # int32 [B]
    slot_mapping: np.ndarray   # int32 [T] (empty while no sequence has blocks)
    block_tables: np.ndarray | None  # int32 [B, max_blocks]
    max_seqlen_q: int
    max_seqlen_k: int

    @property
    def is_prefill(self) -> bool:
        return self.max_seqlen_q != 1


def build(seqs, block_size: int) -> StepMeta:
    """`seqs`: objects with token_ids (or __getitem__/__len__),
    num_cached_tokens, num_scheduled_tokens and block_table."""
    B = len(seqs)
    lens = np.fromiter((len(s) for s in seqs), dtype=np.int64, count=B)
    cached = np.fromiter((s.num_cached_tokens for s in seqs), dtype=np.int64, count=B)
    lq = np.fromiter((s.num_scheduled_tokens for s in seqs), dtype=np.int64, count=B)
    start = np.minimum(cached, lens - 1)
    end = start + lq
    cu_q = np.zeros(B + 1, dtype=np.int32)
    cu_k = np.zeros(B + 1, dtype=np.int32)
    np.cumsum(lq, out=cu_q[1:])
    np.cumsum(end, out=cu_k[1:])
    T = int(cu_q[-1])
    ids = np.empty(T, dtype=np.int64)
    seq_of_tok = np.repeat(np.arange(B), lq)
    positions = (np.arange(T, dtype=np.int64) - np.repeat(cu_q[:-1].astype(np.int64), lq)
                 + np.repeat(start, lq))
    for i, s in enumerate(seqs):
        a, b = int(start[i]), int(end[i])
        toks = s.token_ids if hasattr(s, "token_ids") else [s[j] for j in range(len(s))]
        ids[cu_q[i]:cu_q[i + 1]] = toks[a:b]
    width = max((len(s.block_table) for s in seqs), default=0)
    bt = np.full((B, max(width, 1)), -1, dtype=np.int32)
    has_blocks = np.zeros(B, dtype=bool)
    for i, s in enumerate(seqs):
        if s.block_table:
            bt[i, :len(s.block_table)] = s.block_table
            has_blocks[i] = True
    tok_has = has_blocks[seq_of_tok]
    blk = bt[seq_of_tok[tok_has], positions[tok_has] // block_size].astype(np.int64)
    slots = (blk * block_size + positions[tok_has] % block_size).astype(np.int32)
    block_tables = bt[:, :width] if (cu_k[-1] > cu_q[-1] and width > 0) else None
    return StepMeta(ids, positions, cu_q, cu_k, end.astype(np.int32), slots, block_tables,
                    int(lq.max(initial=0)), int(end.max(initial=0)))


def to_device(meta: StepMeta, device) -> tuple[torch.Tensor, torch.Tensor, Context]:
    """Pinned host copies -> device (non-blocking), wrapped in a Context."""
    def dev(a):
        return torch.from_numpy(np.ascontiguousarray(a)).pin_memory().to(device, non_blocking=True)

    ctx = Context(
        is_prefill=meta.is_prefill,
        cu_seqlens_q=dev(meta.cu_seqlens_q),
        cu_seqlens_k=dev(meta.cu_seqlens_k),
        max_seqlen_q=meta.max_seqlen_q,
        max_seqlen_k=meta.max_seqlen_k,
        slot_mapping=dev(meta.slot_mapping),
        context_lens=dev(meta.context_lens),
        block_tables=dev(meta.block_tables) if meta.block_tables is not None else None,
    )
    return dev(meta.input_ids), dev(meta.positions), ctx


def build_on_device(seqs, block_size: int, device) -> tuple[torch.Tensor, torch.Tensor, Context]:
    """The step's (input_ids, positions, Context) with the per-token expansion
    done by the b200_step_metadata kernel."""
    from src import b200
    B = len(seqs)
    lens = np.fromiter((len(s) for s in seqs), dtype=np.int64, count=B)
    cached = np.fromiter((s.num_cached_tokens for s in seqs), dtype=np.int64, count=B)
    lq = np.fromiter((s.num_scheduled_tokens for s in seqs), dtype=np.int64, count=B)
    nblk = np.fromiter((len(s.block_table) for s in seqs), dtype=np.int64, count=B)
    start = np.minimum(cached, lens - 1)
    end = start + lq
    T = int(lq.sum())
    ids = np.empty(T, dtype=np.int64)
    o = 0
    for i, s in enumerate(seqs):
        n = int(lq[i])
        toks = s.token_ids if hasattr(s, "token_ids") else [s[j] for j in range(len(s))]
        ids[o:o + n] = toks[int(start[i]):int(end[i])]
        o += n
    width = int(nblk.max(initial=0))
    attends_cache = int(end.sum()) > T  # prefix hits / decode (model_runner.py:211-212)
    info = np.stack([start, lq, nblk]).astype(np.int32)
    pinned = torch.from_numpy(info).pin_memory()
    seq_info = pinned.to(device, non_blocking=True)
    bt_dev = None
    if width > 0:
        bt = np.full((B, width), -1, dtype=np.int32)
        for i, s in enumerate(seqs):
            if s.block_table:
                bt[i, :len(s.block_table)] = s.block_table
        bt_dev = torch.from_numpy(bt).pin_memory().to(device, non_blocking=True)
    ids_dev = torch.from_numpy(ids).pin_memory().to(device, non_blocking=True)
    n_slot = int(lq[nblk > 0].sum())
    positions, slots, cu_q, cu_k, ctx_lens = b200.step_metadata(seq_info, bt_dev, block_size, T, n_slot)
    max_q = int(lq.max(initial=0))
    ctx = Context(
        is_prefill=max_q != 1,
        cu_seqlens_q=cu_q,
        cu_seqlens_k=cu_k,
        max_seqlen_q=max_q,
        max_seqlen_k=int(end.max(initial=0)),
        slot_mapping=slots,
        context_lens=ctx_lens,
        block_tables=((bt_dev if width > 0 else torch.empty(B, 0, dtype=torch.int32, device=device))
                      if attends_cache else None),
    )
    return ids_dev, positions, ctx
