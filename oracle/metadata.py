"""Restatement of ModelRunner.prepare_seqs (src/engine/model_runner.py:168-233).

Test infrastructure only.  Integer work, so the result must be bit-exact
against the reference (pinned by tests/golden/metadata.pt).
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np
import torch


@dataclass
class SeqState:
    """The fields of src/engine/sequence.py:Sequence that prepare_seqs reads."""
    token_ids: list[int]
    num_cached_tokens: int = 0
    num_scheduled_tokens: int = 0
    block_table: list[int] = field(default_factory=list)

    def __len__(self) -> int:
        return len(self.token_ids)


def prepare_seqs(seqs: list[SeqState], block_size: int) -> dict:
    """Per sequence (model_runner.py:184-210):
        start = min(num_cached_tokens, len - 1); end = start + num_scheduled
        tokens / positions [start, end); cu_seqlens_q += end - start;
        cu_seqlens_k += end; slot(p) = block_table[p // bs] * bs + p % bs
    Block tables (-1 padded) only when some sequence has cached keys
    (cu_seqlens_k[-1] > cu_seqlens_q[-1], model_runner.py:211-212).
    is_prefill is False only for max_seqlen_q == 1 (model_runner.py:229-232)."""
    ids, pos, slots = [], [], []
    cu_q, cu_k, ctx_lens = [0], [0], []
    max_q = max_k = 0
    for s in seqs:
        n = len(s)
        start = min(s.num_cached_tokens, n - 1)
        lq = s.num_scheduled_tokens
        end = start + lq
        ids.append(np.asarray(s.token_ids[start:end], dtype=np.int64))
        p = np.arange(start, end, dtype=np.int64)
        pos.append(p)
        cu_q.append(cu_q[-1] + lq)
        cu_k.append(cu_k[-1] + end)
        ctx_lens.append(end)
        max_q = max(max_q, lq)
        max_k = max(max_k, end)
        if not s.block_table:
            continue
        bt = np.asarray(s.block_table, dtype=np.int64)
        slots.append(bt[p // block_size] * block_size + p % block_size)
    block_tables = None
    if cu_k[-1] > cu_q[-1]:
        width = max(len(s.block_table) for s in seqs)
        bt = np.full((len(seqs), width), -1, dtype=np.int32)
        for i, s in enumerate(seqs):
            bt[i, :len(s.block_table)] = s.block_table
        block_tables = torch.from_numpy(bt)
    cat = lambda parts, dt: torch.from_numpy(np.concatenate(parts).astype(dt)) if parts else torch.empty(0, dtype=torch.int64 if dt == np.int64 else torch.int32)
    return dict(
        input_ids=cat(ids, np.int64),
        positions=cat(pos, np.int64),
        cu_seqlens_q=torch.tensor(cu_q, dtype=torch.int32),
        cu_seqlens_k=torch.tensor(cu_k, dtype=torch.int32),
        context_lens=torch.tensor(ctx_lens, dtype=torch.int32),
        slot_mapping=cat(slots, np.int32),
        block_tables=block_tables,
        max_seqlen_q=max_q,
        max_seqlen_k=max_k,
        is_prefill=max_q != 1,
    )
