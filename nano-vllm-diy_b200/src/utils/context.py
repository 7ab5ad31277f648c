"""Per-step attention metadata, the same record as the reference's
src/utils/context.py:5-14 (field names, order and defaults are part of the
interface that ModelRunner fills in and the layers read)."""
from dataclasses import dataclass

from torch import Tensor


@dataclass(slots=True)
class Context:
    is_prefill: bool = False
    cu_seqlens_q: Tensor | None = None      # int32 [B + 1]
    cu_seqlens_k: Tensor | None = None      # int32 [B + 1]
    max_seqlen_q: int = 0
    max_seqlen_k: int = 0
    slot_mapping: Tensor | None = None      # int32 [T], -1 = no cache write
    context_lens: Tensor | None = None      # int32 [B]
    block_tables: Tensor | None = None      # int32 [B, max_blocks], -1 padded
