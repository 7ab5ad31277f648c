"""Fused RowParallelLinear (GEMM + all-reduce over NVLink) for tp > 1.

The reference computes y_r = F.linear(x_r, W_r) on every rank and sums with
torch.distributed.all_reduce (src/layers/linear.py:169-173).  Here one kernel
per rank does both: each CTA's bf16 partial goes by NVLink peer stores to
the rank(s) that reduce it, the world's partials are summed in a fixed rank
order (identical results on every rank), and the result lands in every
rank's output buffer (libb200ops: b200_linear_allreduce).

Two exchange patterns (the same on every rank):
  one-shot (world == 2): every rank pushes its partial to every rank and
    sums its own copy -- one NVLink hop;
  two-shot (larger worlds): the rows of each output part are split among
    the ranks; each sums its rows and writes them to every rank -- 2 (w-1)/w
    of the bytes (measured faster from 4 ranks up).

Symmetric memory: every rank allocates one device buffer holding
  stage  bf16 [halves][world][max_tokens][ldo]  partials received
  out    bf16 [2][max_tokens][ldo]              reduced outputs (ping-pong)
  flags  uint32 [halves][MAX_POSITIONS], done uint32 [MAX_POSITIONS]
  keys   int64 [2][world][max_tokens]           token-selection keys received
  emb    bf16 [2][max_tokens][ldo]              embedding rows (ping-pong)
  xflags uint32 [2][8], xstate uint32 [4]       exchange epochs and counter
with halves = 2 for one-shot (alternating by call parity), 1 for two-shot,
and exchanges its CUDA IPC handle through the default process group (after
init_process_group, outside graph capture), so every rank knows every
rank's address of each part.

The same buffers carry the decode step's two other exchanges:
  * the vocabulary-parallel embedding (src/layers/llm_head.py:38-49): the
    rank owning a token's row writes it into every rank's `emb` rows, one
    signal round, instead of a masked lookup + NCCL all_reduce;
  * token selection (src/layers/llm_head.py:60-69 + sampler.py:4-17): every
    rank selects over its own vocabulary shard and only a packed (score,
    index) key per sequence crosses NVLink, instead of gathering the
    [B, V/tp] logits to rank 0.

The returned tensor is a view of an output buffer that the call after the
next one overwrites (two buffers alternate), which is how the decoder
consumes it (the next RMSNorm reads it before the next row-parallel layer).

Which path a call takes is decided the same way on every rank, so that no
rank waits in NCCL while its peers wait on fused-kernel flags:
  * shape conditions known on every rank (more than max_tokens rows, N
    wider than the staged rows) pick GEMM + torch.distributed.all_reduce;
  * the launchability of a shape (every CTA co-resident, flag positions) is
    asked of the library once per (T, N, K) outside graph capture, and the
    ranks agree on the answer with an all_reduce(MIN) before any of them
    uses it;
  * a fused launch that then fails raises instead of switching paths.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from src import b200

MAX_POSITIONS = 4096


class FusedRowParallel:

    def __init__(self, device: torch.device, max_tokens: int = 512, max_hidden: int = 8192,
                 group=None, one_shot: bool | None = None):
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        if self.world > 8:
            raise ValueError("the fused all-reduce supports up to 8 ranks")
        self.device = device
        self.max_tokens = max_tokens
        self.ldo = (max_hidden + 7) // 8 * 8
        # one NVLink hop for small worlds; for larger ones the owner-reduce
        # (two-shot) moves 2 (w-1)/w instead of (w-1) times the output bytes
        self.one_shot = self.world <= 2 if one_shot is None else one_shot
        halves = 2 if self.one_shot else 1
        elt = 2
        self.stage_bytes = halves * self.world * max_tokens * self.ldo * elt
        self.out_bytes = max_tokens * self.ldo * elt
        flag_bytes = halves * MAX_POSITIONS * 4
        self.off_stage = 0
        self.off_out = [self.stage_bytes, self.stage_bytes + self.out_bytes]
        self.off_flags = self.stage_bytes + 2 * self.out_bytes
        self.off_done = self.off_flags + flag_bytes

        def up(n):
            return (n + 255) // 256 * 256
        self.off_keys = up(self.off_done + flag_bytes)
        self.off_emb = [up(self.off_keys + 2 * self.world * max_tokens * 8)]
        self.off_emb.append(self.off_emb[0] + self.out_bytes)
        self.off_xflags = up(self.off_emb[1] + self.out_bytes)
        self.off_xstate = self.off_xflags + 256
        total = self.off_xstate + 256
        self.buf = torch.zeros(total, dtype=torch.uint8, device=device)
        handle, offset = b200.ipc_export(self.buf)
        gathered = [None] * self.world
        dist.all_gather_object(gathered, (handle, offset), group=group)
        self.bases: list[int] = []
        self._opened: list[tuple[int, int]] = []
        for r, (h, off) in enumerate(gathered):
            if r == self.rank:
                self.bases.append(self.buf.data_ptr())
            else:
                ptr = b200.ipc_import(h, off)
                self._opened.append((ptr, off))
                self.bases.append(ptr)
        self.outs = [self.buf[o:o + self.out_bytes].view(torch.bfloat16).view(max_tokens, self.ldo)
                     for o in self.off_out]
        self.embs = [self.buf[o:o + self.out_bytes].view(torch.bfloat16).view(max_tokens, self.ldo)
                     for o in self.off_emb]
        self._eflip = 0
        self._flip = 0
        self.fused_calls = 0
        self.fallback_calls = 0
        self.fallback_reason = ""
        self._plans: dict[tuple[int, int, int], bool] = {}
        dist.barrier(group=group)

    @classmethod
    def create(cls, device: torch.device, max_tokens: int = 512, max_hidden: int = 8192):
        return cls(device, max_tokens, max_hidden)

    def _addrs(self, off: int) -> list[int]:
        return [b + off for b in self.bases]

    def fused_ok(self, T: int, N: int, K: int) -> bool:
        """Whether (T, N, K) runs fused -- the same answer on every rank.  The
        first query of a shape is a collective (outside graph capture)."""
        if T > self.max_tokens or N > self.ldo:
            return False
        key = (T, N, K)
        ok = self._plans.get(key)
        if ok is None:
            if torch.cuda.is_current_stream_capturing():
                raise RuntimeError(f"fused all-reduce: shape {key} first seen inside a CUDA-graph "
                                   "capture; run the batch size eagerly first (warm-up)")
            local = b200.linear_allreduce_supported(T, N, K, self.world, self.max_tokens, self.ldo,
                                                    MAX_POSITIONS)
            flag = torch.tensor([1 if local else 0], dtype=torch.int32, device=self.device)
            dist.all_reduce(flag, op=dist.ReduceOp.MIN, group=self.group)
            ok = self._plans[key] = bool(flag.item())
            if not ok:
                self.fallback_reason = (b200.load_library().b200_last_error().decode(errors="replace")
                                        if not local else f"a peer cannot launch {key} fused")
        return ok

    def linear_allreduce(self, x: torch.Tensor, w: torch.Tensor,
                         bias: torch.Tensor | None = None) -> torch.Tensor:
        T = x.reshape(-1, x.shape[-1]).shape[0]
        N, K = w.shape[0], w.shape[1]
        if self.fused_ok(T, N, K):
            idx = self._flip
            rc = b200.linear_allreduce(
                x, w, bias, self.rank, self.world, self._addrs(self.off_stage),
                self._addrs(self.off_out[idx]), self._addrs(self.off_flags),
                self._addrs(self.off_done), self.max_tokens, self.ldo, MAX_POSITIONS, self.one_shot)
            if rc != 0:
                msg = b200.load_library().b200_last_error().decode(errors="replace")
                raise RuntimeError(f"fused GEMM + all-reduce refused a planned launch: {msg}")
            self._flip ^= 1
            self.fused_calls += 1
            return self.outs[idx][:T, :N].view(*x.shape[:-1], N)
        self.fallback_calls += 1
        y = b200.linear(x, w, bias)
        dist.all_reduce(y, group=self.group)
        return y

    # ------------------------------------------------------------ exchanges
    def can_exchange(self, rows: int, width: int = 0) -> bool:
        """Whether `rows` tokens of `width` features fit the exchange buffers
        (a shape condition: the same answer on every rank)."""
        return 0 < rows <= self.max_tokens and width <= self.ldo

    def embedding(self, ids: torch.Tensor, weight: torch.Tensor, vocab_start: int, vocab_end: int,
                  vocab_size: int) -> torch.Tensor:
        """VocabParallelEmbedding.forward with its all_reduce (llm_head.py:38-49):
        [T, H], a view of this rank's embedding rows (two buffers alternate;
        a call overwrites the buffer of the call before last)."""
        T, H = ids.numel(), weight.shape[1]
        idx = self._eflip
        b200.embedding_exchange(ids, weight, vocab_start, vocab_end, vocab_size, self.rank, self.world,
                                self._addrs(self.off_emb[idx]), self.ldo, self._addrs(self.off_xflags),
                                self.bases[self.rank] + self.off_xstate)
        self._eflip ^= 1
        return self.embs[idx][:T, :H]

    def select_tokens(self, logits: torch.Tensor, vocab_start: int,
                      temperatures: torch.Tensor | None = None, noise: torch.Tensor | None = None,
                      seed: int = 0, offset: int = 0) -> torch.Tensor:
        """Token per row over the whole vocabulary from this rank's logits
        shard [B, V/tp]: the same int64 [B] on every rank."""
        keys = b200.select_tokens(logits, vocab_start, temperatures, noise, seed, offset)
        return b200.tokens_from_keys(keys, self.rank, self.world, self._addrs(self.off_keys),
                                     self._addrs(self.off_xflags),
                                     self.bases[self.rank] + self.off_xstate, self.max_tokens)

    def close(self) -> None:
        if self.buf is None:
            return
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        for ptr, off in self._opened:
            b200.ipc_close(ptr, off)
        self._opened.clear()
        self.buf = None
