"""Per-rank driver of the decoder path: model build, paged KV cache, metadata,
eager prefill and CUDA-graph decode.

This is the subset of the reference's ModelRunner
(src/engine/model_runner.py:14-315) that drives the hot path:
  * the model is built under bf16 / cuda defaults with tp = (rank, world);
  * one KV tensor [2, L, num_blocks, block_size, Hkv / tp, head_dim] whose
    per-layer views are assigned, in modules() order, to every module with
    k_cache and v_cache (model_runner.py:159-165);
  * prefill / mixed batches run eagerly; pure-decode batches (every query
    length 1) replay a CUDA graph captured for the smallest batch size >= B,
    with padded rows marked by slot -1, cu_seqlens 0 and block table -1
    (model_runner.py:241-259, 269-315).
Process-group setup, the scheduler and the shared-memory RPC stay with the
caller.
"""
from __future__ import annotations

import os

import numpy as np
import torch

from src import b200
from src.engine import metadata as M
from src.models.qwen3 import Qwen3ForCausalLM
from src.utils.context import Context
from src.utils.loader import load_weights


class ModelRunner:

    def __init__(self, config, rank: int = 0, world_size: int = 1, block_size: int = 256,
                 max_num_seqs: int = 256, max_seq_len: int = 8192, enforce_eager: bool = False,
                 device: torch.device | None = None):
        self.config = config
        self.rank = rank
        self.world_size = world_size
        self.block_size = block_size
        self.max_num_seqs = max_num_seqs
        self.max_seq_len = max_seq_len
        self.enforce_eager = enforce_eager
        self.device = device or torch.device("cuda", torch.cuda.current_device())
        prev_dtype = torch.get_default_dtype()
        prev_device = torch.get_default_device()
        torch.set_default_dtype(torch.bfloat16)
        torch.set_default_device(self.device)
        try:
            self.model = Qwen3ForCausalLM(config, tp=(rank, world_size))
        finally:
            torch.set_default_device(prev_device)
            torch.set_default_dtype(prev_dtype)
        self.head_dim = getattr(config, "head_dim", None) or config.hidden_size // config.num_attention_heads
        self.local_kv_heads = config.num_key_value_heads // world_size
        self.local_q_heads = config.num_attention_heads // world_size
        self.kv_cache = None
        self.num_kvcache_blocks = 0
        self.graphs: dict[int, torch.cuda.CUDAGraph] = {}
        self.graph_vars: dict[str, torch.Tensor] = {}
        self.graph_pool = None

    # ------------------------------------------------------------------ weights
    def load_weights(self, items) -> None:
        load_weights(self.model, items)

    @torch.no_grad()
    def init_random_weights(self, seed: int = 0, std: float = 0.02) -> None:
        """Linear / embedding weights ~ N(0, std) in bf16 drawn on the device,
        norm weights one (the reference's RMSNorm default)."""
        g = torch.Generator(device=self.device).manual_seed(seed + 7919 * self.rank)
        for name, p in self.model.named_parameters():
            if name.endswith("norm.weight"):
                p.fill_(1.0)
            else:
                p.normal_(0.0, std, generator=g)

    # ------------------------------------------------------------------ cache
    def kv_block_bytes(self) -> int:
        L = self.config.num_hidden_layers
        return 2 * L * self.block_size * self.local_kv_heads * self.head_dim * 2

    def allocate_kv_cache(self, num_blocks: int) -> None:
        L = self.config.num_hidden_layers
        self.kv_cache = torch.empty(2, L, num_blocks, self.block_size, self.local_kv_heads,
                                    self.head_dim, dtype=torch.bfloat16, device=self.device)
        layer = 0
        for module in self.model.modules():
            if hasattr(module, "k_cache") and hasattr(module, "v_cache"):
                module.k_cache = self.kv_cache[0, layer]
                module.v_cache = self.kv_cache[1, layer]
                layer += 1
        assert layer == L
        self.num_kvcache_blocks = num_blocks
        nbytes = b200.attention_workspace_bytes(self.max_num_seqs, self.max_seq_len, self.local_q_heads)
        b200.reserve_workspace("attn", nbytes, self.device)

    # ------------------------------------------------------------------ steps
    def prepare(self, seqs) -> tuple[torch.Tensor, torch.Tensor, Context]:
        """input_ids, positions and the Context of a step: per-sequence values
        from the host, the per-token expansion on the device
        (b200_step_metadata); B200_HOST_METADATA=1 builds everything on the
        host instead."""
        if os.environ.get("B200_HOST_METADATA") == "1":
            return M.to_device(M.build(seqs, self.block_size), self.device)
        return M.build_on_device(seqs, self.block_size, self.device)

    @torch.inference_mode()
    def run_hidden(self, input_ids: torch.Tensor, positions: torch.Tensor,
                   ctx: Context) -> tuple[torch.Tensor, Context]:
        """Final hidden states and the context the LM head takes: eager for
        prefill / mixed batches, the captured graph for pure decode."""
        bs = input_ids.size(0)
        if ctx.max_seqlen_q != 1 or self.enforce_eager or not self.graphs or bs > max(self.graphs):
            return self.model(input_ids, positions, ctx), ctx
        gbs = next(x for x in sorted(self.graphs) if x >= bs)
        v = self.graph_vars
        v["input_ids"][:bs] = input_ids
        v["positions"][:bs] = positions
        v["slot_mapping"].fill_(-1)
        v["slot_mapping"][:bs] = ctx.slot_mapping
        v["cu_seqlens_q"].zero_()
        v["cu_seqlens_q"][:bs + 1] = ctx.cu_seqlens_q
        v["cu_seqlens_k"].zero_()
        v["cu_seqlens_k"][:bs + 1] = ctx.cu_seqlens_k
        v["block_tables"].fill_(-1)
        v["block_tables"][:bs, :ctx.block_tables.size(1)] = ctx.block_tables
        self.graphs[gbs].replay()
        return v["outputs"][:bs], Context(is_prefill=False)

    @torch.inference_mode()
    def run_model(self, input_ids: torch.Tensor, positions: torch.Tensor, ctx: Context) -> torch.Tensor:
        """Logits [B, V] (rank 0; None on other ranks at tp > 1)."""
        hidden, hctx = self.run_hidden(input_ids, positions, ctx)
        return self.model.compute_logits(hidden, hctx)

    @torch.inference_mode()
    def step_tokens(self, seqs, temperatures: torch.Tensor | None = None, seed: int = 0,
                    offset: int = 0) -> list[int]:
        """prepare -> forward -> one token per sequence on every rank, selected
        from the ranks' vocabulary shards (greedy without temperatures)."""
        ids, pos, ctx = self.prepare(seqs)
        hidden, hctx = self.run_hidden(ids, pos, ctx)
        if temperatures is not None:
            temperatures = temperatures.to(device=self.device, dtype=torch.float32)
        return self.model.lm_head.select_tokens(hidden, hctx, temperatures, seed=seed,
                                                offset=offset).tolist()

    @torch.inference_mode()
    def step_greedy(self, seqs) -> list[int]:
        """prepare -> forward -> greedy token per sequence."""
        return self.step_tokens(seqs)

    # ------------------------------------------------------------------ graphs
    @torch.inference_mode()
    def capture_cudagraph(self, batch_sizes: list[int] | None = None,
                          with_sampling: bool = False) -> None:
        """Capture the decode forward for each batch size.  With
        `with_sampling` the graph also runs the LM head and the greedy token
        selection, leaving the tokens in graph_vars["tokens"] (every rank)."""
        max_bs = min(self.max_num_seqs, 512)
        if batch_sizes is None:
            batch_sizes = [b for b in [1, 2, 4, 8] + list(range(16, max_bs + 1, 16)) if b <= max_bs]
        max_bs = max(batch_sizes)
        max_blocks = (self.max_seq_len + self.block_size - 1) // self.block_size
        dev = self.device
        v = dict(
            input_ids=torch.zeros(max_bs, dtype=torch.int64, device=dev),
            positions=torch.zeros(max_bs, dtype=torch.int64, device=dev),
            cu_seqlens_q=torch.zeros(max_bs + 1, dtype=torch.int32, device=dev),
            cu_seqlens_k=torch.zeros(max_bs + 1, dtype=torch.int32, device=dev),
            slot_mapping=torch.full((max_bs,), -1, dtype=torch.int32, device=dev),
            block_tables=torch.full((max_bs, max_blocks), -1, dtype=torch.int32, device=dev),
            outputs=torch.zeros(max_bs, self.config.hidden_size, dtype=torch.bfloat16, device=dev),
            tokens=torch.zeros(max_bs, dtype=torch.int64, device=dev),
        )
        self.graph_with_sampling = with_sampling
        self.graph_vars = v
        for bs in sorted(batch_sizes, reverse=True):
            ctx = Context(is_prefill=False, cu_seqlens_q=v["cu_seqlens_q"][:bs + 1],
                          cu_seqlens_k=v["cu_seqlens_k"][:bs + 1], max_seqlen_q=1,
                          max_seqlen_k=self.max_seq_len, slot_mapping=v["slot_mapping"][:bs],
                          block_tables=v["block_tables"][:bs])
            def step():
                v["outputs"][:bs] = self.model(v["input_ids"][:bs], v["positions"][:bs], ctx)
                if with_sampling:
                    v["tokens"][:bs] = self.model.lm_head.select_tokens(v["outputs"][:bs],
                                                                        Context(is_prefill=False))

            step()  # warm-up outside the graph
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, self.graph_pool):
                step()
            if self.graph_pool is None:
                self.graph_pool = graph.pool()
            self.graphs[bs] = graph
            torch.cuda.synchronize()

    def replay(self, bs: int) -> None:
        """Replay the captured graph of batch size `bs` on the current
        graph_vars (the caller filled them)."""
        self.graphs[bs].replay()

    def release_graphs(self) -> None:
        self.graphs.clear()
        self.graph_pool = None
