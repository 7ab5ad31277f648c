"""Qwen3 decoder forward with tensor-parallel simulation (test infrastructure only).

Restates src/models/qwen3.py:14-234 on CPU over a dict of full (unsharded)
HF-named weights.  Tensor parallelism of degree `tp` is simulated the way the
reference partitions the model (src/layers/linear.py:52-173,
src/layers/llm_head.py:9-69): column-parallel outputs are exact slices, and a
RowParallelLinear output is the bf16-rounded sum over ranks of each rank's
bf16 partial product (linear.py:170-172).
"""
from __future__ import annotations

import torch

from . import layers as L
from .weights import Qwen3Shape


class OracleKV:
    """Per-layer paged caches [num_blocks, page, Hkv, d] (model_runner.py:159-165)."""

    def __init__(self, shape: Qwen3Shape, num_blocks: int, page: int = 256, device="cpu"):
        self.k = [torch.zeros(num_blocks, page, shape.kv_heads, shape.head_dim, dtype=L.BF16,
                              device=device)
                  for _ in range(shape.layers)]
        self.v = [torch.zeros_like(t) for t in self.k]


def _row_parallel(x: torch.Tensor, w: torch.Tensor, tp: int) -> torch.Tensor:
    if tp == 1:
        return L.linear(x, w)
    xs = x.chunk(tp, dim=-1)
    ws = w.chunk(tp, dim=1)
    acc = sum(L.linear(xi, wi).float() for xi, wi in zip(xs, ws))
    return acc.to(L.BF16)


def decoder_layer(shape: Qwen3Shape, W: dict, i: int, h: torch.Tensor,
                  residual: torch.Tensor | None, positions: torch.Tensor, ctx: dict,
                  kv: OracleKV | None = None, tp: int = 1,
                  cos_sin: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """Qwen3DecoderLayer.forward (src/models/qwen3.py:155-169) of layer i:
    (hidden, residual) in -> (MLP output, residual stream) out."""
    d = shape.head_dim
    Hq, Hkv = shape.heads, shape.kv_heads
    eps = shape.eps
    if cos_sin is None:
        cos_sin = L.rope_cos_sin(shape.max_pos, d, shape.theta)
    scale = L.softmax_scale(d)
    p = f"model.layers.{i}."
    if residual is None:
        x, residual = L.rms_norm(h, W[p + "input_layernorm.weight"], eps), h
    else:
        x, residual = L.rms_norm_residual(h, residual, W[p + "input_layernorm.weight"], eps)
    # Qwen3Attention.forward (qwen3.py:74-91)
    # the reference's QKVParallelLinear holds the three projections stacked
    # [q | k | v] (linear.py:130-141); a caller may pass them pre-stacked
    wqkv = W.get(p + "self_attn.qkv_proj.weight")
    if wqkv is None:
        wqkv = torch.cat([W[p + "self_attn.q_proj.weight"], W[p + "self_attn.k_proj.weight"],
                          W[p + "self_attn.v_proj.weight"]], 0)
    qkv = L.linear(x, wqkv)
    q, k, v = qkv.split([Hq * d, Hkv * d, Hkv * d], dim=-1)
    q = q.reshape(-1, Hq, d)
    k = k.reshape(-1, Hkv, d)
    v = v.reshape(-1, Hkv, d)
    q = L.rms_norm(q, W[p + "self_attn.q_norm.weight"], eps)
    k = L.rms_norm(k, W[p + "self_attn.k_norm.weight"], eps)
    q, k = L.rope(q, k, positions, cos_sin)
    # Attention.forward (attention.py:79-104)
    if kv is not None:
        L.store_kvcache(k, v, kv.k[i], kv.v[i], ctx["slot_mapping"])
    bt = ctx.get("block_tables")
    o = L.varlen_attention(q, k, v, ctx["cu_seqlens_q"], ctx["cu_seqlens_k"], scale,
                           kv.k[i] if kv is not None else None,
                           kv.v[i] if kv is not None else None,
                           bt if bt is not None else None)
    h = _row_parallel(o.reshape(-1, Hq * d), W[p + "self_attn.o_proj.weight"], tp)
    x, residual = L.rms_norm_residual(h, residual, W[p + "post_attention_layernorm.weight"], eps)
    # Qwen3MLP.forward (qwen3.py:119-123)
    wgu = W.get(p + "mlp.gate_up_proj.weight")  # [gate | up] (linear.py:98-102)
    if wgu is None:
        wgu = torch.cat([W[p + "mlp.gate_proj.weight"], W[p + "mlp.up_proj.weight"]], 0)
    if tp == 1:
        act = L.silu_and_mul(L.linear(x, wgu))
    else:
        I = shape.inter
        parts = []
        for r in range(tp):
            g = W[p + "mlp.gate_proj.weight"].chunk(tp, 0)[r]
            u = W[p + "mlp.up_proj.weight"].chunk(tp, 0)[r]
            parts.append(L.silu_and_mul(L.linear(x, torch.cat([g, u], 0))))
        act = torch.cat(parts, -1)
        assert act.shape[-1] == I
    h = _row_parallel(act, W[p + "mlp.down_proj.weight"], tp)
    return h, residual


def forward(shape: Qwen3Shape, W: dict, input_ids: torch.Tensor, positions: torch.Tensor,
            ctx: dict, kv: OracleKV | None = None, tp: int = 1,
            cos_sin: torch.Tensor | None = None) -> torch.Tensor:
    """Qwen3Model.forward (src/models/qwen3.py:184-195): final normed hidden [T, H]."""
    if cos_sin is None:
        cos_sin = L.rope_cos_sin(shape.max_pos, shape.head_dim, shape.theta)
    h = W["model.embed_tokens.weight"][input_ids]
    residual = None
    for i in range(shape.layers):
        h, residual = decoder_layer(shape, W, i, h, residual, positions, ctx, kv, tp, cos_sin)
    out, _ = L.rms_norm_residual(h, residual, W["model.norm.weight"], shape.eps)
    return out


def compute_logits(shape: Qwen3Shape, W: dict, hidden: torch.Tensor, ctx: dict) -> torch.Tensor:
    """ParallelLMHead.forward (src/layers/llm_head.py:60-69) after the gather
    to rank 0: last token of each sequence in prefill, logits [B, V]."""
    if ctx["is_prefill"]:
        hidden = hidden[ctx["cu_seqlens_q"][1:].long() - 1]
    w = W.get("lm_head.weight", W["model.embed_tokens.weight"])
    return L.linear(hidden, w)
