"""Qwen3 decoder on the sm_100a kernels (reference: src/models/qwen3.py:1-234).

Module tree, constructor arguments and parameter names are the reference's,
so `packed_modules_mapping` + the weight loaders load a checkpoint the same
way.  The forward passes are fused where the reference calls one module per
step:
  * attention block: qkv GEMM -> one kernel for q/k RMSNorm + RoPE + the K/V
    cache write (+ per-token K/V only when attention reads them) -> paged
    attention -> o_proj (RowParallelLinear: GEMM, or GEMM + all-reduce fused
    at tp > 1);
  * MLP: gate_up GEMM with SiLU-and-mul in its epilogue -> down_proj.
"""
from __future__ import annotations

import torch
from torch import nn

from src import b200
from src.layers.activation import SiluAndMul
from src.layers.attention import Attention, attend
from src.layers.layernorm import RMSNorm
from src.layers.linear import MergedColumnParallelLinear, QKVParallelLinear, RowParallelLinear
from src.layers.llm_head import ParallelLMHead, VocabParallelEmbedding
from src.layers.pos_embedding import RoPE
from src.utils.context import Context


class Qwen3Attention(nn.Module):

    def __init__(self, hidden_size: int, num_heads: int, num_kv_heads: int,
                 max_position: int = 4096 * 32, head_dim: int | None = None,
                 rms_norm_eps: float = 1e-06, qkv_bias: bool = False, rope_theta: float = 10000,
                 rope_scaling: dict | None = None, tp: tuple[int, int] = (0, 1)) -> None:
        super().__init__()
        tp_size = tp[1]
        self.total_num_heads = num_heads
        assert self.total_num_heads % tp_size == 0
        self.num_heads = self.total_num_heads // tp_size
        self.total_num_kv_heads = num_kv_heads
        assert self.total_num_kv_heads % tp_size == 0
        self.num_kv_heads = self.total_num_kv_heads // tp_size
        self.head_dim = head_dim or hidden_size // self.total_num_heads
        self.q_size = self.num_heads * self.head_dim
        self.kv_size = self.num_kv_heads * self.head_dim
        self.scaling = self.head_dim ** -0.5
        self.qkv_bias = qkv_bias
        self.qkv_proj = QKVParallelLinear(hidden_size, self.head_dim, self.total_num_heads,
                                          self.total_num_kv_heads, bias=qkv_bias, tp=tp)
        self.o_proj = RowParallelLinear(self.total_num_heads * self.head_dim, hidden_size,
                                        bias=False, tp=tp)
        if isinstance(rope_scaling, dict):
            rope_theta = rope_scaling.get("rope_theta", rope_theta)
        self.rotary_emb = RoPE(max_seq_len=max_position, head_dim=self.head_dim, base=rope_theta)
        self.attn = Attention(self.head_dim, self.num_heads, self.num_kv_heads, self.scaling)
        self.rms_norm_eps = rms_norm_eps
        if not self.qkv_bias:
            self.q_norm = RMSNorm(self.head_dim, eps=rms_norm_eps)
            self.k_norm = RMSNorm(self.head_dim, eps=rms_norm_eps)

    def forward(self, positions: torch.Tensor, hidden_states: torch.Tensor | None, ctx: Context,
                qkv: torch.Tensor | None = None) -> torch.Tensor:
        """`qkv`: the qkv projection already computed (the decoder layer fuses
        it with the input RMSNorm); else it is computed from hidden_states."""
        if qkv is None:
            qkv = self.qkv_proj(hidden_states)
        T = qkv.shape[0]
        q, k, v = qkv.split([self.q_size, self.kv_size, self.kv_size], dim=-1)
        q = q.view(T, self.num_heads, self.head_dim)
        k = k.view(T, self.num_kv_heads, self.head_dim)
        v = v.view(T, self.num_kv_heads, self.head_dim)
        k_cache, v_cache = self.attn.k_cache, self.attn.v_cache
        cached = k_cache.numel() > 0 and v_cache.numel() > 0
        per_token_kv = ctx.block_tables is None
        q, k, v = b200.qk_norm_rope_store(
            q, k, v,
            None if self.qkv_bias else self.q_norm.weight,
            None if self.qkv_bias else self.k_norm.weight,
            self.q_norm.eps if not self.qkv_bias else 0.0,
            self.rotary_emb.cos_sin, positions,
            ctx.slot_mapping if cached else None,
            k_cache if cached else None, v_cache if cached else None,
            need_kv_out=per_token_kv)
        o = attend(q, k, v, k_cache, v_cache, ctx, self.attn.scale)
        return self.o_proj(o.view(T, -1))


class Qwen3MLP(nn.Module):

    def __init__(self, hidden_size: int, intermediate_size: int, hidden_act: str,
                 tp: tuple[int, int] = (0, 1)) -> None:
        super().__init__()
        self.gate_up_proj = MergedColumnParallelLinear(hidden_size, [intermediate_size] * 2,
                                                       bias=False, tp=tp)
        self.down_proj = RowParallelLinear(intermediate_size, hidden_size, bias=False, tp=tp)
        assert hidden_act == "silu"
        self.act_fn = SiluAndMul()

    def forward(self, x: torch.Tensor | None, act: torch.Tensor | None = None) -> torch.Tensor:
        """`act`: silu(gate) * up already computed (the decoder layer fuses the
        gate_up projection with the post-attention RMSNorm)."""
        if act is None:
            # gate_up GEMM with silu(gate) * up in the epilogue
            act = b200.linear_silu_and_mul(x, self.gate_up_proj.weight)
        return self.down_proj(act)


class Qwen3DecoderLayer(nn.Module):

    def __init__(self, config, tp: tuple[int, int] = (0, 1)) -> None:
        super().__init__()
        self.self_attn = Qwen3Attention(
            hidden_size=config.hidden_size,
            num_heads=config.num_attention_heads,
            num_kv_heads=config.num_key_value_heads,
            max_position=config.max_position_embeddings,
            rms_norm_eps=config.rms_norm_eps,
            qkv_bias=getattr(config, "attention_bias", True),
            head_dim=getattr(config, "head_dim", None),
            rope_theta=getattr(config, "rope_theta", 1000000),
            rope_scaling=getattr(config, "rope_scaling", None),
            tp=tp,
        )
        self.mlp = Qwen3MLP(hidden_size=config.hidden_size,
                            intermediate_size=config.intermediate_size,
                            hidden_act=config.hidden_act, tp=tp)
        self.input_layernorm = RMSNorm(config.hidden_size, eps=config.rms_norm_eps)
        self.post_attention_layernorm = RMSNorm(config.hidden_size, eps=config.rms_norm_eps)

    def forward(self, positions: torch.Tensor, hidden_states: torch.Tensor,
                residual: torch.Tensor | None, ctx: Context) -> tuple[torch.Tensor, torch.Tensor]:
        # The layer order of the reference (src/models/qwen3.py:162-168), with
        # each RMSNorm handed to the projection that consumes it
        # (b200.rmsnorm_linear: two launches, or one with B200_FUSE_NORM=1).
        attn, mlp = self.self_attn, self.mlp
        n1, n2 = self.input_layernorm, self.post_attention_layernorm
        if attn.qkv_bias:  # the fused call carries no bias
            if residual is None:
                hidden_states, residual = n1(hidden_states), hidden_states
            else:
                hidden_states, residual = n1(hidden_states, residual)
            hidden_states = attn(positions, hidden_states, ctx)
        else:
            if residual is None:
                qkv = b200.rmsnorm_linear(hidden_states, n1.weight, n1.eps, attn.qkv_proj.weight)
                residual = hidden_states
            else:
                qkv, residual = b200.rmsnorm_linear(hidden_states, n1.weight, n1.eps, attn.qkv_proj.weight,
                                                    residual=residual)
            hidden_states = attn(positions, None, ctx, qkv=qkv)
        act, residual = b200.rmsnorm_linear(hidden_states, n2.weight, n2.eps, mlp.gate_up_proj.weight,
                                            residual=residual, silu=True)
        hidden_states = mlp(None, act=act)
        return hidden_states, residual


class Qwen3Model(nn.Module):

    def __init__(self, config, tp: tuple[int, int] = (0, 1)) -> None:
        super().__init__()
        self.embed_tokens = VocabParallelEmbedding(config.vocab_size, config.hidden_size, tp=tp)
        self.layers = nn.ModuleList([Qwen3DecoderLayer(config, tp=tp)
                                     for _ in range(config.num_hidden_layers)])
        self.norm = RMSNorm(config.hidden_size, eps=config.rms_norm_eps)

    def forward(self, input_ids: torch.Tensor, positions: torch.Tensor, ctx: Context) -> torch.Tensor:
        hidden_states = self.embed_tokens(input_ids)
        residual = None
        for layer in self.layers:
            hidden_states, residual = layer(positions, hidden_states, residual, ctx)
        hidden_states, _ = self.norm(hidden_states, residual)
        return hidden_states


class Qwen3ForCausalLM(nn.Module):
    packed_modules_mapping = {
        "q_proj": ("qkv_proj", "q"),
        "k_proj": ("qkv_proj", "k"),
        "v_proj": ("qkv_proj", "v"),
        "gate_proj": ("gate_up_proj", 0),
        "up_proj": ("gate_up_proj", 1),
    }

    def __init__(self, config, tp: tuple[int, int] = (0, 1)) -> None:
        super().__init__()
        self.model = Qwen3Model(config, tp=tp)
        self.lm_head = ParallelLMHead(config.vocab_size, config.hidden_size, tp=tp)
        if config.tie_word_embeddings:
            self.lm_head.weight.data = self.model.embed_tokens.weight.data

    def load(self, path: str):
        from src.utils.loader import load_model
        load_model(self, path)

    def forward(self, input_ids: torch.Tensor, positions: torch.Tensor, ctx: Context) -> torch.Tensor:
        return self.model(input_ids, positions, ctx)

    def compute_logits(self, hidden_states: torch.Tensor, ctx: Context) -> torch.Tensor:
        return self.lm_head(hidden_states, ctx)
