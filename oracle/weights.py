"""Seeded random-init Qwen3 weights under the reference's checkpoint names.

Test infrastructure only.  Names are the HF Qwen3 names that
src/utils/loader.py:12-28 dispatches through
Qwen3ForCausalLM.packed_modules_mapping (src/models/qwen3.py:199-205).
Linear and embedding weights ~ N(0, std) in bf16; RMSNorm weights are the
module default of ones (src/layers/layernorm.py:7).
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

BF16 = torch.bfloat16


@dataclass(frozen=True)
class Qwen3Shape:
    hidden: int
    layers: int
    heads: int
    kv_heads: int
    head_dim: int
    inter: int
    vocab: int
    eps: float = 1e-6
    theta: float = 1e6
    tie: bool = False
    max_pos: int = 40960

    def hf_config(self):
        """A transformers Qwen3Config with these dimensions."""
        from transformers import Qwen3Config
        return Qwen3Config(
            hidden_size=self.hidden, num_hidden_layers=self.layers,
            num_attention_heads=self.heads, num_key_value_heads=self.kv_heads,
            head_dim=self.head_dim, intermediate_size=self.inter, vocab_size=self.vocab,
            rms_norm_eps=self.eps, rope_theta=self.theta, tie_word_embeddings=self.tie,
            max_position_embeddings=self.max_pos, attention_bias=False, hidden_act="silu")


QWEN3_0_6B = Qwen3Shape(hidden=1024, layers=28, heads=16, kv_heads=8, head_dim=128, inter=3072,
                        vocab=151936, tie=True)
QWEN3_8B = Qwen3Shape(hidden=4096, layers=36, heads=32, kv_heads=8, head_dim=128, inter=12288,
                      vocab=151936)
QWEN3_32B = Qwen3Shape(hidden=5120, layers=64, heads=64, kv_heads=8, head_dim=128, inter=25600,
                       vocab=151936)


def random_weights(shape: Qwen3Shape, seed: int = 0, std: float = 0.02) -> dict[str, torch.Tensor]:
    g = torch.Generator().manual_seed(seed)

    def rnd(*s):
        return (torch.randn(*s, generator=g) * std).to(BF16)

    H, d = shape.hidden, shape.head_dim
    W: dict[str, torch.Tensor] = {"model.embed_tokens.weight": rnd(shape.vocab, H)}
    for i in range(shape.layers):
        p = f"model.layers.{i}."
        W[p + "self_attn.q_proj.weight"] = rnd(shape.heads * d, H)
        W[p + "self_attn.k_proj.weight"] = rnd(shape.kv_heads * d, H)
        W[p + "self_attn.v_proj.weight"] = rnd(shape.kv_heads * d, H)
        W[p + "self_attn.o_proj.weight"] = rnd(H, shape.heads * d)
        W[p + "self_attn.q_norm.weight"] = torch.ones(d, dtype=BF16)
        W[p + "self_attn.k_norm.weight"] = torch.ones(d, dtype=BF16)
        W[p + "mlp.gate_proj.weight"] = rnd(shape.inter, H)
        W[p + "mlp.up_proj.weight"] = rnd(shape.inter, H)
        W[p + "mlp.down_proj.weight"] = rnd(H, shape.inter)
        W[p + "input_layernorm.weight"] = torch.ones(H, dtype=BF16)
        W[p + "post_attention_layernorm.weight"] = torch.ones(H, dtype=BF16)
    W["model.norm.weight"] = torch.ones(H, dtype=BF16)
    if not shape.tie:
        W["lm_head.weight"] = rnd(shape.vocab, H)
    return W
