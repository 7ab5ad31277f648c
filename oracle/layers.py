"""CPU restatements of the reference's layer ops (test infrastructure only).

Each function cites the reference code it restates.  Tensors are CPU tensors
(the oracle proper); bf16 in, bf16 out, fp32 inside, with bf16 rounding at the
same points as the reference modules.  The functions are device-agnostic, so
a test can also run them on CUDA tensors with NATIVE_BF16_LINEAR set: that is
the reference's own torch path (bf16 F.linear on cuBLAS, the same module
composition) on the GPU, a second yardstick beside the CPU oracle.
"""
from __future__ import annotations

import math

import torch

BF16 = torch.bfloat16

# When True, linear() calls torch's bf16 F.linear -- the op the reference
# itself calls -- instead of the fp32 restatement (used for CPU timing only).
NATIVE_BF16_LINEAR = False


def linear(x: torch.Tensor, w: torch.Tensor, bias: torch.Tensor | None = None) -> torch.Tensor:
    """F.linear in bf16: fp32 accumulation, one rounding of the output.
    src/layers/linear.py:74-75, :169-170; src/layers/llm_head.py:64."""
    if NATIVE_BF16_LINEAR:
        return torch.nn.functional.linear(x, w, bias)
    y = x.float() @ w.float().t()
    if bias is not None:
        y = y + bias.float()
    return y.to(BF16)


def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    """src/layers/layernorm.py:10-16 (RMSNorm.normal_forward)."""
    xf = x.float()
    var = xf.square().mean(-1, keepdim=True) + eps
    return (w * (xf * var.rsqrt())).to(x.dtype)


def rms_norm_residual(x: torch.Tensor, residual: torch.Tensor, w: torch.Tensor, eps: float):
    """src/layers/layernorm.py:18-28 (RMSNorm.residual_forward):
    returns (norm(x + residual), bf16(x + residual))."""
    s = x.float() + residual.float()
    var = s.square().mean(-1, keepdim=True) + eps
    return (w * (s * var.rsqrt())).to(x.dtype), s.to(x.dtype)


def rope_cos_sin(max_seq_len: int, head_dim: int, base: float) -> torch.Tensor:
    """src/layers/pos_embedding.py:6-18: fp32 [max_seq_len, 1, head_dim] table
    holding [cos(pos * f) | sin(pos * f)], f_j = 1 / base^(2j / head_dim)."""
    exps = torch.arange(0, head_dim, 2, dtype=torch.float32) / head_dim
    inv_freq = 1.0 / (base ** exps)
    pos = torch.arange(max_seq_len, dtype=torch.float32)
    ang = pos[:, None] * inv_freq[None, :]
    return torch.cat([ang.cos(), ang.sin()], dim=-1)[:, None, :]


def rope(q: torch.Tensor, k: torch.Tensor, positions: torch.Tensor, cos_sin: torch.Tensor):
    """src/layers/pos_embedding.py:30-52 (neox half rotation in fp32)."""
    cs = cos_sin[positions]
    half = cs.shape[-1] // 2
    c, s = cs[..., :half], cs[..., half:]

    def rot(t):
        tf = t.float()
        a, b = tf[..., :half], tf[..., half:]
        return torch.cat([a * c - b * s, a * s + b * c], dim=-1).to(t.dtype)

    return rot(q), rot(k)


def silu_and_mul(x: torch.Tensor) -> torch.Tensor:
    """src/layers/activation.py:6-10 evaluated eagerly on bf16 tensors:
    silu rounds to bf16, the product rounds again."""
    half = x.shape[-1] // 2
    g, u = x[..., :half], x[..., half:]
    gf = g.float()
    s = (gf / (1.0 + torch.exp(-gf))).to(BF16)
    return (s.float() * u.float()).to(BF16)


def store_kvcache(key, value, k_cache, v_cache, slot_mapping) -> None:
    """src/layers/attention.py:10-61: cache.view(-1, D)[slot] = key row, slot
    -1 skipped.  In place on k_cache / v_cache."""
    T = key.shape[0]
    D = key.shape[1] * key.shape[2]
    kf = k_cache.view(-1, D)
    vf = v_cache.view(-1, D)
    for i in range(T):
        s = int(slot_mapping[i])
        if s == -1:
            continue
        kf[s] = key[i].reshape(D)
        vf[s] = value[i].reshape(D)


def gather_paged(cache: torch.Tensor, block_table_row: torch.Tensor, n: int) -> torch.Tensor:
    """Rows 0..n-1 of one sequence from a [num_blocks, page, Hkv, d] cache."""
    page = cache.shape[1]
    j = torch.arange(n, device=cache.device)
    blocks = block_table_row[(j // page)].long()
    return cache[blocks, j % page]


def varlen_attention(q, k, v, cu_seqlens_q, cu_seqlens_k, scale, k_cache=None, v_cache=None,
                     block_table=None) -> torch.Tensor:
    """Semantics of flash_attn_varlen_func(..., causal=True, block_table) as
    called at src/layers/attention.py:93-104: per sequence, query i of Lq
    sees keys j <= i + Lk - Lq; q head n uses kv head n // (Hq / Hkv); K/V
    come from the paged cache when a block table is given.  Rows with no
    visible key are zero; sequences with Lq <= 0 are skipped.  fp32 softmax."""
    T, Hq, d = q.shape
    out = torch.zeros(T, Hq, d, dtype=q.dtype, device=q.device)
    B = cu_seqlens_q.numel() - 1
    for b in range(B):
        q0, q1 = int(cu_seqlens_q[b]), int(cu_seqlens_q[b + 1])
        Lq = q1 - q0
        if Lq <= 0:
            continue
        Lk = int(cu_seqlens_k[b + 1]) - int(cu_seqlens_k[b])
        if block_table is not None:
            kb = gather_paged(k_cache, block_table[b], Lk)
            vb = gather_paged(v_cache, block_table[b], Lk)
        else:
            k0 = int(cu_seqlens_k[b])
            kb, vb = k[k0:k0 + Lk], v[k0:k0 + Lk]
        Hkv = kb.shape[1]
        G = Hq // Hkv
        qf = q[q0:q1].float().transpose(0, 1)                       # [Hq, Lq, d]
        kf = kb.float().transpose(0, 1).repeat_interleave(G, 0)      # [Hq, Lk, d]
        vf = vb.float().transpose(0, 1).repeat_interleave(G, 0)
        s = (qf @ kf.transpose(1, 2)) * scale
        i = torch.arange(Lq, device=q.device)[:, None]
        j = torch.arange(Lk, device=q.device)[None, :]
        mask = j <= i + (Lk - Lq)
        s = s.masked_fill(~mask, float("-inf"))
        p = torch.softmax(s, dim=-1)
        p = torch.nan_to_num(p, nan=0.0)
        o = p @ vf
        out[q0:q1] = o.transpose(0, 1).to(q.dtype)
    return out


def sample(logits: torch.Tensor, temperatures: torch.Tensor, noise: torch.Tensor) -> torch.Tensor:
    """src/layers/sampler.py:14-17 with its Exp(1) draws given (`noise`, the
    tensor `exponential_(1)` fills there): softmax(logits / T) divided by the
    draws clamped at 1e-10, argmax (first maximum)."""
    scaled = logits.float() / temperatures.float().unsqueeze(1)
    probs = torch.softmax(scaled, dim=-1)
    return (probs / noise.float().clamp_min(1e-10)).argmax(dim=-1)


def vocab_embedding(ids: torch.Tensor, w_shard: torch.Tensor, start: int, end: int) -> torch.Tensor:
    """Local part of src/layers/llm_head.py:38-49: rows of this rank's vocab
    shard, zero for ids outside [start, end)."""
    mask = (ids >= start) & (ids < end)
    local = (ids - start) * mask
    y = w_shard[local]
    return y * mask[:, None].to(y.dtype)


def softmax_scale(head_dim: int) -> float:
    """src/models/qwen3.py:40."""
    return head_dim ** -0.5


def rel_err(a: torch.Tensor, b: torch.Tensor) -> float:
    """max |a - b| / max |b| in fp32."""
    a = a.float()
    b = b.float()
    den = b.abs().max().item()
    return (a - b).abs().max().item() / (den if den > 0 else 1.0)


def allclose_bf16(a: torch.Tensor, b: torch.Tensor, rtol: float = 2e-2) -> bool:
    return rel_err(a, b) <= rtol and not math.isnan(rel_err(a, b))
