"""The library's ops as torch.library custom ops: torch.ops.b200.<name>.

The modules under src/layers call the ctypes binding (src/b200.py) directly.
Importing this module also registers the same ops with the torch dispatcher,
each with a fake (meta) implementation, so code that traces -- torch.compile,
torch.export, FakeTensor shape propagation -- sees one opaque op per kernel
instead of a ctypes call it cannot follow.  The real implementations exist
for CUDA tensors only (there is no CPU path); registration makes no CUDA
call.  Argument meanings are those of the functions in src/b200.py and of
the reference calls they replace (cited there).

The fused RowParallel GEMM + all-reduce is not registered: it depends on the
per-process communicator (src/layers/tp_comm.py), not only on its arguments.
"""
from __future__ import annotations

from typing import Optional

import torch

from . import b200

_NS = "b200"


def _op(name: str, mutates=()):
    return torch.library.custom_op(f"{_NS}::{name}", mutates_args=mutates, device_types="cuda")


@_op("linear")
def linear(x: torch.Tensor, w: torch.Tensor, bias: Optional[torch.Tensor] = None) -> torch.Tensor:
    """F.linear (src/layers/linear.py:75,170; src/layers/llm_head.py:64)."""
    return b200.linear(x, w, bias)


@linear.register_fake
def _(x, w, bias=None):
    return x.new_empty((*x.shape[:-1], w.shape[0]))


@_op("linear_silu_and_mul")
def linear_silu_and_mul(x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """gate_up projection with SiluAndMul fused (linear.py:75 + activation.py:6-10)."""
    return b200.linear_silu_and_mul(x, w)


@linear_silu_and_mul.register_fake
def _(x, w):
    return x.new_empty((*x.shape[:-1], w.shape[0] // 2))


@_op("rms_norm")
def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    """RMSNorm.normal_forward (src/layers/layernorm.py:10-17)."""
    return b200.rms_norm(x, weight, eps)


@rms_norm.register_fake
def _(x, weight, eps):
    return torch.empty_like(x)


@_op("rms_norm_residual")
def rms_norm_residual(x: torch.Tensor, residual: torch.Tensor, weight: torch.Tensor,
                      eps: float) -> tuple[torch.Tensor, torch.Tensor]:
    """RMSNorm.residual_forward (layernorm.py:19-28): (norm(x + r), x + r)."""
    y, r = b200.rms_norm(x, weight, eps, residual=residual)
    return y, r


@rms_norm_residual.register_fake
def _(x, residual, weight, eps):
    return torch.empty_like(x), torch.empty_like(x)


@_op("silu_and_mul")
def silu_and_mul(x: torch.Tensor) -> torch.Tensor:
    """SiluAndMul (src/layers/activation.py:6-10)."""
    return b200.silu_and_mul(x)


@silu_and_mul.register_fake
def _(x):
    return x.new_empty((*x.shape[:-1], x.shape[-1] // 2))


@_op("store_kvcache", mutates=("k_cache", "v_cache"))
def store_kvcache(key: torch.Tensor, value: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                  slot_mapping: torch.Tensor) -> None:
    """store_kvcache (src/layers/attention.py:36-61); slot -1 is skipped."""
    b200.store_kvcache(key, value, k_cache, v_cache, slot_mapping)


@store_kvcache.register_fake
def _(key, value, k_cache, v_cache, slot_mapping):
    return None


@_op("qk_norm_rope_store", mutates=("k_cache", "v_cache"))
def qk_norm_rope_store(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, q_norm_w: torch.Tensor,
                       k_norm_w: torch.Tensor, eps: float, cos_sin: torch.Tensor, positions: torch.Tensor,
                       slot_mapping: torch.Tensor, k_cache: torch.Tensor,
                       v_cache: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """q/k RMSNorm + RoPE + the K/V cache store (src/models/qwen3.py:84-89,
    src/layers/pos_embedding.py:30-52, attention.py:86-87); returns
    (q_out, k_out, v_out)."""
    return b200.qk_norm_rope_store(q, k, v, q_norm_w, k_norm_w, eps, cos_sin, positions, slot_mapping,
                                   k_cache, v_cache)


@qk_norm_rope_store.register_fake
def _(q, k, v, q_norm_w, k_norm_w, eps, cos_sin, positions, slot_mapping, k_cache, v_cache):
    return (q.new_empty(q.shape), k.new_empty(k.shape), v.new_empty(v.shape))


@_op("paged_attention")
def paged_attention(q: torch.Tensor, k: Optional[torch.Tensor], v: Optional[torch.Tensor],
                    k_cache: Optional[torch.Tensor], v_cache: Optional[torch.Tensor],
                    cu_seqlens_q: torch.Tensor, cu_seqlens_k: torch.Tensor, max_seqlen_q: int,
                    max_seqlen_k: int, softmax_scale: float,
                    block_table: Optional[torch.Tensor] = None) -> torch.Tensor:
    """flash_attn_varlen_func(..., causal=True, block_table) (attention.py:89-104)."""
    return b200.paged_attention(q, k, v, k_cache, v_cache, cu_seqlens_q, cu_seqlens_k, max_seqlen_q,
                                max_seqlen_k, softmax_scale, block_table)


@paged_attention.register_fake
def _(q, k, v, k_cache, v_cache, cu_seqlens_q, cu_seqlens_k, max_seqlen_q, max_seqlen_k, softmax_scale,
      block_table=None):
    return q.new_empty(q.shape)


@_op("embedding")
def embedding(ids: torch.Tensor, weight: torch.Tensor, vocab_start: int, vocab_end: int) -> torch.Tensor:
    """VocabParallelEmbedding's masked lookup (src/layers/llm_head.py:38-47)."""
    return b200.embedding(ids, weight, vocab_start, vocab_end)


@embedding.register_fake
def _(ids, weight, vocab_start, vocab_end):
    return weight.new_empty((*ids.shape, weight.shape[1]))


@_op("argmax")
def argmax(logits: torch.Tensor) -> torch.Tensor:
    """Greedy token per row (lowest index on ties)."""
    return b200.argmax(logits)


@argmax.register_fake
def _(logits):
    return logits.new_empty((logits.shape[0],), dtype=torch.int64)


OPS = ("linear", "linear_silu_and_mul", "rms_norm", "rms_norm_residual", "silu_and_mul", "store_kvcache",
       "qk_norm_rope_store", "paged_attention", "embedding", "argmax")
