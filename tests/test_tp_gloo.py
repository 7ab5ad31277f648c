"""Tensor parallelism as two CPU processes over torch.distributed gloo.

What runs on each rank is the host side of the tp > 1 path:
  * the product's module tree, Qwen3ForCausalLM(config, tp=(rank, 2)),
    built on CPU and loaded through its own packed_modules_mapping and
    weight loaders (src/utils/loader.py, src/layers/linear.py), so each rank
    holds exactly the shards the reference's loaders give it
    (reference src/layers/linear.py:71,98-102,130-141,163, llm_head.py:31-36);
  * a forward over those shards with the reference's exchange steps done by
    real collectives: masked vocab-parallel embedding + all_reduce
    (llm_head.py:38-49), RowParallelLinear partial + all_reduce after o_proj
    and down_proj (linear.py:169-173), LM-head partial + gather to rank 0
    (llm_head.py:60-69).  The arithmetic between them is the oracle's.

Checks: both ranks hold bit-identical hidden states after every step, and
rank 0's logits equal the oracle's single-process tp = 2 restatement (the
one the GPU tests compare the fused NVLink kernel against) for a prefill and
two paged decode steps.  CPU only.
"""
import os
import socket

import torch

BF16 = torch.bfloat16


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _all_reduce_bf16(t):
    """Sum over ranks in fp32, rounded once to bf16 (the reduction the
    oracle states for the reference's bf16 all_reduce)."""
    import torch.distributed as dist
    acc = t.float()
    dist.all_reduce(acc)
    return acc.to(BF16)


def _rank_forward(shape, P, ids, pos, ctx, kv, rank, world, cs):
    from oracle import layers as L
    d, eps = shape.head_dim, shape.eps
    hq, hkv = shape.heads // world, shape.kv_heads // world
    # VocabParallelEmbedding.forward: rows outside this rank's shard are zero
    vr = shape.vocab // world
    lo = rank * vr
    inside = (ids >= lo) & (ids < lo + vr)
    h = P["model.embed_tokens.weight"][(ids - lo).clamp(0, vr - 1)] * inside[:, None].to(BF16)
    h = _all_reduce_bf16(h)
    residual = None
    for i in range(shape.layers):
        p = f"model.layers.{i}."
        if residual is None:
            x, residual = L.rms_norm(h, P[p + "input_layernorm.weight"], eps), h
        else:
            x, residual = L.rms_norm_residual(h, residual, P[p + "input_layernorm.weight"], eps)
        qkv = L.linear(x, P[p + "self_attn.qkv_proj.weight"])
        q, k, v = qkv.split([hq * d, hkv * d, hkv * d], dim=-1)
        q = L.rms_norm(q.reshape(-1, hq, d), P[p + "self_attn.q_norm.weight"], eps)
        k = L.rms_norm(k.reshape(-1, hkv, d), P[p + "self_attn.k_norm.weight"], eps)
        v = v.reshape(-1, hkv, d)
        q, k = L.rope(q, k, pos, cs)
        L.store_kvcache(k, v, kv.k[i], kv.v[i], ctx["slot_mapping"])
        o = L.varlen_attention(q, k, v, ctx["cu_seqlens_q"], ctx["cu_seqlens_k"],
                               L.softmax_scale(d), kv.k[i], kv.v[i], ctx.get("block_tables"))
        h = _all_reduce_bf16(L.linear(o.reshape(-1, hq * d), P[p + "self_attn.o_proj.weight"]))
        x, residual = L.rms_norm_residual(h, residual, P[p + "post_attention_layernorm.weight"], eps)
        act = L.silu_and_mul(L.linear(x, P[p + "mlp.gate_up_proj.weight"]))
        h = _all_reduce_bf16(L.linear(act, P[p + "mlp.down_proj.weight"]))
    out, _ = L.rms_norm_residual(h, residual, P["model.norm.weight"], eps)
    return out


def _worker(rank, world, port, result_path):
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    sys.path[:0] = [os.path.dirname(here), os.path.join(os.path.dirname(here), "nano-vllm-diy_b200")]
    import torch.distributed as dist
    from oracle import layers as L
    from oracle import model as OM
    from oracle.metadata import SeqState, prepare_seqs
    from oracle.weights import Qwen3Shape, random_weights
    from src.models.qwen3 import Qwen3ForCausalLM
    from src.utils.loader import load_weights

    torch.set_num_threads(2)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world)
    try:
        shape = Qwen3Shape(hidden=256, layers=2, heads=4, kv_heads=2, head_dim=128, inter=512,
                           vocab=1024, max_pos=4096)
        W = random_weights(shape, seed=31)
        torch.set_default_dtype(BF16)
        model = Qwen3ForCausalLM(shape.hf_config(), tp=(rank, world))
        torch.set_default_dtype(torch.float32)
        load_weights(model, W.items())
        P = {n: p.data for n, p in model.named_parameters()}

        class _KV:  # this rank's kv heads of every layer
            pass
        kv = _KV()
        kv.k = [torch.zeros(8, 256, shape.kv_heads // world, shape.head_dim, dtype=BF16)
                for _ in range(shape.layers)]
        kv.v = [torch.zeros_like(t) for t in kv.k]
        okv = OM.OracleKV(shape, 8, 256)
        cs = L.rope_cos_sin(shape.max_pos, shape.head_dim, shape.theta)
        g = torch.Generator().manual_seed(32)
        seqs = [SeqState(torch.randint(0, shape.vocab, (n,), generator=g).tolist(), 0, n,
                         [2 * i, 2 * i + 1]) for i, n in enumerate((9, 300, 77))]
        worst = 0.0
        for step in range(3):
            meta = prepare_seqs(seqs, 256)
            ctx = {k: meta[k] for k in ("cu_seqlens_q", "cu_seqlens_k", "slot_mapping",
                                        "block_tables", "is_prefill")}
            h = _rank_forward(shape, P, meta["input_ids"], meta["positions"], ctx, kv, rank,
                              world, cs)
            both = [torch.empty_like(h) for _ in range(world)]
            dist.all_gather(both, h)
            assert all(torch.equal(b, both[0]) for b in both), f"ranks disagree at step {step}"
            last = h[ctx["cu_seqlens_q"][1:].long() - 1] if ctx["is_prefill"] else h
            part = L.linear(last, P["lm_head.weight"])
            parts = [torch.empty_like(part) for _ in range(world)] if rank == 0 else None
            dist.gather(part, parts, dst=0)
            ref = OM.compute_logits(shape, W, OM.forward(shape, W, meta["input_ids"],
                                                         meta["positions"], ctx, okv, tp=world,
                                                         cos_sin=cs), ctx)
            if rank == 0:
                logits = torch.cat(parts, -1)
                worst = max(worst, L.rel_err(logits, ref))
                assert torch.equal(logits.float().argmax(-1), ref.float().argmax(-1))
            for s, t in zip(seqs, ref.float().argmax(-1).tolist()):
                s.num_cached_tokens = len(s.token_ids)
                s.token_ids.append(int(t))
                s.num_scheduled_tokens = 1
        if rank == 0:
            torch.save({"worst": worst}, result_path)
    finally:
        dist.destroy_process_group()


def test_tp2_gloo_sharded_forward_matches_oracle(tmp_path):
    import torch.multiprocessing as mp
    out = str(tmp_path / "result.pt")
    mp.spawn(_worker, args=(2, _free_port(), out), nprocs=2, join=True)
    worst = torch.load(out)["worst"]
    # same arithmetic, only head subsets differ between the two restatements
    assert worst <= 1e-3, worst
