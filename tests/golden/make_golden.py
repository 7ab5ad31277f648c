"""Generate the golden vectors that pin the oracle to the reference.

Run in a container where the reference checkout is available, with its path
in the REF_DIR environment variable (required); the outputs are small
.pt files next to this script and are committed.  Nothing on a GPU machine
reads the reference: the tests only load these files.

What runs here is the reference's own code, on CPU:
  * src/layers/{layernorm,pos_embedding,activation,linear,llm_head}.py modules
    (torch.compile disabled with TORCHDYNAMO_DISABLE=1: it cannot build on a
    CPU-only image);
  * the Triton store_kvcache_kernel (src/layers/attention.py:10-34) through
    Triton's CPU interpreter (TRITON_INTERPRET=1), so the scatter golden is the
    reference kernel itself;
  * ModelRunner.prepare_seqs (src/engine/model_runner.py:174-233) with its
    pinned-memory / .cuda() calls turned into CPU no-ops;
  * RowParallelLinear under torch.distributed gloo, world_size 2 (config 1);
  * Qwen3ForCausalLM (src/models/qwen3.py) for a tiny configuration.
flash-attn 2.8.3 (src/layers/attention.py:95) has no CPU implementation; its
call is replaced by `sdpa_varlen` below, torch's scaled_dot_product_attention
applied per sequence with the same varlen / paged / bottom-right causal
semantics.  The attention goldens therefore pin the oracle's independent
restatement against torch's SDPA, not against flash-attn itself.
"""
from __future__ import annotations

import hashlib
import os
import sys

os.environ.setdefault("TORCHDYNAMO_DISABLE", "1")
os.environ.setdefault("TRITON_INTERPRET", "1")

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
REF_DIR = os.environ.get("REF_DIR", "")

import torch  # noqa: E402
import torch.nn.functional as F  # noqa: E402

BF16 = torch.bfloat16


def sdpa_varlen(q, k, v, cu_seqlens_q, cu_seqlens_k, max_seqlen_q, max_seqlen_k,
                softmax_scale=None, causal=True, block_table=None):
    """flash_attn_varlen_func semantics via torch SDPA (fp32 math)."""
    T, Hq, d = q.shape
    out = torch.zeros(T, Hq, d, dtype=q.dtype)
    B = cu_seqlens_q.numel() - 1
    for b in range(B):
        q0, q1 = int(cu_seqlens_q[b]), int(cu_seqlens_q[b + 1])
        Lq = q1 - q0
        if Lq <= 0:
            continue
        Lk = int(cu_seqlens_k[b + 1]) - int(cu_seqlens_k[b])
        if block_table is not None:
            page = k.shape[1]
            j = torch.arange(Lk)
            blocks = block_table[b][j // page].long()
            kb, vb = k[blocks, j % page], v[blocks, j % page]
        else:
            k0 = int(cu_seqlens_k[b])
            kb, vb = k[k0:k0 + Lk], v[k0:k0 + Lk]
        G = Hq // kb.shape[1]
        qh = q[q0:q1].float().transpose(0, 1)
        kh = kb.float().transpose(0, 1).repeat_interleave(G, 0)
        vh = vb.float().transpose(0, 1).repeat_interleave(G, 0)
        i = torch.arange(Lq)[:, None]
        jj = torch.arange(Lk)[None, :]
        mask = jj <= i + (Lk - Lq)
        o = F.scaled_dot_product_attention(qh, kh, vh, attn_mask=mask, scale=softmax_scale)
        o = torch.nan_to_num(o, nan=0.0)
        out[q0:q1] = o.transpose(0, 1).to(q.dtype)
    return out


def import_reference():
    sys.path.insert(0, REF_DIR)
    import src.layers.attention as A
    A.flash_attn_varlen_func = sdpa_varlen
    return A


def g(seed):
    return torch.Generator().manual_seed(seed)


def rnd(*s, std=1.0, seed=0):
    return (torch.randn(*s, generator=g(seed), dtype=torch.float32) * std).to(BF16)


# ---------------------------------------------------------------------------
def make_layers():
    from src.layers.activation import SiluAndMul
    from src.layers.layernorm import RMSNorm
    from src.layers.linear import (ColumnParallelLinear, MergedColumnParallelLinear,
                                   QKVParallelLinear, RowParallelLinear)
    from src.layers.pos_embedding import RoPE
    torch.set_default_dtype(BF16)
    out = {}
    # RMSNorm (layernorm.py:10-28), hidden and head_dim rows
    for dim in (1024, 128):
        x = rnd(8, dim, seed=1)
        r = rnd(8, dim, seed=2)
        m = RMSNorm(dim, eps=1e-6)
        m.weight.data.copy_(rnd(dim, std=0.1, seed=3) + 1)
        y = m(x)
        y2, r2 = m(x, r)
        out[f"rmsnorm{dim}"] = dict(x=x, r=r, w=m.weight.data.clone(), y=y, y_res=y2, r_out=r2)
    # RoPE (pos_embedding.py:30-52)
    rope = RoPE(max_seq_len=4096, head_dim=128, base=1000000.0)
    q = rnd(20, 4, 128, seed=4)
    k = rnd(20, 2, 128, seed=5)
    pos = torch.randint(0, 4096, (20,), generator=g(6))
    qo, ko = rope(q, k, pos)
    out["rope"] = dict(q=q, k=k, pos=pos, q_out=qo, k_out=ko, base=1000000.0, max_pos=4096,
                       table_row_sha=hashlib.sha256(rope.cos_sin[pos].float().numpy().tobytes()).hexdigest())
    # SiluAndMul (activation.py:6-10)
    xs = rnd(16, 2 * 384, seed=7)
    out["silu"] = dict(x=xs, y=SiluAndMul()(xs))
    # linear layers at tp = 1 (forward) and the weight-loader shards at tp = 2
    x = rnd(12, 128, seed=8)
    w = rnd(192, 128, std=0.02, seed=9)
    col = ColumnParallelLinear(128, 192)
    col.weight.weight_loader(col.weight, w)
    out["column"] = dict(x=x, w=w, y=col(x))
    src = dict(w=w, up=rnd(192, 128, std=0.02, seed=10), q=rnd(512, 128, std=0.02, seed=11),
               k=rnd(256, 128, std=0.02, seed=12), v=rnd(256, 128, std=0.02, seed=13),
               row=rnd(128, 192, std=0.02, seed=14))
    shards = {"inputs": src}
    for rank in range(2):
        c = ColumnParallelLinear(128, 192, tp=(rank, 2))
        c.weight.weight_loader(c.weight, src["w"])
        shards[f"column_r{rank}"] = c.weight.data.clone()
        m = MergedColumnParallelLinear(128, [192, 192], tp=(rank, 2))
        m.weight.weight_loader(m.weight, src["w"], 0)
        m.weight.weight_loader(m.weight, src["up"], 1)
        shards[f"merged_r{rank}"] = m.weight.data.clone()
        qkv = QKVParallelLinear(128, 128, 4, 2, tp=(rank, 2))
        qkv.weight.weight_loader(qkv.weight, src["q"], "q")
        qkv.weight.weight_loader(qkv.weight, src["k"], "k")
        qkv.weight.weight_loader(qkv.weight, src["v"], "v")
        shards[f"qkv_r{rank}"] = qkv.weight.data.clone()
        row = RowParallelLinear(192, 128, tp=(rank, 2))
        row.weight.weight_loader(row.weight, src["row"])
        shards[f"row_r{rank}"] = row.weight.data.clone()
    out["shards"] = shards
    torch.set_default_dtype(torch.float32)
    return out


def make_kvcache(A):
    """The reference's Triton kernel, run by Triton's CPU interpreter."""
    T, Hkv, d = 37, 2, 128
    k = rnd(T, Hkv, d, seed=20)
    v = rnd(T, Hkv, d, seed=21)
    kc = rnd(1, 256, Hkv, d, seed=22)
    vc = rnd(1, 256, Hkv, d, seed=23)
    slots = torch.randperm(256, generator=g(24))[:T].to(torch.int32)
    slots[::4] = -1
    kc0, vc0 = kc.clone(), vc.clone()
    A.store_kvcache(k, v, kc, vc, slots)
    return dict(k=k, v=v, k_cache_in=kc0, v_cache_in=vc0, slots=slots, k_cache=kc, v_cache=vc)


def make_attention():
    cases = {}
    gg = g(30)
    # fresh varlen prefill, GQA 4:2
    lens = [1, 37, 64, 70]
    cu = torch.tensor([0] + torch.tensor(lens).cumsum(0).tolist(), dtype=torch.int32)
    T = int(cu[-1])
    q = torch.randn(T, 4, 128, generator=gg).to(BF16)
    k = torch.randn(T, 2, 128, generator=gg).to(BF16)
    v = torch.randn(T, 2, 128, generator=gg).to(BF16)
    cases["fresh"] = dict(q=q, k=k, v=v, cu_q=cu, cu_k=cu, out=sdpa_varlen(q, k, v, cu, cu, max(lens), max(lens), 128 ** -0.5))
    # paged: prefix hits, a chunk and decode rows
    lens_q = [30, 1, 1, 7]
    lens_k = [290, 5, 260, 7]
    page = 256
    nblk = 6
    bt = torch.full((4, 2), -1, dtype=torch.int32)
    perm = torch.randperm(nblk, generator=gg).tolist()
    for b, n in enumerate(lens_k):
        for j in range((n + page - 1) // page):
            bt[b, j] = perm.pop()
    kc = torch.randn(nblk, page, 1, 128, generator=gg).to(BF16)
    vc = torch.randn(nblk, page, 1, 128, generator=gg).to(BF16)
    cu_q = torch.tensor([0] + torch.tensor(lens_q).cumsum(0).tolist(), dtype=torch.int32)
    cu_k = torch.tensor([0] + torch.tensor(lens_k).cumsum(0).tolist(), dtype=torch.int32)
    q = torch.randn(int(cu_q[-1]), 4, 128, generator=gg).to(BF16)
    cases["paged"] = dict(q=q, k_cache=kc, v_cache=vc, block_table=bt, cu_q=cu_q, cu_k=cu_k,
                          out=sdpa_varlen(q, kc, vc, cu_q, cu_k, max(lens_q), max(lens_k), 128 ** -0.5, True, bt))
    return cases


def make_metadata():
    """ModelRunner.prepare_seqs on reference Sequence objects."""
    from src.config.sampling_params import SamplingParams
    from src.engine.model_runner import ModelRunner
    from src.engine.sequence import Sequence
    orig_tensor = torch.tensor
    orig_cuda = torch.Tensor.cuda

    def cpu_tensor(*a, **kw):
        kw.pop("pin_memory", None)
        return orig_tensor(*a, **kw)

    torch.tensor = cpu_tensor
    torch.Tensor.cuda = lambda self, *a, **kw: self
    try:
        class Stub:
            block_size = 256
            prepare_block_tables = ModelRunner.prepare_block_tables

        batches = []
        rng = g(40)
        for bi in range(6):
            seqs = []
            nxt = 0
            for _ in range(int(torch.randint(1, 7, (1,), generator=rng))):
                n = int(torch.randint(1, 1500, (1,), generator=rng))
                s = Sequence(torch.randint(0, 151936, (n,), generator=rng).tolist(), SamplingParams(temperature=0.7))
                mode = int(torch.randint(0, 3, (1,), generator=rng))
                if mode == 0:          # fresh prefill
                    s.num_cached_tokens, s.num_scheduled_tokens = 0, n
                elif mode == 1:        # decode
                    s.num_cached_tokens, s.num_scheduled_tokens = n - 1, 1
                else:                  # cached prefix + rest, or a chunk
                    c = int(torch.randint(0, max(1, (n - 1) // 256 + 1), (1,), generator=rng)) * 256
                    c = min(c, n - 1)
                    s.num_cached_tokens = c
                    s.num_scheduled_tokens = int(torch.randint(1, n - c + 1, (1,), generator=rng))
                nb = (s.num_cached_tokens + s.num_scheduled_tokens + 255) // 256
                s.block_table = [] if bi == 0 else list(range(nxt, nxt + nb))
                nxt += nb
                seqs.append(s)
            ids, pos, ctx, is_prefill = ModelRunner.prepare_seqs(Stub(), seqs)
            batches.append(dict(
                seqs=[dict(token_ids=list(s.token_ids), num_cached_tokens=s.num_cached_tokens,
                           num_scheduled_tokens=s.num_scheduled_tokens, block_table=list(s.block_table))
                      for s in seqs],
                input_ids=ids, positions=pos, cu_seqlens_q=ctx.cu_seqlens_q, cu_seqlens_k=ctx.cu_seqlens_k,
                context_lens=ctx.context_lens, slot_mapping=ctx.slot_mapping, block_tables=ctx.block_tables,
                max_seqlen_q=ctx.max_seqlen_q, max_seqlen_k=ctx.max_seqlen_k, is_prefill=is_prefill))
        return batches
    finally:
        torch.tensor = orig_tensor
        torch.Tensor.cuda = orig_cuda


def _row_parallel_worker(rank, path):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = "29517"
    os.environ["TORCHDYNAMO_DISABLE"] = "1"
    sys.path.insert(0, REF_DIR)
    dist.init_process_group("gloo", rank=rank, world_size=2)
    torch.set_num_threads(4)
    from src.layers.linear import RowParallelLinear
    gen = torch.Generator().manual_seed(0)
    x_full = torch.randn(512, 3072, generator=gen, dtype=torch.float32).to(BF16)
    w_full = (torch.randn(1024, 3072, generator=gen, dtype=torch.float32) * 0.02).to(BF16)
    torch.set_default_dtype(BF16)
    layer = RowParallelLinear(3072, 1024, tp=(rank, 2))
    layer.weight.weight_loader(layer.weight, w_full)
    y = layer(x_full.chunk(2, -1)[rank])
    torch.save(y, path + f".rank{rank}")
    dist.barrier()
    dist.destroy_process_group()


def make_row_parallel_c1():
    """RowParallelLinear under gloo, world_size 2, seed 0:
    x [512, 3072] ~ N(0,1) split into two [512, 1536] shards, W [1024, 3072]
    ~ N(0, 0.02) split into two [1024, 1536] shards."""
    import tempfile
    import torch.multiprocessing as mp
    path = os.path.join(tempfile.mkdtemp(), "row")
    mp.start_processes(_row_parallel_worker, args=(path,), nprocs=2, start_method="spawn")
    y0 = torch.load(path + ".rank0")
    y1 = torch.load(path + ".rank1")
    gen = torch.Generator().manual_seed(0)
    x_full = torch.randn(512, 3072, generator=gen).to(BF16)
    w_full = (torch.randn(1024, 3072, generator=gen) * 0.02).to(BF16)
    ref = x_full.float() @ w_full.float().t()
    err = ((y0.float() - ref).abs().max() / ref.abs().max()).item()
    return dict(ranks_identical=bool(torch.equal(y0, y1)),
                sha256=hashlib.sha256(y0.view(torch.int16).numpy().tobytes()).hexdigest(),
                rows=y0[::64].clone(), fp32_rel_err=err)


def make_tiny_model(A):
    sys.path.insert(0, REPO)
    from oracle.weights import Qwen3Shape, random_weights
    from src.models.qwen3 import Qwen3ForCausalLM
    from src.utils.context import Context
    shape = Qwen3Shape(hidden=256, layers=2, heads=4, kv_heads=2, head_dim=128, inter=512,
                       vocab=1000, max_pos=2048)
    W = random_weights(shape, seed=50)
    torch.set_default_dtype(BF16)
    model = Qwen3ForCausalLM(shape.hf_config())
    packed = model.packed_modules_mapping
    for name, t in W.items():
        for key, (target, sid) in packed.items():
            if key in name:
                p = model.get_parameter(name.replace(key, target))
                p.weight_loader(p, t, sid)
                break
        else:
            p = model.get_parameter(name)
            getattr(p, "weight_loader", lambda p_, t_: p_.data.copy_(t_))(p, t)
    kv = torch.zeros(2, shape.layers, 4, 256, shape.kv_heads, shape.head_dim, dtype=BF16)
    li = 0
    for m in model.modules():
        if hasattr(m, "k_cache") and hasattr(m, "v_cache"):
            m.k_cache, m.v_cache = kv[0, li], kv[1, li]
            li += 1
    # prefill of two prompts (blocks [0], [1, 2]) then 3 greedy decode steps
    prompts = [list(range(3, 40)), list(range(100, 400))]
    tables = [[0], [1, 2]]
    steps = []
    toks = [list(p) for p in prompts]
    cached = [0, 0]
    with torch.no_grad():
        for step in range(4):
            ids, pos, slots, cu_q, cu_k = [], [], [], [0], [0]
            for b in range(2):
                start = cached[b]
                end = len(toks[b])
                ids += toks[b][start:end]
                pos += list(range(start, end))
                slots += [tables[b][p // 256] * 256 + p % 256 for p in range(start, end)]
                cu_q.append(cu_q[-1] + end - start)
                cu_k.append(cu_k[-1] + end)
            prefill = step == 0
            bt = None if prefill else torch.tensor([t + [-1] * (2 - len(t)) for t in tables], dtype=torch.int32)
            ctx = Context(is_prefill=max(cu_q[i + 1] - cu_q[i] for i in range(2)) != 1,
                          cu_seqlens_q=torch.tensor(cu_q, dtype=torch.int32),
                          cu_seqlens_k=torch.tensor(cu_k, dtype=torch.int32),
                          max_seqlen_q=max(cu_q[i + 1] - cu_q[i] for i in range(2)),
                          max_seqlen_k=max(cu_k[i + 1] - cu_k[i] for i in range(2)),
                          slot_mapping=torch.tensor(slots, dtype=torch.int32), block_tables=bt)
            logits = model.compute_logits(model(torch.tensor(ids), torch.tensor(pos), ctx), ctx)
            nxt = logits.float().argmax(-1).tolist()
            steps.append(dict(input_ids=torch.tensor(ids), positions=torch.tensor(pos),
                              cu_seqlens_q=ctx.cu_seqlens_q, cu_seqlens_k=ctx.cu_seqlens_k,
                              slot_mapping=ctx.slot_mapping, block_tables=bt,
                              is_prefill=ctx.is_prefill, logits=logits.clone(), tokens=nxt))
            for b in range(2):
                cached[b] = len(toks[b])
                toks[b].append(nxt[b])
    torch.set_default_dtype(torch.float32)
    return dict(shape=shape.__dict__, seed=50, tables=tables, steps=steps)


def main():
    if not REF_DIR or not os.path.isdir(os.path.join(REF_DIR, "src")):
        raise SystemExit("set REF_DIR to the reference checkout (the directory holding src/)")
    A = import_reference()
    torch.manual_seed(0)
    torch.save(make_layers(), os.path.join(HERE, "layers.pt"))
    torch.save(make_kvcache(A), os.path.join(HERE, "kvcache.pt"))
    torch.save(make_attention(), os.path.join(HERE, "attention.pt"))
    torch.save(make_metadata(), os.path.join(HERE, "metadata.pt"))
    torch.save(make_tiny_model(A), os.path.join(HERE, "qwen3_tiny.pt"))
    torch.save(make_row_parallel_c1(), os.path.join(HERE, "row_parallel_c1.pt"))
    for f in sorted(os.listdir(HERE)):
        if f.endswith(".pt"):
            print(f, os.path.getsize(os.path.join(HERE, f)))


if __name__ == "__main__":
    main()
