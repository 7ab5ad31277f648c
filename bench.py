"""Decode throughput of the B200 Qwen3 decoder path (one JSON line on rank 0).

Workload ("qwen3-8b-decode-mix256"): Qwen3-8B architecture, random-init bf16
weights N(0, 0.02), tensor parallel over the N GPUs (TP = N, strong scaling:
the same 256-sequence batch at every N).  The 256 sequences are the
synthetic serving mix: prompt ~U[100, 1024] tokens, output budget
~U[100, 1024], captured mid-generation (generated ~U[1, budget]), so a decode
step attends over ~843 cached tokens per sequence on average.  The paged KV
cache (block 256, random permutation of physical blocks) holds synthetic
N(0, 1) keys/values.

One step = one greedy decode step for all 256 sequences: embedding, 36
decoder layers (qkv GEMM, q/k norm + RoPE + KV write, paged attention,
o_proj, RMSNorm, gate_up + SiLU, down_proj), final norm, LM head, argmax --
replayed from one CUDA graph.  Each step feeds back its argmax tokens and
advances every position by one.

  value : tok/s with the step metadata already resident in HBM (device-timed
          CUDA events around K steps, max over ranks)
  e2e   : tok/s through the runner's public API with host buffers: metadata
          built on the host, pinned H2D copies, graph replay, tokens copied
          back (D2H) every step
  roofline : the dominant kernel (paged decode attention) timed live with
          CUDA events over its standalone launch on one layer's inputs

`--impl reference` times the oracle (a CPU port of the reference's torch
path) on the host cores instead.
"""
from __future__ import annotations

import argparse
import json
import os
import random
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np
import torch

REPO = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(REPO, "nano-vllm-diy_b200")
for p in (REPO, PKG):
    if p not in sys.path:
        sys.path.insert(0, p)

METRIC = "decode tok/s, Qwen3-8B bf16, TP 1/2/4/8"
UNIT = "tok/s"
WORKLOAD = "qwen3-8b-decode-mix256"
BLOCK = 256


def peaks():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    except Exception:
        return 6650.0, 1590.0, "fallback"


def mix(batch: int, seed: int):
    """Context length (cached tokens + the new one) of each sequence."""
    rng = random.Random(seed)
    lens = []
    for _ in range(batch):
        prompt = rng.randint(100, 1024)
        budget = rng.randint(100, 1024)
        gen = rng.randint(1, budget)
        lens.append(prompt + gen)
    return lens


def qwen3_8b_config():
    from oracle.weights import QWEN3_8B
    import dataclasses
    return dataclasses.replace(QWEN3_8B, max_pos=4096)


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 50 ms."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: torch.device):
        try:
            self.gpu = "GPU-" + str(torch.cuda.get_device_properties(device).uuid)
        except Exception:
            self.gpu = str(device.index)
        self.proc = None
        self.path = None

    def __enter__(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "50"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
        # nvidia-smi can take a second or more to start (eight ranks starting
        # it at once): wait, bounded, for its first sample so that the window
        # really covers the steps that follow
        t_end = time.time() + 5.0
        while self.proc is not None and time.time() < t_end and self.proc.poll() is None:
            if os.path.getsize(self.path) > 0:
                break
            time.sleep(0.05)
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        if not self.path or not os.path.exists(self.path):
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        rows = []
        with open(self.path) as f:
            for line in f:
                parts = [x.strip() for x in line.split(",")]
                if len(parts) >= 9:
                    rows.append(parts)
        os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}

        def num(x):
            try:
                return float(x)
            except ValueError:
                return None
        sm = [num(r[1]) for r in rows if num(r[1]) is not None]
        mx = [num(r[2]) for r in rows if num(r[2]) is not None]
        under = [s for s in sm if s > 0.5 * max(sm)] if sm else []
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(under) if under else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons,
                "samples": len(rows)}


# --------------------------------------------------------------------------
# CPU side: the oracle port of the reference path
# --------------------------------------------------------------------------
class CpuDecodeStep:
    """The oracle (the reference's torch path restated for the CPU) on the host
    cores, on the bench's own workload: one greedy decode step of the 256
    sequences of the mix through all 36 Qwen3-8B decoder layers, the final
    norm, the LM head over the full 151936-entry vocabulary and the argmax.
    GEMMs use torch's bf16 F.linear, the op the reference calls
    (src/layers/linear.py:75,170; src/layers/llm_head.py:64).

    Host memory is kept to a few GB: all 36 layers reference the same random
    layer weights (436 MB, far larger than any CPU cache, so no layer finds
    another's weights cached) and the same paged K/V tensors, which hold the
    whole mix (1 GB).  The arithmetic of a step is exactly that of a step of
    the model; only the values differ."""

    def __init__(self, seed: int = 0, batch: int = 256):
        from oracle import layers as L
        from oracle import model as OM
        from oracle.weights import random_weights
        import dataclasses
        torch.set_num_threads(os.cpu_count() or 1)
        L.NATIVE_BF16_LINEAR = True
        self.L, self.OM = L, OM
        self.shape = qwen3_8b_config()
        one = dataclasses.replace(self.shape, layers=1, vocab=4096)
        W = random_weights(one, seed=seed)
        p0 = "model.layers.0."
        W[p0 + "self_attn.qkv_proj.weight"] = torch.cat(
            [W[p0 + "self_attn.q_proj.weight"], W[p0 + "self_attn.k_proj.weight"],
             W[p0 + "self_attn.v_proj.weight"]], 0)
        W[p0 + "mlp.gate_up_proj.weight"] = torch.cat(
            [W[p0 + "mlp.gate_proj.weight"], W[p0 + "mlp.up_proj.weight"]], 0)
        layer0 = {k[len(p0):]: v for k, v in W.items() if k.startswith(p0)}
        for i in range(1, self.shape.layers):
            for k, v in layer0.items():
                W[f"model.layers.{i}.{k}"] = v
        # full-size embedding and LM head: a random block tiled to 151936 rows
        # (drawing 1.2 G normals would dominate the set-up; the values do not
        # change the CPU time)
        for name in ("model.embed_tokens.weight", "lm_head.weight"):
            small = W[name]
            reps = (self.shape.vocab + small.shape[0] - 1) // small.shape[0]
            W[name] = small.repeat(reps, 1)[:self.shape.vocab].contiguous()
        self.W = W
        self.n = batch
        self.lens = mix(256, seed)[:batch]
        pages = [(n + BLOCK - 1) // BLOCK for n in self.lens]
        nblk = sum(pages)
        kv = OM.OracleKV(one, nblk, BLOCK)
        g = torch.Generator().manual_seed(seed)
        # N(0, 1) K/V (as on the GPU side): a 64 Mi-element random block tiled
        for t in (kv.k[0], kv.v[0]):
            flat = t.view(-1)
            blk = torch.randn(min(flat.numel(), 1 << 26), generator=g).to(torch.bfloat16)
            for o in range(0, flat.numel(), blk.numel()):
                m = min(blk.numel(), flat.numel() - o)
                flat[o:o + m].copy_(blk[:m])
        kv.k = kv.k * self.shape.layers
        kv.v = kv.v * self.shape.layers
        self.kv = kv
        perm = np.random.default_rng(seed).permutation(nblk)
        bt = torch.full((batch, max(pages)), -1, dtype=torch.int32)
        k = 0
        for i, n in enumerate(pages):
            bt[i, :n] = torch.from_numpy(perm[k:k + n].astype(np.int32))
            k += n
        self.pos = torch.tensor([n - 1 for n in self.lens], dtype=torch.int64)
        slots = (bt.long().gather(1, (self.pos // BLOCK)[:, None])[:, 0] * BLOCK
                 + self.pos % BLOCK).to(torch.int32)
        self.ctx = dict(cu_seqlens_q=torch.arange(batch + 1, dtype=torch.int32),
                        cu_seqlens_k=torch.tensor([0] + list(np.cumsum(self.lens)),
                                                  dtype=torch.int32),
                        slot_mapping=slots, block_tables=bt, is_prefill=False)
        self.ids = torch.randint(0, 10000, (batch,), generator=g)
        self.cos_sin = L.rope_cos_sin(self.shape.max_pos, self.shape.head_dim, self.shape.theta)

    def step(self) -> float:
        """One decode step (seconds); feeds its tokens back as the next ids."""
        a = time.perf_counter()
        h = self.OM.forward(self.shape, self.W, self.ids, self.pos, self.ctx, self.kv,
                            cos_sin=self.cos_sin)
        logits = self.OM.compute_logits(self.shape, self.W, h, self.ctx)
        self.ids = logits.argmax(-1)
        return time.perf_counter() - a

    def describe(self, steps: int) -> dict:
        return {"unit": UNIT, "cores": torch.get_num_threads(), "kind": "port",
                "sample": (f"oracle torch-CPU port of the reference path (bf16 F.linear as the "
                           f"reference): {steps} full decode step(s) of the {self.n}-sequence mix "
                           f"(mean ctx {np.mean(self.lens):.0f}) through 36 Qwen3-8B layers, LM head "
                           f"over 151936 tokens and argmax; the 36 layers share one layer's "
                           f"random weights and K/V pages")}


def cpu_baseline(seconds: float, seed: int) -> dict:
    """Full decode steps of the bench's workload on the host cores, as many
    as fit `seconds` (at least one)."""
    smp = CpuDecodeStep(seed=seed)
    times = []
    t0 = time.perf_counter()
    while not times or time.perf_counter() - t0 + times[-1] < seconds:
        times.append(smp.step())
    d = smp.describe(len(times))
    d["value"] = smp.n / float(np.mean(times))
    return d


def run_reference_arm(args, rank: int, world: int):
    """The reference arm: the CPU port on the host cores, full decode steps of
    the same 256-sequence workload.  A CPU step takes tens of seconds, so the
    run does at most `--cpu-max-steps` timed steps after one warm-up step and
    reports the counts it actually ran."""
    if rank != 0:
        return
    smp = CpuDecodeStep(seed=args.seed, batch=args.batch)
    warm = min(args.warmup, 1)
    for _ in range(warm):
        smp.step()
    steps = max(1, min(args.steps, args.cpu_max_steps))
    times = [smp.step() for _ in range(steps)]
    ms = 1000.0 * float(np.mean(times))
    value = smp.n / (ms / 1000.0)
    d = smp.describe(steps)
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT,
        "n_gpus": args.gpus, "steps": steps, "warmup": warm,
        "steps_requested": args.steps, "warmup_requested": args.warmup,
        "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": WORKLOAD, "batch": smp.n, "tp": 1, "parallelism": "tp1",
                   "mean_ctx": float(np.mean(smp.lens)), "block_size": BLOCK,
                   "device": "host CPU"},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": d["cores"], "kind": "port",
                         "sample": d["sample"]},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# --------------------------------------------------------------------------
# GPU side
# --------------------------------------------------------------------------
@torch.inference_mode()
def run_b200(args, rank: int, world: int):
    import torch.distributed as dist
    from src import b200
    from src.engine.model_runner import ModelRunner
    from src.layers import tp_comm

    torch.cuda.set_device(rank % torch.cuda.device_count())
    dev = torch.device("cuda", torch.cuda.current_device())
    if world > 1:
        dist.init_process_group("nccl", device_id=dev,
                                timeout=__import__("datetime").timedelta(seconds=120))
        if args.fused_ar:
            from src.layers import tp_allreduce
            tp_comm.set_comm(tp_allreduce.FusedRowParallel.create(dev))
        else:
            tp_comm.set_enabled(False)
    shape = qwen3_8b_config()
    cfg = shape.hf_config()
    B = args.batch
    lens = mix(B, args.seed)
    steps_total = args.warmup + args.steps + 2
    max_len = max(lens) + steps_total
    runner = ModelRunner(cfg, rank=rank, world_size=world, block_size=BLOCK, max_num_seqs=B,
                         max_seq_len=max(4096, max_len), device=dev)
    runner.init_random_weights(seed=args.seed)
    per_seq = [(n + steps_total + BLOCK - 1) // BLOCK for n in lens]
    nblk = sum(per_seq) + 4
    runner.allocate_kv_cache(nblk)
    g = torch.Generator(device=dev).manual_seed(args.seed + 1)
    for i in range(runner.kv_cache.shape[0]):
        for j in range(runner.kv_cache.shape[1]):
            runner.kv_cache[i, j].normal_(0.0, 1.0, generator=g)
    perm = np.random.default_rng(args.seed).permutation(nblk)
    width = max(per_seq)
    bt = np.full((B, width), -1, dtype=np.int32)
    k = 0
    for i, n in enumerate(per_seq):
        bt[i, :n] = perm[k:k + n]
        k += n

    launches0 = b200.launch_count()
    runner.capture_cudagraph([B], with_sampling=True)
    kernels_per_step = b200.launch_count() - launches0  # warm-up + capture launch the same set
    kernels_per_step //= 2
    v = runner.graph_vars

    # device-resident metadata for every step
    S = steps_total
    lens_t = torch.tensor(lens, dtype=torch.int64)
    pos_all = torch.stack([lens_t - 1 + s for s in range(S)])                     # [S, B]
    bt_t = torch.from_numpy(bt).long()
    slot_all = (bt_t.gather(1, pos_all.t() // BLOCK).t() * BLOCK + pos_all % BLOCK).to(torch.int32)
    cuk_all = torch.zeros(S, B + 1, dtype=torch.int32)
    cuk_all[:, 1:] = torch.cumsum(pos_all + 1, dim=1).to(torch.int32)
    pos_d, slot_d, cuk_d = pos_all.to(dev), slot_all.to(dev), cuk_all.to(dev)
    v["cu_seqlens_q"][:B + 1] = torch.arange(B + 1, dtype=torch.int32, device=dev)
    v["block_tables"][:B, :width] = torch.from_numpy(bt).to(dev)
    v["tokens"][:B] = torch.randint(0, 10000, (B,), device=dev, generator=g)

    def device_step(s):
        v["input_ids"][:B].copy_(v["tokens"][:B])
        v["positions"][:B].copy_(pos_d[s])
        v["slot_mapping"][:B].copy_(slot_d[s])
        v["cu_seqlens_k"][:B + 1].copy_(cuk_d[s])
        runner.replay(B)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[dev.index])
        torch.cuda.synchronize()

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    stream = torch.cuda.current_stream()
    # clocks are sampled over the whole loaded window (warm-up, the timed steps
    # and the e2e steps below): the timed region alone is a few tenths of a
    # second, a handful of samples
    clocks = ClockSampler(dev).__enter__()
    for s in range(args.warmup):
        device_step(s)
    barrier()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    for s in range(args.warmup, args.warmup + args.steps):
        device_step(s)
    ev1.record(stream)
    barrier()
    ms = max_over_ranks(ev0.elapsed_time(ev1) / args.steps)
    value = B / (ms / 1000.0)

    # ---- e2e: host metadata -> pinned H2D -> replay -> D2H tokens, per step
    h_lens = np.asarray(lens, dtype=np.int64)
    pin = {
        "ids": torch.empty(B, dtype=torch.int64).pin_memory(),
        "pos": torch.empty(B, dtype=torch.int64).pin_memory(),
        "slot": torch.empty(B, dtype=torch.int32).pin_memory(),
        "cuq": torch.empty(B + 1, dtype=torch.int32).pin_memory(),
        "cuk": torch.empty(B + 1, dtype=torch.int32).pin_memory(),
        "bt": torch.from_numpy(bt).pin_memory(),
        "tok": torch.empty(B, dtype=torch.int64).pin_memory(),
    }
    h2d = sum(pin[k].numel() * pin[k].element_size() for k in ("ids", "pos", "slot", "cuq", "cuk", "bt"))
    d2h = pin["tok"].numel() * pin["tok"].element_size()
    tokens_host = np.random.default_rng(args.seed).integers(0, 10000, B)

    def e2e_step(s):
        pos = h_lens - 1 + s
        pin["ids"].numpy()[:] = tokens_host
        pin["pos"].numpy()[:] = pos
        pin["slot"].numpy()[:] = bt[np.arange(B), pos // BLOCK] * BLOCK + pos % BLOCK
        pin["cuq"].numpy()[:] = np.arange(B + 1)
        pin["cuk"].numpy()[0] = 0
        np.cumsum(pos + 1, out=pin["cuk"].numpy()[1:])
        v["input_ids"][:B].copy_(pin["ids"], non_blocking=True)
        v["positions"][:B].copy_(pin["pos"], non_blocking=True)
        v["slot_mapping"][:B].copy_(pin["slot"], non_blocking=True)
        v["cu_seqlens_q"][:B + 1].copy_(pin["cuq"], non_blocking=True)
        v["cu_seqlens_k"][:B + 1].copy_(pin["cuk"], non_blocking=True)
        v["block_tables"][:B, :width].copy_(pin["bt"], non_blocking=True)
        runner.replay(B)
        pin["tok"].copy_(v["tokens"][:B], non_blocking=True)
        stream.synchronize()
        tokens_host[:] = pin["tok"].numpy()

    for s in range(args.warmup):
        e2e_step(s)
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for s in range(args.warmup, args.warmup + args.steps):
        e2e_step(s)
    e1.record(stream)
    barrier()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1) / args.steps)
    clocks.__exit__(None, None, None)
    clock_summary = clocks.summary()
    clock_summary["window"] = "warm-up, timed and e2e steps"

    # ---- roofline: decode attention of one layer, timed standalone
    hbm_peak, _, peak_kind = peaks()
    from src.layers.attention import attend
    from src.utils.context import Context
    attn_mod = runner.model.model.layers[0].self_attn
    s_last = args.warmup + args.steps - 1
    ctx = Context(is_prefill=False, cu_seqlens_q=v["cu_seqlens_q"][:B + 1].clone(),
                  cu_seqlens_k=cuk_d[s_last].clone(), max_seqlen_q=1,
                  max_seqlen_k=runner.max_seq_len, slot_mapping=slot_d[s_last].clone(),
                  block_tables=v["block_tables"][:B].clone())
    Hq = runner.local_q_heads
    q = torch.randn(B, Hq, 128, device=dev, dtype=torch.bfloat16)
    out = torch.empty_like(q)
    with torch.inference_mode():
        for _ in range(3):
            attend(q, None, None, attn_mod.attn.k_cache, attn_mod.attn.v_cache, ctx, attn_mod.scaling, out=out)
        torch.cuda.synchronize()
        a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        reps = 20
        a0.record(stream)
        for _ in range(reps):
            attend(q, None, None, attn_mod.attn.k_cache, attn_mod.attn.v_cache, ctx, attn_mod.scaling, out=out)
        a1.record(stream)
        torch.cuda.synchronize()
    attn_ms = a0.elapsed_time(a1) / reps
    ctx_sum = int((pos_all[s_last] + 1).sum())
    kv_bytes = ctx_sum * runner.local_kv_heads * 128 * 2 * 2
    qo_bytes = 2 * B * Hq * 128 * 2
    attn_bytes = kv_bytes + qo_bytes
    achieved = attn_bytes / (attn_ms / 1000.0) / 1e9
    # whole-step bytes: weights + KV read + KV write of the new tokens
    w_bytes = sum(p.numel() * p.element_size() for n, p in runner.model.named_parameters()
                  if "embed_tokens" not in n)
    step_bytes = w_bytes + kv_bytes * shape.layers + B * runner.local_kv_heads * 128 * 4 * shape.layers
    step_gbs = step_bytes / (ms / 1000.0) / 1e9
    traffic = None
    tpath = os.path.join(REPO, "profiles", "decode_attention_traffic.txt")
    if os.path.exists(tpath):
        try:
            with open(tpath) as f:
                tr = json.load(f)
            # captured on a smaller case: scale by the KV bytes processed
            traffic = tr["dram_bytes"] * attn_bytes / tr["algorithmic_bytes"]
        except Exception:
            traffic = None

    # any bounded wait that gave up or index that was out of range during the
    # run would have set the device error word
    dev_err = b200.device_error(clear=True)
    cpu = None
    # the CPU port is timed at N = 1 only: under torchrun the other ranks would
    # wait in the next collective for as long as rank 0 keeps the host's cores
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu = cpu_baseline(args.cpu_seconds, args.seed)

    if world > 1:
        tp_comm.clear()
    runner.release_graphs()
    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "bf16", "data": "synthetic (random-init weights, N(0,1) KV, seeded mix)",
            "config": {"workload": WORKLOAD, "batch": B, "tp": world, "parallelism": f"tp{world}",
                       "mean_ctx": float(np.mean(lens)), "block_size": BLOCK,
                       "l2": "inputs larger than L2 (16.4 GB weights + KV per step)",
                       "fused_allreduce": bool(world > 1 and args.fused_ar)},
            "roofline": {"bound": "hbm", "kernel": "decode_attn_kernel",
                         "achieved": achieved, "peak": hbm_peak, "unit": "GB/s",
                         "frac": achieved / hbm_peak, "peak_source": peak_kind,
                         "traffic": traffic, "algorithmic_bytes": attn_bytes,
                         "launch_ms": attn_ms},
            "step_roofline": {"bytes": step_bytes, "achieved_gbs": step_gbs,
                              "frac": step_gbs / hbm_peak},
            "cpu_baseline": cpu,
            "e2e": {"value": B / (e2e_ms / 1000.0), "unit": UNIT, "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "ms_per_step": e2e_ms},
            "gpu_launches": kernels_per_step * args.steps,
            "clocks": clock_summary,
            "device_error": dev_err,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier(device_ids=[dev.index])
        dist.destroy_process_group()


def run_microbench(args):
    """Kernel microbenchmarks (one JSON line each), used for ncu captures.
      attn    : BASELINE config 3 -- paged decode attention, B=256, ctx ~U[128,4096],
                32 q / 8 kv heads, N(0,1) bf16, block 256, random block permutation,
                seed 1 -- plus the slot_mapping scatter of 256 new tokens
      gemm    : the Qwen3-8B TP1 decode GEMMs at 256 tokens
      prefill : prefill attention, fresh varlen and chunked over paged prefixes,
                FLOPs against the tensor peak"""
    from src import b200
    from src.layers.attention import attend
    from src.utils.context import Context
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    hbm, tflops, kind = peaks()
    reps = args.steps

    def timeit(fn):
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / reps

    with torch.inference_mode():
        if args.workload == "attn":
            g = torch.Generator().manual_seed(1)
            B, Hq, Hkv = 256, 32, 8
            lens = torch.randint(128, 4097, (B,), generator=g)
            pages = (lens + BLOCK - 1) // BLOCK
            nblk = int(pages.sum()) + 1
            perm = torch.randperm(nblk, generator=g)
            width = int(pages.max())
            bt = torch.full((B, width), -1, dtype=torch.int32)
            k = 0
            for i, n in enumerate(pages.tolist()):
                bt[i, :n] = perm[k:k + n].to(torch.int32)
                k += n
            gd = torch.Generator(device=dev).manual_seed(1)
            kc = torch.randn(nblk, BLOCK, Hkv, 128, generator=gd, device=dev).to(torch.bfloat16)
            vc = torch.randn(nblk, BLOCK, Hkv, 128, generator=gd, device=dev).to(torch.bfloat16)
            q = torch.randn(B, Hq, 128, generator=gd, device=dev).to(torch.bfloat16)
            cu_q = torch.arange(B + 1, dtype=torch.int32, device=dev)
            cu_k = torch.zeros(B + 1, dtype=torch.int32)
            cu_k[1:] = torch.cumsum(lens, 0)
            ctx = Context(is_prefill=False, cu_seqlens_q=cu_q, cu_seqlens_k=cu_k.to(dev),
                          max_seqlen_q=1, max_seqlen_k=4096, block_tables=bt.to(dev))
            out = torch.empty_like(q)
            ms = timeit(lambda: attend(q, None, None, kc, vc, ctx, 128 ** -0.5, out=out))
            byts = int(lens.sum()) * Hkv * 128 * 2 * 2 + 2 * B * Hq * 128 * 2
            # the scatter of 256 new tokens into their slots
            pos = lens - 1
            slots = (bt.long().gather(1, (pos // BLOCK)[:, None])[:, 0] * BLOCK + pos % BLOCK).to(torch.int32).to(dev)
            knew = torch.randn(B, Hkv, 128, generator=gd, device=dev).to(torch.bfloat16)
            # a 2 MiB scatter takes a few microseconds, less than one host
            # launch: time it from a CUDA graph of 20 calls
            b200.store_kvcache(knew, knew, kc, vc, slots)
            torch.cuda.synchronize()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                for _ in range(20):
                    b200.store_kvcache(knew, knew, kc, vc, slots)
            ms_sc = timeit(graph.replay) / 20
            sc_bytes = 2 * B * Hkv * 128 * 2 * 2
            print(json.dumps({"workload": "attn-microbench (config 3)", "decode_attn_ms": ms,
                              "bytes": byts, "gbs": byts / ms / 1e6, "frac": byts / ms / 1e6 / hbm,
                              "scatter_ms": ms_sc, "scatter_gbs": sc_bytes / ms_sc / 1e6,
                              "peak_gbs": hbm, "peak_source": kind}), flush=True)
        elif args.workload == "prefill":
            # Qwen3-8B heads (32 q / 8 kv, d 128): (a) fresh varlen prefill of 8
            # prompts of 2048 tokens (per-token K / V); (b) chunked prefill: 16
            # chunks of 512 tokens over 1536 cached tokens each (the scheduler's
            # chunk size, src/engine/scheduler.py:90-98), K / V paged, block 256
            Hq, Hkv = 32, 8
            res = {}
            gd = torch.Generator(device=dev).manual_seed(3)
            scale = 128 ** -0.5
            # (a) fresh
            lens = [2048] * 8
            cu = torch.tensor([0] + list(np.cumsum(lens)), dtype=torch.int32, device=dev)
            T = sum(lens)
            q = torch.randn(T, Hq, 128, generator=gd, device=dev).to(torch.bfloat16)
            k = torch.randn(T, Hkv, 128, generator=gd, device=dev).to(torch.bfloat16)
            v = torch.randn(T, Hkv, 128, generator=gd, device=dev).to(torch.bfloat16)
            pairs = sum(n * (n + 1) // 2 for n in lens)
            ctx_a = Context(is_prefill=True, cu_seqlens_q=cu, cu_seqlens_k=cu, max_seqlen_q=2048,
                            max_seqlen_k=2048)
            out = torch.empty_like(q)
            ms = timeit(lambda: attend(q, k, v, None, None, ctx_a, scale, out=out))
            fl = 4.0 * 128 * Hq * pairs
            res["fresh_8x2048"] = {"ms": ms, "tflops": fl / ms / 1e9, "frac": fl / ms / 1e9 / tflops}
            # (b) chunked over paged prefixes
            B, chunk, cached = 16, 512, 1536
            Lk = chunk + cached
            pages = (Lk + BLOCK - 1) // BLOCK
            nblk = B * pages + 1
            perm = torch.randperm(nblk, generator=torch.Generator().manual_seed(5))
            bt = perm[:B * pages].view(B, pages).to(torch.int32).to(dev)
            kc = torch.randn(nblk, BLOCK, Hkv, 128, generator=gd, device=dev).to(torch.bfloat16)
            vc = torch.randn(nblk, BLOCK, Hkv, 128, generator=gd, device=dev).to(torch.bfloat16)
            cu_q = torch.arange(0, (B + 1) * chunk, chunk, dtype=torch.int32, device=dev)
            cu_k = torch.arange(0, (B + 1) * Lk, Lk, dtype=torch.int32, device=dev)
            q2 = torch.randn(B * chunk, Hq, 128, generator=gd, device=dev).to(torch.bfloat16)
            ctx_b = Context(is_prefill=True, cu_seqlens_q=cu_q, cu_seqlens_k=cu_k, max_seqlen_q=chunk,
                            max_seqlen_k=Lk, block_tables=bt)
            out2 = torch.empty_like(q2)
            ms = timeit(lambda: attend(q2, None, None, kc, vc, ctx_b, scale, out=out2))
            pairs = B * (chunk * cached + chunk * (chunk + 1) // 2)
            fl = 4.0 * 128 * Hq * pairs
            res["chunked_16x512_over_1536"] = {"ms": ms, "tflops": fl / ms / 1e9, "frac": fl / ms / 1e9 / tflops}
            print(json.dumps({"workload": "prefill-attention (Qwen3-8B heads)",
                              "kernel": os.environ.get("B200_PREFILL") or "tcgen05", "kernels": res,
                              "tensor_peak_tflops": tflops, "peak_source": kind}), flush=True)
        else:
            T = 256
            shapes = {"qkv": (6144, 4096), "o_proj": (4096, 4096), "gate_up": (24576, 4096),
                      "down": (4096, 12288), "lm_head": (151936, 4096)}
            res = {}
            if args.gemm_shapes:
                shapes = {k: v for k, v in shapes.items() if k in args.gemm_shapes.split(",")}
            for name, (N, K) in shapes.items():
                x = torch.randn(T, K, device=dev).to(torch.bfloat16)
                # enough weight copies that consecutive calls stream from HBM
                # (> 300 MB between reuses of one copy, L2 is 126 MB)
                copies = max(1, -(-300 * 2 ** 20 // (N * K * 2)))
                ws = [(torch.randn(N, K, device=dev) * 0.02).to(torch.bfloat16) for _ in range(copies)]
                y = torch.empty(T, N // 2 if name == "gate_up" else N, device=dev, dtype=torch.bfloat16)
                if name == "gate_up":
                    fn = lambda w: b200.linear_silu_and_mul(x, w, out=y)
                else:
                    fn = lambda w: b200.linear(x, w, out=y)
                # device time per call from a CUDA graph of `per` calls (a
                # host-launched loop would time the Python launch path)
                fn(ws[0])
                torch.cuda.synchronize()
                per = 2 * copies if copies > 1 else 10
                graph = torch.cuda.CUDAGraph()
                with torch.cuda.graph(graph):
                    for i in range(per):
                        fn(ws[i % copies])
                ms = timeit(graph.replay) / per
                del graph, ws
                byts = N * K * 2 + T * K * 2 + T * (N // 2 if name == "gate_up" else N) * 2
                res[name] = {"ms": ms, "gbs": byts / ms / 1e6, "frac": byts / ms / 1e6 / hbm}
                del x
            print(json.dumps({"workload": "gemm-microbench (Qwen3-8B TP1 decode, T=256)",
                              "kernels": res, "peak_gbs": hbm}), flush=True)


def run_allreduce_microbench(args, rank: int, world: int):
    """Fused RowParallelLinear (GEMM + all-reduce over NVLink) of the Qwen3-8B
    decode step at TP = world, T = 256 tokens: o_proj (K = 4096 / world) and
    down_proj (K = 12288 / world), N = 4096.  Device time per call with CUDA
    events, max over ranks, against GEMM + NCCL all_reduce.  Roofline target
    = slowest of FLOPs / tensor peak, HBM bytes / HBM peak and NVLink bytes /
    770 GB/s (measured peer-copy bandwidth per direction), with NVLink bytes
    per rank = 2 (world - 1) / world x T x N x 2 (reduce-scatter + all-gather)."""
    import datetime
    import torch.distributed as dist
    from src import b200
    from src.layers.tp_allreduce import FusedRowParallel
    torch.cuda.set_device(rank % torch.cuda.device_count())
    dev = torch.device("cuda", torch.cuda.current_device())
    dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=120))
    mode = {"auto": None, "oneshot": True, "twoshot": False}[args.ar_mode]
    comm = FusedRowParallel(dev, max_tokens=512, max_hidden=4096, one_shot=mode)
    hbm, tflops, kind = peaks()
    nvlink = 770.0
    T, N = 256, 4096
    out = {}
    stream = torch.cuda.current_stream()

    def time_fn(fn):
        """Device time per call: `steps` calls captured in one CUDA graph, the
        graph replayed after warm-up (no host launch gaps), max over ranks."""
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for _ in range(args.steps):
                fn()
        for _ in range(2):
            graph.replay()
        dist.barrier(device_ids=[dev.index])
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        graph.replay()
        e1.record(stream)
        torch.cuda.synchronize()
        del graph
        t = torch.tensor([e0.elapsed_time(e1) / args.steps], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    with torch.inference_mode():
        for name, Kfull in (("o_proj", 4096), ("down_proj", 12288)):
            K = Kfull // world
            g = torch.Generator(device=dev).manual_seed(rank + 1)
            x = torch.randn(T, K, device=dev, generator=g).to(torch.bfloat16)
            w = (torch.randn(N, K, device=dev, generator=g) * 0.02).to(torch.bfloat16)
            fused_ms = time_fn(lambda: comm.linear_allreduce(x, w))

            def unfused():
                y = b200.linear(x, w)
                dist.all_reduce(y)
            base_ms = time_fn(unfused)
            gemm_ms = time_fn(lambda: b200.linear(x, w))
            yy = b200.linear(x, w)
            nccl_ms = time_fn(lambda: dist.all_reduce(yy))
            flops = 2.0 * T * N * K
            hbm_bytes = N * K * 2 + T * K * 2 + T * N * 2
            nv_bytes = 2.0 * (world - 1) / world * T * N * 2
            target_ms = max(flops / (tflops * 1e12), hbm_bytes / (hbm * 1e9), nv_bytes / (nvlink * 1e9)) * 1e3
            out[name] = {"K_per_rank": K, "fused_ms": fused_ms, "gemm_plus_nccl_ms": base_ms,
                         "gemm_only_ms": gemm_ms, "nccl_allreduce_ms": nccl_ms,
                         "roofline_ms": target_ms, "frac": target_ms / fused_ms,
                         "nvlink_bytes_per_rank": nv_bytes, "hbm_bytes": hbm_bytes}
    fused_ok = comm.fallback_calls == 0
    comm.close()
    if rank == 0:
        print(json.dumps({"workload": "fused-rowparallel-allreduce (Qwen3-8B decode, T=256)",
                          "tp": world, "mode": "one-shot" if comm.one_shot else "two-shot",
                          "kernels": out, "fused_path_taken": fused_ok,
                          "nvlink_gbs_per_direction": nvlink, "hbm_peak_gbs": hbm,
                          "tensor_peak_tflops": tflops, "peak_source": kind}), flush=True)
    dist.barrier(device_ids=[dev.index])
    dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--batch", type=int, default=256)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline sample")
    ap.add_argument("--cpu-seconds", type=float, default=25.0,
                    help="CPU baseline sample length (whole decode steps, at least one)")
    ap.add_argument("--cpu-max-steps", type=int, default=3,
                    help="reference arm: timed CPU steps at most (each takes tens of seconds)")
    ap.add_argument("--no-fused-ar", dest="fused_ar", action="store_false")
    ap.add_argument("--gemm-shapes", default="",
                    help="gemm workload: comma list of qkv,o_proj,gate_up,down,lm_head (default all)")
    ap.add_argument("--ar-mode", default="auto", choices=["auto", "oneshot", "twoshot"],
                    help="fused all-reduce exchange (allreduce workload)")
    ap.add_argument("--workload", default="decode", choices=["decode", "attn", "gemm", "allreduce", "prefill"],
                    help="decode = the headline line; attn / gemm / prefill / allreduce = kernel microbenchmarks")
    args = ap.parse_args()
    if args.warmup < 3 and args.workload == "decode":
        ap.error("--warmup must be >= 3")
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if args.impl == "reference":
        run_reference_arm(args, rank, world)
        return
    if args.workload == "allreduce":
        run_allreduce_microbench(args, rank, world)
        return
    if args.workload != "decode":
        run_microbench(args)
        return
    run_b200(args, rank, world)


if __name__ == "__main__":
    main()
