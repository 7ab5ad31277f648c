"""Oracle for the tensor-parallel Qwen3 decoder forward path of nano-vllm-diy.

TEST INFRASTRUCTURE ONLY.  This package is a CPU restatement (torch on CPU,
fp32 arithmetic with bf16 rounding exactly where the reference rounds) of the
reference's algorithm for this path.  Only tests/, __graft_entry__.smoke()
and bench.py (its cpu_baseline leg and `--impl reference` arm) may import it,
and there only as the checker or as the timed CPU baseline; the product path
(nano-vllm-diy_b200/src) never imports it and has no CPU fallback.

Pinning: tests/golden/ holds vectors produced by running the reference's own
modules (src/layers/*, src/models/qwen3.py, ModelRunner.prepare_seqs, and the
Triton store_kvcache kernel under TRITON_INTERPRET=1) on CPU; the generating
script is tests/golden/make_golden.py.  flash-attn 2.8.3 cannot run on a CPU,
so the attention goldens come from torch's scaled_dot_product_attention on
the same paged/varlen inputs; the oracle's attention is an independent
restatement checked against them.

Modules:
  layers    per-op restatements (linear, RMSNorm, RoPE, SiLU-and-mul,
            store_kvcache, varlen/paged attention, vocab embedding, LM head)
  metadata  ModelRunner.prepare_seqs: slot_mapping, cu_seqlens, block tables
  model     Qwen3 forward composition with tensor-parallel simulation
  weights   seeded random-init weights under the reference's HF names
"""
