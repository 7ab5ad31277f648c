"""B200-native (sm_100a) tensor-parallel Qwen3 decoder forward path.

Mirrors the `src` package layout of nano-vllm-diy (src.layers, src.models,
src.utils.context) so the reference's engine can drive these modules; the
kernels live in nano-vllm-diy_b200/lib/libb200ops.so (C-ABI:
include/b200ops.h), bound by src.b200.
"""
