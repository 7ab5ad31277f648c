"""libb200ops.so: loads without a GPU and exports every function that
include/b200ops.h declares (CPU only, no compute calls)."""
import ctypes
import os
import re

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def header_functions():
    with open(os.path.join(REPO, "include", "b200ops.h")) as f:
        text = f.read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(b200_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_function():
    from src import b200
    lib = b200.load_library()
    names = header_functions()
    assert len(names) >= 15
    for name in names:
        assert hasattr(lib, name), name


def test_python_binding_covers_the_header():
    from src import b200
    assert set(b200.exported_symbols()) == set(header_functions())


def test_version_and_error_string():
    from src import b200
    lib = b200.load_library()
    assert lib.b200_version() == 1
    assert isinstance(lib.b200_last_error(), bytes)


def test_invalid_arguments_fail_before_any_launch():
    """Shape / alignment validation happens on the host: no CUDA call needed."""
    from src import b200
    lib = b200.load_library()
    # K not a multiple of 8
    rc = lib.b200_linear(ctypes.c_void_p(16), 12, ctypes.c_void_p(16), 12, None,
                         ctypes.c_void_p(16), 16, 4, 16, 12, None, 0, None)
    assert rc == -1
    assert b"multiples of 8" in lib.b200_last_error()
    # rms_norm dim not a multiple of 8
    rc = lib.b200_rms_norm(ctypes.c_void_p(16), 12, None, ctypes.c_void_p(16), ctypes.c_void_p(16),
                           12, None, 1, 12, 1e-6, None)
    assert rc == -2
    # token selection: the vocabulary start must leave room for 32-bit indices
    rc = lib.b200_select_tokens_partial(ctypes.c_void_p(16), 100, 2, 100, 1 << 33, None, None, 0,
                                        0, 0, ctypes.c_void_p(16), None)
    assert rc == -1
    # the keys exchange needs the peers' key slots at world > 1, and rows <= max_rows
    rc = lib.b200_select_tokens_exchange(ctypes.c_void_p(16), 4, 0, 2, None, None, None, 4,
                                         ctypes.c_void_p(16), None)
    assert rc == -1
    # the embedding exchange needs 8-element rows
    rc = lib.b200_embedding_exchange(ctypes.c_void_p(16), ctypes.c_void_p(16), 4, 12, 0, 10, 10, 0, 1,
                                     (ctypes.c_void_p * 1)(16), 12, None, None, None)
    assert rc == -1
    # step metadata: a block table needs a slot mapping output, pages are positive
    rc = lib.b200_step_metadata(ctypes.c_void_p(16), None, 0, 4, 0, ctypes.c_void_p(16), None,
                                ctypes.c_void_p(16), ctypes.c_void_p(16), ctypes.c_void_p(16), None)
    assert rc == -1
    # RMSNorm + projection: the norm width (K) must be a multiple of 8, and a
    # residual needs somewhere to write the sum
    rc = lib.b200_rmsnorm_linear(ctypes.c_void_p(16), 12, None, None, ctypes.c_void_p(16), 1e-6,
                                 ctypes.c_void_p(16), 12, ctypes.c_void_p(16), 12, ctypes.c_void_p(16),
                                 16, 4, 16, 12, 0, None, 0, None)
    assert rc == -1
    rc = lib.b200_rmsnorm_linear(ctypes.c_void_p(16), 16, ctypes.c_void_p(16), None,
                                 ctypes.c_void_p(16), 1e-6, ctypes.c_void_p(16), 16, ctypes.c_void_p(16),
                                 16, ctypes.c_void_p(16), 16, 4, 16, 16, 0, None, 0, None)
    assert rc == -1 and b"residual_out" in lib.b200_last_error()
    # the fused all-reduce's plan query rejects a bad shape without a device call
    ok = ctypes.c_int(7)
    rc = lib.b200_linear_allreduce_supported(256, 4100, 4096, 2, 512, 4096, 4096, ctypes.byref(ok))
    assert rc == -1 and ok.value == 0


def test_gemm_schedule_partitions_the_work():
    """The SM-pair GEMM's work split (grouped split-K and stream-K), walked on
    the host with the kernel's own segment iterator: every (tile, K block)
    unit exactly once, groups of consecutive pairs, flags inside the flag
    area.  Covers the Qwen3-8B decode shapes at every TP (tiles 3..594, 64 or
    192 K blocks over 74 pairs) and forced pair counts."""
    from src import b200
    lib = b200.load_library()
    cases = 0
    for tiles in (1, 2, 3, 6, 12, 16, 23, 24, 37, 38, 48, 73, 74, 75, 96, 149, 297, 594):
        for num_kb in (1, 2, 3, 7, 16, 64, 192):
            for max_pairs in (1, 3, 17, 64, 74):
                for grouped in (0, 1):
                    bad = lib.b200_gemm_schedule_check(tiles, num_kb, max_pairs, grouped)
                    assert bad == 0, (tiles, num_kb, max_pairs, grouped, bad)
                    cases += 1
    assert cases > 1000
    assert lib.b200_gemm_schedule_check(0, 64, 74, 1) < 0


def test_every_python_op_refuses_cpu_tensors():
    """The product path has no CPU fallback: each op of the binding raises on
    CPU tensors before it reaches the library (no launch, no silent torch
    substitute)."""
    import pytest
    import torch
    from src import b200
    bf = torch.bfloat16
    x = torch.zeros(4, 64, dtype=bf)
    w = torch.zeros(128, 64, dtype=bf)
    q = torch.zeros(4, 2, 128, dtype=bf)
    kv = torch.zeros(4, 1, 128, dtype=bf)
    cache = torch.zeros(2, 256, 1, 128, dtype=bf)
    i32 = torch.zeros(5, dtype=torch.int32)
    calls = [
        lambda: b200.linear(x, w),
        lambda: b200.linear_silu_and_mul(x, w),
        lambda: b200.rms_norm(x, torch.zeros(64, dtype=bf), 1e-6),
        lambda: b200.silu_and_mul(x),
        lambda: b200.store_kvcache(kv, kv, cache, cache, torch.zeros(4, dtype=torch.int32)),
        lambda: b200.qk_norm_rope_store(q, kv, kv, None, None, 1e-6, torch.zeros(16, 128),
                                        torch.zeros(4, dtype=torch.int64)),
        lambda: b200.paged_attention(q, kv, kv, None, None, i32, i32, 1, 4, 0.1),
        lambda: b200.embedding(torch.zeros(4, dtype=torch.int64), w, 0, 128),
        lambda: b200.argmax(x),
        lambda: b200.select_tokens(x),
        lambda: b200.tokens_from_keys(torch.zeros(4, dtype=torch.int64)),
        lambda: b200.embedding_exchange(torch.zeros(4, dtype=torch.int64), w, 0, 128, 128, 0, 1,
                                        [0], 64, None, None),
        lambda: b200.step_metadata(torch.zeros(3, 4, dtype=torch.int32), None, 256, 4, 0),
    ]
    for call in calls:
        with pytest.raises(RuntimeError, match="CUDA tensors"):
            call()
