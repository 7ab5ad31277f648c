"""ctypes binding of libb200ops.so (the sm_100a kernels of the decoder path).

Every wrapper takes torch tensors, checks dtype / device / layout, passes raw
pointers plus the current CUDA stream to the C-ABI declared in
include/b200ops.h and raises RuntimeError on a non-zero status.  There is no
fallback: if the shared library is missing or a tensor is not on a CUDA
device, the call fails.

The decode-attention workspace (its scheduler counters and split-KV partials)
and the GEMM workspace (split-K flags and fp32 partials of the SM-pair GEMM)
are per-device torch buffers that grow on demand outside CUDA-graph capture
and are reused by every call.
"""
from __future__ import annotations

import ctypes
import os

import torch

_PKG = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
# B200_OPS_LIB points at the library when these modules are copied into
# another `src` tree (the reference checkout); default: the package's lib/
LIB_PATH = os.environ.get("B200_OPS_LIB") or os.path.join(_PKG, "lib", "libb200ops.so")

_lib = None

_c_void_p = ctypes.c_void_p
_ll = ctypes.c_longlong
_i = ctypes.c_int
_f = ctypes.c_float
_sz = ctypes.c_size_t

_SIGNATURES = {
    "b200_last_error": ([], ctypes.c_char_p),
    "b200_version": ([], _i),
    "b200_launch_count": ([], ctypes.c_ulonglong),
    "b200_device_error": ([ctypes.POINTER(ctypes.c_uint), _i], _i),
    "b200_linear_workspace_bytes": ([_i, _i, _i, ctypes.POINTER(_sz)], _i),
    "b200_gemm_schedule_check": ([ctypes.c_longlong, _i, _i, _i], _i),
    "b200_linear": ([_c_void_p, _ll, _c_void_p, _ll, _c_void_p, _c_void_p, _ll, _i, _i, _i,
                     _c_void_p, _sz, _c_void_p], _i),
    "b200_linear_silu_and_mul": ([_c_void_p, _ll, _c_void_p, _ll, _c_void_p, _ll, _i, _i, _i,
                                  _c_void_p, _sz, _c_void_p], _i),
    "b200_rmsnorm_linear": ([_c_void_p, _ll, _c_void_p, _c_void_p, _c_void_p, _f, _c_void_p, _ll,
                             _c_void_p, _ll, _c_void_p, _ll, _i, _i, _i, _i, _c_void_p, _sz,
                             _c_void_p], _i),
    "b200_linear_allreduce": ([_c_void_p, _ll, _c_void_p, _ll, _c_void_p, _i, _i, _i, _i, _i,
                               _c_void_p, _c_void_p, _c_void_p, _c_void_p, _ll, _ll, _ll, _i,
                               _c_void_p], _i),
    "b200_linear_allreduce_supported": ([_i, _i, _i, _i, _ll, _ll, _ll, ctypes.POINTER(_i)], _i),
    "b200_ipc_export": ([_c_void_p, _c_void_p, ctypes.POINTER(ctypes.c_ulonglong)], _i),
    "b200_ipc_import": ([_c_void_p, ctypes.c_ulonglong, ctypes.POINTER(_c_void_p)], _i),
    "b200_ipc_close": ([_c_void_p, ctypes.c_ulonglong], _i),
    "b200_rms_norm": ([_c_void_p, _ll, _c_void_p, _c_void_p, _c_void_p, _ll, _c_void_p, _i, _i,
                       _f, _c_void_p], _i),
    "b200_qk_norm_rope_store": ([_c_void_p, _ll, _c_void_p, _ll, _c_void_p, _ll, _i, _i, _i,
                                 _c_void_p, _c_void_p, _f, _c_void_p, _ll, _c_void_p, _c_void_p,
                                 _c_void_p, _c_void_p, _ll, _c_void_p, _c_void_p, _c_void_p,
                                 _c_void_p], _i),
    "b200_store_kvcache": ([_c_void_p, _ll, _c_void_p, _ll, _c_void_p, _c_void_p, _c_void_p, _i,
                            _i, _ll, _c_void_p], _i),
    "b200_silu_and_mul": ([_c_void_p, _ll, _c_void_p, _ll, _i, _i, _c_void_p], _i),
    "b200_embedding": ([_c_void_p, _c_void_p, _c_void_p, _i, _i, _ll, _ll, _c_void_p], _i),
    "b200_argmax": ([_c_void_p, _ll, _i, _i, _c_void_p, _c_void_p], _i),
    "b200_step_metadata": ([_c_void_p, _c_void_p, _i, _i, _i, _c_void_p, _c_void_p, _c_void_p,
                            _c_void_p, _c_void_p, _c_void_p], _i),
    "b200_embedding_exchange": ([_c_void_p, _c_void_p, _i, _i, _ll, _ll, _ll, _i, _i, _c_void_p, _ll,
                                 _c_void_p, _c_void_p, _c_void_p], _i),
    "b200_select_tokens_partial": ([_c_void_p, _ll, _i, _i, _ll, _c_void_p, _c_void_p, _ll,
                                    ctypes.c_ulonglong, ctypes.c_ulonglong, _c_void_p, _c_void_p], _i),
    "b200_select_tokens_exchange": ([_c_void_p, _i, _i, _i, _c_void_p, _c_void_p, _c_void_p, _ll,
                                     _c_void_p, _c_void_p], _i),
    "b200_attention_workspace_bytes": ([_i, _i, _i, ctypes.POINTER(_sz)], _i),
    "b200_paged_decode_attention_static": ([_c_void_p, _ll, _i, _c_void_p, _c_void_p, _ll,
                                            _c_void_p, _i, _i, _c_void_p, _c_void_p, _i, _i,
                                            _i, _i, _i, _f, _c_void_p, _ll, _c_void_p], _i),
    "b200_paged_attention": ([_c_void_p, _ll, _i, _c_void_p, _ll, _c_void_p, _ll, _c_void_p,
                              _c_void_p, _ll, _c_void_p, _i, _i, _c_void_p, _c_void_p, _i, _i, _i,
                              _i, _i, _i, _f, _c_void_p, _ll, _c_void_p, _sz, _c_void_p], _i),
}


def load_library(path: str = LIB_PATH) -> ctypes.CDLL:
    """Load libb200ops.so and declare its signatures (no CUDA calls)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(path):
        raise RuntimeError(f"{path} is missing: build it with `python __graft_entry__.py build` "
                           "(the decoder path has no CPU fallback)")
    lib = ctypes.CDLL(path)
    for name, (args, res) in _SIGNATURES.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = res
    _lib = lib
    return lib


def exported_symbols() -> list[str]:
    return sorted(_SIGNATURES)


def _check(rc: int, name: str) -> None:
    if rc != 0:
        msg = load_library().b200_last_error().decode(errors="replace")
        raise RuntimeError(f"{name} failed with status {rc}: {msg}")


def _p(t: torch.Tensor | None):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _cuda(*ts: torch.Tensor | None) -> None:
    for t in ts:
        if t is not None and not t.is_cuda:
            raise RuntimeError("b200 kernels need CUDA tensors (there is no CPU path)")


def _bf16(*ts: torch.Tensor | None) -> None:
    for t in ts:
        if t is not None and t.dtype != torch.bfloat16:
            raise TypeError(f"expected bfloat16, got {t.dtype}")


def _rows(t: torch.Tensor) -> tuple[int, int]:
    """(rows, row_stride) of a tensor whose last dim is contiguous and whose
    leading dims collapse into uniformly strided rows."""
    if t.stride(-1) != 1:
        raise ValueError("last dimension must be contiguous")
    if t.dim() == 1:
        return 1, t.shape[0]
    if t.dim() == 2:
        return t.shape[0], t.stride(0)
    lead = t.reshape(-1, t.shape[-1]) if t.is_contiguous() else None
    if lead is None:
        raise ValueError("tensor rows are not uniformly strided")
    return lead.shape[0], lead.stride(0)


# ---------------------------------------------------------------------------
# workspaces
# ---------------------------------------------------------------------------
_workspaces: dict[tuple[int, str], torch.Tensor] = {}


def workspace(kind: str, nbytes: int, device: torch.device) -> torch.Tensor:
    """Zero-filled on (re)allocation: both workspaces start with counters or
    flags that must be zero before the first call (every call leaves them
    zero)."""
    key = (device.index if device.index is not None else torch.cuda.current_device(), kind)
    buf = _workspaces.get(key)
    if buf is None or buf.numel() < nbytes:
        if torch.cuda.is_current_stream_capturing():
            raise RuntimeError(f"workspace '{kind}' must be sized before CUDA-graph capture "
                               f"({nbytes} bytes requested)")
        buf = torch.zeros(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
        _workspaces[key] = buf
    return buf


def reserve_workspace(kind: str, nbytes: int, device: torch.device) -> None:
    workspace(kind, nbytes, device)




def launch_count() -> int:
    """Kernels launched by libb200ops from the host so far."""
    return int(load_library().b200_launch_count())


# device error bits (include/b200ops.h): a bounded wait ran out
_TIMEOUT_BITS = 0x1 | 0x2
# the GEMM workspace starts with 4 KiB of split-K flags and counters
_GEMM_FLAG_BYTES = 4096


def device_error(clear: bool = True) -> int:
    """The device error word (synchronises the device).  With `clear`, it is
    reset; if a bounded wait ran out, the counters at the head of this
    device's attention and GEMM workspaces are zeroed too: a kernel that gave
    up waiting can leave counts that the next call would trust."""
    v = ctypes.c_uint(0)
    _check(load_library().b200_device_error(ctypes.byref(v), int(clear)), "b200_device_error")
    if clear and v.value & _TIMEOUT_BITS:
        dev = torch.cuda.current_device()
        heads = {"attn": attention_workspace_bytes(0, 0, 1), "gemm": _GEMM_FLAG_BYTES}
        for (d, kind), buf in _workspaces.items():
            if d == dev and kind in heads:
                buf[:heads[kind]].zero_()
        torch.cuda.synchronize()
    return v.value


# ---------------------------------------------------------------------------
# GEMMs
# ---------------------------------------------------------------------------
_gemm_ws_bytes: dict[int, int] = {}


def _gemm_workspace(device: torch.device) -> torch.Tensor:
    """The GEMM's split-K workspace of this device (zeroed on allocation,
    sized before any graph capture by the first eager call)."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    n = _gemm_ws_bytes.get(idx)
    if n is None:
        size = ctypes.c_size_t(0)
        _check(load_library().b200_linear_workspace_bytes(1, 1, 1, ctypes.byref(size)),
               "b200_linear_workspace_bytes")
        n = _gemm_ws_bytes[idx] = int(size.value)
    return workspace("gemm", n, device)


def linear(x: torch.Tensor, w: torch.Tensor, bias: torch.Tensor | None = None,
           out: torch.Tensor | None = None) -> torch.Tensor:
    """y = x @ w.T (+ bias); x [..., K], w [N, K] -> [..., N] (F.linear)."""
    lib = load_library()
    _cuda(x, w, bias)
    _bf16(x, w, bias)
    K = x.shape[-1]
    N = w.shape[0]
    if w.shape[1] != K:
        raise ValueError(f"linear: x has K={K}, weight is {tuple(w.shape)}")
    x2 = x.reshape(-1, K)
    if x2.stride(-1) != 1:
        x2 = x2.contiguous()
    T = x2.shape[0]
    if out is None:
        out = torch.empty(*x.shape[:-1], N, dtype=x.dtype, device=x.device)
    y2 = out.view(-1, N)
    if w.stride(-1) != 1:
        raise ValueError("linear: weight rows must be contiguous")
    ws = _gemm_workspace(x.device)
    _check(lib.b200_linear(_p(x2), x2.stride(0), _p(w), w.stride(0), _p(bias), _p(y2), y2.stride(0),
                           T, N, K, _p(ws), ws.numel(), _stream()), "b200_linear")
    return out


def linear_silu_and_mul(x: torch.Tensor, w: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """silu(x @ w[:I].T) * (x @ w[I:].T) with w = [gate ; up] of shape [2I, K]."""
    lib = load_library()
    _cuda(x, w)
    _bf16(x, w)
    K = x.shape[-1]
    I = w.shape[0] // 2
    x2 = x.reshape(-1, K)
    if x2.stride(-1) != 1:
        x2 = x2.contiguous()
    T = x2.shape[0]
    if I % 64:
        # the fused epilogue pairs 64-row gate / up blocks; other widths run
        # the GEMM and the activation as two kernels
        act = silu_and_mul(linear(x2, w))
        if out is None:
            return act.view(*x.shape[:-1], I)
        out.view(-1, I).copy_(act)
        return out
    if out is None:
        out = torch.empty(*x.shape[:-1], I, dtype=x.dtype, device=x.device)
    y2 = out.view(-1, I)
    ws = _gemm_workspace(x.device)
    _check(lib.b200_linear_silu_and_mul(_p(x2), x2.stride(0), _p(w), w.stride(0), _p(y2),
                                        y2.stride(0), T, I, K, _p(ws), ws.numel(), _stream()),
           "b200_linear_silu_and_mul")
    return out


def rmsnorm_linear(x: torch.Tensor, norm_weight: torch.Tensor, eps: float, w: torch.Tensor,
                   residual: torch.Tensor | None = None, silu: bool = False):
    """RMSNorm of x (+ residual) followed by the projection that consumes it:
    y = norm(x [+ residual]) @ w.T, or with silu=True the gate_up projection
    silu(n @ w[:I].T) * (n @ w[I:].T).  Returns y, or (y, x + residual) with a
    residual, as RMSNorm.forward then the linear layer would
    (src/models/qwen3.py:162-168).  The rms_norm kernel then the GEMM; with
    B200_FUSE_NORM=1 one launch where the GEMM runs on the persistent SM-pair
    kernel."""
    lib = load_library()
    _cuda(x, norm_weight, w, residual)
    _bf16(x, norm_weight, w, residual)
    K = x.shape[-1]
    N = w.shape[0]
    if w.shape[1] != K or norm_weight.shape != (K,):
        raise ValueError(f"rmsnorm_linear: x has K={K}, weight {tuple(w.shape)}, "
                         f"norm weight {tuple(norm_weight.shape)}")
    if w.stride(-1) != 1:
        raise ValueError("rmsnorm_linear: weight rows must be contiguous")
    if silu and (N % 2 or (N // 2) % 64):
        # widths the fused SiLU epilogue does not pair: two steps
        if residual is None:
            return linear_silu_and_mul(rms_norm(x, norm_weight, eps), w)
        n, r = rms_norm(x, norm_weight, eps, residual=residual)
        return linear_silu_and_mul(n, w), r
    x2 = x.reshape(-1, K)
    if x2.stride(-1) != 1:
        x2 = x2.contiguous()
    T = x2.shape[0]
    res_out = None
    if residual is not None:
        if residual.shape != x.shape:
            raise ValueError(f"rmsnorm_linear: residual {tuple(residual.shape)}, x {tuple(x.shape)}")
        residual = residual.reshape(-1, K).contiguous()
        res_out = torch.empty(T, K, dtype=x.dtype, device=x.device)
    xn = torch.empty(T, K, dtype=x.dtype, device=x.device)
    width = N // 2 if silu else N
    y = torch.empty(T, width, dtype=x.dtype, device=x.device)
    ws = _gemm_workspace(x.device)
    _check(lib.b200_rmsnorm_linear(_p(x2), x2.stride(0), _p(residual), _p(res_out), _p(norm_weight),
                                   float(eps), _p(xn), xn.stride(0), _p(w), w.stride(0), _p(y), y.stride(0),
                                   T, N, K, int(silu), _p(ws), ws.numel(), _stream()),
           "b200_rmsnorm_linear")
    y = y.view(*x.shape[:-1], width)
    if residual is None:
        return y
    return y, res_out.view(x.shape)


ERR_UNSUPPORTED = -2


def ipc_export(t: torch.Tensor) -> tuple[bytes, int]:
    """(64-byte CUDA IPC handle of the allocation holding t, offset of t in it)."""
    h = ctypes.create_string_buffer(64)
    off = ctypes.c_ulonglong(0)
    _check(load_library().b200_ipc_export(_p(t), h, ctypes.byref(off)), "b200_ipc_export")
    return h.raw, off.value


def ipc_import(handle: bytes, offset: int) -> int:
    """Device address, in this process, of a peer's exported buffer."""
    ptr = ctypes.c_void_p()
    _check(load_library().b200_ipc_import(handle, offset, ctypes.byref(ptr)), "b200_ipc_import")
    return ptr.value


def ipc_close(ptr: int, offset: int) -> None:
    _check(load_library().b200_ipc_close(ctypes.c_void_p(ptr), offset), "b200_ipc_close")


def linear_allreduce_supported(T: int, N: int, K: int, world: int, stage_rows: int, ldo: int,
                               max_positions: int) -> bool:
    """Whether the fused GEMM + all-reduce would launch this shape (no launch)."""
    ok = ctypes.c_int(0)
    _check(load_library().b200_linear_allreduce_supported(T, N, K, world, stage_rows, ldo,
                                                          max_positions, ctypes.byref(ok)),
           "b200_linear_allreduce_supported")
    return bool(ok.value)


def linear_allreduce(x: torch.Tensor, w: torch.Tensor, bias: torch.Tensor | None, rank: int,
                     world: int, stage: list[int], out: list[int], flags: list[int],
                     done: list[int], stage_rows: int, ldo: int, max_positions: int,
                     one_shot: bool = False) -> int:
    """Fused GEMM + all-reduce; returns the C status (0, or ERR_UNSUPPORTED when
    the caller must fall back) and raises on any other failure."""
    lib = load_library()
    _cuda(x, w, bias)
    _bf16(x, w, bias)
    K = x.shape[-1]
    x2 = x.reshape(-1, K)
    if x2.stride(-1) != 1:
        x2 = x2.contiguous()
    arr = ctypes.c_void_p * world
    rc = lib.b200_linear_allreduce(_p(x2), x2.stride(0), _p(w), w.stride(0), _p(bias), x2.shape[0],
                                   w.shape[0], K, rank, world, arr(*stage), arr(*out), arr(*flags),
                                   arr(*done), stage_rows, ldo, max_positions, int(one_shot),
                                   _stream())
    if rc not in (0, ERR_UNSUPPORTED):
        _check(rc, "b200_linear_allreduce")
    return rc


# ---------------------------------------------------------------------------
# norms / rope / activation
# ---------------------------------------------------------------------------
def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float,
             residual: torch.Tensor | None = None,
             out: torch.Tensor | None = None,
             residual_out: torch.Tensor | None = None):
    """RMSNorm over the last dim; with `residual` returns (norm(x + r), x + r)."""
    lib = load_library()
    _cuda(x, weight, residual)
    _bf16(x, weight, residual)
    dim = x.shape[-1]
    try:
        rows, xs = _rows(x)
    except ValueError:
        x = x.contiguous()
        rows, xs = _rows(x)
    # the kernel indexes out, residual and residual_out as contiguous rows of
    # `dim` elements: anything else would be read or written out of bounds
    if weight.shape != (dim,):
        raise ValueError(f"rms_norm: weight {tuple(weight.shape)} for rows of {dim}")
    for name, t in (("out", out), ("residual", residual), ("residual_out", residual_out)):
        if t is not None and t.shape != x.shape:
            raise ValueError(f"rms_norm: {name} has shape {tuple(t.shape)}, x has {tuple(x.shape)}")
    for name, t in (("out", out), ("residual_out", residual_out)):
        if t is not None and not t.is_contiguous():
            raise ValueError(f"rms_norm: {name} must be contiguous")
    _cuda(out, residual_out)
    _bf16(out, residual_out)
    if out is None:
        out = torch.empty(x.shape, dtype=x.dtype, device=x.device)
    if residual is not None:
        residual = residual.contiguous()
        if residual_out is None:
            residual_out = torch.empty(x.shape, dtype=x.dtype, device=x.device)
    _check(lib.b200_rms_norm(_p(x), xs, _p(residual), _p(weight), _p(out), dim, _p(residual_out),
                             rows, dim, float(eps), _stream()), "b200_rms_norm")
    return out if residual is None else (out, residual_out)


def qk_norm_rope_store(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor | None,
                       q_norm_w: torch.Tensor | None, k_norm_w: torch.Tensor | None, eps: float,
                       cos_sin: torch.Tensor, positions: torch.Tensor,
                       slot_mapping: torch.Tensor | None = None,
                       k_cache: torch.Tensor | None = None, v_cache: torch.Tensor | None = None,
                       need_kv_out: bool = True):
    """q [T, Hq, 128], k/v [T, Hkv, 128] (views into the qkv projection are
    fine) -> (q_out, k_out, v_out); K/V are also written to the cache."""
    lib = load_library()
    _cuda(q, k, v, cos_sin, positions)
    _bf16(q, k, v)
    T, Hq, D = q.shape
    Hkv = k.shape[1]
    if D != 128 or k.shape[2] != 128:
        raise ValueError("head_dim must be 128")
    for t in (q, k, v):
        if t is not None and (t.stride(-1) != 1 or t.stride(-2) != 128):
            raise ValueError("heads must be contiguous 128-element rows")
    if positions.dtype != torch.int64 or cos_sin.dtype != torch.float32:
        raise TypeError("positions must be int64 and cos_sin float32")
    q_out = torch.empty(T, Hq, 128, dtype=q.dtype, device=q.device)
    k_out = torch.empty(T, Hkv, 128, dtype=q.dtype, device=q.device) if need_kv_out else None
    v_out = torch.empty(T, Hkv, 128, dtype=q.dtype, device=q.device) if (need_kv_out and v is not None) else None
    store = k_cache is not None and k_cache.numel() > 0
    if store:
        if slot_mapping is None or slot_mapping.dtype != torch.int32:
            raise TypeError("slot_mapping must be int32")
        num_slots = k_cache.numel() // (Hkv * 128)
    else:
        num_slots = 0
    cs = cos_sin.reshape(cos_sin.shape[0], -1)
    _check(lib.b200_qk_norm_rope_store(
        _p(q), q.stride(0), _p(k), k.stride(0), _p(v), v.stride(0) if v is not None else 0,
        T, Hq, Hkv, _p(q_norm_w), _p(k_norm_w), float(eps), _p(cs), cs.shape[0], _p(positions),
        _p(slot_mapping) if store else None, _p(k_cache) if store else None,
        _p(v_cache) if store else None, num_slots, _p(q_out), _p(k_out), _p(v_out), _stream()),
        "b200_qk_norm_rope_store")
    return q_out, k_out, v_out


def silu_and_mul(x: torch.Tensor) -> torch.Tensor:
    lib = load_library()
    _cuda(x)
    _bf16(x)
    I = x.shape[-1] // 2
    x2 = x.reshape(-1, x.shape[-1])
    if x2.stride(-1) != 1:
        x2 = x2.contiguous()
    out = torch.empty(*x.shape[:-1], I, dtype=x.dtype, device=x.device)
    o2 = out.view(-1, I)
    _check(lib.b200_silu_and_mul(_p(x2), x2.stride(0), _p(o2), o2.stride(0), x2.shape[0], I,
                                 _stream()), "b200_silu_and_mul")
    return out


# ---------------------------------------------------------------------------
# KV cache, attention
# ---------------------------------------------------------------------------
def store_kvcache(key: torch.Tensor, value: torch.Tensor, k_cache: torch.Tensor,
                  v_cache: torch.Tensor, slot_mapping: torch.Tensor) -> None:
    lib = load_library()
    _cuda(key, value, k_cache, v_cache, slot_mapping)
    _bf16(key, value, k_cache, v_cache)
    T, Hkv, D = key.shape
    Dt = Hkv * D
    # layout contract of src/layers/attention.py:51-56
    assert key.stride(-1) == 1 and value.stride(-1) == 1
    assert key.stride(1) == D and value.stride(1) == D
    assert k_cache.stride(1) == Dt and v_cache.stride(1) == Dt
    assert slot_mapping.numel() == T
    if slot_mapping.dtype != torch.int32:
        raise TypeError("slot_mapping must be int32")
    num_slots = k_cache.shape[0] * k_cache.shape[1]
    _check(lib.b200_store_kvcache(_p(key), key.stride(0), _p(value), value.stride(0), _p(k_cache),
                                  _p(v_cache), _p(slot_mapping), T, Dt, num_slots, _stream()),
           "b200_store_kvcache")


def attention_workspace_bytes(max_seqs: int, max_seqlen_k: int, num_heads: int) -> int:
    n = ctypes.c_size_t(0)
    _check(load_library().b200_attention_workspace_bytes(max_seqs, max_seqlen_k, num_heads,
                                                         ctypes.byref(n)),
           "b200_attention_workspace_bytes")
    return n.value


def paged_attention(q: torch.Tensor, k: torch.Tensor | None, v: torch.Tensor | None,
                    k_cache: torch.Tensor | None, v_cache: torch.Tensor | None,
                    cu_seqlens_q: torch.Tensor, cu_seqlens_k: torch.Tensor, max_seqlen_q: int,
                    max_seqlen_k: int, softmax_scale: float,
                    block_table: torch.Tensor | None = None,
                    out: torch.Tensor | None = None) -> torch.Tensor:
    """flash_attn_varlen_func(q, k, v, cu_q, cu_k, max_q, max_k, scale,
    causal=True, block_table) with head_dim 128."""
    lib = load_library()
    _cuda(q, k, v, k_cache, v_cache, cu_seqlens_q, cu_seqlens_k, block_table)
    T, Hq, D = q.shape
    if D != 128:
        raise ValueError("head_dim must be 128")
    if q.stride(-1) != 1 or q.stride(1) != 128:
        q = q.contiguous()
    B = cu_seqlens_q.numel() - 1
    if out is None:
        out = torch.empty(T, Hq, 128, dtype=q.dtype, device=q.device)
    if block_table is not None:
        Hkv = k_cache.shape[2]
        page = k_cache.shape[1]
        num_slots = k_cache.shape[0] * page
        if block_table.dtype != torch.int32 or block_table.stride(-1) != 1:
            raise TypeError("block_table must be int32 with contiguous rows")
        bt_stride = block_table.stride(0)
        bt_width = block_table.shape[1]
        k_arg = v_arg = None
        ks = vs = 0
    else:
        Hkv = k.shape[1]
        page = 0
        num_slots = 0
        bt_stride = 0
        bt_width = 0
        k_arg, v_arg = k, v
        if k.stride(-1) != 1 or k.stride(1) != 128:
            k_arg = k.contiguous()
        if v.stride(-1) != 1 or v.stride(1) != 128:
            v_arg = v.contiguous()
        ks, vs = k_arg.stride(0), v_arg.stride(0)
    ws = None
    nbytes = 0
    if max_seqlen_q == 1 and block_table is not None:
        nbytes = attention_workspace_bytes(B, max_seqlen_k, Hq)
        ws = workspace("attn", nbytes, q.device)
        nbytes = ws.numel()
    _check(lib.b200_paged_attention(
        _p(q), q.stride(0), T, _p(k_arg), ks, _p(v_arg), vs,
        _p(k_cache) if block_table is not None else None,
        _p(v_cache) if block_table is not None else None, num_slots, _p(block_table), bt_stride, bt_width,
        _p(cu_seqlens_q), _p(cu_seqlens_k), B, int(max_seqlen_q), int(max_seqlen_k), Hq, Hkv, page,
        float(softmax_scale), _p(out), out.stride(0), _p(ws), nbytes, _stream()),
        "b200_paged_attention")
    return out


# ---------------------------------------------------------------------------
# vocabulary
# ---------------------------------------------------------------------------
def embedding(ids: torch.Tensor, weight: torch.Tensor, vocab_start: int, vocab_end: int) -> torch.Tensor:
    lib = load_library()
    _cuda(ids, weight)
    if ids.dtype != torch.int64:
        ids = ids.to(torch.int64)
    ids = ids.contiguous()
    T = ids.numel()
    H = weight.shape[1]
    out = torch.empty(T, H, dtype=weight.dtype, device=weight.device)
    _check(lib.b200_embedding(_p(ids), _p(weight), _p(out), T, H, int(vocab_start), int(vocab_end),
                              _stream()), "b200_embedding")
    return out.view(*ids.shape, H)


def argmax(logits: torch.Tensor) -> torch.Tensor:
    lib = load_library()
    _cuda(logits)
    _bf16(logits)
    if logits.stride(-1) != 1:
        logits = logits.contiguous()
    rows, V = logits.shape
    out = torch.empty(rows, dtype=torch.int64, device=logits.device)
    _check(lib.b200_argmax(_p(logits), logits.stride(0), rows, V, _p(out), _stream()), "b200_argmax")
    return out


# ---------------------------------------------------------------------------
# vocabulary-parallel token selection and embedding exchange
# ---------------------------------------------------------------------------
def select_tokens(logits: torch.Tensor, vocab_start: int = 0,
                  temperatures: torch.Tensor | None = None, noise: torch.Tensor | None = None,
                  seed: int = 0, offset: int = 0) -> torch.Tensor:
    """Packed (score, global index) key of each row's best column of this
    vocabulary shard: greedy without `temperatures`, else the Gumbel-max form
    of src/layers/sampler.py:4-17 (Exp(1) draws from `noise`, or Philox keyed
    by seed / offset).  int64 [rows]."""
    lib = load_library()
    _cuda(logits, temperatures, noise)
    _bf16(logits)
    if logits.stride(-1) != 1:
        logits = logits.contiguous()
    rows, V = logits.shape
    if temperatures is not None:
        if temperatures.dtype != torch.float32 or temperatures.shape != (rows,):
            raise TypeError("temperatures must be float32 [rows]")
        temperatures = temperatures.contiguous()
    if noise is not None:
        if noise.dtype != torch.float32 or noise.shape != (rows, V) or noise.stride(-1) != 1:
            raise TypeError("noise must be float32 [rows, V] with contiguous rows")
    keys = torch.empty(rows, dtype=torch.int64, device=logits.device)
    _check(lib.b200_select_tokens_partial(_p(logits), logits.stride(0), rows, V, int(vocab_start),
                                          _p(temperatures), _p(noise),
                                          noise.stride(0) if noise is not None else 0,
                                          int(seed) & (2 ** 64 - 1), int(offset) & (2 ** 64 - 1),
                                          _p(keys), _stream()), "b200_select_tokens_partial")
    return keys


def tokens_from_keys(keys: torch.Tensor, rank: int = 0, world: int = 1,
                     key_slots: list[int] | None = None, flags: list[int] | None = None,
                     state: int | None = None, max_rows: int = 0,
                     out: torch.Tensor | None = None) -> torch.Tensor:
    """Tokens int64 [rows]: the maximum key of each row over the ranks (the
    exchange needs the symmetric buffers at world > 1)."""
    lib = load_library()
    _cuda(keys)
    rows = keys.numel()
    if out is None:
        out = torch.empty(rows, dtype=torch.int64, device=keys.device)
    arr = ctypes.c_void_p * max(world, 1)
    ks = arr(*key_slots) if key_slots else None
    fl = arr(*flags) if flags else None
    _check(lib.b200_select_tokens_exchange(_p(keys), rows, rank, world, ks, fl,
                                           ctypes.c_void_p(state) if state else None, max_rows,
                                           _p(out), _stream()), "b200_select_tokens_exchange")
    return out


def embedding_exchange(ids: torch.Tensor, weight: torch.Tensor, vocab_start: int, vocab_end: int,
                       vocab_size: int, rank: int, world: int, outs: list[int], ld_out: int,
                       flags: list[int] | None, state: int | None) -> None:
    """Rows of `ids` from every rank's vocabulary shard into outs[rank] of
    every rank (src/layers/llm_head.py:38-49 with its all-reduce)."""
    lib = load_library()
    _cuda(ids, weight)
    _bf16(weight)
    if ids.dtype != torch.int64:
        ids = ids.to(torch.int64)
    ids = ids.contiguous()
    arr = ctypes.c_void_p * world
    _check(lib.b200_embedding_exchange(_p(ids), _p(weight), ids.numel(), weight.shape[1],
                                       int(vocab_start), int(vocab_end), int(vocab_size), rank, world,
                                       arr(*outs), ld_out, arr(*flags) if flags else None,
                                       ctypes.c_void_p(state) if state else None, _stream()),
           "b200_embedding_exchange")


# ---------------------------------------------------------------------------
# step metadata
# ---------------------------------------------------------------------------
def step_metadata(seq_info: torch.Tensor, block_tables: torch.Tensor | None, page: int,
                  num_tokens: int, num_slot_tokens: int):
    """(positions int64 [T], slot_mapping int32 [slot tokens], cu_seqlens_q,
    cu_seqlens_k int32 [B + 1], context_lens int32 [B]) from the per-sequence
    int32 [3, B] (start, query length, block-table length) and the -1-padded
    block tables (src/engine/model_runner.py:174-233 expanded on the device)."""
    lib = load_library()
    _cuda(seq_info, block_tables)
    if seq_info.dtype != torch.int32 or seq_info.dim() != 2 or seq_info.shape[0] != 3:
        raise TypeError("seq_info must be int32 [3, B]")
    seq_info = seq_info.contiguous()
    B = seq_info.shape[1]
    dev = seq_info.device
    positions = torch.empty(num_tokens, dtype=torch.int64, device=dev)
    slots = torch.empty(num_slot_tokens, dtype=torch.int32, device=dev)
    cu_q = torch.empty(B + 1, dtype=torch.int32, device=dev)
    cu_k = torch.empty(B + 1, dtype=torch.int32, device=dev)
    ctx_lens = torch.empty(B, dtype=torch.int32, device=dev)
    if block_tables is not None:
        if block_tables.dtype != torch.int32 or block_tables.stride(-1) != 1:
            raise TypeError("block_tables must be int32 with contiguous rows")
    _check(lib.b200_step_metadata(_p(seq_info), _p(block_tables),
                                  block_tables.stride(0) if block_tables is not None else 0, B, page,
                                  _p(positions), _p(slots), _p(cu_q), _p(cu_k), _p(ctx_lens), _stream()),
           "b200_step_metadata")
    return positions, slots, cu_q, cu_k, ctx_lens
