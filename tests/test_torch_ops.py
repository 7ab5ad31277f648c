"""torch.ops.b200.*: the library's ops registered as torch.library custom ops.

CPU only: registration, output shapes and dtypes from the fake implementations
(FakeTensor mode, as torch.compile / torch.export trace them), and no CPU
implementation (the real ops run on CUDA tensors only).
"""
import pytest
import torch
from torch._subclasses.fake_tensor import FakeTensorMode

BF = torch.bfloat16


def test_every_op_is_registered():
    from src import torch_ops
    for name in torch_ops.OPS:
        assert hasattr(torch.ops.b200, name), name


def test_fake_shapes_and_dtypes():
    from src import torch_ops  # noqa: F401  (registers the ops)
    ops = torch.ops.b200
    with FakeTensorMode():
        dev = "cuda"
        x = torch.empty(7, 1024, dtype=BF, device=dev)
        assert ops.linear(x, torch.empty(4096, 1024, dtype=BF, device=dev)).shape == (7, 4096)
        assert ops.linear_silu_and_mul(x, torch.empty(6144, 1024, dtype=BF, device=dev)).shape == (7, 3072)
        wn = torch.empty(1024, dtype=BF, device=dev)
        assert ops.rms_norm(x, wn, 1e-6).shape == (7, 1024)
        y, r = ops.rms_norm_residual(x, x, wn, 1e-6)
        assert y.shape == r.shape == (7, 1024) and y.dtype == r.dtype == BF
        assert ops.silu_and_mul(torch.empty(7, 6144, dtype=BF, device=dev)).shape == (7, 3072)
        q = torch.empty(7, 32, 128, dtype=BF, device=dev)
        k = torch.empty(7, 8, 128, dtype=BF, device=dev)
        v = torch.empty(7, 8, 128, dtype=BF, device=dev)
        kc = torch.empty(4, 256, 8, 128, dtype=BF, device=dev)
        vc = torch.empty(4, 256, 8, 128, dtype=BF, device=dev)
        slots = torch.empty(7, dtype=torch.int32, device=dev)
        assert ops.store_kvcache(k, v, kc, vc, slots) is None
        qw = torch.empty(128, dtype=BF, device=dev)
        cs = torch.empty(4096, 1, 128, dtype=torch.float32, device=dev)
        pos = torch.empty(7, dtype=torch.int64, device=dev)
        qo, ko, vo = ops.qk_norm_rope_store(q, k, v, qw, qw, 1e-6, cs, pos, slots, kc, vc)
        assert qo.shape == q.shape and ko.shape == k.shape and vo.shape == v.shape
        cu_q = torch.empty(8, dtype=torch.int32, device=dev)
        cu_k = torch.empty(8, dtype=torch.int32, device=dev)
        bt = torch.empty(7, 4, dtype=torch.int32, device=dev)
        o = ops.paged_attention(q, None, None, kc, vc, cu_q, cu_k, 1, 1024, 128 ** -0.5, bt)
        assert o.shape == q.shape and o.dtype == BF
        ids = torch.empty(7, dtype=torch.int64, device=dev)
        emb = ops.embedding(ids, torch.empty(151936, 1024, dtype=BF, device=dev), 0, 151936)
        assert emb.shape == (7, 1024)
        am = ops.argmax(torch.empty(7, 151936, dtype=BF, device=dev))
        assert am.shape == (7,) and am.dtype == torch.int64


def test_no_cpu_implementation():
    from src import torch_ops  # noqa: F401
    with pytest.raises(NotImplementedError):
        torch.ops.b200.linear(torch.empty(2, 8, dtype=BF), torch.empty(4, 8, dtype=BF))


@pytest.mark.gpu
def test_custom_ops_run_the_same_kernels():
    """On a GPU the registered ops give exactly what the direct binding gives."""
    from src import b200, torch_ops  # noqa: F401
    g = torch.Generator().manual_seed(5)
    x = torch.randn(37, 512, generator=g).to(BF).cuda()
    w = (torch.randn(640, 512, generator=g) * 0.02).to(BF).cuda()
    assert torch.equal(torch.ops.b200.linear(x, w), b200.linear(x, w))
    logits = torch.randn(5, 1000, generator=g).to(BF).cuda()
    assert torch.equal(torch.ops.b200.argmax(logits), b200.argmax(logits))
