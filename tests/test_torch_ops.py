"""The custom-operator boundary (torch.library): registration and the fake
implementations that graph capture traces through, checked on the CPU with fake
CUDA tensors (no kernel runs)."""
import torch
from torch._subclasses.fake_tensor import FakeTensorMode

import mosaic_b200.torch_ops  # noqa: F401  (registers the ops)


def test_ops_registered():
    assert hasattr(torch.ops.mosaic_b200, "attn_func")
    assert hasattr(torch.ops.mosaic_b200, "sparse_attn")


def test_fake_attn_func_shapes():
    with FakeTensorMode():
        for dt in (torch.bfloat16, torch.float16, torch.float32):
            q = torch.empty(2, 3072, 8, 64, dtype=dt, device="cuda")
            k = torch.empty(2, 3072, 2, 64, dtype=dt, device="cuda")
            w = torch.empty(3, 2, 3072, 8, 1, dtype=dt, device="cuda")
            o = torch.ops.mosaic_b200.attn_func(q, k, k, w, 1024, 64, 8, False, False)
            assert o.shape == q.shape and o.dtype == dt and o.device.type == "cuda"
            o = torch.ops.mosaic_b200.attn_func(q, k, k, None, 1024, 64, 8, True, False)
            assert o.shape == q.shape


def test_fake_sparse_attn_shapes():
    with FakeTensorMode():
        q = torch.empty(1, 768, 12, 64, dtype=torch.bfloat16, device="cuda")
        k = torch.empty(1, 768, 3, 64, dtype=torch.bfloat16, device="cuda")
        idx = torch.empty(1, 12, 3, 4, dtype=torch.int64, device="cuda")
        o = torch.ops.mosaic_b200.sparse_attn(q, k, k, idx, 64, 0.125)
        assert o.shape == q.shape and o.dtype == q.dtype


def test_fake_sparse_attn_training_ops():
    assert hasattr(torch.ops.mosaic_b200, "sparse_attn_fwd")
    assert hasattr(torch.ops.mosaic_b200, "sparse_attn_bwd")
    with FakeTensorMode():
        q = torch.empty(2, 1024, 8, 64, dtype=torch.bfloat16, device="cuda")
        k = torch.empty(2, 1024, 2, 64, dtype=torch.bfloat16, device="cuda")
        idx = torch.empty(2, 16, 2, 3, dtype=torch.int64, device="cuda")
        o, lse = torch.ops.mosaic_b200.sparse_attn_fwd(q, k, k, idx, 64, 0.125)
        assert o.shape == q.shape and o.dtype == q.dtype
        assert lse.shape == (2, 1024, 8) and lse.dtype == torch.float32
        dq, dk, dv = torch.ops.mosaic_b200.sparse_attn_bwd(q, k, k, o, lse, o, idx, 64, 0.125)
        assert dq.shape == q.shape and dk.shape == k.shape and dv.shape == k.shape
        assert dq.dtype == dk.dtype == torch.bfloat16
