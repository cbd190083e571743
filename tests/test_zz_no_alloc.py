"""mosaic_bsa_fwd_noalloc: the forward for callers that cannot allocate device
memory (a foreign-language host with no device allocator, or a service with a
fixed memory budget that must not call cudaMalloc per request). It keeps its
scratch in an 8 MiB array inside the library instead of a caller workspace.

Checked through the C ABI against mosaic_bsa_fwd (the workspace entry point) on
two calls in a row with different inputs, so that scratch left over from the
first call cannot leak into the second. This file is collected last on purpose.
"""
import ctypes

import pytest
import torch

from mosaic_b200 import _lib

MAX_ABS, MEAN_ABS = 2e-2, 2e-3  # the tolerance of the other parity tests


def _args(q, k, v, w, out, idx, ws=None, B=1, N=49152, Hq=12, Hk=3, bas=1024, bs=64, K=24):
    a = _lib.MosaicBsaArgs()
    a.q, a.k, a.v = q.data_ptr(), k.data_ptr(), v.data_ptr()
    a.gates = w.data_ptr()
    a.out = out.data_ptr()
    a.block_indices = idx.data_ptr()
    a.workspace = ws.data_ptr() if ws is not None else None
    a.workspace_bytes = ws.numel() if ws is not None else 0
    a.batch, a.seq_len, a.num_q_heads, a.num_kv_heads, a.head_dim = B, N, Hq, Hk, 64
    a.block_attn_size, a.sparse_block_size, a.sparse_block_count = bas, bs, K
    return a


@pytest.mark.gpu
def test_noalloc_matches_workspace_entry_point_on_two_calls():
    lib = _lib.load()
    dev = torch.device("cuda", 0)
    B, N, Hq, Hk, bs, K = 1, 49152, 12, 3, 64, 24
    stream = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
    ws = torch.empty(lib.mosaic_bsa_workspace_bytes(B, N, Hq, Hk, 64, bs, K, 0), dtype=torch.uint8, device=dev)
    for seed in (0, 1):
        g = torch.Generator(device=dev).manual_seed(seed)
        q = torch.randn(B, N, Hq, 64, generator=g, device=dev).bfloat16()
        k = torch.randn(B, N, Hk, 64, generator=g, device=dev).bfloat16()
        v = torch.randn(B, N, Hk, 64, generator=g, device=dev).bfloat16()
        w = torch.sigmoid(torch.randn(3, B, N, Hq, generator=g, device=dev)).bfloat16()
        out_ref = torch.empty(B, N, Hq, 64, dtype=torch.bfloat16, device=dev)
        out_new = torch.full_like(out_ref, float("nan"))
        idx_ref = torch.empty(B, N // bs, Hk, K, dtype=torch.int64, device=dev)
        idx_new = torch.full_like(idx_ref, -1)
        a_ref = _args(q, k, v, w, out_ref, idx_ref, ws)
        assert lib.mosaic_bsa_fwd(ctypes.byref(a_ref), stream) == _lib.MOSAIC_OK
        a_new = _args(q, k, v, w, out_new, idx_new)
        assert lib.mosaic_bsa_fwd_noalloc(ctypes.byref(a_new), stream) == _lib.MOSAIC_OK
        torch.cuda.synchronize()
        assert torch.equal(idx_new, idx_ref)
        d = (out_new.float() - out_ref.float()).abs()
        assert torch.isfinite(out_new.float()).all()
        assert d.max().item() <= MAX_ABS and d.mean().item() <= MEAN_ABS, (d.max().item(), d.mean().item())


def test_noalloc_rejects_what_does_not_fit():
    # validation happens on the host before any CUDA call, so this runs anywhere
    lib = _lib.load()
    a = _lib.MosaicBsaArgs()
    a.q = a.k = a.v = a.gates = a.out = 0x10000
    a.batch, a.seq_len, a.num_q_heads, a.num_kv_heads, a.head_dim = 4, 49152, 12, 3, 64  # 13.6 MB > 8 MiB
    a.block_attn_size, a.sparse_block_size, a.sparse_block_count = 1024, 64, 24
    assert lib.mosaic_bsa_fwd_noalloc(ctypes.byref(a), None) == _lib.MOSAIC_ERR_WORKSPACE
    a.batch = 1
    a.rope_cos = a.rope_sin = 0x10000
    assert lib.mosaic_bsa_fwd_noalloc(ctypes.byref(a), None) == _lib.MOSAIC_ERR_UNSUPPORTED
    assert lib.mosaic_bsa_fwd_noalloc(None, None) == _lib.MOSAIC_ERR_INVALID_ARGUMENT
