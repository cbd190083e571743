"""mosaic_bsa_fwd_noalloc: the forward for callers that cannot allocate device
memory (a foreign-language host with no device allocator, or a service with a
fixed memory budget that must not call cudaMalloc per request). It keeps its
scratch in an 8 MiB array inside the library instead of a caller workspace.

Checked through the C ABI against mosaic_bsa_fwd (the workspace entry point) on
two calls in a row with different inputs, so that scratch left over from the
first call cannot leak into the second: both entry points run the same kernels on
the same inputs, so outputs and indices must be bitwise equal (which is inside the
max-abs 2e-2 / mean-abs 2e-3 tolerance of the other parity tests). Covered: the
full forward with the block indices written to caller memory or kept in the
scratch, no_compression, block_attn_only (no scratch used), and fp16 activations.
This file is collected last on purpose.
"""
import ctypes
import os

import pytest
import torch

from mosaic_b200 import _lib


def _args(q, k, v, w, out, idx, ws=None, B=1, N=49152, Hq=12, Hk=3, bas=1024, bs=64, K=24, dtype=0):
    a = _lib.MosaicBsaArgs()
    a.q, a.k, a.v = q.data_ptr(), k.data_ptr(), v.data_ptr()
    a.gates = w.data_ptr()
    a.out = out.data_ptr()
    a.block_indices = idx.data_ptr() if idx is not None else None
    a.workspace = ws.data_ptr() if ws is not None else None
    a.workspace_bytes = ws.numel() if ws is not None else 0
    a.batch, a.seq_len, a.num_q_heads, a.num_kv_heads, a.head_dim = B, N, Hq, Hk, 64
    a.block_attn_size, a.sparse_block_size, a.sparse_block_count = bas, bs, K
    a.dtype = dtype
    return a


MODES = {
    "full, indices to caller memory": dict(indices=True),
    "full, indices in the scratch": dict(indices=False),
    "no_compression": dict(indices=True, no_compression=1),
    "block_attn_only": dict(indices=False, block_attn_only=1),
    "fp16": dict(indices=True, dtype=_lib.MOSAIC_DTYPE_F16),
}


@pytest.mark.gpu
@pytest.mark.parametrize("mode", list(MODES))
def test_noalloc_matches_workspace_entry_point_on_two_calls(mode):
    cfg = MODES[mode]
    lib = _lib.load()
    dev = torch.device("cuda", 0)
    B, N, Hq, Hk, bs, K = 1, 49152, 12, 3, 64, 24
    dt = torch.float16 if cfg.get("dtype") == _lib.MOSAIC_DTYPE_F16 else torch.bfloat16
    stream = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
    ws = torch.empty(lib.mosaic_bsa_workspace_bytes(B, N, Hq, Hk, 64, bs, K, 0), dtype=torch.uint8, device=dev)
    for seed in (0, 1):
        g = torch.Generator(device=dev).manual_seed(seed)
        q = torch.randn(B, N, Hq, 64, generator=g, device=dev).to(dt)
        k = torch.randn(B, N, Hk, 64, generator=g, device=dev).to(dt)
        v = torch.randn(B, N, Hk, 64, generator=g, device=dev).to(dt)
        w = torch.sigmoid(torch.randn(3, B, N, Hq, generator=g, device=dev)).to(dt)
        out_ref = torch.empty(B, N, Hq, 64, dtype=dt, device=dev)
        out_new = torch.full_like(out_ref, float("nan"))
        idx_ref = torch.empty(B, N // bs, Hk, K, dtype=torch.int64, device=dev)
        idx_new = torch.full_like(idx_ref, -1) if cfg["indices"] else None
        a_ref = _args(q, k, v, w, out_ref, idx_ref, ws, dtype=cfg.get("dtype", 0))
        a_new = _args(q, k, v, w, out_new, idx_new, dtype=cfg.get("dtype", 0))
        for a in (a_ref, a_new):
            a.no_compression = cfg.get("no_compression", 0)
            a.block_attn_only = cfg.get("block_attn_only", 0)
        assert lib.mosaic_bsa_fwd(ctypes.byref(a_ref), stream) == _lib.MOSAIC_OK
        assert lib.mosaic_bsa_fwd_noalloc(ctypes.byref(a_new), stream) == _lib.MOSAIC_OK
        torch.cuda.synchronize()
        if idx_new is not None and not cfg.get("block_attn_only"):
            assert torch.equal(idx_new, idx_ref)
        assert torch.isfinite(out_new.float()).all()
        assert torch.equal(out_new, out_ref)


@pytest.mark.skipif(not os.path.exists(_lib.LIB_PATH), reason="libmosaic_b200.so is not built")
def test_noalloc_rejects_what_does_not_fit():
    # validation happens on the host before any CUDA call, so no GPU is needed
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
