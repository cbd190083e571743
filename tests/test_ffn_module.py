"""The FFN drop-ins (mosaic_b200.MosaicSwiGLU, MosaicBlock) on the CPU: parameter names
of primitives.cSwiGLU / MosaicBlock (so reference state dicts load), the interleaved
w13 row order the GEMM takes, the C ABI's argument checks (host-side, no kernel runs),
and the oracle's restatement pinned to the reference's own cSwiGLU module."""
import ctypes
import os
import types

import pytest
import torch

import mosaic_b200 as M
from baseline import reference as R
from mosaic_b200 import _lib
from mosaic_b200 import ffn as F
from oracle import bsa_oracle as O


def block_cfg(dim=256, heads=4, noise_dim=32, affine=False):
    return types.SimpleNamespace(num_heads=heads, gqa_ratio=4, dim=dim, qkv_compress_ratio=1, rope=True,
                                 rope_theta=10000, block_attn_size=1024, sparse_block_size=64, sparse_block_count=24,
                                 noise_dim=noise_dim, mlp_ratio=4.0, rmsnorm_elementwise_affine=affine)


def test_swiglu_state_dict_names():
    m = M.MosaicSwiGLU(256, 1024, 32)
    assert set(m.state_dict()) == {"w13.weight", "w2.weight", "noise_bias.weight"}
    assert tuple(m.w13.weight.shape) == (2048, 256) and tuple(m.w2.weight.shape) == (256, 1024)
    assert set(M.MosaicSwiGLU(256, 1024, 0).state_dict()) == {"w13.weight", "w2.weight"}


@pytest.mark.parametrize("affine", [False, True])
def test_block_state_dict_names(affine):
    m = M.MosaicBlock(block_cfg(affine=affine), block_attn_only=False)
    keys = {k for k in m.state_dict() if not k.startswith("attention.")}
    want = {"ffn.w13.weight", "ffn.w2.weight", "ffn.noise_bias.weight"}
    if affine:
        want |= {"norm1.weight", "norm2.weight"}
    assert keys == want


def test_interleave_w13_layout():
    hidden, dim = 384, 8
    w13 = torch.arange(2 * hidden, dtype=torch.float32).unsqueeze(1).expand(2 * hidden, dim).contiguous()
    wi = F.interleave_w13(w13)
    rows = wi[:, 0].long()
    for i in range(hidden // 128):
        assert torch.equal(rows[256 * i:256 * i + 128], torch.arange(128 * i, 128 * i + 128))           # w1
        assert torch.equal(rows[256 * i + 128:256 * i + 256], hidden + torch.arange(128 * i, 128 * i + 128))  # w3
    with pytest.raises(ValueError):
        F.interleave_w13(torch.zeros(2 * 200, dim))


def test_forward_requiring_gradients_raises():
    m = M.MosaicSwiGLU(256, 1024, 32)
    with pytest.raises(NotImplementedError):
        m(torch.randn(16, 1, 256))


LIB_BUILT = os.path.exists(_lib.LIB_PATH)
FAKE = ctypes.c_void_p(0x10000)


@pytest.mark.skipif(not LIB_BUILT, reason="libmosaic_b200.so is not built")
def test_capi_rejects_bad_arguments():
    lib = _lib.load()
    sw = lambda rows=64, dim=256, hidden=1024, batch=2, x=FAKE, noise=None: lib.mosaic_ffn_swiglu(
        x, FAKE, None, noise, FAKE, None, rows, dim, hidden, batch, None)
    assert sw(hidden=1000) == _lib.MOSAIC_ERR_UNSUPPORTED        # hidden not a multiple of 128
    assert sw(dim=100) == _lib.MOSAIC_ERR_UNSUPPORTED            # dim not a multiple of 64
    assert sw(rows=63) == _lib.MOSAIC_ERR_INVALID_ARGUMENT       # rows not a multiple of batch
    assert sw(batch=0) == _lib.MOSAIC_ERR_INVALID_ARGUMENT
    assert sw(x=None) == _lib.MOSAIC_ERR_INVALID_ARGUMENT
    assert sw(noise=ctypes.c_void_p(0x10008)) == _lib.MOSAIC_ERR_INVALID_ARGUMENT  # misaligned
    assert sw(rows=0) == _lib.MOSAIC_OK
    lr = lambda rows=64, k=256, n=256, res=FAKE, dt=0: lib.mosaic_linear_residual(FAKE, FAKE, res, FAKE, None, None,
                                                                                 rows, k, n, dt, None)
    assert lr(k=100) == _lib.MOSAIC_ERR_UNSUPPORTED
    assert lr(n=40) == _lib.MOSAIC_ERR_UNSUPPORTED
    assert lr(res=None) == _lib.MOSAIC_ERR_INVALID_ARGUMENT
    assert lr(dt=5) == _lib.MOSAIC_ERR_INVALID_ARGUMENT
    assert lr(rows=0) == _lib.MOSAIC_OK
    rn = lambda x=FAKE, y=ctypes.c_void_p(0x20000), dt=0: lib.mosaic_rms_norm(x, None, y, 64, 256, ctypes.c_float(1e-6),
                                                                              dt, None)
    assert rn(dt=7) == _lib.MOSAIC_ERR_INVALID_ARGUMENT
    assert rn(y=FAKE, dt=_lib.MOSAIC_DTYPE_F16) == _lib.MOSAIC_ERR_INVALID_ARGUMENT  # fp16 in, bf16 out: not in place
    op = lambda dt=0: lib.mosaic_attn_out_proj_residual(FAKE, FAKE, FAKE, FAKE, None, 64, 1, 256, 4, 64, dt, None)
    assert op(dt=3) == _lib.MOSAIC_ERR_INVALID_ARGUMENT


@pytest.mark.skipif(not R.available(), reason="baseline/_ref holds no reference copy")
@pytest.mark.parametrize("affine", [False, True])
def test_oracle_matches_reference_cswiglu(affine):
    ref = R.load()
    torch.manual_seed(0)
    m = ref.primitives.cSwiGLU(128, 512, 32)
    norm = torch.nn.RMSNorm(128, elementwise_affine=affine)
    if affine:
        with torch.no_grad():
            norm.weight.uniform_(0.5, 1.5)
    x, z = torch.randn(40, 3, 128), torch.randn(3, 32)
    with torch.no_grad():
        want = m(x, z)
        got = O.swiglu_ffn(x, m.w13.weight, m.w2.weight, m.noise_bias.weight, z)
        torch.testing.assert_close(got, want, rtol=1e-5, atol=1e-6)
        want_block = x + m(norm(x), z)
        got_block = O.mosaic_block_ffn(x, z, m.w13.weight, m.w2.weight, m.noise_bias.weight,
                                       torch.finfo(torch.float32).eps, norm.weight if affine else None)
        torch.testing.assert_close(got_block, want_block, rtol=1e-5, atol=1e-5)


def test_pad_head_dim():
    from mosaic_b200 import ops as mops
    q = torch.randn(1, 8, 2, 32)
    (p,) = mops.pad_head_dim(q)
    assert p.shape == (1, 8, 2, 64) and torch.equal(p[..., :32], q) and not p[..., 32:].any()
    assert mops.pad_head_dim(torch.randn(1, 8, 2, 64))[0].shape[-1] == 64
    with pytest.raises(ValueError):
        mops.pad_head_dim(torch.randn(1, 8, 2, 96))
