"""The fused FFN of a Mosaic block on the B200 (mosaic_b200.ffn: mosaic_ffn_swiglu and
mosaic_linear_residual on the tcgen05 projection GEMM) against the fp32 oracle
(oracle.swiglu_ffn / mosaic_block_ffn, restating primitives.py:92-106 and :229) and
against a bf16 torch emulation of the epilogue's rounding points.

Bounds: the bf16 outputs against the fp32 oracle within max-abs 2e-2 and mean-abs 2e-3,
both relative to the largest magnitude of the oracle's output (the FFN's scale depends
on the random weights: the reference's nn.Linear initialisation). Against the bf16
emulation (same rounding points, cuBLAS accumulation order instead of the tensor-core
tile order) every hidden value within 2 bf16 ulps of its magnitude."""
import ctypes

import pytest
import torch

import mosaic_b200 as M
from mosaic_b200 import _lib
from mosaic_b200 import ffn as F
from oracle import bsa_oracle as O

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")


def close_rel(got, ref, max_rel=2e-2, mean_rel=2e-3):
    got, ref = got.float().cpu(), ref.float().cpu()
    assert torch.isfinite(got).all(), "non-finite output"
    scale = ref.abs().max().item()
    d = (got - ref).abs()
    assert d.max().item() <= max_rel * scale and d.mean().item() <= mean_rel * scale, \
        (d.max().item(), d.mean().item(), scale)


def weights(dim, hidden, noise_dim, seed):
    torch.manual_seed(seed)
    m = M.MosaicSwiGLU(dim, hidden, noise_dim)
    return m


@pytest.mark.parametrize("cfg", [(3072, 2, 768, 4), (1024, 3, 1024, 4), (512, 1, 1280, 4), (256, 2, 256, 2)])
def test_swiglu_module_matches_oracle(cfg):
    S, B, dim, ratio = cfg
    m = weights(dim, dim * ratio, 32, seed=S + B)
    g = torch.Generator().manual_seed(S)
    x = torch.randn(S, B, dim, generator=g).bfloat16()
    z = torch.randn(B, 32, generator=g).bfloat16()
    ref = O.swiglu_ffn(x, m.w13.weight, m.w2.weight, m.noise_bias.weight, z)
    md = m.to(DEV).bfloat16()
    with torch.no_grad():
        out = md(x.to(DEV), z.to(DEV))
    torch.cuda.synchronize()
    assert out.dtype == torch.bfloat16 and out.shape == (S, B, dim)
    close_rel(out, ref)


@pytest.mark.parametrize("cfg", [(3072, 2, 768), (1024, 3, 1024), (512, 2, 1280)])
@pytest.mark.parametrize("affine", [False, True])
def test_block_ffn_matches_oracle(cfg, affine):
    S, B, dim = cfg
    m = weights(dim, 4 * dim, 32, seed=dim)
    norm = torch.nn.RMSNorm(dim, elementwise_affine=affine)
    g = torch.Generator().manual_seed(dim + S)
    if affine:
        with torch.no_grad():
            norm.weight.copy_(1 + 0.2 * torch.randn(dim, generator=g))
    x = (3 * torch.randn(S, B, dim, generator=g)).bfloat16()
    z = torch.randn(B, 32, generator=g).bfloat16()
    eps = torch.finfo(torch.float32).eps  # torch.nn.RMSNorm's eps=None default, for bf16 too
    ref = O.mosaic_block_ffn(x, z, m.w13.weight, m.w2.weight, m.noise_bias.weight, eps,
                             norm.weight if affine else None)
    md, nd = m.to(DEV), norm.to(DEV)
    md.bfloat16()
    with torch.no_grad():
        out = md.residual_forward(x.to(DEV), z.to(DEV), nd)
    torch.cuda.synchronize()
    close_rel(out, ref)
    # the FFN's own contribution on its own scale, beside the bf16 rounding of x + ffn
    # (half an ulp of |out|, as in the reference's bf16 add)
    ffn_scale = (ref - x.float()).abs().max().item()
    d = (out.float().cpu() - ref).abs()
    assert (d <= 2e-2 * ffn_scale + 2 ** -8 * ref.abs()).all(), d.max().item()
    assert d.mean().item() <= 2e-3 * ffn_scale + (2 ** -9 * ref.abs()).mean().item()


def test_swiglu_epilogue_rounding_points():
    """mosaic_ffn_swiglu through the C ABI against torch bf16 ops at the reference's
    rounding points (w13 output, + noise, SiLU, product) on the same rows."""
    S, B, dim, hidden = 512, 2, 768, 3072
    g = torch.Generator(device=DEV).manual_seed(3)
    x = torch.randn(S, B, dim, generator=g, device=DEV).bfloat16()
    w13 = (torch.randn(2 * hidden, dim, generator=g, device=DEV) * dim ** -0.5).bfloat16()
    noise = torch.randn(B, hidden, generator=g, device=DEV).bfloat16()
    h = torch.empty(S * B, hidden, dtype=torch.bfloat16, device=DEV)
    wi = F.interleave_w13(w13).contiguous()
    lib = _lib.load()
    rc = lib.mosaic_ffn_swiglu(x.data_ptr(), wi.data_ptr(), None, noise.data_ptr(), h.data_ptr(), None, S * B, dim,
                               hidden, B, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == _lib.MOSAIC_OK
    torch.cuda.synchronize()
    x1, x3 = (x @ w13.t()).chunk(2, dim=-1)  # bf16 Linear outputs
    ref = torch.nn.functional.silu(x1 + noise.unsqueeze(0)) * x3
    d = (h.reshape(S, B, hidden).float() - ref.float()).abs()
    assert (d <= 2 * 2 ** -8 * ref.float().abs() + 1e-3).float().mean() > 0.995, d.max()
    close_rel(h.reshape(S, B, hidden), ref, max_rel=2e-2, mean_rel=2e-4)


def test_linear_residual_in_place_equals_out_of_place():
    M_, K, N = 2048, 3072, 768
    g = torch.Generator(device=DEV).manual_seed(4)
    a = torch.randn(M_, K, generator=g, device=DEV).bfloat16()
    w = (torch.randn(N, K, generator=g, device=DEV) * K ** -0.5).bfloat16()
    r = torch.randn(M_, N, generator=g, device=DEV).bfloat16()
    out = F.linear_residual(a, w, r)
    r2 = r.clone()
    F.linear_residual(a, w, r2, out=r2)
    torch.cuda.synchronize()
    assert torch.equal(out, r2)
    ref = r.float() + (a @ w.t()).float()
    close_rel(out, ref, max_rel=1e-2, mean_rel=1e-3)


def test_block_ffn_keeps_an_fp32_stream():
    """A residual stream in fp32 (the reference's fp32 model under fp16 autocast) stays
    fp32: the FFN runs in bf16 and is added in fp32."""
    S, B, dim = 1024, 2, 768
    m = weights(dim, 4 * dim, 32, seed=9)
    norm = torch.nn.RMSNorm(dim, elementwise_affine=False)
    g = torch.Generator().manual_seed(9)
    x = torch.randn(S, B, dim, generator=g)
    z = torch.randn(B, 32, generator=g)
    ref = O.mosaic_block_ffn(x, z, m.w13.weight, m.w2.weight, m.noise_bias.weight, torch.finfo(torch.float32).eps)
    with torch.no_grad():
        out = m.to(DEV).residual_forward(x.to(DEV), z.to(DEV), norm.to(DEV))
    torch.cuda.synchronize()
    assert out.dtype == torch.float32
    close_rel(out.cpu() - x, ref - x)


def test_rms_norm_matches_torch():
    g = torch.Generator(device=DEV).manual_seed(6)
    x = (2 * torch.randn(4096, 768, generator=g, device=DEV)).bfloat16()
    for affine in (False, True):
        norm = torch.nn.RMSNorm(768, elementwise_affine=affine).to(DEV)
        if affine:
            with torch.no_grad():
                norm.weight.uniform_(0.5, 1.5)
        eps = torch.finfo(torch.float32).eps  # what torch.nn.RMSNorm(eps=None) applies
        got = F.rms_norm(x, eps, norm.weight if affine else None)
        with torch.no_grad():
            want = norm(x)
        d = (got.float() - want.float()).abs()
        # the same fp32 arithmetic; the sum of squares in another order can move a value
        # across a rounding boundary (one bf16 ulp), rarely
        assert (d <= 2 ** -7 * want.float().abs()).all() and (d > 0).float().mean() < 0.01


def test_attention_residual_in_the_output_projection():
    import types
    cfg = types.SimpleNamespace(num_heads=12, gqa_ratio=4, dim=768, qkv_compress_ratio=1, rope=True, rope_theta=10000,
                                block_attn_size=1024, sparse_block_size=64, sparse_block_count=8)
    torch.manual_seed(1)
    m = M.MosaicAttention(cfg, block_attn_only=False)
    grid = O.healpix_grid(16)
    m.q_rope.initialize_rope(grid)
    m.k_rope.initialize_rope(grid)
    m = m.to(DEV).bfloat16()
    g = torch.Generator(device=DEV).manual_seed(7)
    x = torch.randn(3072, 2, 768, generator=g, device=DEV).bfloat16()
    r = torch.randn(3072, 2, 768, generator=g, device=DEV).bfloat16()
    with torch.no_grad():
        a = m(x)
        b = m(x, residual=r)
    torch.cuda.synchronize()
    assert torch.equal(b, r + a)


def test_block_ffn_fp16_stream():
    """A residual stream in fp16 (the model under fp16 autocast) runs fused as well: the
    norm reads fp16, the w2 epilogue rounds the Linear's output to fp16 and adds in fp16."""
    S, B, dim = 2048, 2, 768
    m = weights(dim, 4 * dim, 32, seed=11)
    norm = torch.nn.RMSNorm(dim, elementwise_affine=False)
    g = torch.Generator().manual_seed(11)
    x = (3 * torch.randn(S, B, dim, generator=g)).half()
    z = torch.randn(B, 32, generator=g)  # fp32 weights: the noise projection runs in fp32 here
    ref = O.mosaic_block_ffn(x, z, m.w13.weight, m.w2.weight, m.noise_bias.weight, torch.finfo(torch.float32).eps)
    md = m.to(DEV)
    with torch.no_grad():
        out = md.residual_forward(x.to(DEV), z.to(DEV), norm.to(DEV))
    torch.cuda.synchronize()
    assert out.dtype == torch.float16
    ffn_scale = (ref - x.float()).abs().max().item()
    d = (out.float().cpu() - ref).abs()
    # the FFN runs in bf16 (2e-2 of its scale), then the fp16 add rounds (half an fp16 ulp)
    assert (d <= 2e-2 * ffn_scale + 2 ** -11 * ref.abs()).all(), d.max().item()
    assert d.mean().item() <= 2e-3 * ffn_scale + (2 ** -12 * ref.abs()).mean().item()


def test_rms_norm_reads_fp16():
    g = torch.Generator(device=DEV).manual_seed(12)
    x = (2 * torch.randn(4096, 1024, generator=g, device=DEV)).half()
    eps = torch.finfo(torch.float32).eps
    got = F.rms_norm(x, eps)
    assert got.dtype == torch.bfloat16
    xf = x.float()
    want = (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)).bfloat16()
    d = (got.float() - want.float()).abs()
    assert (d <= 2 ** -7 * want.float().abs()).all() and (d > 0).float().mean() < 0.01


def test_linear_residual_fp16_residual():
    M_, K, N = 1024, 3072, 768
    g = torch.Generator(device=DEV).manual_seed(13)
    a = torch.randn(M_, K, generator=g, device=DEV).bfloat16()
    w = (torch.randn(N, K, generator=g, device=DEV) * K ** -0.5).bfloat16()
    r = torch.randn(M_, N, generator=g, device=DEV).half()
    out = F.linear_residual(a, w, r)
    torch.cuda.synchronize()
    assert out.dtype == torch.float16
    # the Linear's output rounded to fp16, then the fp16 add (autocast's rounding points)
    y = (a.float() @ w.float().t()).half()
    ref = (r.float() + y.float()).half()
    d = (out.float() - ref.float()).abs()
    # y may differ by one fp16 ulp (accumulation order), the sum by one more: both scale
    # with |y| as well as |out| (the residual can cancel y)
    assert (d <= 2 ** -9 * (y.float().abs() + ref.float().abs()) + 1e-3).all(), d.max().item()
