"""Drop-ins for the feed-forward half of a Mosaic layer: primitives.cSwiGLU
(primitives.py:92-106) and primitives.MosaicBlock (primitives.py:212-229), on
libmosaic_b200.so.

    MosaicBlock.forward(x [S, B, dim], z [B, noise_dim]), bf16 or fp16 stream:
        y = norm1(x)                        --mosaic_rms_norm-->
        x = x + attention(y)                --mosaic_b200.MosaicAttention, the residual add
                                              in its output projection's epilogue
        y = norm2(x)                        --mosaic_rms_norm-->
        h = silu(x1 + noise) * x3           --mosaic_ffn_swiglu-->  one tcgen05 GEMM over the
                                              interleaved w13; the epilogue does the rest
        x = x + w2(h)                       --mosaic_linear_residual-->

The reference's cSwiGLU splits `w13(x)` with `chunk(2)` and runs the noise add, the
SiLU and the product as elementwise passes over the two strided halves; here they are
the epilogue of the w13 GEMM, with the reference's bf16 rounding after every tensor op
(the norms write the same bf16 rows torch.nn.RMSNorm does, and each GEMM's output is
rounded before its epilogue arithmetic), so only the GEMMs' accumulation order differs.

Both modules keep the reference's constructor and submodule names (`w13`, `w2`,
`act_fn`, `noise_bias`; `attention`, `norm1`, `norm2`, `ffn`), so reference state
dicts load, and rebinding the block class mosaic.py imports (`_MosaicBlock`, or
primitives.MosaicBlock before mosaic.py is imported) swaps them in. They serve
inference (no backward). The GEMMs run in bf16. A residual stream in fp16 (the
reference's model under fp16 autocast, where every Linear outputs fp16) stays fp16:
the norms read it, and the residual epilogues round the Linear's output to fp16 and add
in fp16, as autocast does. Any other stream dtype keeps its dtype, with the module's
own torch.nn.RMSNorm and the adds done by torch.
"""
import torch
import torch.nn as nn

from . import _lib
from .attention import MosaicAttention
from .interp import linear, norm_eps
from .ops import _ptr, _require_cuda, _stream_ptr

__all__ = ["interleave_w13", "ffn_swiglu", "linear_residual", "rms_norm", "MosaicSwiGLU", "MosaicBlock"]

_BLOCK = 128  # hidden units per interleaved block of w13 (half a GEMM tile)


def _bf16c(t):
    t = t if t.dtype == torch.bfloat16 else t.to(torch.bfloat16)
    return t.contiguous()


def interleave_w13(w13):
    """cSwiGLU.w13.weight [2 hidden, dim] -> the row order mosaic_ffn_swiglu takes: blocks
    of 128 w1 rows, each followed by the w3 rows of the same hidden units."""
    two_h, dim = w13.shape
    hidden = two_h // 2
    if two_h % 2 or hidden % _BLOCK:
        raise ValueError(f"mosaic_ffn_swiglu needs a hidden size that is a multiple of {_BLOCK} (got {hidden})")
    w1, w3 = w13[:hidden], w13[hidden:]
    return torch.stack((w1.reshape(-1, _BLOCK, dim), w3.reshape(-1, _BLOCK, dim)), dim=1).reshape(two_h, dim)


def ffn_swiglu(x, w13_interleaved, batch, row_scale=None, noise=None, status=None):
    """h [..., hidden] = bf16(silu(bf16(x1 + noise[b])) * x3), x1 / x3 = bf16(row_scale * x w1^T / w3^T),
    for x [S, batch, dim] (any leading shape whose flattened rows are (s, b))."""
    _require_cuda(x, w13_interleaved)
    dim = x.shape[-1]
    xb, wb = _bf16c(x).reshape(-1, dim), _bf16c(w13_interleaved)
    hidden = wb.shape[0] // 2
    h = torch.empty(xb.shape[0], hidden, dtype=torch.bfloat16, device=x.device)
    rs = None if row_scale is None else row_scale.float().contiguous()
    nz = None if noise is None else _bf16c(noise).reshape(batch, hidden)
    with torch.cuda.device(x.device):
        rc = _lib.load().mosaic_ffn_swiglu(_ptr(xb), _ptr(wb), _ptr(rs), _ptr(nz), _ptr(h), _ptr(status),
                                           xb.shape[0], dim, hidden, batch, _stream_ptr(x.device))
    _lib.check("mosaic_ffn_swiglu", rc)
    return h.reshape(*x.shape[:-1], hidden)


def _stream_dtype(t):
    """A 16-bit residual stream's dtype code (bf16, or fp16 under fp16 autocast)."""
    if t.dtype == torch.float16:
        return _lib.MOSAIC_DTYPE_F16
    if t.dtype == torch.bfloat16:
        return _lib.MOSAIC_DTYPE_BF16
    raise TypeError(f"expected a bf16 or fp16 tensor, got {t.dtype}")


def linear_residual(a, w, residual, out=None, row_scale=None, status=None):
    """out = T(residual + T(row_scale * a w^T)) with T the residual's dtype (bf16 or fp16;
    out may be residual: in place). a and w run in bf16."""
    _require_cuda(a, w, residual)
    k_in, n_out = a.shape[-1], w.shape[0]
    ab, wb = _bf16c(a).reshape(-1, k_in), _bf16c(w)
    rb = residual.contiguous().reshape(-1, n_out)
    o = torch.empty_like(rb) if out is None else out.reshape(-1, n_out)
    rs = None if row_scale is None else row_scale.float().contiguous()
    with torch.cuda.device(a.device):
        rc = _lib.load().mosaic_linear_residual(_ptr(ab), _ptr(wb), _ptr(rb), _ptr(o), _ptr(rs), _ptr(status),
                                                ab.shape[0], k_in, n_out, _stream_dtype(rb), _stream_ptr(a.device))
    _lib.check("mosaic_linear_residual", rc)
    return o.reshape(residual.shape)


def rms_norm(x, eps, weight=None):
    """torch.nn.RMSNorm of a bf16 or fp16 x [..., dim] through mosaic_rms_norm: bf16(x *
    rsqrt(mean(x^2) + eps) * weight) in fp32 arithmetic, the norm a Mosaic block feeds
    its attention and its FFN (primitives.py:228-229); the result is bf16 either way
    (the GEMMs behind it take bf16)."""
    _require_cuda(x)
    dim = x.shape[-1]
    xb = (x if x.dtype in (torch.bfloat16, torch.float16) else x.to(torch.bfloat16)).contiguous().reshape(-1, dim)
    y = torch.empty(xb.shape, dtype=torch.bfloat16, device=x.device)
    w = None if weight is None else weight.detach().float().contiguous()
    with torch.cuda.device(x.device):
        rc = _lib.load().mosaic_rms_norm(_ptr(xb), _ptr(w), _ptr(y), xb.shape[0], dim, float(eps),
                                         _stream_dtype(xb), _stream_ptr(x.device))
    _lib.check("mosaic_rms_norm", rc)
    return y.reshape(x.shape)


def _no_grad_check(mod, x):
    if torch.is_grad_enabled() and (x.requires_grad or any(p.requires_grad for p in mod.parameters())):
        raise NotImplementedError(
            f"mosaic_b200.{type(mod).__name__} serves inference (the fused FFN has no backward); run it under "
            "torch.no_grad() or torch.inference_mode()")


class MosaicSwiGLU(nn.Module):
    """Drop-in for primitives.cSwiGLU (primitives.py:92-106): same constructor, weights
    and forward(x, z) on an already normalised x [S, B, dim]; `residual_forward` is the
    form MosaicBlock uses (its norm2, then the FFN with the residual add in the w2 GEMM)."""

    def __init__(self, dim, hidden_dim, noise_dim):
        super().__init__()
        self.w13 = nn.Linear(dim, 2 * hidden_dim, bias=False)
        self.w2 = nn.Linear(hidden_dim, dim, bias=False)
        self.act_fn = nn.SiLU()
        if noise_dim > 0:
            self.noise_bias = nn.Linear(noise_dim, hidden_dim, bias=False)

    def _w13_interleaved(self):
        """w13 in bf16 with its rows interleaved; rebuilt only when the weight changes
        (another tensor or an in-place update, which bumps its version counter)."""
        w = self.w13.weight
        key = (w.data_ptr(), w._version, w.dtype, w.device)
        if getattr(self, "_w13_key", None) != key:
            self._w13_cache = interleave_w13(w.detach().to(torch.bfloat16))
            self._w13_key = key
        return self._w13_cache

    def _noise(self, z):
        if z is None or not hasattr(self, "noise_bias"):
            return None
        return self.noise_bias(z)

    def forward(self, x, z=None):
        _no_grad_check(self, x)
        h = ffn_swiglu(x, self._w13_interleaved(), x.shape[1], noise=self._noise(z))
        return linear(h, self.w2.weight).to(x.dtype)

    def residual_forward(self, x, z, norm):
        """x + self(norm(x), z) for the block's torch.nn.RMSNorm `norm`."""
        _no_grad_check(self, x)
        if x.dtype in (torch.bfloat16, torch.float16):
            y = rms_norm(x, norm_eps(norm), norm.weight)
            h = ffn_swiglu(y, self._w13_interleaved(), x.shape[1], noise=self._noise(z))
            return linear_residual(h, self.w2.weight, x)
        h = ffn_swiglu(norm(x), self._w13_interleaved(), x.shape[1], noise=self._noise(z))
        return x + linear(h, self.w2.weight).to(x.dtype)


class MosaicBlock(nn.Module):
    """Drop-in for primitives.MosaicBlock (primitives.py:212-229): the same submodules
    (`attention` = mosaic_b200.MosaicAttention, `norm1`, `norm2`, `ffn` =
    MosaicSwiGLU) and forward(x [S, B, dim], z [B, noise_dim]): norm, attention with
    the residual add in its output projection, norm, w13 + noise + SiLU + product,
    w2 + residual."""

    def __init__(self, config, block_attn_only: bool, no_compression: bool = False):
        super().__init__()
        dim = config.dim
        self.attention = MosaicAttention(config, block_attn_only, no_compression)
        self.norm1 = nn.RMSNorm(dim, elementwise_affine=config.rmsnorm_elementwise_affine)
        self.norm2 = nn.RMSNorm(dim, elementwise_affine=config.rmsnorm_elementwise_affine)
        self.ffn = MosaicSwiGLU(dim, int(dim * config.mlp_ratio), config.noise_dim)

    def forward(self, x, z=None):
        if x.dtype in (torch.bfloat16, torch.float16):
            x = self.attention(rms_norm(x, norm_eps(self.norm1), self.norm1.weight), residual=x)
        else:
            x = x + self.attention(self.norm1(x))
        return self.ffn.residual_forward(x, z, self.norm2)
