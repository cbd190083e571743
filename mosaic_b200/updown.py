"""Drop-ins for primitives.HEALPixDownsample and primitives.HEALPixUpsample
(primitives.py:305-359), the resolution changes of Mosaic's U-Net between HEALPix
levels (nside 64 -> 32 -> 16 and back):

    down: x [(n f), B, C] --mosaic_healpix_downsample--> RMSNorm(proj_x(x as [n, B, (f C)])
                                                          + proj_pos(rel_pos)) [n, B, out]
    up:   x [n, B, C], shortcut --mosaic_healpix_upsample--> RMSNorm(rearrange(proj_x(x)
                                                          + proj_pos(rel_pos)) + shortcut)

Each is one tcgen05 GEMM whose epilogue adds the position bias (and the shortcut) and
writes the reference's output layout directly (the rearranges are addressing), then one
pass that applies the RMSNorm (one warp per row sums the squares of the stored bf16 row in
a fixed order, so the layer is deterministic).
proj_pos(rel_pos) does not depend on the input: it is computed once per weight version
and kept. The modules keep the reference's constructor, submodules (`proj_x`,
`proj_pos`, `norm`) and `rel_pos` buffer, so a reference state dict loads. Inference only.
"""
import torch
import torch.nn as nn

from . import _lib
from .healpix import get_healpix_grid
from .interp import norm_eps, rad_to_xyz
from .ops import _ptr, _require_cuda, _stream_ptr

__all__ = ["HEALPixDownsample", "HEALPixUpsample", "healpix_downsample", "healpix_upsample", "updown_rel_pos"]


def updown_rel_pos(nside_fine, nside_coarse):
    """The rel_pos buffer (primitives.py:317-322, 345-350): per coarse pixel, its nested
    children's unit vectors minus its own, [n, (f xyz)], standardised per column."""
    F = (nside_fine // nside_coarse) ** 2
    fine = rad_to_xyz(torch.deg2rad(get_healpix_grid(nside_fine)))
    coarse = rad_to_xyz(torch.deg2rad(get_healpix_grid(nside_coarse)))
    rel = (fine.reshape(-1, F, 3) - coarse[:, None]).reshape(-1, 3 * F)
    return ((rel - rel.mean(dim=0, keepdim=True)) / (rel.std(dim=0, keepdim=True) + 1e-6)).contiguous()


def _bf16c(t):
    return (t if t.dtype == torch.bfloat16 else t.to(torch.bfloat16)).contiguous()


def healpix_downsample(x, w_x, pos_bias, factor, eps, norm_weight=None, status=None):
    """x [(n f), B, C] -> [n, B, out] through mosaic_healpix_downsample."""
    _require_cuda(x, w_x, pos_bias)
    nF, B, C = x.shape
    n = nF // factor
    out_dim = w_x.shape[0]
    out = torch.empty(n, B, out_dim, dtype=torch.bfloat16, device=x.device)
    nw = None if norm_weight is None else norm_weight.float().contiguous()
    xb, wb, pb = _bf16c(x), _bf16c(w_x), _bf16c(pos_bias)
    with torch.cuda.device(x.device):
        rc = _lib.load().mosaic_healpix_downsample(_ptr(xb), _ptr(wb), _ptr(pb), _ptr(nw), _ptr(out),
                                                   _ptr(status), n, int(factor), B, C, out_dim, float(eps),
                                                   _stream_ptr(x.device))
    _lib.check("mosaic_healpix_downsample", rc)
    return out


def healpix_upsample(x, shortcut, w_x, pos_bias, factor, eps, norm_weight=None, status=None):
    """x [n, B, C], shortcut [(n f), B, out] -> [(n f), B, out] through mosaic_healpix_upsample."""
    _require_cuda(x, w_x, pos_bias)
    n, B, C = x.shape
    out_dim = w_x.shape[0] // factor
    out = torch.empty(n * factor, B, out_dim, dtype=torch.bfloat16, device=x.device)
    nw = None if norm_weight is None else norm_weight.float().contiguous()
    sc = None if shortcut is None else _bf16c(shortcut)
    xb, wb, pb = _bf16c(x), _bf16c(w_x), _bf16c(pos_bias)
    with torch.cuda.device(x.device):
        rc = _lib.load().mosaic_healpix_upsample(_ptr(xb), _ptr(sc), _ptr(wb), _ptr(pb), _ptr(nw), _ptr(out),
                                                 _ptr(status), n, int(factor), B, C, out_dim, float(eps),
                                                 _stream_ptr(x.device))
    _lib.check("mosaic_healpix_upsample", rc)
    return out


class _UpDown(nn.Module):
    space_dim = 3

    def _pos_bias(self):
        """bf16 proj_pos(rel_pos), recomputed only when the weight or the buffer changed."""
        w, rel = self.proj_pos.weight, self.rel_pos
        key = (w.data_ptr(), w._version, rel.data_ptr(), rel._version, w.device)
        if getattr(self, "_pos_key", None) != key:
            with torch.no_grad():
                self._pos_cache = torch.nn.functional.linear(rel.float(), w.float()).to(torch.bfloat16).contiguous()
            self._pos_key = key
        return self._pos_cache

    def _norm_args(self, x):
        eps = norm_eps(self.norm)
        return eps, self.norm.weight

    def _check_inference(self, *xs):
        if torch.is_grad_enabled() and (any(t is not None and t.requires_grad for t in xs)
                                        or any(p.requires_grad for p in self.parameters())):
            raise NotImplementedError(
                f"mosaic_b200.{type(self).__name__} serves inference; run it under torch.no_grad() or "
                "torch.inference_mode()")


class HEALPixDownsample(_UpDown):
    """primitives.HEALPixDownsample (primitives.py:305-329) on libmosaic_b200.so."""

    def __init__(self, in_dim, out_dim, nside_before, nside_after, rmsnorm_elementwise_affine=True):
        super().__init__()
        self.factor = (nside_before // nside_after) ** 2
        self.proj_x = nn.Linear(self.factor * in_dim, out_dim, bias=False)
        self.proj_pos = nn.Linear(self.factor * self.space_dim, out_dim, bias=False)
        self.norm = nn.RMSNorm(out_dim, elementwise_affine=rmsnorm_elementwise_affine)
        self.register_buffer("rel_pos", updown_rel_pos(nside_before, nside_after), persistent=True)

    def forward(self, x):
        self._check_inference(x)
        eps, w = self._norm_args(x)
        out = healpix_downsample(x, self.proj_x.weight, self._pos_bias(), self.factor, eps, w)
        return out.to(x.dtype)


class HEALPixUpsample(_UpDown):
    """primitives.HEALPixUpsample (primitives.py:332-359) on libmosaic_b200.so."""

    def __init__(self, in_dim, out_dim, nside_before, nside_after, rmsnorm_elementwise_affine=True):
        super().__init__()
        self.factor = (nside_after // nside_before) ** 2
        self.proj_x = nn.Linear(in_dim, out_dim * self.factor, bias=False)
        self.proj_pos = nn.Linear(self.factor * self.space_dim, out_dim * self.factor, bias=False)
        self.norm = nn.RMSNorm(out_dim, elementwise_affine=rmsnorm_elementwise_affine)
        self.register_buffer("rel_pos", updown_rel_pos(nside_after, nside_before), persistent=True)

    def forward(self, x, shortcut):
        self._check_inference(x, shortcut)
        eps, w = self._norm_args(x)
        out = healpix_upsample(x, shortcut, self.proj_x.weight, self._pos_bias(), self.factor, eps, w)
        return out.to(x.dtype)
