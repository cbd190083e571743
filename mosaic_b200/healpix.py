"""HEALPix nested-order pixel centres and Mosaic's 2D RoPE tables (host-side init).

`get_healpix_grid(nside)` replaces utils.get_healpix_grid (utils.py:19-30), which
calls healpy.pix2ang(nside, arange(12*nside**2), nest=True) and returns
(lon deg, lat deg = 90 - colatitude deg) as float32 [npix, 2]. healpy is not a
dependency here: pix2ang for the NESTED scheme is restated from the HEALPix
definition (Gorski et al. 2005, ApJ 622:759, section 4 and the nest2ring
geometry): a nested index splits into a base face f = ipix // nside^2 and
bit-interleaved in-face coordinates (x, y); the ring index is
jr = jrll[f]*nside - x - y - 1 and the position along the ring is
jp = (jpll[f]*nr + x - y + 1 + s) / 2 with s the ring shift. Vectorised numpy,
float64 throughout like healpy.

Because the ordering is nested, every run of 4^k consecutive pixels is one
spatially compact patch; this is why Mosaic's sparse blocks are contiguous
index ranges.
"""
import math

import numpy as np
import torch

_JRLL = np.array([2, 2, 2, 2, 3, 3, 3, 3, 4, 4, 4, 4], dtype=np.int64)
_JPLL = np.array([1, 3, 5, 7, 0, 2, 4, 6, 1, 3, 5, 7], dtype=np.int64)


def _compress_bits(v):
    """Keep the even bits of v packed together (inverse of bit interleaving)."""
    v = v & 0x5555555555555555
    v = (v | (v >> 1)) & 0x3333333333333333
    v = (v | (v >> 2)) & 0x0F0F0F0F0F0F0F0F
    v = (v | (v >> 4)) & 0x00FF00FF00FF00FF
    v = (v | (v >> 8)) & 0x0000FFFF0000FFFF
    v = (v | (v >> 16)) & 0x00000000FFFFFFFF
    return v


def pix2ang_nest(nside, ipix):
    """(theta, phi) in radians of NESTED pixel centres, like healpy.pix2ang(..., nest=True)."""
    if nside < 1 or (nside & (nside - 1)) != 0:
        raise ValueError(f"nside must be a power of two, got {nside}")
    ipix = np.asarray(ipix, dtype=np.int64)
    npface = nside * nside
    npix = 12 * npface
    if ipix.size and (ipix.min() < 0 or ipix.max() >= npix):
        raise ValueError("pixel index out of range")
    face = ipix // npface
    ipf = ipix % npface
    ix = _compress_bits(ipf)
    iy = _compress_bits(ipf >> 1)
    jr = _JRLL[face] * nside - ix - iy - 1

    nr = np.where(jr < nside, jr, np.where(jr > 3 * nside, 4 * nside - jr, nside))
    z = np.empty(ipix.shape, dtype=np.float64)
    north = jr < nside
    south = jr > 3 * nside
    equ = ~(north | south)
    fact2 = 4.0 / npix
    z[north] = 1.0 - nr[north].astype(np.float64) ** 2 * fact2
    z[south] = -(1.0 - nr[south].astype(np.float64) ** 2 * fact2)
    z[equ] = (2 * nside - jr[equ]).astype(np.float64) * (2.0 * nside * fact2)
    kshift = np.where(equ, (jr - nside) & 1, 0)

    jp = (_JPLL[face] * nr + ix - iy + 1 + kshift) // 2
    jp = np.where(jp > 4 * nside, jp - 4 * nside, jp)
    jp = np.where(jp < 1, jp + 4 * nside, jp)
    phi = (jp - (kshift + 1) * 0.5) * (0.5 * math.pi / nr)
    theta = np.arccos(np.clip(z, -1.0, 1.0))
    return theta, phi


def get_healpix_grid(nside):
    """float32 [12*nside^2, 2] of (lon deg, lat deg) in nested order (utils.py:19-30)."""
    theta, phi = pix2ang_nest(nside, np.arange(12 * nside * nside))
    phi = np.rad2deg(phi)
    lat = 90.0 - np.rad2deg(theta)
    return torch.stack((torch.from_numpy(phi), torch.from_numpy(lat)), dim=-1).float()


def rope_tables(positions, head_dim=64, theta=10000.0):
    """(cos, sin), each fp32 [N, head_dim // 2], of Mosaic's 2D RoPE.

    Follows RoPE.initialize_rope (primitives.py:115-123): 16 base frequencies
    theta ** -(2i / (head_dim/2)), applied to lon (first half) and lat (second
    half) in radians.
    """
    base = 1.0 / (theta ** (torch.arange(0, head_dim // 2, 2).float() / (head_dim // 2)))
    lon = torch.deg2rad(positions[:, 0:1])
    lat = torch.deg2rad(positions[:, 1:2])
    freqs = torch.cat([lon @ base.unsqueeze(0), lat @ base.unsqueeze(0)], dim=-1)
    return freqs.cos().contiguous(), freqs.sin().contiguous()


def healpix_rope_tables(nside, head_dim=64, theta=10000.0):
    """RoPE tables for the nested HEALPix grid of `nside` (what Transformer.initialize_rope builds)."""
    return rope_tables(get_healpix_grid(nside), head_dim, theta)
