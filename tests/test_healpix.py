"""HEALPix nested pixel centres and RoPE tables (utils.py:19-30, primitives.py:115-123).

healpy is absent, so the reference side of this piece is unpinned; the product's
vectorised restatement is checked against the oracle's independent scalar one and
against HEALPix known answers (Gorski et al. 2005)."""
import math

import numpy as np
import pytest
import torch

from mosaic_b200 import healpix as H
from oracle import bsa_oracle as O


def test_nside1_known_answers():
    th, ph = H.pix2ang_nest(1, np.arange(12))
    lat = 90 - np.degrees(th)
    z23 = math.degrees(math.asin(2.0 / 3.0))
    np.testing.assert_allclose(lat, [z23] * 4 + [0.0] * 4 + [-z23] * 4, atol=1e-12)
    np.testing.assert_allclose(np.degrees(ph), [45, 135, 225, 315, 0, 90, 180, 270, 45, 135, 225, 315], atol=1e-12)


@pytest.mark.parametrize("nside", [1, 2, 4, 8, 16])
def test_vectorised_matches_scalar_oracle(nside):
    th, ph = H.pix2ang_nest(nside, np.arange(12 * nside * nside))
    for p in range(12 * nside * nside):
        t2, p2 = O.pix2ang_nest_scalar(nside, p)
        assert abs(th[p] - t2) < 1e-12 and abs(ph[p] - p2) < 1e-12


@pytest.mark.parametrize("nside", [4, 16, 64])
def test_rings_and_equal_area(nside):
    th, _ = H.pix2ang_nest(nside, np.arange(12 * nside * nside))
    z = np.round(np.cos(th), 12)
    vals, counts = np.unique(z, return_counts=True)
    assert len(vals) == 4 * nside - 1
    # polar rings hold 4*i pixels, equatorial rings 4*nside
    counts = counts[::-1]  # north to south
    for i in range(1, nside):
        assert counts[i - 1] == 4 * i
    assert np.all(counts[nside - 1: 3 * nside] == 4 * nside)


def test_nested_children_surround_parent():
    child = H.get_healpix_grid(32).double()
    parent = H.get_healpix_grid(16).double()
    # children 4p..4p+3 are the four sub-pixels of p: their centroid is close to it
    for p in range(0, 12 * 16 * 16, 97):
        c = child[4 * p: 4 * p + 4]
        if abs(parent[p, 1]) > 80:  # skip the poles where longitude wraps
            continue
        lon = c[:, 0]
        if lon.max() - lon.min() > 180:
            continue
        assert abs(lon.mean() - parent[p, 0]) < 1.0 and abs(c[:, 1].mean() - parent[p, 1]) < 1.0


def test_rope_tables_match_oracle_exactly():
    pos = H.get_healpix_grid(16)
    assert torch.equal(pos, O.healpix_grid(16))
    cos, sin = H.rope_tables(pos, 64)
    c2, s2 = O.rope_tables(pos, 64)
    assert cos.shape == (3072, 32)
    assert torch.equal(cos, c2) and torch.equal(sin, s2)
