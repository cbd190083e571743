"""Parity of the cross-attention interpolation (mosaic_row_rms, mosaic_linear,
mosaic_interp_attend, mosaic_interp_attend_tiled and the CrossAttentionInterpolate module) with the CPU oracle's
restatement of primitives.CrossAttentionInterpolate.forward and with the fixtures of
the reference module. Tolerance: bf16 tensors with fp32 arithmetic inside, compared
with the fp32 oracle at max-abs 2e-2 and mean-abs 2e-3 of the output's largest
magnitude."""
import types

import pytest
import torch

import mosaic_b200 as M
from mosaic_b200 import interp as I
from mosaic_b200 import ops as mops
from oracle import bsa_oracle as O
from tests import golden_util as GU

pytestmark = pytest.mark.gpu
DEV = "cuda"


def close_rel(got, ref, max_rel=2e-2, mean_rel=2e-3):
    got = got.float().cpu()
    assert torch.isfinite(got).all(), "non-finite output"
    m = max(1e-6, ref.abs().max().item())
    d = (got - ref.float()).abs()
    assert d.max().item() <= max_rel * m and d.mean().item() <= mean_rel * m, (d.max().item(), d.mean().item(), m)


def scheme(n_lon, n_lat, nside, to_hp, k):
    ll, hp = GU.interp_grids(n_lon, n_lat, nside)
    pf, pt = (ll, hp) if to_hp else (hp, ll)
    nb = I.knn_neighbors(pf, pt, k)
    rel = torch.nn.functional.normalize(I.rad_to_xyz(pt).unsqueeze(1) - I.rad_to_xyz(pf)[nb], dim=-1)
    return pf, pt, nb, rel


@pytest.mark.parametrize("cfg", [(48, 25, 8, True, 1, 256, 4, 24), (48, 25, 8, False, 3, 768, 12, 20),
                                 (24, 13, 4, True, 2, 512, 8, 8)])
def test_interp_attend_matches_oracle(cfg):
    n_lon, n_lat, nside, to_hp, B, dim, H, k = cfg
    pf, pt, nb, rel = scheme(n_lon, n_lat, nside, to_hp, k)
    g = torch.Generator().manual_seed(dim + k)
    kv = torch.randn(pf.shape[0], B, 2 * dim, generator=g).bfloat16()
    w_q = torch.randn(dim, 3, generator=g)
    status = mops.status_buffer(DEV)
    out = I.interp_attend(kv.to(DEV), nb.to(DEV), rel.to(DEV), w_q.to(DEV), H, pf.shape[0], status=status)
    torch.cuda.synchronize()
    assert mops.check_status(status) == 0
    # the oracle's attention on the same kv (identity norm / projections)
    D = dim // H
    q = (rel @ w_q.t()).reshape(*rel.shape[:2], 1, H, D)
    kvr = kv.float().reshape(pf.shape[0], B, 2, H, D).permute(2, 0, 1, 3, 4)
    kk, vv = kvr[:, nb]
    a = torch.softmax((q * kk).sum(-1, keepdim=True) * D ** -0.5, dim=1)
    close_rel(out, (a * vv).sum(1).reshape(pt.shape[0], B, dim))


def oracle_attend(kv, nb, rel, w_q, H):
    S_from, B, two_dim = kv.shape
    dim = two_dim // 2
    D = dim // H
    q = (rel @ w_q.t()).reshape(*rel.shape[:2], 1, H, D)
    kvr = kv.float().reshape(S_from, B, 2, H, D).permute(2, 0, 1, 3, 4)
    kk, vv = kvr[:, nb]
    a = torch.softmax((q * kk).sum(-1, keepdim=True) * D ** -0.5, dim=1)
    return (a * vv).sum(1).reshape(nb.shape[0], B, dim)


def dev_tiles(t):
    return {key: (val.to(DEV) if torch.is_tensor(val) else val) for key, val in t.items()}


@pytest.mark.parametrize("cfg", [(48, 25, 8, True, 1, 256, 4, 24, 80, 32), (48, 25, 8, False, 3, 768, 12, 20, 96, 32),
                                 (24, 13, 4, True, 2, 512, 8, 8, 80, 32), (48, 25, 8, True, 1, 256, 4, 32, 48, 3),
                                 (24, 13, 4, False, 2, 256, 4, 1, 16, 1), (48, 25, 8, False, 1, 512, 8, 17, 256, 32),
                                 (24, 13, 4, True, 1, 384, 6, 24, 112, 17), (24, 13, 4, False, 2, 128, 2, 12, 32, 20)])
def test_interp_attend_tiled_matches_oracle(cfg):
    """Tiles from the default packing, from small unions / few targets (many ragged tiles),
    one neighbour per target, unions up to 256 points, and dims of 384 and 128 (a last
    chunk of one head pair, a single chunk)."""
    n_lon, n_lat, nside, to_hp, B, dim, H, k, umax, tmax = cfg
    pf, pt, nb, rel = scheme(n_lon, n_lat, nside, to_hp, k)
    tiles = I.build_tiles(nb, pt, max_union=umax, max_targets=tmax)
    assert tiles["max_union"] <= umax
    g = torch.Generator().manual_seed(dim + k + 1)
    kv = torch.randn(pf.shape[0], B, 2 * dim, generator=g).bfloat16()
    w_q = torch.randn(dim, 3, generator=g)
    status = mops.status_buffer(DEV)
    out = I.interp_attend_tiled(kv.to(DEV), dev_tiles(tiles), rel.to(DEV), w_q.to(DEV), H, pf.shape[0],
                                status=status)
    torch.cuda.synchronize()
    assert mops.check_status(status) == 0
    close_rel(out, oracle_attend(kv, nb, rel, w_q, H))
    if dim % 256 == 0:
        untiled = I.interp_attend(kv.to(DEV), nb.to(DEV), rel.to(DEV), w_q.to(DEV), H, pf.shape[0])
        close_rel(out, untiled.float().cpu())


def test_tiled_bad_local_index_is_reported_not_faulted():
    pf, pt, nb, rel = scheme(24, 13, 4, True, 8)
    tiles = I.build_tiles(nb, pt)
    tiles["local"] = tiles["local"].clone()
    tiles["local"][5, 3] = 254  # planted on the host: beyond its tile's union
    kv = torch.randn(pf.shape[0], 1, 512).bfloat16()
    status = mops.status_buffer(DEV)
    out = I.interp_attend_tiled(kv.to(DEV), dev_tiles(tiles), rel.to(DEV), torch.randn(256, 3).to(DEV), 4,
                                pf.shape[0], status=status)
    torch.cuda.synchronize()
    assert status.item() & 2
    assert torch.isfinite(out.float()).all()


def test_module_above_32_neighbours_takes_untiled_kernel():
    pf, pt, nb, rel = scheme(24, 13, 4, True, 40)
    m, x, (w_q, w_kv, w_o) = module(256, 4, 40, pf, pt, nb, seed=3, B=2)
    assert m._tiles() is None
    with torch.no_grad():
        out = m(x.to(DEV))
    ref = O.cross_attention_interpolate(x, nb, rel, w_q, w_kv, w_o, 4, torch.finfo(torch.float32).eps)
    close_rel(out, ref)


def test_module_after_state_dict_load_rebuilds_tiles():
    pf, pt, nb, rel = scheme(48, 25, 8, True, 24)
    m, x, (w_q, w_kv, w_o) = module(256, 4, 24, pf, pt, nb, seed=5, B=1)
    cfg = types.SimpleNamespace(k_neighbors=24, dim=256, num_heads=4, rmsnorm_elementwise_affine=False)
    m2 = M.CrossAttentionInterpolate(cfg)
    m2.initialize_interpolation_scheme(pf, pt)
    with torch.no_grad():
        m2.neighbors.copy_(torch.roll(m2.neighbors, 1, dims=0))  # a stale table, replaced by the load
    m2._tiles()
    m2.load_state_dict(m.state_dict())
    assert m2._tile_max_union is None
    m2 = m2.to(DEV)
    for lin in (m2.to_kv, m2.to_o):
        lin.to(torch.bfloat16)
    with torch.no_grad():
        out = m2(x.to(DEV))
    ref = O.cross_attention_interpolate(x, nb, rel, w_q, w_kv, w_o, 4, torch.finfo(torch.float32).eps)
    close_rel(out, ref)


def test_tiled_attend_takes_callers_key_vectors():
    """kw_ready: key vectors (to_q.weight_h^T k_h, 0) supplied by the caller give the
    same output as the ones the call computes itself (two members)."""
    g = torch.Generator().manual_seed(4)
    dim, H = 768, 12
    w_q = torch.randn(dim, 3, generator=g).to(DEV)
    pf, pt, nb, rel = scheme(24, 13, 4, True, 8)
    kv = torch.randn(pf.shape[0], 2, 2 * dim, generator=g).bfloat16().to(DEV)
    tiles = dev_tiles(I.build_tiles(nb, pt))
    a = I.interp_attend_tiled(kv, tiles, rel.to(DEV), w_q, H, pf.shape[0])
    kw = torch.einsum("pbhd,hdc->pbhc", kv[..., :dim].float().reshape(pf.shape[0], 2, H, 64), w_q.reshape(H, 64, 3))
    kw = torch.cat([kw, torch.zeros_like(kw[..., :1])], -1).contiguous()
    b = I.interp_attend_tiled(kv, tiles, rel.to(DEV), None, H, pf.shape[0], kw=kw)
    close_rel(a, b.float().cpu(), max_rel=1e-2, mean_rel=1e-4)


def test_linear_and_row_rms():
    g = torch.Generator().manual_seed(1)
    a = torch.randn(1000, 768, generator=g).bfloat16()
    w = (torch.randn(1536, 768, generator=g) * 768 ** -0.5).bfloat16()
    rinv = I.row_rms(a.to(DEV), 1e-6)
    torch.testing.assert_close(rinv.cpu(), torch.rsqrt(a.float().pow(2).mean(-1) + 1e-6), rtol=1e-5, atol=0)
    out = I.linear(a.to(DEV), w.to(DEV), rinv)
    close_rel(out, (a.float() @ w.float().t()) * rinv.cpu().unsqueeze(1))
    close_rel(I.linear(a.to(DEV), w.to(DEV)), a.float() @ w.float().t())


def module(dim, H, k, pf, pt, nb, seed, B):
    cfg = types.SimpleNamespace(k_neighbors=k, dim=dim, num_heads=H, rmsnorm_elementwise_affine=False)
    m = M.CrossAttentionInterpolate(cfg)
    x, w_q, w_kv, w_o = GU.draw_interp_inputs(pf.shape[0], B, dim, seed)
    with torch.no_grad():
        m.to_q.weight.copy_(w_q)
        m.to_kv.weight.copy_(w_kv)
        m.to_o.weight.copy_(w_o)
    m._set_scheme(nb, pf, pt)
    m = m.to(DEV)
    for lin in (m.to_kv, m.to_o):
        lin.to(torch.bfloat16)
    return m, x, (w_q, w_kv, w_o)


@pytest.mark.parametrize("cfg", [(48, 25, 8, True, 2, 256, 4, 24), (48, 25, 8, False, 1, 768, 12, 20)])
def test_module_matches_oracle(cfg):
    n_lon, n_lat, nside, to_hp, B, dim, H, k = cfg
    pf, pt, nb, rel = scheme(n_lon, n_lat, nside, to_hp, k)
    m, x, (w_q, w_kv, w_o) = module(dim, H, k, pf, pt, nb, seed=dim + B, B=B)
    with torch.no_grad():
        out = m(x.to(DEV))
    assert out.shape == (pt.shape[0], B, dim) and out.dtype == torch.bfloat16
    ref = O.cross_attention_interpolate(x, nb, rel, w_q, w_kv, w_o, H, torch.finfo(torch.float32).eps)
    close_rel(out, ref)


@pytest.mark.parametrize("name", GU.interp_fixture_names())
def test_module_matches_reference_fixture(name):
    """Against primitives.CrossAttentionInterpolate itself, with its BallTree neighbours and
    its fp32 RMSNorm epsilon (the fixture ran in fp32)."""
    d = GU.load_interp(name)
    ll, hp = GU.interp_grids(d["n_lon"], d["n_lat"], d["nside"])
    pf, pt = (ll, hp) if d["to_hp"] else (hp, ll)
    nb = torch.from_numpy(d["neighbors"]).long()
    m, x, _ = module(d["dim"], d["H"], d["k"], pf, pt, nb, d["seed"], d["B"])
    m.kv_norm.eps = torch.finfo(torch.float32).eps
    with torch.no_grad():
        out = m(x.to(DEV)).float().cpu()
    rows = torch.from_numpy(d["rows"]).long()
    close_rel(out[rows], GU.t(d["out_rows"]))


def test_full_size_ll_to_healpix():
    """The model's own sizes: 240 x 121 lat-lon points to HEALPix nside 64 (49,152 targets),
    dim 768, 12 heads, 24 neighbours, against the oracle on all targets."""
    pf, pt, nb, rel = scheme(240, 121, 64, True, 24)
    m, x, (w_q, w_kv, w_o) = module(768, 12, 24, pf, pt, nb, seed=7, B=1)
    with torch.no_grad():
        out = m(x.to(DEV))
    ref = O.cross_attention_interpolate(x, nb, rel, w_q, w_kv, w_o, 12, torch.finfo(torch.float32).eps)
    close_rel(out, ref)


def test_bad_neighbour_is_reported_not_faulted():
    pf, pt, nb, rel = scheme(24, 13, 4, True, 8)
    nb = nb.clone()
    nb[5, 3] = 10 ** 6  # planted on the host: out of range
    kv = torch.randn(pf.shape[0], 1, 512).bfloat16()
    status = mops.status_buffer(DEV)
    I.interp_attend(kv.to(DEV), nb.to(DEV), rel.to(DEV), torch.randn(256, 3).to(DEV), 4, pf.shape[0], status=status)
    torch.cuda.synchronize()
    assert status.item() & 2
