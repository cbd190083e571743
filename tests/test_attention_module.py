"""The attention-block drop-in (mosaic_b200.MosaicAttention) on the CPU: parameter and
buffer names of primitives.MosaicAttention (so reference state dicts load), the RoPE
module against the oracle, and the inference-only guard. No kernel runs here."""
import types

import pytest
import torch

import mosaic_b200 as M
from oracle import bsa_oracle as O


def cfg(dim=768, heads=12):
    return types.SimpleNamespace(num_heads=heads, gqa_ratio=4, dim=dim, qkv_compress_ratio=1, rope=True,
                                 rope_theta=10000, block_attn_size=1024, sparse_block_size=64, sparse_block_count=24)


def test_state_dict_names_match_the_reference_module():
    m = M.MosaicAttention(cfg(), block_attn_only=False)
    grid = O.healpix_grid(4)
    m.q_rope.initialize_rope(grid)
    m.k_rope.initialize_rope(grid)
    keys = set(m.state_dict())
    assert keys == {"to_q.weight", "to_k.weight", "to_v.weight", "to_o.weight", "to_strategy_combine_mlp.weight",
                    "q_rope.cos_freqs", "q_rope.sin_freqs", "k_rope.cos_freqs", "k_rope.sin_freqs"}
    assert tuple(m.to_q.weight.shape) == (768, 768) and tuple(m.to_k.weight.shape) == (192, 768)
    assert tuple(m.to_strategy_combine_mlp.weight.shape) == (36, 768)
    m2 = M.MosaicAttention(cfg(), block_attn_only=True)
    assert m2.to_strategy_combine_mlp is None
    m2.load_state_dict({k: v for k, v in m.state_dict().items() if "strategy" not in k}, strict=False)


def test_rope_module_matches_oracle():
    grid = O.healpix_grid(4)
    r = M.attention.RoPE(64)
    r.initialize_rope(grid)
    cos, sin = O.rope_tables(grid)
    torch.testing.assert_close(r.cos_freqs, cos)
    x = torch.randn(2, grid.shape[0], 3, 64).bfloat16()
    torch.testing.assert_close(r(x).float(), O.rope_apply(x, cos, sin).float(), atol=0, rtol=0)


def test_forward_requiring_gradients_raises():
    m = M.MosaicAttention(cfg(dim=256, heads=4), block_attn_only=False)
    with pytest.raises(NotImplementedError):
        m(torch.randn(768, 1, 256))


def test_interpolate_module_names_and_scheme():
    from tests import golden_util as GU
    cfg_i = types.SimpleNamespace(k_neighbors=6, dim=256, num_heads=4, rmsnorm_elementwise_affine=False)
    m = M.CrossAttentionInterpolate(cfg_i)
    ll, hp = GU.interp_grids(24, 13, 4)
    m.initialize_interpolation_scheme(ll, hp)
    assert set(m.state_dict()) == {"to_q.weight", "to_kv.weight", "to_o.weight", "neighbors", "rel_pos"}
    assert tuple(m.neighbors.shape) == (192, 6) and tuple(m.rel_pos.shape) == (192, 6, 3)
    n = m.rel_pos.norm(dim=-1)  # unit vectors, or 0 where a target coincides with a source point
    assert (((n - 1).abs() < 1e-5) | (n == 0)).all() and (n == 0).float().mean() < 0.05
    with pytest.raises(NotImplementedError):
        m(torch.randn(312, 1, 256))


@pytest.mark.parametrize("grids,k,umax,tmax", [((24, 13, 4, True), 8, 80, 32), ((48, 25, 8, False), 24, 64, 16),
                                               ((24, 13, 4, False), 1, 16, 1), ((24, 13, 4, True), 32, 32, 4),
                                               ((48, 25, 8, True), 24, 256, 32)])
def test_interp_tiles_reconstruct_the_neighbour_table(grids, k, umax, tmax):
    """build_tiles: every target in exactly one tile (the order is a permutation), each
    tile's union within max_union and max_targets, sorted and duplicate-free up to the
    padding (repeats of its first point to a multiple of 16), and tile_points[local] gives
    back the neighbour table exactly."""
    from mosaic_b200 import interp as I
    from tests import golden_util as GU
    n_lon, n_lat, nside, to_hp = grids
    ll, hp = GU.interp_grids(n_lon, n_lat, nside)
    pf, pt = (ll, hp) if to_hp else (hp, ll)
    nb = I.knn_neighbors(pf, pt, k)
    t = I.build_tiles(nb, pt, max_union=umax, max_targets=tmax)
    order = torch.arange(pt.shape[0]) if t["order"] is None else t["order"].long()
    assert sorted(order.tolist()) == list(range(pt.shape[0]))
    tt, po = t["tile_targets"].long(), t["tile_point_off"].long()
    pts, loc = t["tile_points"].long(), t["local"].long()
    assert tt[0] == 0 and tt[-1] == pt.shape[0] and po[-1] == pts.numel() and t["local"].dtype == torch.uint8
    assert t["max_union"] == int((po[1:] - po[:-1]).max()) <= umax
    for i in range(tt.numel() - 1):
        ts = order[tt[i]:tt[i + 1]]
        assert 1 <= ts.numel() <= tmax
        u = pts[po[i]:po[i + 1]]
        n_uni = torch.unique(nb[ts]).numel()
        assert u.numel() % 16 == 0 and u.numel() - n_uni < 16
        assert (u[1:n_uni] > u[:n_uni - 1]).all() and (u[n_uni:] == u[0]).all()
        assert torch.equal(u[loc[ts]], nb[ts])


def test_interp_tiles_reject_bad_tables():
    from mosaic_b200 import interp as I
    with pytest.raises(ValueError):  # more neighbours than a union holds
        I.build_tiles(torch.arange(40).reshape(2, 20), None, max_union=16)
    with pytest.raises(ValueError):  # repeated neighbour
        I.build_tiles(torch.tensor([[0, 1, 2], [3, 4, 3]]), None)
    with pytest.raises(ValueError):  # union not a multiple of the mma k step
        I.build_tiles(torch.arange(6).reshape(2, 3), None, max_union=40)


@pytest.mark.parametrize("kind", ["down", "up"])
def test_updown_modules_match_the_reference_structure(kind):
    """HEALPixDownsample / HEALPixUpsample: the reference's parameters and buffer, and a
    rel_pos equal to the reference module's own (from the fixtures)."""
    from tests import golden_util as GU
    name = [n for n in GU.updown_fixture_names() if n.startswith(kind + "_")][0]
    d = GU.load_updown(name)
    cls = M.HEALPixDownsample if kind == "down" else M.HEALPixUpsample
    m = cls(d["c_in"], d["c_out"], d["nside_before"], d["nside_after"], rmsnorm_elementwise_affine=d["affine"])
    keys = {"proj_x.weight", "proj_pos.weight", "rel_pos"} | ({"norm.weight"} if d["affine"] else set())
    assert set(m.state_dict()) == keys
    F = m.factor
    fan = d["c_in"] * (F if kind == "down" else 1)
    assert tuple(m.proj_x.weight.shape) == ((d["c_out"], fan) if kind == "down" else (F * d["c_out"], fan))
    torch.testing.assert_close(m.rel_pos, torch.from_numpy(d["rel_pos"]), atol=1e-5, rtol=1e-5)
    x = torch.randn(m.rel_pos.shape[0] * (F if kind == "down" else 1), 1, d["c_in"])
    with pytest.raises(NotImplementedError):
        m(x) if kind == "down" else m(x, None)
