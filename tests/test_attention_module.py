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
