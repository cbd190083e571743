"""The CPU oracle against fixtures produced by running the reference code itself
(tests/golden/make_golden.py). This pins the oracle before it is trusted as the
checker of the CUDA path."""
import pytest
import torch

from oracle import bsa_oracle as O
from tests import golden_util as GU

NAMES = GU.fixture_names()


def test_fixtures_present():
    assert len(NAMES) >= 3


@pytest.mark.parametrize("name", NAMES)
def test_rope_and_pool_bit_exact(name):
    d = GU.load(name)
    x = GU.inputs(d)
    rows = torch.from_numpy(d["rows"]).long()
    # RoPE.forward of the reference == oracle.rope_apply, bit for bit (bf16 -> fp16 storage is exact here)
    assert torch.equal(x["q"][:, rows].float().half().float(), GU.t(d["q_rot_rows"]))
    assert torch.equal(x["k"][:, rows].float().half().float(), GU.t(d["k_rot_rows"]))
    # reference einops mean-pool == oracle.pool_mean
    assert torch.equal(O.pool_mean(x["q"], d["bs"]).float(), GU.t(d["q_cmp"]))
    assert torch.equal(O.pool_mean(x["k"], d["bs"]).float(), GU.t(d["k_cmp"]))


@pytest.mark.parametrize("name", NAMES)
def test_topk_matches_reference(name):
    d = GU.load(name)
    x = GU.inputs(d)
    qc, kc = O.pool_mean(x["q"], d["bs"]), O.pool_mean(x["k"], d["bs"])
    idx = O.attn_topk(qc, kc, d["K"])
    ref = torch.from_numpy(d["block_indices"]).long()
    ok, ndiff = O.topk_matches(idx, ref, O.topk_scores(qc, kc))
    assert ok, f"{ndiff} rows differ beyond score ties"


@pytest.mark.parametrize("name", NAMES)
def test_branches_and_combine_match_reference(name):
    d = GU.load(name)
    x = GU.inputs(d)
    rows = torch.from_numpy(d["rows"]).long()
    idx = torch.from_numpy(d["block_indices"]).long()
    parts = {}
    out = O.mosaic_attn_func(x["q"], x["k"], x["v"], x["w"], d["bas"], d["bs"], d["K"], False,
                             block_indices=idx, parts=parts)
    # fp32 vs fp32 (fp16 storage) for the dense branches
    torch.testing.assert_close(parts["o_ba"][:, rows], GU.t(d["o_ba_rows"]), atol=2e-3, rtol=2e-3)
    o_cmp_small = O.dense_attention(O.pool_mean(x["q"], d["bs"]), O.pool_mean(x["k"], d["bs"]),
                                    O.pool_mean(x["v"], d["bs"]))
    torch.testing.assert_close(o_cmp_small, GU.t(d["o_cmp"]), atol=2e-3, rtol=2e-3)
    # the reference sparse branch is the Triton kernel, which rounds q*scale*log2e and P to bf16
    diff = (parts["o_slc"][:, rows] - GU.t(d["o_slc_rows"])).abs()
    assert diff.max() < 2e-2 and diff.mean() < 2e-3, (diff.max(), diff.mean())
    diff = (out[:, rows] - GU.t(d["out_rows"])).abs()
    assert diff.max() < 2e-2 and diff.mean() < 2e-3, (diff.max(), diff.mean())
    # whole-tensor sums (fp64) of the reference outputs
    for key, val in (("out_sums", out), ("o_ba_sums", parts["o_ba"]), ("o_slc_sums", parts["o_slc"])):
        s = val.double().sum(dim=(1, 3))
        torch.testing.assert_close(s, torch.from_numpy(d[key]), atol=0.05 * d["N"] ** 0.5, rtol=1e-3)


@pytest.mark.parametrize("name", NAMES)
def test_sparse_lse_and_modes_match_reference(name):
    d = GU.load(name)
    x = GU.inputs(d)
    rows = torch.from_numpy(d["rows"]).long()
    idx = torch.from_numpy(d["block_indices"]).long()
    _, lse = O.sparse_attention(x["q"], x["k"], x["v"], idx, d["bs"], return_lse=True)
    assert (lse[:, rows] - GU.t(d["lse_rows"])).abs().max() < 3e-2
    out_nocmp = O.mosaic_attn_func(x["q"], x["k"], x["v"], x["w"], d["bas"], d["bs"], d["K"], False, True,
                                   block_indices=idx)
    diff = (out_nocmp[:, rows] - GU.t(d["out_nocmp_rows"])).abs()
    assert diff.max() < 2e-2 and diff.mean() < 2e-3
    out_k0 = O.mosaic_attn_func(x["q"], x["k"], x["v"], x["w"], d["bas"], d["bs"], 0, False)
    torch.testing.assert_close(out_k0[:, rows], GU.t(d["out_k0_rows"]), atol=2e-3, rtol=2e-3)


def test_topk_checker_rejects_wrong_selection():
    # a mistake planted in the oracle's output must be caught by the parity checker
    d = GU.load(NAMES[0])
    x = GU.inputs(d)
    qc, kc = O.pool_mean(x["q"], d["bs"]), O.pool_mean(x["k"], d["bs"])
    sc = O.topk_scores(qc, kc)
    idx = O.attn_topk(qc, kc, d["K"])
    bad = idx.clone()
    worst = sc.float().argmin(dim=-1)
    bad[..., -1] = worst
    ok, _ = O.topk_matches(bad, idx, sc)
    assert not ok


# ----------------------------------------------------------------------------- backward
BWD_NAMES = GU.bwd_fixture_names()


def test_bwd_fixtures_present():
    assert len(BWD_NAMES) >= 2


@pytest.mark.parametrize("name", BWD_NAMES)
def test_backward_matches_reference(name):
    """oracle.sparse_attention_bwd against the reference's two Triton backward kernels.
    The reference rounds q*scale*log2e, P and dS to bf16 before its dots, hence the
    bf16-level tolerance; one fixture repeats a block inside selections, so this also
    pins the counting of repeats (twice for dq, once for dk / dv)."""
    d = GU.load_bwd(name)
    q, k, v, go, idx = GU.bwd_inputs(d)
    assert torch.equal(idx, torch.from_numpy(d["block_indices"]).long())
    dq, dk, dv = O.sparse_attention_bwd(q, k, v, idx, d["bs"], go)
    rows = torch.from_numpy(d["rows"]).long()
    for key, val in (("dq", dq), ("dk", dk), ("dv", dv)):
        diff = (val[:, rows] - GU.t(d[key + "_rows"])).abs()
        assert diff.max() < 3e-2 and diff.mean() < 3e-3, (key, diff.max(), diff.mean())
        s = val.double().sum(dim=(1, 3))
        torch.testing.assert_close(s, torch.from_numpy(d[key + "_sums"]), atol=0.5, rtol=2e-2)


def test_backward_oracle_is_the_gradient_of_the_forward_oracle():
    """With distinct selections the restated backward is autograd's gradient of the
    forward restatement; with a repeated block only dq still is (dk / dv count the
    repeat once, like the reference's boolean block mask)."""
    torch.manual_seed(0)
    B, N, Hq, Hk, bs, K = 2, 256, 8, 2, 64, 3
    q, k, v, go = torch.randn(B, N, Hq, 64), torch.randn(B, N, Hk, 64), torch.randn(B, N, Hk, 64), \
        torch.randn(B, N, Hq, 64)
    nb = N // bs
    idx = torch.stack([torch.randperm(nb)[:K] for _ in range(B * nb * Hk)]).reshape(B, nb, Hk, K)
    for repeat in (False, True):
        if repeat:
            idx[..., 1] = idx[..., 0]
        qa, ka, va = (t.clone().requires_grad_() for t in (q, k, v))
        O.sparse_attention(qa, ka, va, idx, bs).backward(go)
        dq, dk, dv = O.sparse_attention_bwd(q, k, v, idx, bs, go)
        torch.testing.assert_close(dq, qa.grad, atol=1e-5, rtol=1e-5)
        if not repeat:
            torch.testing.assert_close(dk, ka.grad, atol=1e-5, rtol=1e-5)
            torch.testing.assert_close(dv, va.grad, atol=1e-5, rtol=1e-5)
        else:
            assert (dk - ka.grad).abs().max() > 1e-2


# ----------------------------------------------------------------------------- attention block
BLOCK_NAMES = GU.block_fixture_names()


def test_block_fixtures_present():
    assert len(BLOCK_NAMES) >= 2


@pytest.mark.parametrize("name", BLOCK_NAMES)
def test_attention_block_matches_reference(name):
    """oracle.mosaic_attention against primitives.MosaicAttention.forward run on the same
    seeded weights (projections, RoPE, strategy gates, attention, to_o; B = 2 in one
    fixture, so the sequence-first rearranges are pinned too)."""
    d = GU.load_block(name)
    x, w_q, w_k, w_v, w_g, w_o = GU.draw_block_inputs(d["S"], d["B"], d["dim"], d["Hq"], d["Hk"], d["seed"])
    cos, sin = O.rope_tables(O.healpix_grid(int(round((d["S"] / 12) ** 0.5))))
    idx = torch.from_numpy(d["block_indices"]).long()
    out = O.mosaic_attention(x, w_q, w_k, w_v, w_g, w_o, d["Hq"], d["Hk"], cos, sin, d["bas"], d["bs"], d["K"],
                             d["block_attn_only"], d["no_compression"], block_indices=idx)
    rows = torch.from_numpy(d["rows"]).long()
    diff = (out[rows] - GU.t(d["out_rows"])).abs()
    assert diff.max() < 1e-2 and diff.mean() < 1e-3, (diff.max(), diff.mean())
    torch.testing.assert_close(out.double().sum(dim=(0, 2)), torch.from_numpy(d["out_sums"]), atol=1.0, rtol=1e-2)


# ----------------------------------------------------------------------------- interpolation
INTERP_NAMES = GU.interp_fixture_names()


def test_interp_fixtures_present():
    assert len(INTERP_NAMES) >= 2


def _interp_case(d):
    from mosaic_b200 import interp as I
    ll, hp = GU.interp_grids(d["n_lon"], d["n_lat"], d["nside"])
    pf, pt = (ll, hp) if d["to_hp"] else (hp, ll)
    nb = torch.from_numpy(d["neighbors"]).long()
    rel = torch.nn.functional.normalize(I.rad_to_xyz(pt).unsqueeze(1) - I.rad_to_xyz(pf)[nb], dim=-1)
    return pf, pt, nb, rel


@pytest.mark.parametrize("name", INTERP_NAMES)
def test_cross_attention_interpolate_matches_reference(name):
    """oracle.cross_attention_interpolate against primitives.CrossAttentionInterpolate
    run with its own BallTree neighbours (both grid directions, batch 2 in one)."""
    d = GU.load_interp(name)
    pf, pt, nb, rel = _interp_case(d)
    x, w_q, w_kv, w_o = GU.draw_interp_inputs(pf.shape[0], d["B"], d["dim"], d["seed"])
    out = O.cross_attention_interpolate(x, nb, rel, w_q, w_kv, w_o, d["H"], torch.finfo(torch.float32).eps)
    rows = torch.from_numpy(d["rows"]).long()
    diff = (out[rows] - GU.t(d["out_rows"])).abs()
    assert diff.max() < 3e-3 and diff.mean() < 3e-4, (diff.max(), diff.mean())
    torch.testing.assert_close(out.double().sum(dim=(0, 2)), torch.from_numpy(d["out_sums"]), atol=1e-2, rtol=1e-4)


@pytest.mark.parametrize("name", INTERP_NAMES)
def test_neighbour_search_matches_balltree_up_to_ties(name):
    """mosaic_b200.interp.knn_neighbors (exact search by unit-vector dot product) against
    the reference's BallTree haversine query: per target the same multiset of distances
    (the grids are symmetric, so equidistant points may be swapped at the k-th place)."""
    from mosaic_b200 import interp as I
    d = GU.load_interp(name)
    pf, pt, nb, _ = _interp_case(d)
    mine = I.knn_neighbors(pf, pt, d["k"])
    a, b = I.rad_to_xyz(pt.double()), I.rad_to_xyz(pf.double())
    dist = lambda idx: torch.sort((a.unsqueeze(1) * b[idx]).sum(-1), 1).values
    assert (dist(mine) - dist(nb)).abs().max() < 1e-12
    assert (torch.sort(mine, 1).values == torch.sort(nb, 1).values).all(1).float().mean() > 0.9


# ----------------------------------------------------------------------------- HEALPix down/upsampling
UPDOWN_NAMES = GU.updown_fixture_names()


def test_updown_fixtures_present():
    assert len(UPDOWN_NAMES) >= 3


def updown_oracle(d):
    """The oracle's forward of a down/upsampling fixture case (fp32, RMSNorm epsilon of
    the fp32 run the fixture made)."""
    fine, coarse = max(d["nside_before"], d["nside_after"]), min(d["nside_before"], d["nside_after"])
    F = (fine // coarse) ** 2
    rel = O.healpix_updown_rel_pos(fine, coarse)
    x, sc, w_x, w_pos, w_norm = GU.draw_updown_inputs(d["kind"], 12 * coarse ** 2, F, d["B"], d["c_in"], d["c_out"],
                                                      d["affine"], d["seed"])
    eps = torch.finfo(torch.float32).eps
    if d["kind"] == "down":
        return rel, O.healpix_downsample(x, w_x, w_pos, rel, eps, w_norm)
    return rel, O.healpix_upsample(x, sc, w_x, w_pos, rel, eps, w_norm)


@pytest.mark.parametrize("name", UPDOWN_NAMES)
def test_healpix_updown_matches_reference(name):
    """oracle.healpix_downsample / healpix_upsample and healpix_updown_rel_pos against
    primitives.HEALPixDownsample / HEALPixUpsample (factor 4 and 16, batch 1 and 2,
    with and without the affine RMSNorm)."""
    d = GU.load_updown(name)
    rel, out = updown_oracle(d)
    torch.testing.assert_close(rel, torch.from_numpy(d["rel_pos"]), atol=1e-5, rtol=1e-5)
    flat = out.reshape(-1, out.shape[-1])
    diff = (flat[torch.from_numpy(d["rows"]).long()] - GU.t(d["out_rows"])).abs()
    assert diff.max() < 3e-3 and diff.mean() < 3e-4, (diff.max(), diff.mean())
    torch.testing.assert_close(out.double().sum(dim=(0, 2)), torch.from_numpy(d["out_sums"]), atol=1e-2, rtol=1e-4)


def test_sampled_oracle_equals_full_oracle_on_its_windows():
    """The CPU baseline's sample (global part once + chosen windows) computes exactly the
    full oracle's rows of those windows."""
    x = O.make_inputs(1, 3072, 4, 1, seed=0, rope=False)
    full = O.mosaic_attn_func(x["q"], x["k"], x["v"], x["w"], 1024, 64, 8, False)
    s = O.mosaic_attn_func_sample(x["q"], x["k"], x["v"], x["w"], 1024, 64, 8, windows=[0, 2])
    assert torch.equal(torch.cat([full[:, :1024], full[:, 2048:]], 1), s)
