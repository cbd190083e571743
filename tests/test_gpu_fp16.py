"""The native fp16 path: the reference's production dtype. Its rollout runs under
torch.autocast(float16) (inference.py:59,379), so attn_topk pools, scores and averages
in fp16 (primitives.py:37-49: every tensor op rounds its result to fp16) and the
local / coarse branches run flash-attn in fp16. Here fp16 inputs keep fp16 through
every kernel: pooled means rounded to fp16, per-head scores and their group mean
rounded to fp16, attention operands fp16 on the tensor core.

Checks, against the oracle run on the same fp16 tensors (its rounding points follow
the input dtype): RoPE bit-exact; pooled means within one fp16 ulp (fp32 sums of 64
fp16 values are order-dependent, and the reference's own CUDA reduction has its own
order); top-k exact up to 1e-3-relative ties; outputs (fp16, returned in q's dtype)
within max-abs 2e-2 / mean-abs 2e-3 at C1, S2 and the full S1 size; the drop-in
entry points (mosaic_sparse_attn, block_attention, attn_topk) in fp16."""
import pytest
import torch

import mosaic_b200 as M
from mosaic_b200 import ops as mops
from oracle import bsa_oracle as O

pytestmark = pytest.mark.gpu

MAX_ABS, MEAN_ABS = 2e-2, 2e-3
DEV = "cuda"
F16 = torch.float16


def close(got, ref, max_abs=MAX_ABS, mean_abs=MEAN_ABS):
    d = (got.float().cpu() - ref.float().cpu()).abs()
    assert torch.isfinite(got.float()).all(), "non-finite output"
    assert d.max().item() <= max_abs and d.mean().item() <= mean_abs, (d.max().item(), d.mean().item())


def within_one_ulp(got, ref):
    """|got - ref| <= one fp16 ulp of ref, elementwise; returns the fraction that is exact."""
    g, r = got.float().cpu(), ref.float().cpu()
    ulp = torch.where(r.abs() >= 2 ** -14, 2.0 ** (torch.floor(torch.log2(r.abs().clamp_min(2 ** -14))) - 10),
                      torch.full_like(r, 2.0 ** -24))
    assert ((g - r).abs() <= ulp).all(), (g - r).abs().max().item()
    return (g == r).float().mean().item()


def cuda(*ts):
    return [t.to(DEV) if t is not None else None for t in ts]


@pytest.mark.parametrize("cfg", [(1, 3072, 4, 1, 64), (1, 12288, 16, 4, 64), (2, 3072, 8, 2, 128)])
def test_pool_fp16(cfg):
    B, N, Hq, Hk, bs = cfg
    x = O.make_inputs(B, N, Hq, Hk, seed=31, dtype=F16, rope=False)
    qc, kc, vc = M.block_pool(*cuda(x["q"], x["k"], x["v"]), bs)
    assert qc.dtype == F16
    exact = [within_one_ulp(g, O.pool_mean(t, bs)) for g, t in ((qc, x["q"]), (kc, x["k"]), (vc, x["v"]))]
    assert min(exact) > 0.99, exact


def test_rope_pool_fp16_bit_exact_rotation():
    x = O.make_inputs(1, 3072, 12, 3, seed=32, dtype=F16, rope=True)
    q, k, v, cos, sin = cuda(x["q_raw"], x["k_raw"], x["v"], x["cos"], x["sin"])
    qc, kc, vc, q_rot, k_rot = M.block_pool(q, k, v, 64, rope_tables=(cos, sin))
    assert q_rot.dtype == F16
    assert torch.equal(q_rot.cpu(), x["q"]) and torch.equal(k_rot.cpu(), x["k"])
    within_one_ulp(qc, O.pool_mean(x["q"], 64))


@pytest.mark.parametrize("cfg", [(1, 48, 4, 1, 8), (1, 768, 12, 3, 24), (2, 192, 16, 4, 20), (1, 3072, 12, 3, 24),
                                 (1, 2600, 8, 4, 32)])
def test_topk_fp16_rounding_points(cfg):
    """Scores rounded to fp16 (not bf16): both the mma.sync kernel (< 2048 blocks) and
    the tcgen05 kernel (from 2048 blocks on)."""
    B, nb, Hq, Hk, K = cfg
    g = torch.Generator().manual_seed(nb + 1)
    qc = (torch.randn(B, nb, Hq, 64, generator=g) * 0.3).to(F16)
    kc = (torch.randn(B, nb, Hk, 64, generator=g) * 0.3).to(F16)
    idx = M.attn_topk(*cuda(qc, kc), K).cpu()
    scores = O.topk_scores(qc, kc)
    assert scores.dtype == F16
    ok, ndiff = O.topk_matches(idx, O.attn_topk(qc, kc, K), scores)
    assert ok, f"{ndiff} rows differ beyond ties"
    # fp16 rounding resolves scores that bf16 rounding would merge: the fp16 selection
    # differs from a bf16 one somewhere on these inputs, so the fp16 points matter
    if nb >= 768:
        idx_bf16 = O.attn_topk(qc.bfloat16(), kc.bfloat16(), K)
        assert not torch.equal(torch.sort(idx, -1).values, torch.sort(idx_bf16, -1).values)


def full_check_fp16(B, N, Hq, Hk, bas, bs, K, seed):
    x = O.make_inputs(B, N, Hq, Hk, seed=seed, dtype=F16, rope=True)
    status = mops.status_buffer(DEV)
    out, idx = M.mosaic_attn_func(*cuda(x["q"], x["k"], x["v"], x["w"]), bas, bs, K, False,
                                  return_block_indices=True, status=status)
    torch.cuda.synchronize()
    assert mops.check_status(status) == 0
    assert out.dtype == F16
    qc, kc = O.pool_mean(x["q"], bs), O.pool_mean(x["k"], bs)
    ok, ndiff = O.topk_matches(idx.cpu(), O.attn_topk(qc, kc, K), O.topk_scores(qc, kc))
    assert ok, f"{ndiff} rows differ beyond ties"
    ref = O.mosaic_attn_func(x["q"], x["k"], x["v"], x["w"], bas, bs, K, False, block_indices=idx.cpu())
    close(out, ref)


@pytest.mark.parametrize("cfg", [
    (1, 3072, 4, 1, 1024, 64, 8),      # BASELINE config 1 (C1) shapes
    (1, 12288, 16, 4, 1024, 64, 20),   # S2
    (2, 3072, 8, 2, 512, 128, 4),      # reference-preset block size 128, batch 2
])
def test_mosaic_attn_func_fp16(cfg):
    full_check_fp16(*cfg, seed=40)


def test_mosaic_attn_func_fp16_stage1_full_size():
    """BASELINE config 2 (S1) in fp16: N=49152, 12/3 heads, bs 64, K 24, window 1024."""
    full_check_fp16(1, 49152, 12, 3, 1024, 64, 24, seed=41)


def test_drop_in_entry_points_fp16():
    B, N, Hq, Hk, bs, K = 1, 3072, 8, 2, 64, 6
    x = O.make_inputs(B, N, Hq, Hk, seed=42, dtype=F16, rope=False)
    q, k, v = cuda(x["q"], x["k"], x["v"])
    g = torch.Generator().manual_seed(3)
    idx = torch.stack([torch.randperm(N // bs, generator=g)[:K] for _ in range(B * (N // bs) * Hk)])
    idx = idx.reshape(B, N // bs, Hk, K)
    out = M.mosaic_sparse_attn(q, k, v, idx.to(DEV), bs)
    assert out.dtype == F16
    close(out, O.sparse_attention(x["q"], x["k"], x["v"], idx, bs))
    loc = M.block_attention(q, k, v, 1024)
    assert loc.dtype == F16
    close(loc, O.block_attention(x["q"], x["k"], x["v"], 1024))
    qc, kc, vc = M.block_pool(q, k, v, bs)
    close(M.cmp_attention(qc, kc, vc), O.dense_attention(qc.cpu(), kc.cpu(), vc.cpu()))
