"""Parity with the reference's own GPU code on the same B200 (baseline/reference.py loads
the reference's unmodified modules from baseline/_ref; skipped when that copy is absent).

* The reference Triton kernel ops.mosaic_attn_fwd_kernel (launched with q_tile_size 64,
  as the autotuner's q_tile_size 128 is undefined at 64-token blocks, ops.py:54-55)
  against mosaic_sparse_attn on the same selections: outputs within max-abs 2e-2 /
  mean-abs 2e-3, log-sum-exp within 3e-2 (both round q*scale*log2e or P to bf16 at
  different points).
* The reference's whole primitives.mosaic_attn_func on the GPU (flash-attn local and
  coarse branches, torch top-k, the Triton kernel) against ours: on every query block
  whose selected set is the same (the two top-k implementations may order a score tie
  differently), the same bound."""
import pytest
import torch

import mosaic_b200 as M
from baseline import reference as R
from oracle import bsa_oracle as O

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not R.available(), reason="baseline/_ref holds no reference copy")]

MAX_ABS, MEAN_ABS = 2e-2, 2e-3
DEV = "cuda"


@pytest.fixture(scope="module")
def ref():
    return R.load(torch.device(DEV))


def close(got, want, max_abs=MAX_ABS, mean_abs=MEAN_ABS):
    d = (got.float() - want.float()).abs()
    assert torch.isfinite(got.float()).all()
    assert d.max().item() <= max_abs and d.mean().item() <= mean_abs, (d.max().item(), d.mean().item())


@pytest.mark.parametrize("cfg", [(1, 3072, 4, 1, 64, 8), (1, 12288, 12, 3, 64, 24), (2, 4096, 8, 2, 128, 6),
                                 (1, 49152, 12, 3, 128, 24),
                                 # 1, 2 and 8 query heads per kv head (the Triton kernel takes any)
                                 (1, 3072, 2, 2, 64, 8), (1, 4096, 4, 2, 128, 6), (1, 3072, 8, 1, 64, 8)])
def test_sparse_attention_matches_reference_triton_kernel(ref, cfg):
    B, N, Hq, Hk, bs, K = cfg
    g = torch.Generator(device=DEV).manual_seed(N + K)
    q = torch.randn(B, N, Hq, 64, generator=g, device=DEV).bfloat16()
    k = torch.randn(B, N, Hk, 64, generator=g, device=DEV).bfloat16()
    v = torch.randn(B, N, Hk, 64, generator=g, device=DEV).bfloat16()
    nb = N // bs
    idx = torch.argsort(torch.rand(B, nb, Hk, nb, generator=g, device=DEV), dim=-1)[..., :K].contiguous()
    r_out, r_lse = ref.sparse_attn_fwd(q, k, v, idx, bs)
    out, lse = M.mosaic_sparse_attn_with_lse(q, k, v, idx, bs)
    torch.cuda.synchronize()
    close(out, r_out)
    assert (lse - r_lse).abs().max().item() < 3e-2


@pytest.mark.parametrize("cfg", [(1, 3072, 4, 1, 1024, 64, 8, torch.bfloat16),
                                 (1, 49152, 12, 3, 1024, 64, 24, torch.bfloat16),
                                 (2, 12288, 16, 4, 1024, 128, 12, torch.bfloat16),
                                 # fp16, the reference rollout's dtype: its attn_topk then scores in fp16
                                 (1, 3072, 4, 1, 1024, 64, 8, torch.float16),
                                 (1, 49152, 12, 3, 1024, 64, 24, torch.float16),
                                 # 1, 2 and 8 query heads per kv head
                                 (1, 3072, 2, 2, 1024, 64, 8, torch.bfloat16),
                                 (1, 3072, 2, 1, 1024, 64, 8, torch.bfloat16),
                                 (1, 3072, 8, 1, 1024, 64, 8, torch.bfloat16)])
def test_mosaic_attn_func_matches_reference_gpu_path(ref, cfg):
    B, N, Hq, Hk, bas, bs, K, dtype = cfg
    x = O.make_inputs(B, N, Hq, Hk, seed=N + bs, dtype=dtype, rope=True)
    q, k, v, w = (t.to(DEV) for t in (x["q"], x["k"], x["v"], x["w"]))
    r_out = ref.primitives.mosaic_attn_func(q, k, v, w, bas, bs, K, False)
    out, idx = M.mosaic_attn_func(q, k, v, w, bas, bs, K, False, return_block_indices=True)
    qc, kc = M.block_pool(q, k, v, bs)[:2]
    r_idx = ref.primitives.attn_topk(qc, kc, K)
    torch.cuda.synchronize()
    same = (torch.sort(r_idx, -1).values == torch.sort(idx, -1).values).all(-1).all(-1)  # [B, nb]
    assert same.float().mean().item() > 0.9, "selections differ on more than a tenth of the query blocks"
    rows = same.repeat_interleave(bs, dim=1)  # [B, N]
    assert out.dtype == r_out.dtype == dtype
    close(out[rows], r_out[rows])


@pytest.mark.parametrize("q_gain", [4.0, 8.0])
def test_sharp_softmax_at_least_as_accurate_as_reference_gpu_path(ref, q_gain):
    """Sharp rows (q scaled so outputs approach single v rows, |out| up to ~6): against the
    fp32 oracle the reference's own GPU path (flash-attn + its Triton kernel) reaches
    max-abs 0.028 / 0.049 at q x4 / x8 on these inputs, above the 2e-2 north-star bound;
    ours must stay within the mean bound and no worse than the reference's maximum."""
    B, N, Hq, Hk = 1, 3072, 8, 2
    x = O.make_inputs(B, N, Hq, Hk, seed=23, rope=False)
    q = (x["q"].float() * q_gain).bfloat16()
    qd, kd, vd, wd = (t.to(DEV) for t in (q, x["k"], x["v"], x["w"]))
    out, idx = M.mosaic_attn_func(qd, kd, vd, wd, 1024, 64, 8, False, return_block_indices=True)
    r_out = ref.primitives.mosaic_attn_func(qd, kd, vd, wd, 1024, 64, 8, False)
    qc, kc = O.pool_mean(q, 64), O.pool_mean(x["k"], 64)
    r_idx = ref.primitives.attn_topk(qc.to(DEV), kc.to(DEV), 8).cpu()
    d = (out.float().cpu() - O.mosaic_attn_func(q, x["k"], x["v"], x["w"], 1024, 64, 8, False,
                                                block_indices=idx.cpu())).abs()
    dr = (r_out.float().cpu() - O.mosaic_attn_func(q, x["k"], x["v"], x["w"], 1024, 64, 8, False,
                                                   block_indices=r_idx)).abs()
    assert d.mean().item() <= MEAN_ABS
    assert d.max().item() <= dr.max().item(), (d.max().item(), dr.max().item())
