"""Parity of the attention block (mosaic_attn_qkv_proj, mosaic_attn_out_proj and the
MosaicAttention module) with the CPU oracle's restatement of
primitives.MosaicAttention.forward and with the fixtures of the reference module.

Tolerances: the projections are bf16 GEMMs with fp32 accumulation whose outputs are
rounded to bf16, as the reference's bf16 Linear layers; they are compared with the
fp32 oracle at max-abs 2e-2 and mean-abs 2e-3 of the output's largest magnitude, the
gates (softmax weights in [0, 1]) at 1e-2 / 1e-3 absolute."""
import types

import pytest
import torch

import mosaic_b200 as M
from mosaic_b200 import attention as A
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


def tables(S):
    return O.rope_tables(O.healpix_grid(int(round((S / 12) ** 0.5))))


@pytest.mark.parametrize("cfg", [
    (3072, 1, 768, 12, 3, True),     # the S1 stage's dims on a shorter sequence
    (3072, 1, 1024, 16, 4, True),    # stage 2
    (3072, 1, 1280, 20, 5, True),    # bottleneck (3 Hq = 60 gate columns)
    (768, 2, 256, 4, 1, True),       # batch 2: sequence-first input rows (s, b)
    (700, 1, 512, 8, 2, False),      # rows not a multiple of 128, no gates
])
def test_qkv_projection_matches_oracle(cfg):
    S, B, dim, Hq, Hk, gates = cfg
    x, w_q, w_k, w_v, w_g, _ = GU.draw_block_inputs(S, B, dim, Hq, Hk, seed=S + dim)
    rope = S % 12 == 0 and round((S / 12) ** 0.5) ** 2 * 12 == S
    cos, sin = tables(S) if rope else (None, None)
    w = torch.cat([w_q, w_k, w_v] + ([w_g] if gates else []))
    status = mops.status_buffer(DEV)
    q, k, v, g = A.qkv_projection(x.to(DEV), w.to(DEV), Hq, Hk, None if cos is None else cos.to(DEV),
                                  None if sin is None else sin.to(DEV), with_gates=gates, status=status)
    torch.cuda.synchronize()
    assert mops.check_status(status) == 0
    rq, rk, rv, rg = O.attention_projections(x, w_q, w_k, w_v, w_g if gates else None, Hq, Hk, cos, sin)
    close_rel(q, rq)
    close_rel(k, rk)
    close_rel(v, rv)
    if gates:
        d = (g.float().cpu() - rg).abs()
        assert d.max() < 1e-2 and d.mean() < 1e-3, (d.max(), d.mean())
        torch.testing.assert_close(g.float().sum(0).cpu(), torch.ones(B, S, Hq), atol=1e-2, rtol=0)


def test_rope_epilogue_matches_reference_rounding():
    """RoPE in the epilogue rotates the bf16-rounded projection exactly as RoPE.forward
    does: against the oracle's rotation of the kernel's own unrotated output, the rotated
    q and k are bit-identical."""
    S, B, dim, Hq, Hk = 3072, 1, 768, 12, 3
    x, w_q, w_k, w_v, _, _ = GU.draw_block_inputs(S, B, dim, Hq, Hk, seed=5)
    cos, sin = tables(S)
    w = torch.cat([w_q, w_k, w_v]).to(DEV)
    q0, k0, _, _ = A.qkv_projection(x.to(DEV), w, Hq, Hk, with_gates=False)
    q1, k1, _, _ = A.qkv_projection(x.to(DEV), w, Hq, Hk, cos.to(DEV), sin.to(DEV), with_gates=False)
    assert torch.equal(q1.cpu(), O.rope_apply(q0.cpu(), cos, sin))
    assert torch.equal(k1.cpu(), O.rope_apply(k0.cpu(), cos, sin))


@pytest.mark.parametrize("cfg", [(3072, 1, 768, 12), (768, 2, 256, 4), (700, 1, 512, 8)])
def test_out_projection_matches_oracle(cfg):
    S, B, dim, Hq = cfg
    g = torch.Generator().manual_seed(S + Hq)
    attn = torch.randn(B, S, Hq, 64, generator=g).bfloat16()
    w_o = (torch.randn(dim, Hq * 64, generator=g) * (Hq * 64) ** -0.5).bfloat16()
    out = A.out_projection(attn.to(DEV), w_o.to(DEV))
    ref = attn.float().permute(1, 0, 2, 3).reshape(S, B, Hq * 64) @ w_o.float().t()
    assert out.shape == (S, B, dim)
    close_rel(out, ref)


def module(S, B, dim, Hq, Hk, bas, bs, K, bao, noc, seed):
    cfg = types.SimpleNamespace(num_heads=Hq, gqa_ratio=Hq // Hk, dim=dim, qkv_compress_ratio=1, rope=True,
                                rope_theta=10000, block_attn_size=bas, sparse_block_size=bs, sparse_block_count=K)
    m = M.MosaicAttention(cfg, bao, noc)
    x, w_q, w_k, w_v, w_g, w_o = GU.draw_block_inputs(S, B, dim, Hq, Hk, seed)
    with torch.no_grad():
        m.to_q.weight.copy_(w_q)
        m.to_k.weight.copy_(w_k)
        m.to_v.weight.copy_(w_v)
        m.to_o.weight.copy_(w_o)
        if m.to_strategy_combine_mlp is not None:
            m.to_strategy_combine_mlp.weight.copy_(w_g)
    grid = O.healpix_grid(int(round((S / 12) ** 0.5)))
    m.q_rope.initialize_rope(grid)
    m.k_rope.initialize_rope(grid)
    m = m.to(DEV)  # the RoPE tables stay fp32; the Linear weights become bf16
    for lin in (m.to_q, m.to_k, m.to_v, m.to_o, m.to_strategy_combine_mlp):
        if lin is not None:
            lin.to(torch.bfloat16)
    return m, x, (w_q, w_k, w_v, w_g, w_o)


def gpu_selection(m, x):
    """The block selection the module's attention makes (same q, k as inside forward)."""
    q, k, _, _ = A.qkv_projection(x.to(DEV), m._w_qkvg(), m.q_heads, m.kv_heads, m.q_rope.cos_freqs,
                                  m.q_rope.sin_freqs, with_gates=not m.block_attn_only)
    qc, kc, _ = M.block_pool(q, k, k, m.sparse_block_size)
    return M.attn_topk(qc, kc, m.sparse_block_count).cpu()


@pytest.mark.parametrize("cfg", [
    (3072, 1, 768, 12, 3, 1024, 64, 8, False, False),
    (768, 2, 512, 8, 2, 256, 128, 2, False, True),
    (3072, 1, 1024, 16, 4, 1024, 64, 4, True, False),
])
def test_mosaic_attention_module_matches_oracle(cfg):
    S, B, dim, Hq, Hk, bas, bs, K, bao, noc = cfg
    m, x, (w_q, w_k, w_v, w_g, w_o) = module(S, B, dim, Hq, Hk, bas, bs, K, bao, noc, seed=S + K)
    with torch.no_grad():
        out = m(x.to(DEV))
    idx = None if bao else gpu_selection(m, x)
    cos, sin = tables(S)
    ref = O.mosaic_attention(x, w_q, w_k, w_v, w_g, w_o, Hq, Hk, cos, sin, bas, bs, K, bao, noc, block_indices=idx)
    assert out.shape == (S, B, dim) and out.dtype == torch.bfloat16
    close_rel(out, ref)


@pytest.mark.parametrize("name", GU.block_fixture_names())
def test_mosaic_attention_module_matches_reference_fixture(name):
    """Against primitives.MosaicAttention.forward itself (fixture; same seeded weights).
    The module's top-k runs on bf16 q/k, the fixture's on fp32, so a query block whose
    selection differs inside a score tie has a different output: the comparison covers
    the sampled rows of query blocks whose selections agree (most of them)."""
    d = GU.load_block(name)
    m, x, _ = module(d["S"], d["B"], d["dim"], d["Hq"], d["Hk"], d["bas"], d["bs"], d["K"], d["block_attn_only"],
                      d["no_compression"], d["seed"])
    with torch.no_grad():
        out = m(x.to(DEV)).float().cpu()
    rows = torch.from_numpy(d["rows"]).long()
    idx_ref = torch.from_numpy(d["block_indices"]).long()
    idx = gpu_selection(m, x)
    same = (torch.sort(idx, -1).values == torch.sort(idx_ref, -1).values).all(-1).all(-1)  # [B, nb]
    keep = same[:, rows // d["bs"]].all(0)
    assert keep.float().mean() > 0.5
    ref = GU.t(d["out_rows"])
    diff = (out[rows][keep] - ref[keep]).abs()
    m_ = ref.abs().max().item()
    assert diff.max() <= 2e-2 * m_ + 1e-3 and diff.mean() <= 2e-3 * m_ + 1e-4, (diff.max(), diff.mean(), m_)
