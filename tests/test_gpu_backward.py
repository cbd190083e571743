"""Parity of the selected-block attention backward (mosaic_sparse_attn_bwd through
the C ABI) with the CPU oracle's restatement of ops.mosaic_attn_bwd and with the
golden fixtures of the reference's own Triton backward kernels.

Tolerance: the kernels round P and dS to bf16 before their tensor-core products
and return bf16 gradients, like the reference; gradients are compared after
normalising by their largest magnitude (max-abs 2e-2, mean-abs 2e-3 of it)."""
import pytest
import torch

import mosaic_b200 as M
from mosaic_b200 import ops as mops
from oracle import bsa_oracle as O
from tests import golden_util as GU

pytestmark = pytest.mark.gpu

DEV = "cuda"


def close_grad(got, ref, max_rel=2e-2, mean_rel=2e-3):
    got = got.float().cpu()
    assert torch.isfinite(got).all(), "non-finite gradient"
    m = max(1.0, ref.abs().max().item())
    d = (got - ref.float()).abs()
    assert d.max().item() <= max_rel * m and d.mean().item() <= mean_rel * m, (d.max().item(), d.mean().item(), m)


def random_indices(B, nb, Hk, K, seed, repeat=False):
    g = torch.Generator().manual_seed(seed)
    idx = torch.stack([torch.randperm(nb, generator=g)[:K] for _ in range(B * nb * Hk)]).reshape(B, nb, Hk, K)
    if repeat:
        idx[..., -1] = idx[..., 0]
    return idx


def inputs(B, N, Hq, Hk, seed):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, N, Hq, 64, generator=g).bfloat16()
    k = torch.randn(B, N, Hk, 64, generator=g).bfloat16()
    v = torch.randn(B, N, Hk, 64, generator=g).bfloat16()
    go = torch.randn(B, N, Hq, 64, generator=g).bfloat16()
    return q, k, v, go


def gpu_bwd(q, k, v, go, idx, bs, scale=None):
    """Forward then backward on the GPU through the library; checks the status word."""
    scale = 64 ** -0.5 if scale is None else scale
    qd, kd, vd, gd, idd = (t.to(DEV) for t in (q, k, v, go, idx))
    status = mops.status_buffer(DEV)
    out, lse = mops.mosaic_attn_fwd(qd, kd, vd, idd, bs, scale, status=status)
    dq, dk, dv = mops.mosaic_attn_bwd(qd, kd, vd, out, lse, gd, scale, idd, bs, status=status)
    torch.cuda.synchronize()
    assert mops.check_status(status) == 0
    return dq, dk, dv


@pytest.mark.parametrize("cfg", [
    (1, 768, 4, 1, 64, 4),
    (2, 1024, 8, 2, 128, 3),
    (1, 3072, 12, 3, 64, 16),
    (1, 2048, 4, 1, 256, 2),
    (1, 320, 4, 1, 64, 2),    # N % 128 == 64: the last 128-key tile has one segment
    (1, 1024, 2, 2, 64, 4),   # 1 query head per kv head (an odd G: half-empty head pairs)
    (1, 1024, 4, 2, 64, 3),   # 2
    (1, 1024, 8, 1, 64, 4),   # 8: two head groups per kv head
    (1, 768, 6, 2, 64, 4),    # 3
    (1, 512, 4, 1, 64, 8),    # every block selected by every query block
    (2, 640, 8, 2, 64, 1),
])
def test_sparse_bwd_matches_oracle(cfg):
    B, N, Hq, Hk, bs, K = cfg
    q, k, v, go = inputs(B, N, Hq, Hk, seed=N + K)
    idx = random_indices(B, N // bs, Hk, K, seed=K)
    dq, dk, dv = gpu_bwd(q, k, v, go, idx, bs)
    rq, rk, rv = O.sparse_attention_bwd(q, k, v, idx, bs, go)
    close_grad(dq, rq)
    close_grad(dk, rk)
    close_grad(dv, rv)


def test_sparse_bwd_repeated_block_counts_like_the_reference():
    """A block selected twice: dq counts it twice, dk / dv once (ops.py:277-297)."""
    B, N, Hq, Hk, bs, K = 1, 1024, 8, 2, 64, 4
    q, k, v, go = inputs(B, N, Hq, Hk, seed=5)
    idx = random_indices(B, N // bs, Hk, K, seed=6, repeat=True)
    dq, dk, dv = gpu_bwd(q, k, v, go, idx, bs)
    rq, rk, rv = O.sparse_attention_bwd(q, k, v, idx, bs, go)
    close_grad(dq, rq)
    close_grad(dk, rk)
    close_grad(dv, rv)


@pytest.mark.parametrize("name", GU.bwd_fixture_names())
def test_sparse_bwd_matches_golden(name):
    """Against the reference's own Triton backward kernels (run in the interpreter)."""
    d = GU.load_bwd(name)
    q, k, v, go, idx = GU.bwd_inputs(d)
    dq, dk, dv = gpu_bwd(q, k, v, go, idx, d["bs"])
    rows = torch.from_numpy(d["rows"]).long()
    for key, val in (("dq", dq), ("dk", dk), ("dv", dv)):
        diff = (val.float().cpu()[:, rows] - GU.t(d[key + "_rows"])).abs()
        assert diff.max() < 3e-2 and diff.mean() < 3e-3, (key, diff.max().item(), diff.mean().item())


def test_unselected_blocks_get_zero_gradients():
    """Every query block selects blocks 0 and 1 only: the other keys' dk / dv are 0."""
    B, N, Hq, Hk, bs, K = 1, 1024, 4, 1, 64, 2
    q, k, v, go = inputs(B, N, Hq, Hk, seed=9)
    idx = torch.tensor([0, 1]).expand(B, N // bs, Hk, K).contiguous()
    dq, dk, dv = gpu_bwd(q, k, v, go, idx, bs)
    assert torch.count_nonzero(dk[:, 2 * bs:]) == 0 and torch.count_nonzero(dv[:, 2 * bs:]) == 0
    rq, rk, rv = O.sparse_attention_bwd(q, k, v, idx, bs, go)
    close_grad(dq, rq)
    close_grad(dk, rk)
    close_grad(dv, rv)


def test_sparse_bwd_is_deterministic():
    B, N, Hq, Hk, bs, K = 1, 2048, 8, 2, 64, 8
    q, k, v, go = inputs(B, N, Hq, Hk, seed=11)
    idx = random_indices(B, N // bs, Hk, K, seed=12)
    a = gpu_bwd(q, k, v, go, idx, bs)
    b = gpu_bwd(q, k, v, go, idx, bs)
    for x, y in zip(a, b):
        assert torch.equal(x, y)


def test_autograd_through_mosaic_sparse_attn():
    """mosaic_sparse_attn(...).backward() gives the library's gradients, in the inputs' dtype."""
    B, N, Hq, Hk, bs, K = 1, 768, 8, 2, 64, 3
    q, k, v, go = inputs(B, N, Hq, Hk, seed=13)
    idx = random_indices(B, N // bs, Hk, K, seed=14)
    for dt in (torch.bfloat16, torch.float32):
        qa, ka, va = (t.to(DEV, dt).requires_grad_() for t in (q, k, v))
        out = M.mosaic_sparse_attn(qa, ka, va, idx.to(DEV), bs)
        out.backward(go.to(DEV, dt))
        assert qa.grad.dtype == dt and ka.grad.dtype == dt
        dq, dk, dv = gpu_bwd(q, k, v, go, idx, bs)
        assert torch.equal(qa.grad.bfloat16(), dq) and torch.equal(ka.grad.bfloat16(), dk)
        assert torch.equal(va.grad.bfloat16(), dv)


def test_no_lse_is_kept_without_grad():
    """Inference calls keep nothing for a backward."""
    B, N, Hq, Hk, bs, K = 1, 512, 4, 1, 64, 2
    q, k, v, _ = inputs(B, N, Hq, Hk, seed=15)
    idx = random_indices(B, N // bs, Hk, K, seed=16)
    out = M.mosaic_sparse_attn(*(t.to(DEV) for t in (q, k, v, idx)), bs)
    assert out.grad_fn is None


def test_sparse_bwd_bad_index_is_reported_not_faulted():
    B, N, Hq, Hk, bs, K = 1, 512, 4, 1, 64, 2
    q, k, v, go = inputs(B, N, Hq, Hk, seed=17)
    idx = random_indices(B, N // bs, Hk, K, seed=18)
    qd, kd, vd, gd, idd = (t.to(DEV) for t in (q, k, v, go, idx))
    out, lse = mops.mosaic_attn_fwd(qd, kd, vd, idd, bs, 0.125)
    idd[0, 2, 0, 1] = 10_000  # planted on the host side: out of range
    status = mops.status_buffer(DEV)
    mops.mosaic_attn_bwd(qd, kd, vd, out, lse, gd, 0.125, idd, bs, status=status)
    torch.cuda.synchronize()
    assert status.item() & 2


def test_sparse_bwd_full_size_linearity():
    """At the benchmark's selected-branch size (N = 49152, 12 / 3 heads, bs 64, K 24)
    the gradients are linear in grad_out: g(2 a + b) = 2 g(a) + g(b) up to bf16
    rounding, and finite."""
    B, N, Hq, Hk, bs, K = 1, 49152, 12, 3, 64, 24
    g = torch.Generator(device=DEV).manual_seed(19)
    q, k, v = (torch.randn(B, N, h, 64, device=DEV, generator=g).bfloat16() for h in (Hq, Hk, Hk))
    ga = torch.randn(B, N, Hq, 64, device=DEV, generator=g).bfloat16()
    gb = torch.randn(B, N, Hq, 64, device=DEV, generator=g).bfloat16()
    idx = random_indices(B, N // bs, Hk, K, seed=20).to(DEV)
    status = mops.status_buffer(DEV)
    out, lse = mops.mosaic_attn_fwd(q, k, v, idx, bs, 0.125, status=status)
    ra = mops.mosaic_attn_bwd(q, k, v, out, lse, ga, 0.125, idx, bs, status=status)
    rb = mops.mosaic_attn_bwd(q, k, v, out, lse, gb, 0.125, idx, bs, status=status)
    rc = mops.mosaic_attn_bwd(q, k, v, out, lse, (2 * ga.float() + gb.float()).bfloat16(), 0.125, idx, bs,
                              status=status)
    torch.cuda.synchronize()
    assert mops.check_status(status) == 0
    for a, b, c in zip(ra, rb, rc):
        assert torch.isfinite(c.float()).all()
        expect = 2 * a.float() + b.float()
        m = expect.abs().max().item()
        d = (c.float() - expect).abs()
        assert d.max().item() <= 3e-2 * m and d.mean().item() <= 3e-3 * m, (d.max().item(), d.mean().item(), m)


def test_backward_head_dim_32():
    """The gradient through the zero-padding of a head_dim below 64 (pad_head_dim)."""
    B, N, Hq, Hk, D, bs = 1, 1024, 4, 1, 32, 64
    g = torch.Generator().manual_seed(32)
    q, k, v, go = (torch.randn(B, N, h, D, generator=g).bfloat16() for h in (Hq, Hk, Hk, Hq))
    sel = torch.stack([torch.randperm(N // bs, generator=g)[:4] for _ in range(N // bs)]).reshape(B, N // bs, Hk, 4)
    qa, ka, va = (t.cuda().requires_grad_() for t in (q, k, v))
    out = M.mosaic_sparse_attn(qa, ka, va, sel.cuda(), bs)
    assert out.shape == (B, N, Hq, D)
    out.backward(go.cuda())
    torch.cuda.synchronize()
    for got, ref in zip((qa.grad, ka.grad, va.grad), O.sparse_attention_bwd(q, k, v, sel, bs, go)):
        assert got.shape == ref.shape
        m = max(1.0, ref.abs().max().item())
        e = (got.float().cpu() - ref).abs()
        assert e.max() <= 2e-2 * m and e.mean() <= 2e-3 * m, (e.max().item(), e.mean().item())
