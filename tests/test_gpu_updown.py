"""Parity of the HEALPix down/upsampling layers (mosaic_healpix_downsample /
mosaic_healpix_upsample and the HEALPixDownsample / HEALPixUpsample modules) with the
CPU oracle's restatement of primitives.py:305-359 and with the fixtures of the reference
modules. Tolerance: bf16 outputs compared with the fp32 oracle at max-abs 2e-2 and
mean-abs 2e-3 of the output's largest magnitude."""
import pytest
import torch

import mosaic_b200 as M
from mosaic_b200 import ops as mops
from mosaic_b200 import updown as U
from oracle import bsa_oracle as O
from tests import golden_util as GU

pytestmark = pytest.mark.gpu
DEV = "cuda"
# torch.nn.RMSNorm with eps=None takes fp32's epsilon for bf16 inputs too
NORM_EPS = torch.finfo(torch.float32).eps


def close_rel(got, ref, max_rel=2e-2, mean_rel=2e-3):
    got = got.float().cpu()
    assert got.shape == ref.shape, (got.shape, ref.shape)
    assert torch.isfinite(got).all(), "non-finite output"
    m = max(1e-6, ref.abs().max().item())
    d = (got - ref.float()).abs()
    assert d.max().item() <= max_rel * m and d.mean().item() <= mean_rel * m, (d.max().item(), d.mean().item(), m)


def module(kind, c_in, c_out, nb, na, affine, seed, B):
    F = (max(nb, na) // min(nb, na)) ** 2
    n = 12 * min(nb, na) ** 2
    x, sc, w_x, w_pos, w_norm = GU.draw_updown_inputs(kind, n, F, B, c_in, c_out, affine, seed)
    cls = M.HEALPixDownsample if kind == "down" else M.HEALPixUpsample
    m = cls(c_in, c_out, nb, na, rmsnorm_elementwise_affine=affine)
    with torch.no_grad():
        m.proj_x.weight.copy_(w_x.float())
        m.proj_pos.weight.copy_(w_pos.float())
        if affine:
            m.norm.weight.copy_(w_norm.float())
    m = m.to(DEV)
    m.proj_x.to(torch.bfloat16)
    return m, x, sc, (w_x, w_pos, w_norm)


def oracle(kind, m, x, sc, w, eps):
    w_x, w_pos, w_norm = w
    rel = m.rel_pos.cpu()
    if kind == "down":
        return O.healpix_downsample(x, w_x, w_pos, rel, eps, w_norm)
    return O.healpix_upsample(x, sc, w_x, w_pos, rel, eps, w_norm)


@pytest.mark.parametrize("cfg", [
    ("down", 768, 1024, 64, 32, False, 1),   # the U-Net's first downsample
    ("down", 1024, 1280, 32, 16, True, 2),   # the second, two members, affine norm
    ("up", 1280, 1024, 16, 32, True, 1),     # the first upsample
    ("up", 1024, 768, 32, 64, False, 2),     # the last, two members
    ("down", 64, 128, 16, 4, False, 3),      # factor 16, three members (rows not a multiple of 128)
    ("up", 192, 640, 4, 8, True, 1),         # out_dim not a multiple of 256
])
def test_module_matches_oracle(cfg):
    kind, c_in, c_out, nb, na, affine, B = cfg
    m, x, sc, w = module(kind, c_in, c_out, nb, na, affine, seed=c_in + B, B=B)
    with torch.no_grad():
        out = m(x.to(DEV)) if kind == "down" else m(x.to(DEV), sc.to(DEV))
    assert out.dtype == torch.bfloat16
    close_rel(out, oracle(kind, m, x, sc, w, NORM_EPS))


@pytest.mark.parametrize("name", GU.updown_fixture_names())
def test_module_matches_reference_fixture(name):
    """Against primitives.HEALPixDownsample / HEALPixUpsample themselves (fp32 run, so the
    RMSNorm epsilon is fp32's)."""
    d = GU.load_updown(name)
    m, x, sc, _ = module(d["kind"], d["c_in"], d["c_out"], d["nside_before"], d["nside_after"], d["affine"],
                         d["seed"], d["B"])
    m.norm.eps = torch.finfo(torch.float32).eps
    with torch.no_grad():
        out = m(x.to(DEV)) if d["kind"] == "down" else m(x.to(DEV), sc.to(DEV))
    flat = out.float().cpu().reshape(-1, out.shape[-1])
    close_rel(flat[torch.from_numpy(d["rows"]).long()], GU.t(d["out_rows"]))


def test_upsample_without_shortcut_and_in_place():
    """shortcut=None is the projection and bias alone; out may be the shortcut's buffer."""
    m, x, sc, (w_x, w_pos, w_norm) = module("up", 256, 128, 4, 8, True, seed=9, B=2)
    xd, scd = x.to(DEV), sc.to(DEV)
    pos = m._pos_bias()
    eps = NORM_EPS
    no_sc = U.healpix_upsample(xd, None, m.proj_x.weight, pos, 4, eps, m.norm.weight)
    close_rel(no_sc, O.healpix_upsample(x, torch.zeros_like(sc), w_x, w_pos, m.rel_pos.cpu(), eps, w_norm))
    ref = U.healpix_upsample(xd, scd, m.proj_x.weight, pos, 4, eps, m.norm.weight)
    buf = scd.clone()
    from mosaic_b200 import _lib
    from mosaic_b200.ops import _ptr, _stream_ptr
    rc = _lib.load().mosaic_healpix_upsample(_ptr(xd), _ptr(buf), _ptr(m.proj_x.weight), _ptr(pos),
                                             _ptr(m.norm.weight.float().contiguous()), _ptr(buf), None,
                                             x.shape[0], 4, 2, 256, 128, float(eps), _stream_ptr(xd.device))
    assert rc == 0
    torch.cuda.synchronize()
    assert torch.equal(buf, ref)


def test_outputs_repeatable_and_rows_normalised():
    """Two runs agree to one bf16 rounding step (a row's partial sums of squares are added
    atomically, in an order that may vary); without affine every output row has mean
    square 1 up to bf16 rounding."""
    m, x, _, _ = module("down", 768, 1024, 64, 32, False, seed=3, B=1)
    with torch.no_grad():
        a = m(x.to(DEV))
        b = m(x.to(DEV))
    ms = a.float().pow(2).mean(-1)
    assert ((ms - 1).abs() < 2e-2).all()
    assert ((a.float() - b.float()).abs().max() <= 2 ** -7 * a.float().abs().max())


def test_pos_bias_follows_weight_updates():
    m, x, _, _ = module("down", 64, 128, 8, 4, False, seed=5, B=1)
    p0 = m._pos_bias().clone()
    with torch.no_grad():
        m.proj_pos.weight.mul_(2)
    assert not torch.equal(m._pos_bias(), p0)
