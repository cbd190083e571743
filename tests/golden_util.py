"""Loading of the golden fixtures (written by tests/golden/make_golden.py from the
reference code) and regeneration of their seeded inputs."""
import glob
import os

import numpy as np
import torch

from oracle import bsa_oracle as O

GOLDEN_DIR = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def fixture_names():
    """The forward fixtures."""
    return sorted(n for n in _all_names() if not n.startswith(("bwd_", "block_", "interp_", "down_", "up_")))


def bwd_fixture_names():
    """The backward fixtures (bwd_*.npz)."""
    return sorted(n for n in _all_names() if n.startswith("bwd_"))


def _all_names():
    return [os.path.basename(p)[:-4] for p in glob.glob(os.path.join(GOLDEN_DIR, "*.npz"))]


def load(name):
    z = np.load(os.path.join(GOLDEN_DIR, name + ".npz"))
    d = {k: z[k] for k in z.files}
    B, N, Hq, Hk, bs, K, bas, seed = (int(x) for x in d["meta"])
    d.update(B=B, N=N, Hq=Hq, Hk=Hk, bs=bs, K=K, bas=bas, seed=seed)
    return d


def load_bwd(name):
    z = np.load(os.path.join(GOLDEN_DIR, name + ".npz"))
    d = {k: z[k] for k in z.files}
    B, N, Hq, Hk, bs, K, seed, repeat = (int(x) for x in d["meta"])
    d.update(B=B, N=N, Hq=Hq, Hk=Hk, bs=bs, K=K, seed=seed, repeat=bool(repeat))
    return d


def bwd_inputs(d):
    """A backward fixture's inputs (q, k, v, grad_out, block_indices)."""
    return draw_bwd_inputs(d["B"], d["N"], d["Hq"], d["Hk"], d["bs"], d["K"], d["seed"], d["repeat"])


def draw_bwd_inputs(B, N, Hq, Hk, bs, K, seed, repeat):
    """Seeded bf16 inputs of a backward fixture; make_golden.py draws them with this
    function too. `repeat`: every other q block selects its first block twice."""
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, N, Hq, 64, generator=g).bfloat16()
    k = torch.randn(B, N, Hk, 64, generator=g).bfloat16()
    v = torch.randn(B, N, Hk, 64, generator=g).bfloat16()
    go = torch.randn(B, N, Hq, 64, generator=g).bfloat16()
    nb = N // bs
    idx = torch.stack([torch.randperm(nb, generator=g)[:K] for _ in range(B * nb * Hk)]).reshape(B, nb, Hk, K)
    if repeat:
        idx[:, ::2, :, 1] = idx[:, ::2, :, 0]
    return q, k, v, go, idx


def inputs(d):
    """The fixture's inputs, drawn exactly as make_golden.py drew them."""
    return O.make_inputs(d["B"], d["N"], d["Hq"], d["Hk"], seed=d["seed"], rope=True)


def t(a):
    return torch.from_numpy(np.asarray(a)).float()


def block_fixture_names():
    """The attention-block fixtures (block_*.npz)."""
    return sorted(n for n in _all_names() if n.startswith("block_"))


def load_block(name):
    z = np.load(os.path.join(GOLDEN_DIR, name + ".npz"))
    d = {k: z[k] for k in z.files}
    S, B, dim, Hq, Hk, bas, bs, K, seed, bao, noc = (int(x) for x in d["meta"])
    d.update(S=S, B=B, dim=dim, Hq=Hq, Hk=Hk, bas=bas, bs=bs, K=K, seed=seed, block_attn_only=bool(bao),
             no_compression=bool(noc))
    return d


def draw_block_inputs(S, B, dim, Hq, Hk, seed):
    """Seeded bf16 input and weights of an attention-block fixture: x [S, B, dim] ~ N(0, 1),
    weights ~ N(0, 1/dim) (to_q, to_k, to_v, gate, to_o); make_golden.py uses this too."""
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(S, B, dim, generator=g).bfloat16()
    sd = dim ** -0.5
    w_q = (torch.randn(Hq * 64, dim, generator=g) * sd).bfloat16()
    w_k = (torch.randn(Hk * 64, dim, generator=g) * sd).bfloat16()
    w_v = (torch.randn(Hk * 64, dim, generator=g) * sd).bfloat16()
    w_g = (torch.randn(3 * Hq, dim, generator=g) * sd).bfloat16()
    w_o = (torch.randn(dim, Hq * 64, generator=g) * (Hq * 64) ** -0.5).bfloat16()
    return x, w_q, w_k, w_v, w_g, w_o


def interp_fixture_names():
    """The cross-attention interpolation fixtures (interp_*.npz)."""
    return sorted(n for n in _all_names() if n.startswith("interp_"))


def load_interp(name):
    z = np.load(os.path.join(GOLDEN_DIR, name + ".npz"))
    d = {k: z[k] for k in z.files}
    n_lon, n_lat, nside, to_hp, B, dim, H, kn, seed = (int(x) for x in d["meta"])
    d.update(n_lon=n_lon, n_lat=n_lat, nside=nside, to_hp=bool(to_hp), B=B, dim=dim, H=H, k=kn, seed=seed)
    return d


def interp_grids(n_lon, n_lat, nside):
    """(lat-lon grid, HEALPix grid), each [npoints, 2] (lon, lat) radians, built as
    Transformer.initialize_interpolation builds them (mosaic.py:272-276): the lat-lon
    grid is meshgrid(lon, lat, 'ij') flattened, lon 0..360 and lat -90..90 evenly."""
    lon = torch.linspace(0, 360, n_lon + 1)[:-1]
    lat = torch.linspace(-90, 90, n_lat)
    ll = torch.deg2rad(torch.stack(torch.meshgrid(lon, lat, indexing="ij"), -1).reshape(-1, 2))
    hp = torch.deg2rad(O.healpix_grid(nside))
    return ll, hp


def draw_updown_inputs(kind, n_coarse, F, B, c_in, c_out, affine, seed):
    """Seeded bf16 input and weights of a HEALPix down/upsampling case (make_golden.py uses
    this too): for "down" x [(n f), B, c_in], proj_x.weight [c_out, F c_in]; for "up"
    x [n, B, c_in], shortcut [(n f), B, c_out], proj_x.weight [F c_out, c_in]; proj_pos.weight
    [cols, 3 F]; norm weight 1 + 0.1 N(0, 1) when affine, else None. Values ~ N(0, 1),
    weights ~ N(0, 1 / fan_in)."""
    g = torch.Generator().manual_seed(seed)
    if kind == "down":
        x = torch.randn(n_coarse * F, B, c_in, generator=g).bfloat16()
        shortcut = None
        w_x = (torch.randn(c_out, F * c_in, generator=g) * (F * c_in) ** -0.5).bfloat16()
        cols = c_out
    else:
        x = torch.randn(n_coarse, B, c_in, generator=g).bfloat16()
        shortcut = torch.randn(n_coarse * F, B, c_out, generator=g).bfloat16()
        w_x = (torch.randn(F * c_out, c_in, generator=g) * c_in ** -0.5).bfloat16()
        cols = F * c_out
    w_pos = (torch.randn(cols, 3 * F, generator=g) * (3 * F) ** -0.5).bfloat16()
    w_norm = (1 + 0.1 * torch.randn(c_out, generator=g)).bfloat16() if affine else None
    return x, shortcut, w_x, w_pos, w_norm


def updown_fixture_names():
    """The HEALPix down/upsampling fixtures (down_*.npz, up_*.npz)."""
    return sorted(n for n in _all_names() if n.startswith(("down_", "up_")))


def load_updown(name):
    d = dict(np.load(os.path.join(GOLDEN_DIR, name + ".npz")))
    kind, nside_before, nside_after, B, c_in, c_out, affine, seed = (int(v) for v in d.pop("meta"))
    d.update(kind="down" if kind == 0 else "up", nside_before=nside_before, nside_after=nside_after, B=B, c_in=c_in,
             c_out=c_out, affine=bool(affine), seed=seed)
    return d


def draw_interp_inputs(S_from, B, dim, seed):
    """Seeded bf16 input and weights of an interpolation fixture: x_from [S_from, B, dim]
    ~ N(0, 1), to_q.weight [dim, 3] ~ N(0, 1), to_kv.weight [2 dim, dim] and to_o.weight
    [dim, dim] ~ N(0, 1/dim); make_golden.py uses this too."""
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(S_from, B, dim, generator=g).bfloat16()
    w_q = torch.randn(dim, 3, generator=g).bfloat16()
    w_kv = (torch.randn(2 * dim, dim, generator=g) * dim ** -0.5).bfloat16()
    w_o = (torch.randn(dim, dim, generator=g) * dim ** -0.5).bfloat16()
    return x, w_q, w_kv, w_o
