"""Drop-in for primitives.CrossAttentionInterpolate (primitives.py:228-284), the k-nearest
neighbour cross-attention that moves fields between the lat-lon and HEALPix grids.

    x_from [S_from, B, dim] --mosaic_row_rms + mosaic_linear--> kv = to_kv(RMSNorm(x_from))
                            --mosaic_interp_attend_tiled-----> per target: softmax over its k
                                                               neighbours, q from rel_pos
                            --mosaic_linear------------------> to_o -> [S_to, B, dim]

The neighbour table is static, so the module packs the targets once into tiles of
spatially adjacent points (`build_tiles`) whose merged neighbour lists fit in shared
memory; the tiled kernel then reads each source point once per tile instead of once
per (target, neighbour). Neighbour counts above 32 take mosaic_interp_attend.

The module keeps the reference's constructor (`config.k_neighbors`, `dim`, `num_heads`,
`rmsnorm_elementwise_affine`), submodules (`kv_norm`, `to_q`, `to_kv`, `to_o`) and
buffers (`neighbors`, `rel_pos`), so a reference state dict loads. The neighbour search
of `initialize_interpolation_scheme` (sklearn's BallTree with the haversine metric in
the reference, utils.py:33-40) is an exact k-nearest search on the device: haversine
distance is monotonic in the dot product of the points' unit vectors, computed in
fp64. Inference only, like MosaicAttention here.
"""
import torch
import torch.nn as nn

from . import _lib
from .ops import _ptr, _require_cuda, _stream_ptr

__all__ = ["CrossAttentionInterpolate", "rad_to_xyz", "knn_neighbors", "linear", "norm_eps", "row_rms", "interp_attend",
           "build_tiles", "interp_attend_tiled"]

TILE_MAX_UNION = 80  # source points per tile (a multiple of 16: the tensor-core k step)
TILE_MAX_TARGETS = 32  # 2 blocks of 16 rows
TILED_MAX_NEIGHBORS = 32


def rad_to_xyz(lonlat):
    """utils.rad_to_xyz (utils.py:7-16): (lon, lat) radians -> unit xyz."""
    lon, lat = lonlat[..., 0], lonlat[..., 1]
    return torch.stack([torch.cos(lat) * torch.cos(lon), torch.cos(lat) * torch.sin(lon), torch.sin(lat)], dim=-1)


def knn_neighbors(pos_from_rad, pos_to_rad, k, chunk=2048):
    """int64 [S_to, k]: the k points of pos_from nearest to each point of pos_to on the
    sphere (both (lon, lat) radians), nearest first. Same sets as the reference's
    BallTree haversine query up to ties in distance."""
    a = rad_to_xyz(pos_to_rad.double())
    b = rad_to_xyz(pos_from_rad.double())
    out = []
    for i in range(0, a.shape[0], chunk):
        out.append(torch.topk(a[i:i + chunk] @ b.t(), k, dim=1).indices)
    return torch.cat(out).contiguous()


def _bf16c(t):
    t = t if t.dtype == torch.bfloat16 else t.to(torch.bfloat16)
    return t.contiguous()


def linear(a, w, row_scale=None, status=None):
    """a [..., in] @ w^T -> [..., out] bf16 through mosaic_linear (optionally times row_scale
    per row of the flattened a)."""
    _require_cuda(a, w)
    lead, k_in = a.shape[:-1], a.shape[-1]
    ab, wb = _bf16c(a).reshape(-1, k_in), _bf16c(w)
    rows, n_out = ab.shape[0], wb.shape[0]
    out = torch.empty(rows, n_out, dtype=torch.bfloat16, device=a.device)
    rs = None if row_scale is None else row_scale.float().contiguous()
    with torch.cuda.device(a.device):
        rc = _lib.load().mosaic_linear(_ptr(ab), _ptr(wb), _ptr(out), _ptr(rs), _ptr(status), rows, k_in, n_out,
                                       _stream_ptr(a.device))
    _lib.check("mosaic_linear", rc)
    return out.reshape(*lead, n_out)


def norm_eps(norm):
    """The epsilon torch.nn.RMSNorm `norm` applies: its own eps, or when that is None the
    epsilon of the op's math type, which is fp32 for bf16, fp16 and fp32 inputs alike
    (torch upcasts half-precision inputs and takes numeric_limits<float>::epsilon), not
    the input dtype's epsilon."""
    return norm.eps if norm.eps is not None else torch.finfo(torch.float32).eps


def row_rms(x, eps):
    """fp32 1 / sqrt(mean(x^2, -1) + eps) per row of x (flattened to [rows, dim])."""
    _require_cuda(x)
    xb = _bf16c(x).reshape(-1, x.shape[-1])
    rinv = torch.empty(xb.shape[0], dtype=torch.float32, device=x.device)
    with torch.cuda.device(x.device):
        rc = _lib.load().mosaic_row_rms(_ptr(xb), _ptr(rinv), xb.shape[0], xb.shape[1], float(eps),
                                        _stream_ptr(x.device))
    _lib.check("mosaic_row_rms", rc)
    return rinv


def interp_attend(kv, neighbors, rel_pos, w_q, num_heads, points_from, status=None):
    """The gather-attention of CrossAttentionInterpolate.forward through mosaic_interp_attend:
    kv [S_from, B, 2 dim] bf16, neighbors [S_to, k], rel_pos [S_to, k, 3], w_q [dim, 3] ->
    [S_to, B, dim] bf16 (before to_o)."""
    _require_cuda(kv, neighbors, rel_pos, w_q)
    S_from, B, two_dim = kv.shape
    dim = two_dim // 2
    S_to, kn = neighbors.shape
    out = torch.empty(S_to, B, dim, dtype=torch.bfloat16, device=kv.device)
    nb = neighbors.to(torch.int32).contiguous()
    rp = rel_pos.float().contiguous()
    wq = w_q.float().contiguous()
    kvb = _bf16c(kv)
    with torch.cuda.device(kv.device):
        rc = _lib.load().mosaic_interp_attend(_ptr(kvb), _ptr(nb), _ptr(rp), _ptr(wq), _ptr(out), _ptr(status), S_to,
                                              int(points_from), B, dim, int(num_heads), kn, (dim // num_heads) ** -0.5,
                                              _stream_ptr(kv.device))
    _lib.check("mosaic_interp_attend", rc)
    return out


def _morton3(xyz, bits=10):
    """3D Morton (Z-order) key of unit vectors: targets sorted by it form compact patches."""
    q = ((xyz + 1) * 0.5 * ((1 << bits) - 1)).round().long().clamp(0, (1 << bits) - 1)
    key = torch.zeros(xyz.shape[0], dtype=torch.long)
    for bit in range(bits):
        for d in range(3):
            key |= ((q[:, d] >> bit) & 1) << (3 * bit + d)
    return key


def _pack(nb, order, max_union, max_targets):
    """Greedy packing of targets, in `order`, into tiles whose neighbour union stays within
    max_union points and max_targets targets; list of target lists."""
    tiles, cur, cur_set = [], [], set()
    for t in order:
        merged = cur_set.union(nb[t])
        if cur and (len(merged) > max_union or len(cur) >= max_targets):
            tiles.append(cur)
            cur, merged = [], set(nb[t])
        cur.append(t)
        cur_set = merged
    if cur:
        tiles.append(cur)
    return tiles


def build_tiles(neighbors, pos_to_rad, max_union=TILE_MAX_UNION, max_targets=TILE_MAX_TARGETS):
    """The tile tables of mosaic_interp_attend_tiled for a static neighbour table
    [S_to, k] and the targets' (lon, lat) radians: the targets in index order and (when
    pos_to_rad is given) in 3D Morton order are each packed greedily, and the packing that
    stages fewer source points in total is kept. Each tile's union is padded with repeats of
    its first point to a multiple of 16. Returns a dict of CPU tensors (tile_targets,
    tile_point_off, tile_points, local int32/uint8, order int32 or None) and max_union (the
    largest padded union). Neighbour lists must not repeat a point (a k-nearest search
    never does): the tiled kernel scatters each weight to its point's position."""
    nb = neighbors.detach().cpu().long()
    S_to, kn = nb.shape
    if max_union % 16 or not 16 <= max_union <= 256 or not 1 <= max_targets <= TILE_MAX_TARGETS:
        raise ValueError(f"max_union {max_union} (a multiple of 16 up to 256), max_targets {max_targets} (<= 32)")
    if kn > max_union:
        raise ValueError(f"{kn} neighbours do not fit a tile of {max_union} points")
    srt = nb.sort(dim=1).values
    if kn > 1 and bool((srt[:, 1:] == srt[:, :-1]).any()):
        raise ValueError("a neighbour list repeats a point")
    rows = nb.tolist()
    best = None
    orders = [None]
    if pos_to_rad is not None:
        orders.append(torch.argsort(_morton3(rad_to_xyz(pos_to_rad.detach().cpu().double())), stable=True))
    for order in orders:
        seq = range(S_to) if order is None else order.tolist()
        tiles = _pack(rows, seq, max_union, max_targets)
        staged = sum(len(set().union(*(rows[t] for t in tl))) for tl in tiles)
        if best is None or staged < best[0]:
            best = (staged, order, tiles)
    _, order, tiles = best
    tile_targets, point_off, points = [0], [0], []
    local = torch.empty(S_to, kn, dtype=torch.uint8)
    for tl in tiles:
        ts = torch.tensor(tl)
        uni, inv = torch.unique(nb[ts], sorted=True, return_inverse=True)
        local[ts] = inv.to(torch.uint8)
        pad = -uni.numel() % 16
        points.append(torch.cat([uni, uni[:1].expand(pad)]) if pad else uni)
        uni = points[-1]
        tile_targets.append(tile_targets[-1] + len(tl))
        point_off.append(point_off[-1] + uni.numel())
    return {
        "tile_targets": torch.tensor(tile_targets, dtype=torch.int32),
        "tile_point_off": torch.tensor(point_off, dtype=torch.int32),
        "tile_points": torch.cat(points).to(torch.int32),
        "local": local,
        "order": None if order is None else order.to(torch.int32),
        "max_union": max(b - a for a, b in zip(point_off[:-1], point_off[1:])),
    }


def interp_attend_tiled(kv, tiles, rel_pos, w_q, num_heads, points_from, status=None, kw=None):
    """interp_attend through mosaic_interp_attend_tiled with the tables of build_tiles
    (tensors on kv's device). `kw` [S_from, B, H, 4] fp32 = (to_q.weight_h^T k_h, 0) per
    point and head, when the caller has it, skips the kernel that computes it (w_q may
    then be None)."""
    _require_cuda(kv, rel_pos, *(() if w_q is None else (w_q,)))
    S_from, B, two_dim = kv.shape
    dim = two_dim // 2
    S_to, kn = tiles["local"].shape
    out = torch.empty(S_to, B, dim, dtype=torch.bfloat16, device=kv.device)
    kw_ready = kw is not None
    if kw is None:  # the call writes (x, y, z, 0) per point and head
        kw = torch.empty(S_from, B, num_heads, 4, dtype=torch.float32, device=kv.device)
    rp = rel_pos.float().contiguous()
    wq = None if w_q is None else w_q.float().contiguous()
    kvb = _bf16c(kv)
    n_tiles = tiles["tile_targets"].numel() - 1
    with torch.cuda.device(kv.device):
        rc = _lib.load().mosaic_interp_attend_tiled(
            _ptr(kvb), _ptr(kw), _ptr(tiles["tile_targets"]), _ptr(tiles["tile_point_off"]),
            _ptr(tiles["tile_points"]), _ptr(tiles["local"]), _ptr(tiles["order"]), _ptr(rp), _ptr(wq), _ptr(out),
            _ptr(status), n_tiles, int(tiles["max_union"]), int(points_from), B, dim, int(num_heads), kn,
            int(kw_ready), (dim // num_heads) ** -0.5, _stream_ptr(kv.device))
    _lib.check("mosaic_interp_attend_tiled", rc)
    return out


_TILE_KEYS = ("tile_targets", "tile_point_off", "tile_points", "local", "order")


class CrossAttentionInterpolate(nn.Module):
    """primitives.CrossAttentionInterpolate (primitives.py:228-284) on libmosaic_b200.so."""

    space_dim = 3

    def __init__(self, config):
        super().__init__()
        self.k_neighbors = config.k_neighbors
        dim = config.dim
        num_heads = config.num_heads
        head_dim = dim // num_heads
        self.num_heads = num_heads
        self.head_dim = head_dim
        self.scale = head_dim ** -0.5
        self.kv_norm = nn.RMSNorm(dim, elementwise_affine=config.rmsnorm_elementwise_affine)
        self.to_q = nn.Linear(self.space_dim, dim, bias=False)
        self.to_kv = nn.Linear(dim, 2 * dim, bias=False)
        self.to_o = nn.Linear(dim, dim, bias=False)
        self.register_buffer("neighbors", None, persistent=True)
        self.register_buffer("rel_pos", None, persistent=True)
        self.points_from = None
        for key in _TILE_KEYS:  # tile tables of the tiled kernel, derived from `neighbors`
            self.register_buffer("_tile_" + key, None, persistent=False)
        self._tile_max_union = None

    @torch.no_grad()
    def initialize_interpolation_scheme(self, pos_from_rad, pos_to_rad):
        """neighbors [S_to, k] and the unit relative positions [S_to, k, 3] of
        primitives.py:253-261, computed on pos_to_rad's device."""
        dev = pos_to_rad.device
        neighbors = knn_neighbors(pos_from_rad.to(dev), pos_to_rad, self.k_neighbors)
        self._set_scheme(neighbors, pos_from_rad.to(dev), pos_to_rad)

    def _set_scheme(self, neighbors, pos_from_rad, pos_to_rad):
        pos_to_xyz = rad_to_xyz(pos_to_rad)
        pos_from_xyz = rad_to_xyz(pos_from_rad)
        rel = (pos_to_xyz.unsqueeze(1) - pos_from_xyz[neighbors]).contiguous()
        self.register_buffer("neighbors", neighbors.long().contiguous(), persistent=True)
        self.register_buffer("rel_pos", torch.nn.functional.normalize(rel, dim=-1).contiguous(), persistent=True)
        self.points_from = pos_from_rad.shape[0]
        self._pos_to_rad = pos_to_rad.detach().cpu()
        self._drop_tiles()
        self._tiles()

    def _drop_tiles(self):
        for key in _TILE_KEYS:
            setattr(self, "_tile_" + key, None)
        self._tile_max_union = None

    def _load_from_state_dict(self, *args, **kwargs):
        super()._load_from_state_dict(*args, **kwargs)
        self._drop_tiles()  # rebuilt from the loaded neighbour table on first use

    def _tiles(self):
        """The tile tables for the current neighbour table (built on first use), or None
        when the neighbour count is above what the tiled kernel takes."""
        if self.neighbors.shape[1] > TILED_MAX_NEIGHBORS:
            return None
        if self._tile_max_union == 0:  # neighbour lists with repeats: untiled kernel
            return None
        if self._tile_max_union is None:
            # after a state-dict load the target positions are unknown: index order only
            try:
                t = build_tiles(self.neighbors, getattr(self, "_pos_to_rad", None))
            except ValueError:
                self._tile_max_union = 0
                return None
            dev = self.neighbors.device
            for key in _TILE_KEYS:
                setattr(self, "_tile_" + key, None if t[key] is None else t[key].to(dev))
            self._tile_max_union = t["max_union"]
        tiles = {key: getattr(self, "_tile_" + key) for key in _TILE_KEYS}
        tiles["max_union"] = self._tile_max_union
        return tiles

    def forward(self, x_from):
        if self.neighbors is None or self.rel_pos is None:
            raise ValueError("Interpolation scheme not initialized.")
        if torch.is_grad_enabled() and (x_from.requires_grad or any(p.requires_grad for p in self.parameters())):
            raise NotImplementedError(
                "mosaic_b200.CrossAttentionInterpolate serves inference; run it under torch.no_grad() or "
                "torch.inference_mode()")
        S_from = x_from.shape[0] if self.points_from is None else self.points_from
        eps = norm_eps(self.kv_norm)
        w_kv = self.to_kv.weight
        if self.kv_norm.weight is not None:  # affine RMSNorm: fold the weight into to_kv's input columns
            w_kv = w_kv * self.kv_norm.weight.unsqueeze(0)
        rinv = row_rms(x_from, eps)
        kv = linear(x_from, w_kv, rinv)
        tiles = self._tiles()
        if tiles is not None:
            o = interp_attend_tiled(kv, tiles, self.rel_pos, self.to_q.weight, self.num_heads, S_from)
        else:
            o = interp_attend(kv, self.neighbors, self.rel_pos, self.to_q.weight, self.num_heads, S_from)
        return linear(o, self.to_o.weight).to(x_from.dtype)
