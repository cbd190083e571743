"""CPU restatement of the reference's block-sparse attention forward, its backward
and the layers around it (the attention block, the cross-attention interpolation,
the HEALPix down/upsampling layers).

TEST INFRASTRUCTURE: the checker for the CUDA path and the timed CPU baseline.
Only tests/, __graft_entry__.smoke() and bench.py's CPU legs use it; the product
path never does.

Each function restates one piece of maxxxzdn/mosaic in plain torch on the CPU
(fp32 arithmetic unless stated), citing the reference file:line it follows.
Two pieces of the reference live in third-party code that is absent here and are
restated from their published definitions:
  * flash_attn.flash_attn_func (flash-attn, unpinned `flash-attn>=2.0` in
    requirements.txt:9; 2.8.3 in the build image): non-causal softmax attention,
    default scale head_dim**-0.5, query head j reads kv head j // (Hq // Hk);
  * healpy.pix2ang(nest=True) (healpy>=1.16, requirements.txt:3): see
    `pix2ang_nest_scalar` below (HEALPix nested geometry, Gorski et al. 2005).
Pinning: tests/golden/make_golden.py runs the reference code itself (imported
from the reference checkout, its Triton kernel under TRITON_INTERPRET=1) on
seeded inputs and commits the results as fixtures; tests/test_oracle_golden.py
checks this module against them. The HEALPix restatement has no reference-side
fixture (healpy is not installed), so it is pinned by HEALPix known answers only.
"""
import math

import torch

LOG2_E = 1.44269504089


# --------------------------------------------------------------------------- geometry
_JRLL = [2, 2, 2, 2, 3, 3, 3, 3, 4, 4, 4, 4]
_JPLL = [1, 3, 5, 7, 0, 2, 4, 6, 1, 3, 5, 7]


def pix2ang_nest_scalar(nside, ipix):
    """(theta, phi) radians of one NESTED pixel centre (healpy.pix2ang(nest=True)).

    Pure-Python restatement (Gorski et al. 2005): de-interleave the in-face index
    into (x, y), ring jr = jrll[face]*nside - x - y - 1, then z and phi from the
    polar-cap / equatorial-belt formulas."""
    npface = nside * nside
    face, ipf = divmod(ipix, npface)
    ix = iy = 0
    bit = 0
    while ipf:
        ix |= (ipf & 1) << bit
        iy |= ((ipf >> 1) & 1) << bit
        ipf >>= 2
        bit += 1
    jr = _JRLL[face] * nside - ix - iy - 1
    npix = 12 * npface
    if jr < nside:
        nr = jr
        z = 1.0 - nr * nr * 4.0 / npix
        kshift = 0
    elif jr > 3 * nside:
        nr = 4 * nside - jr
        z = -(1.0 - nr * nr * 4.0 / npix)
        kshift = 0
    else:
        nr = nside
        z = (2 * nside - jr) * 2.0 * nside * 4.0 / npix
        kshift = (jr - nside) & 1
    jp = (_JPLL[face] * nr + ix - iy + 1 + kshift) // 2
    if jp > 4 * nside:
        jp -= 4 * nside
    if jp < 1:
        jp += 4 * nside
    phi = (jp - (kshift + 1) * 0.5) * (0.5 * math.pi / nr)
    return math.acos(max(-1.0, min(1.0, z))), phi


def healpix_grid(nside):
    """float32 [npix, 2] (lon deg, lat deg): utils.get_healpix_grid (utils.py:19-30)."""
    rows = []
    for p in range(12 * nside * nside):
        th, ph = pix2ang_nest_scalar(nside, p)
        rows.append((math.degrees(ph), 90.0 - math.degrees(th)))
    return torch.tensor(rows, dtype=torch.float64).float()


def rope_tables(positions, dim=64, theta=10000):
    """(cos, sin) [N, dim/2] fp32: RoPE.initialize_rope (primitives.py:115-123)."""
    base = 1.0 / (theta ** (torch.arange(0, dim // 2, 2).float() / (dim // 2)))
    lon = torch.deg2rad(positions[:, 0:1])
    lat = torch.deg2rad(positions[:, 1:2])
    freqs = torch.cat([lon @ base.unsqueeze(0), lat @ base.unsqueeze(0)], dim=-1)
    return freqs.cos(), freqs.sin()


def rope_apply(x, cos, sin):
    """RoPE.forward (primitives.py:126-135): interleaved-pair rotation in fp32, cast back."""
    c = cos.unsqueeze(0).unsqueeze(2).repeat_interleave(2, dim=-1)
    s = sin.unsqueeze(0).unsqueeze(2).repeat_interleave(2, dim=-1)
    xf = x.float()
    pairs = xf.unflatten(-1, (-1, 2))
    rot = torch.stack((-pairs[..., 1], pairs[..., 0]), dim=-1).flatten(-2)
    return (xf * c + rot * s).to(x.dtype)


# --------------------------------------------------------------------------- attention pieces
def dense_attention(q, k, v, scale=None):
    """flash_attn_func semantics (third-party; see module docstring): q [B, L, Hq, D],
    k/v [B, S, Hk, D] -> [B, L, Hq, D] fp32, query head j reads kv head j // G."""
    B, L, Hq, D = q.shape
    Hk = k.shape[2]
    G = Hq // Hk
    scale = D ** -0.5 if scale is None else scale
    qf = q.float().transpose(1, 2)                                   # B Hq L D
    kf = k.float().repeat_interleave(G, dim=2).transpose(1, 2)       # B Hq S D
    vf = v.float().repeat_interleave(G, dim=2).transpose(1, 2)
    att = torch.softmax((qf @ kf.transpose(-1, -2)) * scale, dim=-1)
    return (att @ vf).transpose(1, 2)


def block_attention(q, k, v, block_size):
    """primitives.block_attention (primitives.py:28-32): dense attention per window."""
    B, N, Hq, D = q.shape
    nb = N // block_size
    r = lambda x: x.reshape(B * nb, block_size, x.shape[2], D)
    return dense_attention(r(q), r(k), r(v)).reshape(B, N, Hq, D)


def pool_mean(x, block_size):
    """reduce(x, 'b (nb bs) h d -> b nb h d', 'mean') (primitives.py:65-66,76):
    fp32 sum, one rounding to x's dtype."""
    B, N, H, D = x.shape
    return x.float().reshape(B, N // block_size, block_size, H, D).mean(dim=2).to(x.dtype)


def topk_scores(q_cmp, k_cmp):
    """The score matrix attn_topk ranks (primitives.py:37-49), with the reference's
    rounding points for bf16 inputs: S_j = q_j . k_{j//G} rounded to the input
    dtype, then the mean over the STRIDED group (g h), h fastest
    ('b (g h) t k -> b h t k', :47), again rounded. Returns [B, nb, Hk, nb]."""
    Hq, Hk = q_cmp.shape[2], k_cmp.shape[2]
    G = Hq // Hk
    dt = q_cmp.dtype
    kk = k_cmp.repeat_interleave(G, dim=2)
    s = (q_cmp.float().transpose(1, 2) @ kk.float().transpose(1, 2).transpose(-1, -2)).to(dt)  # B Hq t k
    if Hq != Hk:
        s = s.float().reshape(s.shape[0], G, Hk, s.shape[2], s.shape[3]).mean(dim=1).to(dt)
    return s.transpose(1, 2)  # B t Hk k


def attn_topk(q_cmp, k_cmp, block_count):
    """primitives.attn_topk (primitives.py:35-51): int64 [B, nb, Hk, K], scores descending,
    ties to the lower index (torch leaves tie order unspecified; the checker accepts
    any order inside a tie)."""
    t = topk_scores(q_cmp, k_cmp).float()
    order = torch.sort(-t, dim=-1, stable=True).indices  # descending, equal scores keep index order
    return order[..., :block_count].contiguous()


def sparse_attention(q, k, v, block_indices, block_size, softmax_scale=None, return_lse=False, qblocks=None):
    """ops.mosaic_attn_fwd_kernel (ops.py:25-134) in fp32: query n of head j attends to
    the keys of blocks block_indices[b, n // block_size, j // G, :] of kv head j // G
    (the CONTIGUOUS group, ops.py:47-49). LSE in log2 units (ops.py:131).
    `qblocks=(lo, hi)` restricts the work to query blocks lo..hi-1 (other rows are
    left uninitialised); the CPU timing sample uses it."""
    B, N, Hq, D = q.shape
    nb = N // block_size
    out = torch.empty(B, N, Hq, D, dtype=torch.float32)
    lse = torch.empty(B, N, Hq, dtype=torch.float32)
    lo, hi = (0, nb) if qblocks is None else qblocks
    n0, n1 = lo * block_size, hi * block_size
    out[:, n0:n1], lse[:, n0:n1] = sparse_attention_rows(q, k, v, block_indices, block_size, lo, hi, softmax_scale)
    return (out, lse) if return_lse else out


def sparse_attention_rows(q, k, v, block_indices, block_size, lo, hi, softmax_scale=None):
    """The rows of query blocks lo..hi-1 of `sparse_attention` (ops.py:25-134), compact:
    (out [B, (hi-lo)*bs, Hq, D], lse [B, (hi-lo)*bs, Hq]) fp32. Works on full-size
    inputs without allocating an output of the whole sequence."""
    B, N, Hq, D = q.shape
    Hk = k.shape[2]
    G = Hq // Hk
    K = block_indices.shape[-1]
    scale = D ** -0.5 if softmax_scale is None else softmax_scale
    n0, n1 = lo * block_size, hi * block_size
    out = torch.empty(B, n1 - n0, Hq, D, dtype=torch.float32)
    lse = torch.empty(B, n1 - n0, Hq, dtype=torch.float32)
    ar = torch.arange(block_size)
    for b in range(B):
        for h in range(Hk):
            sel = block_indices[b, lo:hi, h, :].long()
            rows = (sel.unsqueeze(-1) * block_size + ar).reshape(hi - lo, K * block_size)
            ks = k[b, :, h][rows].float()                            # nblk, K*bs, D
            vs = v[b, :, h][rows].float()
            for g in range(G):
                j = h * G + g
                qq = q[b, n0:n1, j].float().reshape(hi - lo, block_size, D) * (scale * LOG2_E)
                s2 = qq @ ks.transpose(-1, -2)                       # nblk, bs, K*bs  (log2 domain)
                m = s2.amax(dim=-1, keepdim=True)
                p = torch.exp2(s2 - m)
                l = p.sum(dim=-1, keepdim=True)
                out[b, :, j] = ((p @ vs) / l).reshape(n1 - n0, D)
                lse[b, :, j] = (m + torch.log2(l)).reshape(n1 - n0)
    return out, lse


def sparse_attention_bwd(q, k, v, block_indices, block_size, grad_out, softmax_scale=None, out=None, lse=None):
    """ops.mosaic_attn_bwd (ops.py:436-507) in fp32: returns (dq, dk, dv).

    With c = scale*log2(e), S2 = (q c).k, P = exp2(S2 - lse), dP = dO.v and
    D = rowsum(out * dO) (ops.py:461):
      dq = scale * sum_keys P (dP - D) k over every selected slot, a block selected
           twice counting twice (mosaic_attn_bwd_q_kernel, ops.py:184-274);
      dk = scale * sum_queries P (dP - D) q and dv = sum_queries P dO over the
           DISTINCT q blocks that selected the key's block (the boolean block mask
           of mosaic_block_mask, ops.py:277-297, read by mosaic_attn_bwd_kv_kernel,
           ops.py:305-433).
    The reference folds LN_2 and LOG2_E into its bf16 operands (ops.py:249,267,
    273,420,426); they cancel, so in exact arithmetic these are the same sums.
    out / lse default to this module's sparse_attention forward."""
    B, N, Hq, D = q.shape
    Hk = k.shape[2]
    G = Hq // Hk
    K = block_indices.shape[-1]
    scale = D ** -0.5 if softmax_scale is None else softmax_scale
    nb = N // block_size
    if out is None or lse is None:
        out, lse = sparse_attention(q, k, v, block_indices, block_size, scale, return_lse=True)
    qf, kf, vf, gof = q.float(), k.float(), v.float(), grad_out.float()
    delta = (out.float() * gof).sum(-1)                               # B, N, Hq
    dq = torch.zeros(B, N, Hq, D)
    dk = torch.zeros(B, N, Hk, D)
    dv = torch.zeros(B, N, Hk, D)
    ar = torch.arange(block_size)
    for b in range(B):
        for h in range(Hk):
            sel = block_indices[b, :, h, :].long()                    # nb, K
            first = torch.ones(nb, K, dtype=torch.bool)               # first occurrence of each block in its row
            for s in range(1, K):
                first[:, s] = (sel[:, :s] != sel[:, s:s + 1]).all(dim=1)
            rows = (sel.unsqueeze(-1) * block_size + ar).reshape(nb, K * block_size)
            keep = first.repeat_interleave(block_size, dim=1).float()  # nb, K*bs
            ks = kf[b, :, h][rows]                                    # nb, K*bs, D
            vs = vf[b, :, h][rows]
            for g in range(G):
                j = h * G + g
                qq = qf[b, :, j].reshape(nb, block_size, D)
                s2 = (qq * (scale * LOG2_E)) @ ks.transpose(-1, -2)   # nb, bs, K*bs
                p = torch.exp2(s2 - lse[b, :, j].reshape(nb, block_size, 1))
                go = gof[b, :, j].reshape(nb, block_size, D)
                dp = go @ vs.transpose(-1, -2)
                ds = p * (dp - delta[b, :, j].reshape(nb, block_size, 1))
                dq[b, :, j] = (scale * (ds @ ks)).reshape(N, D)
                dk_slots = scale * (ds * keep.unsqueeze(1)).transpose(-1, -2) @ qq   # nb, K*bs, D
                dv_slots = (p * keep.unsqueeze(1)).transpose(-1, -2) @ go
                dk[b, :, h].index_add_(0, rows.reshape(-1), dk_slots.reshape(-1, D))
                dv[b, :, h].index_add_(0, rows.reshape(-1), dv_slots.reshape(-1, D))
    return dq, dk, dv


def mosaic_attn_func(q, k, v, weight_ba_cmp_slc, block_attn_size, sparse_block_size, sparse_block_count,
                     block_attn_only, no_compression=False, block_indices=None, parts=None):
    """primitives.mosaic_attn_func (primitives.py:54-89), fp32 arithmetic.

    `block_indices` overrides the top-k selection (to compare outputs against a
    kernel whose selection differs from this oracle's only inside score ties);
    `parts`, if a dict, receives o_ba / o_cmp / o_slc / block_indices."""
    o_ba = block_attention(q, k, v, block_attn_size)
    if parts is not None:
        parts["o_ba"] = o_ba
    if block_attn_only:
        return o_ba
    w = weight_ba_cmp_slc.float()
    q_cmp = pool_mean(q, sparse_block_size)
    k_cmp = pool_mean(k, sparse_block_size)
    if no_compression:
        idx = attn_topk(q_cmp, k_cmp, sparse_block_count) if block_indices is None else block_indices
        o_slc = sparse_attention(q, k, v, idx, sparse_block_size)
        if parts is not None:
            parts.update(o_slc=o_slc, block_indices=idx)
        w_sum = w[0] + w[2] + 1e-8
        return o_ba * (w[0] / w_sum) + o_slc * (w[2] / w_sum)
    v_cmp = pool_mean(v, sparse_block_size)
    o_cmp = dense_attention(q_cmp, k_cmp, v_cmp).repeat_interleave(sparse_block_size, dim=1)
    if parts is not None:
        parts["o_cmp"] = o_cmp
    if sparse_block_count == 0:
        w_sum = w[0] + w[1] + 1e-8
        return o_ba * (w[0] / w_sum) + o_cmp * (w[1] / w_sum)
    idx = attn_topk(q_cmp, k_cmp, sparse_block_count) if block_indices is None else block_indices
    o_slc = sparse_attention(q, k, v, idx, sparse_block_size)
    if parts is not None:
        parts.update(o_slc=o_slc, block_indices=idx)
    return o_ba * w[0] + o_cmp * w[1] + o_slc * w[2]


def attention_projections(x, w_q, w_k, w_v, w_g, num_q_heads, num_kv_heads, rope_cos=None, rope_sin=None):
    """The projections of MosaicAttention.forward (primitives.py:182-194), fp32:
    x [S, B, dim] -> q [B, S, Hq, 64], k, v [B, S, Hk, 64] (q, k rotated by RoPE.forward,
    primitives.py:132-135, when the tables are given) and the strategy weights
    [3, B, S, Hq] = softmax over the three strategies of x w_g^T laid out (head,
    strategy) (generate_strategy_weights, primitives.py:172-178), or None without w_g."""
    xf = x.float()
    S, B, _ = xf.shape
    q = (xf @ w_q.float().t()).reshape(S, B, num_q_heads, -1).permute(1, 0, 2, 3)
    k = (xf @ w_k.float().t()).reshape(S, B, num_kv_heads, -1).permute(1, 0, 2, 3)
    v = (xf @ w_v.float().t()).reshape(S, B, num_kv_heads, -1).permute(1, 0, 2, 3)
    if rope_cos is not None:
        q, k = rope_apply(q, rope_cos, rope_sin), rope_apply(k, rope_cos, rope_sin)
    g = None
    if w_g is not None:
        logits = (xf @ w_g.float().t()).reshape(S, B, num_q_heads, 3)      # 't b (h s)'
        g = torch.softmax(logits, dim=-1).permute(3, 1, 0, 2)               # -> 's b t h'
    return q.contiguous(), k.contiguous(), v.contiguous(), None if g is None else g.contiguous()


def mosaic_attention(x, w_q, w_k, w_v, w_g, w_o, num_q_heads, num_kv_heads, rope_cos, rope_sin, block_attn_size,
                     sparse_block_size, sparse_block_count, block_attn_only, no_compression=False,
                     block_indices=None, parts=None):
    """MosaicAttention.forward (primitives.py:182-209), fp32: projections, the
    attention of mosaic_attn_func, and to_o applied to rearrange(o, 'b s h d -> s b (h d)').
    `block_indices` / `parts` as in mosaic_attn_func; `parts` also receives q, k, v, g."""
    q, k, v, g = attention_projections(x, w_q, w_k, w_v, None if block_attn_only else w_g, num_q_heads,
                                       num_kv_heads, rope_cos, rope_sin)
    if parts is not None:
        parts.update(q=q, k=k, v=v, g=g)
    o = mosaic_attn_func(q, k, v, None if g is None else g.unsqueeze(-1), block_attn_size, sparse_block_size,
                         sparse_block_count, block_attn_only, no_compression, block_indices=block_indices, parts=parts)
    B, S, H, D = o.shape
    return o.permute(1, 0, 2, 3).reshape(S, B, H * D) @ w_o.float().t()


def cross_attention_interpolate(x_from, neighbors, rel_pos, w_q, w_kv, w_o, num_heads, eps, norm_weight=None):
    """CrossAttentionInterpolate.forward (primitives.py:264-284), fp32: x_from [S_from, B, dim],
    neighbors [S_to, k], rel_pos [S_to, k, 3] -> [S_to, B, dim]. kv_norm is torch.nn.RMSNorm
    (x / sqrt(mean(x^2) + eps), times norm_weight when affine)."""
    xf = x_from.float()
    S_from, B, dim = xf.shape
    H = num_heads
    D = dim // H
    q = (rel_pos.float() @ w_q.float().t()).reshape(*rel_pos.shape[:2], 1, H, D)          # s k 1 h d
    x = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    if norm_weight is not None:
        x = x * norm_weight.float()
    kv = (x @ w_kv.float().t()).reshape(S_from, B, 2, H, D).permute(2, 0, 1, 3, 4)         # n s b h d
    k, v = kv[:, neighbors.long()]                                                          # s k b h d
    scores = (q * k).sum(-1, keepdim=True) * D ** -0.5
    a = torch.softmax(scores, dim=1)
    out = (a * v).sum(dim=1).reshape(neighbors.shape[0], B, dim)
    return out @ w_o.float().t()


def swiglu_ffn(x, w13, w2, noise_w=None, z=None):
    """cSwiGLU.forward (primitives.py:102-106), fp32: x [S, B, dim], z [B, noise_dim];
    x1, x3 = (x w13^T).chunk(2); w2(silu(x1 + noise_bias(z)) * x3)."""
    xf = x.float()
    x1, x3 = (xf @ w13.float().t()).chunk(2, dim=-1)
    noise = (z.float() @ noise_w.float().t()).unsqueeze(0) if z is not None else 0.0
    return (torch.nn.functional.silu(x1 + noise) * x3) @ w2.float().t()


def mosaic_block_ffn(x, z, w13, w2, noise_w, eps, norm_weight=None):
    """The FFN half of MosaicBlock.forward (primitives.py:229), fp32:
    x + ffn(norm2(x), z) with norm2 = torch.nn.RMSNorm (times norm_weight when affine)."""
    xf = x.float()
    return xf + swiglu_ffn(rms_norm(xf, eps, norm_weight), w13, w2, noise_w, z)


def rad_to_xyz(lonlat):
    """utils.rad_to_xyz (utils.py:7-16): (lon, lat) radians -> unit xyz."""
    lon, lat = lonlat[..., 0], lonlat[..., 1]
    return torch.stack([torch.cos(lat) * torch.cos(lon), torch.cos(lat) * torch.sin(lon), torch.sin(lat)], dim=-1)


def healpix_updown_rel_pos(nside_fine, nside_coarse):
    """The rel_pos buffer of HEALPixDownsample / HEALPixUpsample (primitives.py:317-322,
    345-350): per coarse pixel n, its F = (nside_fine / nside_coarse)^2 nested children's
    unit vectors minus its own, flattened to [n, (f xyz)], then standardised per column
    (torch.std, unbiased) with 1e-6 added to the deviation. fp32 [n_coarse, 3 F]."""
    F = (nside_fine // nside_coarse) ** 2
    fine = rad_to_xyz(torch.deg2rad(healpix_grid_fast(nside_fine).float()))
    coarse = rad_to_xyz(torch.deg2rad(healpix_grid_fast(nside_coarse).float()))
    rel = (fine.reshape(-1, F, 3) - coarse[:, None]).reshape(-1, 3 * F)
    return (rel - rel.mean(dim=0, keepdim=True)) / (rel.std(dim=0, keepdim=True) + 1e-6)


def rms_norm(x, eps, weight=None):
    """torch.nn.RMSNorm.forward in fp32: x / sqrt(mean(x^2, -1) + eps), times weight."""
    x = x.float()
    y = x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps)
    return y if weight is None else y * weight.float()


def healpix_downsample(x, w_x, w_pos, rel_pos, eps, norm_weight=None):
    """HEALPixDownsample.forward (primitives.py:325-329), fp32: x [(n f), B, C] ->
    rearrange '(n f) b c -> n b (f c)', proj_x, + proj_pos(rel_pos) broadcast over b,
    RMSNorm. w_x [out, F C], w_pos [out, 3 F], rel_pos [n, 3 F] -> [n, B, out]."""
    F = rel_pos.shape[1] // 3
    nF, B, C = x.shape
    xr = x.float().reshape(nF // F, F, B, C).permute(0, 2, 1, 3).reshape(nF // F, B, F * C)
    y = xr @ w_x.float().t() + (rel_pos.float() @ w_pos.float().t()).unsqueeze(1)
    return rms_norm(y, eps, norm_weight)


def healpix_upsample(x, shortcut, w_x, w_pos, rel_pos, eps, norm_weight=None):
    """HEALPixUpsample.forward (primitives.py:352-357), fp32: x [n, B, C_in] -> proj_x +
    proj_pos(rel_pos) broadcast over b -> [n, B, (f d)] -> rearrange 'n b (f d) -> (n f) b d',
    + shortcut [(n f), B, d], RMSNorm. w_x [F d, C_in], w_pos [F d, 3 F] -> [(n f), B, d]."""
    F = rel_pos.shape[1] // 3
    n, B, _ = x.shape
    y = x.float() @ w_x.float().t() + (rel_pos.float() @ w_pos.float().t()).unsqueeze(1)
    d = y.shape[-1] // F
    y = y.reshape(n, B, F, d).permute(0, 2, 1, 3).reshape(n * F, B, d) + shortcut.float()
    return rms_norm(y, eps, norm_weight)


def mosaic_attn_func_sample(q, k, v, weight_ba_cmp_slc, block_attn_size, sparse_block_size, sparse_block_count,
                            windows):
    """mosaic_attn_func restricted to the queries of the given local windows: the
    compression and top-k run over the whole sequence (they are global), the
    local and selected branches only for those windows. A bounded, proportional
    sample of the full forward for CPU timing. Returns [B, len(windows)*bas, Hq, D]."""
    o_cmp, idx = mosaic_attn_global(q, k, v, sparse_block_size, sparse_block_count)
    return torch.cat([mosaic_attn_window(q, k, v, weight_ba_cmp_slc, block_attn_size, sparse_block_size, win,
                                         o_cmp, idx) for win in windows], dim=1)


def mosaic_attn_global(q, k, v, sparse_block_size, sparse_block_count):
    """The sequence-global part of mosaic_attn_func (primitives.py:65-78, 86): pooled
    coarse attention o_cmp [B, nb, Hq, D] (not yet repeated) and the top-k indices."""
    bs = sparse_block_size
    q_cmp, k_cmp, v_cmp = pool_mean(q, bs), pool_mean(k, bs), pool_mean(v, bs)
    return dense_attention(q_cmp, k_cmp, v_cmp), attn_topk(q_cmp, k_cmp, sparse_block_count)


def mosaic_attn_window(q, k, v, weight_ba_cmp_slc, block_attn_size, sparse_block_size, win, o_cmp, idx):
    """mosaic_attn_func's output rows of local window `win` (primitives.py:31, 87-89) given
    the global part: [B, block_attn_size, Hq, D] fp32."""
    bas, bs = block_attn_size, sparse_block_size
    w = weight_ba_cmp_slc.float()
    n0, n1 = win * bas, (win + 1) * bas
    o_ba = dense_attention(q[:, n0:n1], k[:, n0:n1], v[:, n0:n1])
    o_slc, _ = sparse_attention_rows(q, k, v, idx, bs, n0 // bs, n1 // bs)
    o_c = o_cmp[:, n0 // bs:n1 // bs].repeat_interleave(bs, dim=1)
    return o_ba * w[0, :, n0:n1] + o_c * w[1, :, n0:n1] + o_slc * w[2, :, n0:n1]


# --------------------------------------------------------------------------- checkers
def topk_matches(idx_test, idx_ref, scores, rel=1e-3):
    """Top-k parity up to score ties: for every row the two index SETS must agree,
    except for entries whose score lies within `rel` (relative) of that row's K-th
    score (the tie boundary). Returns (ok, number_of_rows_that_differ)."""
    idx_test = idx_test.long()
    idx_ref = idx_ref.long()
    sc = scores.float()
    K = idx_ref.shape[-1]
    kth = torch.gather(sc, -1, idx_ref).amin(dim=-1, keepdim=True)       # reference K-th score
    tol = kth.abs() * rel + 1e-30
    a = torch.zeros_like(sc, dtype=torch.bool).scatter_(-1, idx_test, True)
    b = torch.zeros_like(sc, dtype=torch.bool).scatter_(-1, idx_ref, True)
    diff = a ^ b
    near = (sc - kth).abs() <= tol
    bad = diff & ~near
    # a kernel row must also hold K distinct indices
    distinct = a.sum(dim=-1) == K
    ok = bool((~bad).all()) and bool(distinct.all())
    return ok, int(diff.any(dim=-1).sum())


def make_inputs(B, N, Hq, Hk, D=64, seed=0, dtype=torch.bfloat16, rope=True):
    """Seeded synthetic inputs (draw order q, k, v, gate logits): q/k/v ~ N(0,1),
    gates = sigmoid(N(0,1)) [3, B, N, Hq, 1]; with `rope`, q and k are rotated by
    the nested-HEALPix 2D RoPE of nside = sqrt(N / 12) (as MosaicAttention.forward
    does before calling the op, primitives.py:193-195). Returns a dict with the
    un-rotated tensors too."""
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, N, Hq, D, generator=g).to(dtype)
    k = torch.randn(B, N, Hk, D, generator=g).to(dtype)
    v = torch.randn(B, N, Hk, D, generator=g).to(dtype)
    w = torch.sigmoid(torch.randn(3, B, N, Hq, 1, generator=g)).to(dtype)
    out = dict(q_raw=q, k_raw=k, v=v, w=w, q=q, k=k, cos=None, sin=None)
    if rope:
        nside = int(round(math.sqrt(N / 12)))
        if 12 * nside * nside != N:
            raise ValueError(f"N={N} is not a HEALPix pixel count")
        cos, sin = rope_tables(healpix_grid_fast(nside), D)
        out.update(q=rope_apply(q, cos, sin), k=rope_apply(k, cos, sin), cos=cos, sin=sin)
    return out


def healpix_grid_fast(nside):
    """healpix_grid for large nside (the scalar loop is slow at nside 64+); same maths,
    cached per nside."""
    if nside not in _GRID_CACHE:
        _GRID_CACHE[nside] = healpix_grid(nside)
    return _GRID_CACHE[nside]


_GRID_CACHE = {}
