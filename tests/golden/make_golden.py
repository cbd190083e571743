"""Generate the golden fixtures in this directory by running the REFERENCE code.

Run from the repository root in a container that has the reference checkout:

    TRITON_INTERPRET=1 python tests/golden/make_golden.py /path/to/mosaic/reference [part ...]

(parts: attn bwd block interp updown; all by default).

It imports the reference's `ops` and `primitives` modules and runs, on the CPU:
  * primitives.mosaic_attn_func / attn_topk / RoPE / the einops pooling as-is;
  * ops.mosaic_attn_fwd_kernel (the Triton kernel itself) through Triton's
    interpreter, as the selected-branch attention (primitives.mosaic_sparse_attn
    is rebound to that launch);
  * primitives.flash_attn_func rebound to torch SDPA with GQA (flash-attn is a
    CUDA-only third-party op; its published semantics are non-causal softmax
    attention, scale head_dim**-0.5, query head j -> kv head j // G).
healpy is not installed: the nested pixel centres for the RoPE angles (and the
interpolation grids) come from the restatement in oracle/bsa_oracle.py (pinned
separately by known answers); sklearn (the reference's BallTree) is installed.

Harness patches (test-side only, to the Triton interpreter): bf16 operands of
tl.dot are up-converted to fp32 before numpy's matmul (the stock interpreter
stores bf16 as uint16 and would multiply the raw bits). Kernel inputs are fp32
tensors holding bf16-representable values; the kernel casts them to bf16 itself
(ops.py:92,115-116), so this is the bf16 computation of the reference.

Outputs are fp32 (the reference run in fp32 on bf16-valued inputs); top-k is
taken from the bf16 run of attn_topk on bf16 pooled tensors, which is the
precision of the B200 path, and the fp32 run is driven with those indices.
Fixtures keep the full indices, the small pooled outputs, 64 sampled query rows
of every larger output (fp16) and fp64 per-head sums of the full outputs.

The backward fixtures (bwd_*.npz) run ops.mosaic_attn_bwd's two Triton kernels
(mosaic_attn_bwd_q_kernel, mosaic_attn_bwd_kv_kernel) in the interpreter on the
forward kernel's own output and lse, with the block mask from ops.mosaic_block_mask
(its eager function; the reference wraps it in torch.compile) and delta computed as
ops.py:461 does. They keep 64 sampled rows of dq, dk, dv (fp16) and fp64 per-head
sums. One config repeats a block inside some selections, which pins the
reference's counting of repeated blocks (twice for dq, once for dk / dv).

The attention-block fixtures (block_*.npz) run primitives.MosaicAttention.forward
(projections, RoPE, strategy gates, mosaic_attn_func as above, to_o) in fp32 on
seeded bf16-valued weights and input, and keep the selected block indices, 64
sampled token rows of the output and fp64 per-batch sums.

The interpolation fixtures (interp_*.npz) run primitives.CrossAttentionInterpolate
(its BallTree neighbour search, relative positions and forward) in fp32 on seeded
bf16-valued weights and input between a small lat-lon grid and HEALPix nside 4, in
both directions, and keep the neighbour table, 64 sampled target rows and fp64 sums.

The down/upsampling fixtures (down_*.npz, up_*.npz) run primitives.HEALPixDownsample /
HEALPixUpsample (their rel_pos construction and forward, with and without the affine
RMSNorm, factor 4 and 16, batch 1 and 2) in fp32 on seeded bf16-valued weights and input,
and keep rel_pos, 64 sampled output rows and fp64 per-member sums.
"""
import os
import sys
import types

import numpy as np
import torch
import torch.nn.functional as F

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
HERE = os.path.dirname(os.path.abspath(__file__))


def _import_reference(ref_dir):
    if os.environ.get("TRITON_INTERPRET") != "1":
        raise SystemExit("set TRITON_INTERPRET=1 (the reference Triton kernel runs in the interpreter)")
    sys.path.insert(0, ref_dir)
    sys.modules.setdefault("healpy", types.ModuleType("healpy"))
    import triton.language as tl
    import triton.runtime.interpreter as interp

    def create_dot(self, a, b, d, input_precision, max_num_imprecise_acc):
        def up(h):
            if h.dtype.scalar == tl.bfloat16:
                return interp._convert_float(h.data, tl.bfloat16, tl.float32, None).view(np.float32)
            return h.data
        return interp.TensorHandle(np.matmul(up(a), up(b), dtype=d.data.dtype) + d.data, d.dtype.scalar)

    interp.InterpreterBuilder.create_dot = create_dot
    import ops
    import primitives
    return ops, primitives


def sdpa_gqa(q, k, v):
    """flash_attn_func(q, k, v) semantics on CPU (fp32)."""
    G = q.shape[2] // k.shape[2]
    o = F.scaled_dot_product_attention(q.transpose(1, 2).float(), k.transpose(1, 2).float(),
                                       v.transpose(1, 2).float(), enable_gqa=G > 1)
    return o.transpose(1, 2)


def make_triton_sparse(ops):
    def triton_sparse(q, k, v, block_indices, block_size, softmax_scale=None):
        B, N, Hq, D = q.shape
        Hk = k.shape[2]
        scale = D ** -0.5 if softmax_scale is None else softmax_scale
        q, k, v = (t.float().contiguous() for t in (q, k, v))
        idx = block_indices.contiguous()
        out = torch.empty(B, N, Hq, D)
        lse = torch.empty(B, N, Hq)
        ops.mosaic_attn_fwd_kernel.fn[(N // 64, Hq // Hk, B * Hk)](
            q, k, v, out, lse, idx, softmax_scale=scale, seq_len=N, num_kv_heads=Hk, num_q_heads=Hq,
            q_heads_per_kv_head=Hq // Hk, feature_dim=D, kv_block_size=block_size,
            num_kv_blocks_per_q_block=idx.shape[-1], q_tile_size=64)
        triton_sparse.last_lse = lse
        return out
    return triton_sparse


CONFIGS = {
    # name: B, N, Hq, Hk, bs, K, bas, seed
    "g1_n768_h4x1_bs64_k4": (1, 768, 4, 1, 64, 4, 256, 0),
    "c1_n3072_h4x1_bs64_k8": (1, 3072, 4, 1, 64, 8, 1024, 1),
    "g3_n3072_h8x2_bs128_k4": (1, 3072, 8, 2, 128, 4, 512, 2),
}


BWD_CONFIGS = {
    # name: B, N, Hq, Hk, bs, K, seed, repeat_a_block
    "bwd_n512_h8x2_bs64_k3": (1, 512, 8, 2, 64, 3, 10, False),
    "bwd_n768_h4x1_bs128_k3_rep": (2, 768, 4, 1, 128, 3, 11, True),
}


def main_bwd(ops):
    sys.path.insert(0, ROOT)
    from tests.golden_util import draw_bwd_inputs
    triton_sparse = make_triton_sparse(ops)
    block_mask_fn = getattr(ops.mosaic_block_mask, "_torchdynamo_orig_callable", ops.mosaic_block_mask)
    for name, (B, N, Hq, Hk, bs, K, seed, repeat) in BWD_CONFIGS.items():
        q, k, v, go, idx = draw_bwd_inputs(B, N, Hq, Hk, bs, K, seed, repeat)
        qf, kf, vf, gof = (t.float().contiguous() for t in (q, k, v, go))
        scale = 64 ** -0.5
        out = triton_sparse(qf, kf, vf, idx, bs)
        lse = triton_sparse.last_lse
        mask = block_mask_fn(idx)
        delta = (out * gof).sum(dim=-1)
        dq, dk, dv = torch.empty_like(qf), torch.empty_like(kf), torch.empty_like(vf)
        ops.mosaic_attn_bwd_q_kernel.fn[(N // 64, Hq // Hk, B * Hk)](
            q_ptr=qf, k_ptr=kf, v_ptr=vf, lse_ptr=lse, delta_ptr=delta, grad_o_ptr=gof, grad_q_ptr=dq,
            block_indices_ptr=idx, softmax_scale=scale, seq_len=N, num_kv_heads=Hk, num_q_heads=Hq,
            q_heads_per_kv_head=Hq // Hk, feature_dim=64, kv_block_size=bs, num_kv_blocks_per_q_block=K,
            q_tile_size=64)
        ops.mosaic_attn_bwd_kv_kernel.fn[(N // bs, B * Hk)](
            q_ptr=qf, k_ptr=kf, v_ptr=vf, lse_ptr=lse, delta_ptr=delta, grad_o_ptr=gof, grad_k_ptr=dk,
            grad_v_ptr=dv, block_mask_ptr=mask, softmax_scale=scale, seq_len=N, num_kv_heads=Hk,
            num_q_heads=Hq, q_heads_per_kv_head=Hq // Hk, feature_dim=64, kv_block_size=bs, q_tile_size=64)
        rows = torch.sort(torch.randperm(N, generator=torch.Generator().manual_seed(200 + seed))[:64]).values
        f16 = lambda t: t[:, rows].to(torch.float16).numpy()
        sums = lambda t: t.double().sum(dim=(1, 3)).numpy()
        np.savez_compressed(
            os.path.join(HERE, f"{name}.npz"),
            meta=np.array([B, N, Hq, Hk, bs, K, seed, int(repeat)], dtype=np.int64),
            rows=rows.numpy().astype(np.int32),
            block_indices=idx.numpy().astype(np.int16),
            dq_rows=f16(dq), dk_rows=f16(dk), dv_rows=f16(dv),
            dq_sums=sums(dq), dk_sums=sums(dk), dv_sums=sums(dv),
        )
        print(name, "written")


BLOCK_CONFIGS = {
    # name: S, B, dim, Hq, Hk, bas, bs, K, seed, block_attn_only, no_compression
    "block_n768_d256_h4x1": (768, 1, 256, 4, 1, 256, 64, 4, 20, False, False),
    "block_n768_b2_d512_h8x2_nocmp": (768, 2, 512, 8, 2, 256, 128, 2, 21, False, True),
}


def main_block(P):
    """primitives.MosaicAttention.forward itself (fp32 on the CPU, bf16-valued weights and
    input, its Triton sparse kernel in the interpreter, flash-attn as SDPA)."""
    import types as _types
    sys.path.insert(0, ROOT)
    from oracle import bsa_oracle as O
    from tests.golden_util import draw_block_inputs
    real_topk = P.attn_topk
    for name, (S, B, dim, Hq, Hk, bas, bs, K, seed, bao, noc) in BLOCK_CONFIGS.items():
        x, w_q, w_k, w_v, w_g, w_o = draw_block_inputs(S, B, dim, Hq, Hk, seed)
        cfg = _types.SimpleNamespace(num_heads=Hq, gqa_ratio=Hq // Hk, dim=dim, qkv_compress_ratio=dim // Hq // 64,
                                     rope=True, rope_theta=10000, block_attn_size=bas, sparse_block_size=bs,
                                     sparse_block_count=K)
        mod = P.MosaicAttention(cfg, bao, noc)
        with torch.no_grad():
            mod.to_q.weight.copy_(w_q.float())
            mod.to_k.weight.copy_(w_k.float())
            mod.to_v.weight.copy_(w_v.float())
            mod.to_o.weight.copy_(w_o.float())
            if mod.to_strategy_combine_mlp is not None:
                mod.to_strategy_combine_mlp.weight.copy_(w_g.float())
        grid = O.healpix_grid(int(round((S / 12) ** 0.5)))
        mod.q_rope.initialize_rope(grid)
        mod.k_rope.initialize_rope(grid)
        seen = {}

        def topk_rec(qc, kc, kk, _seen=seen):
            idx = real_topk(qc, kc, kk)
            _seen["idx"] = idx
            return idx
        P.attn_topk = topk_rec
        with torch.no_grad():
            out = mod(x.float())
        P.attn_topk = real_topk
        rows = torch.sort(torch.randperm(S, generator=torch.Generator().manual_seed(300 + seed))[:64]).values
        idx = seen.get("idx")
        np.savez_compressed(
            os.path.join(HERE, f"{name}.npz"),
            meta=np.array([S, B, dim, Hq, Hk, bas, bs, K, seed, int(bao), int(noc)], dtype=np.int64),
            rows=rows.numpy().astype(np.int32),
            block_indices=(idx.numpy().astype(np.int16) if idx is not None else np.zeros(0, np.int16)),
            out_rows=out[rows].to(torch.float16).numpy(),
            out_sums=out.double().sum(dim=(0, 2)).numpy(),
        )
        print(name, "written")


INTERP_CONFIGS = {
    # name: n_lon, n_lat, nside, to_hp, B, dim, heads, k, seed
    "interp_ll24x13_to_hp4_d256_h4_k8": (24, 13, 4, True, 2, 256, 4, 8, 30),
    "interp_hp4_to_ll24x13_d512_h8_k6": (24, 13, 4, False, 1, 512, 8, 6, 31),
}


def main_interp(P):
    """primitives.CrossAttentionInterpolate itself (fp32 on the CPU): the reference's
    neighbour search (utils.get_neighbors, sklearn BallTree, haversine), relative
    positions and forward on seeded bf16-valued weights and input. The HEALPix pixel
    centres come from the oracle's restatement (healpy is not installed)."""
    import types as _types
    sys.path.insert(0, ROOT)
    from tests.golden_util import draw_interp_inputs, interp_grids
    for name, (n_lon, n_lat, nside, to_hp, B, dim, H, kn, seed) in INTERP_CONFIGS.items():
        ll, hp = interp_grids(n_lon, n_lat, nside)
        pos_from, pos_to = (ll, hp) if to_hp else (hp, ll)
        x, w_q, w_kv, w_o = draw_interp_inputs(pos_from.shape[0], B, dim, seed)
        cfg = _types.SimpleNamespace(k_neighbors=kn, dim=dim, num_heads=H, rmsnorm_elementwise_affine=False)
        mod = P.CrossAttentionInterpolate(cfg)
        with torch.no_grad():
            mod.to_q.weight.copy_(w_q.float())
            mod.to_kv.weight.copy_(w_kv.float())
            mod.to_o.weight.copy_(w_o.float())
        mod.initialize_interpolation_scheme(pos_from, pos_to)
        with torch.no_grad():
            out = mod(x.float())
        rows = torch.sort(torch.randperm(pos_to.shape[0], generator=torch.Generator().manual_seed(400 + seed))[:64]).values
        np.savez_compressed(
            os.path.join(HERE, f"{name}.npz"),
            meta=np.array([n_lon, n_lat, nside, int(to_hp), B, dim, H, kn, seed], dtype=np.int64),
            neighbors=mod.neighbors.numpy().astype(np.int32),
            rows=rows.numpy().astype(np.int32),
            out_rows=out[rows].to(torch.float16).numpy(),
            out_sums=out.double().sum(dim=(0, 2)).numpy(),
        )
        print(name, "written")


UPDOWN_CONFIGS = {
    # name: kind, nside_before, nside_after, B, c_in, c_out, affine, seed
    "down_hp8_to_hp4_c64_o128_b2": ("down", 8, 4, 2, 64, 128, False, 40),
    "down_hp16_to_hp4_c64_o128_b1_affine": ("down", 16, 4, 1, 64, 128, True, 41),
    "up_hp4_to_hp8_c128_o128_b2_affine": ("up", 4, 8, 2, 128, 128, True, 42),
}


def main_updown(P):
    """primitives.HEALPixDownsample / HEALPixUpsample themselves (fp32 on the CPU): their
    rel_pos construction (with the oracle's HEALPix centres, healpy being absent) and
    forward on seeded bf16-valued weights and input. Keeps rel_pos, 64 sampled output rows
    (fp16) and fp64 per-member sums."""
    sys.path.insert(0, ROOT)
    from oracle import bsa_oracle as O
    from tests.golden_util import draw_updown_inputs
    P.get_healpix_grid = O.healpix_grid
    for name, (kind, nb, na, B, c_in, c_out, affine, seed) in UPDOWN_CONFIGS.items():
        F = (max(nb, na) // min(nb, na)) ** 2
        n_coarse = 12 * min(nb, na) ** 2
        x, sc, w_x, w_pos, w_norm = draw_updown_inputs(kind, n_coarse, F, B, c_in, c_out, affine, seed)
        cls = P.HEALPixDownsample if kind == "down" else P.HEALPixUpsample
        mod = cls(c_in, c_out, nb, na, rmsnorm_elementwise_affine=affine)
        with torch.no_grad():
            mod.proj_x.weight.copy_(w_x.float())
            mod.proj_pos.weight.copy_(w_pos.float())
            if affine:
                mod.norm.weight.copy_(w_norm.float())
            out = mod(x.float()) if kind == "down" else mod(x.float(), sc.float())
        flat = out.reshape(-1, out.shape[-1])
        rows = torch.sort(torch.randperm(flat.shape[0], generator=torch.Generator().manual_seed(500 + seed))[:64]).values
        np.savez_compressed(
            os.path.join(HERE, f"{name}.npz"),
            meta=np.array([0 if kind == "down" else 1, nb, na, B, c_in, c_out, int(affine), seed], dtype=np.int64),
            rel_pos=mod.rel_pos.numpy().astype(np.float32),
            rows=rows.numpy().astype(np.int32),
            out_rows=flat[rows].to(torch.float16).numpy(),
            out_sums=out.double().sum(dim=(0, 2)).numpy(),
        )
        print(name, "written")


def main(ref_dir, parts=("attn", "bwd", "block", "interp", "updown")):
    sys.path.insert(0, ROOT)
    from oracle import bsa_oracle as O
    ops, P = _import_reference(ref_dir)
    if "updown" in parts:
        main_updown(P)
    if "attn" not in parts and "block" not in parts:
        if "bwd" in parts:
            main_bwd(ops)
        if "interp" in parts:
            main_interp(P)
        return
    triton_sparse = make_triton_sparse(ops)
    P.flash_attn_func = sdpa_gqa
    P.mosaic_sparse_attn = triton_sparse
    real_topk = P.attn_topk

    for name, (B, N, Hq, Hk, bs, K, bas, seed) in (CONFIGS.items() if "attn" in parts else ()):
        g = torch.Generator().manual_seed(seed)
        q_raw = torch.randn(B, N, Hq, 64, generator=g).bfloat16()
        k_raw = torch.randn(B, N, Hk, 64, generator=g).bfloat16()
        v = torch.randn(B, N, Hk, 64, generator=g).bfloat16()
        w = torch.sigmoid(torch.randn(3, B, N, Hq, 1, generator=g)).bfloat16()
        nside = int(round((N / 12) ** 0.5))
        rope = P.RoPE(64, 10000)
        rope.initialize_rope(O.healpix_grid(nside))
        q = rope(q_raw)  # bf16 out, like MosaicAttention.forward (primitives.py:193-195)
        k = rope(k_raw)
        # bf16 top-k, exactly as the reference computes it on bf16 activations
        from einops import reduce
        q_cmp = reduce(q, 'b (nb bs) h d -> b nb h d', 'mean', bs=bs)
        k_cmp = reduce(k, 'b (nb bs) h d -> b nb h d', 'mean', bs=bs)
        idx = real_topk(q_cmp, k_cmp, K)
        # fp32 run of the orchestration on the same (bf16-valued) inputs, driven by that selection
        P.attn_topk = lambda qc, kc, kk, _idx=idx: _idx
        qf, kf, vf, wf = q.float(), k.float(), v.float(), w.float()
        out = P.mosaic_attn_func(qf, kf, vf, wf, bas, bs, K, False, False)
        o_ba = P.block_attention(qf, kf, vf, bas)
        o_slc = triton_sparse(qf, kf, vf, idx, bs)
        lse = triton_sparse.last_lse
        qc, kc, vc = (reduce(t, 'b (nb bs) h d -> b nb h d', 'mean', bs=bs) for t in (qf, kf, vf))
        o_cmp = sdpa_gqa(qc, kc, vc)
        out_nocmp = P.mosaic_attn_func(qf, kf, vf, wf, bas, bs, K, False, True)
        out_k0 = P.mosaic_attn_func(qf, kf, vf, wf, bas, bs, 0, False, False)
        P.attn_topk = real_topk
        rows = torch.sort(torch.randperm(N, generator=torch.Generator().manual_seed(100 + seed))[:64]).values
        f16 = lambda t: t[:, rows].to(torch.float16).numpy()
        sums = lambda t: t.double().sum(dim=(1, 3)).numpy()  # [B, Hq]
        np.savez_compressed(
            os.path.join(HERE, f"{name}.npz"),
            meta=np.array([B, N, Hq, Hk, bs, K, bas, seed], dtype=np.int64),
            rows=rows.numpy().astype(np.int32),
            block_indices=idx.numpy().astype(np.int16),
            q_rot_rows=f16(q.float()), k_rot_rows=f16(k.float()),
            q_cmp=q_cmp.float().numpy().astype(np.float16), k_cmp=k_cmp.float().numpy().astype(np.float16),
            o_cmp=o_cmp.numpy().astype(np.float16),
            out_rows=f16(out), o_ba_rows=f16(o_ba), o_slc_rows=f16(o_slc),
            lse_rows=lse[:, rows].numpy(),
            out_nocmp_rows=f16(out_nocmp), out_k0_rows=f16(out_k0),
            out_sums=sums(out), o_ba_sums=sums(o_ba), o_slc_sums=sums(o_slc),
        )
        print(name, "written")
    if "bwd" in parts:
        main_bwd(ops)
    if "block" in parts:
        main_block(P)
    if "interp" in parts:
        main_interp(P)


if __name__ == "__main__":
    ref = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("MOSAIC_REFERENCE_DIR", "")
    if not ref or not os.path.isdir(ref):
        raise SystemExit("usage: TRITON_INTERPRET=1 python tests/golden/make_golden.py <reference checkout> [part ...]")
    main(ref, tuple(sys.argv[2:]) or ("attn", "bwd", "block", "interp", "updown"))
