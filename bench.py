#!/usr/bin/env python
"""Benchmark of the Mosaic block-sparse attention forward on B200.

Default workload ("S1", the stage-1 attention of the headline metric): one
mosaic_attn_func forward at Nside 64 —
B=1 per GPU, N=49152 tokens, 12 query / 3 kv heads, head_dim 64, sparse block 64,
top-k 24, local window 1024, bf16, synthetic q/k/v ~ N(0,1) and gates
sigmoid(N(0,1)). A step = the four kernels of the op on one member's inputs:
(a) block pool, coarse attention, (b) scores + top-k, (c) fused local + selected
attention with the gated combine. Ensemble members are independent, so with
--gpus N every rank runs its own member (weak scaling, no collective in the step).

Timing: W untimed warm-up steps, then K steps of `mosaic_bsa_fwd` (the C-ABI
entry point of the whole op) between barrier + synchronize, CUDA events on the
launching stream, max over ranks. Several input sets (S1: 4 x 117 MB against the
126 MB L2) rotate so no step reads inputs left in L2 by the previous ones. Per-kernel
durations come from a second loop of K steps right after the timed one that
launches the same kernels one entry point at a time with CUDA events between
them; `roofline` uses the fused kernel (c) from that loop.

--workload S1_bas64 | S1_bs128 | S2 | BN | X128 | X256 runs the other configurations
(S1 with a 64-token local window or the reference preset's 128-token blocks, the
deeper U-Net stages, the Nside 128 / 256 stress cases) instead; X128 / X256 also
time cuDNN dense SDPA on the same inputs (`dense_sdpa`).

The line also carries `backward`: the device time of mosaic_sparse_attn's backward
(the training path of the selected branch, ops.mosaic_attn_bwd) on the same workload
and its FLOP rate against the measured bf16 peak (--no-backward skips it); and
`attention_block`: the whole MosaicAttention forward at the stage's dims (fused
projections + attention + output projection, stage times, the projection GEMMs' FLOP
rates) next to the reference module's eager sequence on the same GPU (--no-block
skips it); and, for S1, `interpolation`: CrossAttentionInterpolate in both grid
directions at the model's sizes, likewise beside its eager sequence (--no-interp), and
`updown`: HEALPixDownsample 64 -> 32 and HEALPixUpsample 32 -> 64 at the U-Net's first
stage dims, beside their eager sequences (--no-updown).

For S1 the line also carries `ensemble`: one 24-member ensemble step of the U-Net's
attention work sharded by member over the ranks (the 14 mosaic_attn_func calls of a step
per member at the reference presets, then an NCCL all-gather of per-member output
fields), as step/s with the gather's share (--no-ensemble skips it); and, on one GPU,
`reference_gpu`: the reference's own GPU code from baseline/_ref (its Triton
selected-block kernel, its flash-attn local branch, its whole mosaic_attn_func) timed
on the same inputs beside ours, with the output differences (--no-reference-gpu).

`unet_step` (S1 default run; --no-model skips it): one 24-member forward step of the
whole U-Net — the reference's Transformer from baseline/_ref with mosaic_b200's modules
rebound into it, random weights, bf16 — sharded by member over the ranks with the
output fields all-gathered over NCCL in the step, eager and replayed from one CUDA
graph, and on one GPU beside the same model with the reference's own modules.

`--impl reference` times the reference algorithm on the host cores instead: the
reference's CPU form is the oracle port (oracle/bsa_oracle.py; the reference itself
needs CUDA for flash-attn and Triton), run on a bounded sample of the same workload
per step: the sequence-global part (pooling, coarse attention, top-k over all tokens)
once and the local + selected branches of 4 of the 48 windows; the full call is
extrapolated as t_global + t_windows x 48 / 4.
"""
import argparse
import ctypes
import json
import os
import statistics
import sys
import threading
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "BSA fwd tokens/s/GPU @Nside64 (N=49152,12h,d64,k24); 24-member step/s @1-8 GPU"
UNIT = "tokens/s"
S1 = dict(B=1, N=49152, Hq=12, Hk=3, D=64, bs=64, K=24, bas=1024)
# The metric's configurations as bench workloads. S1 is the default and the headline; the
# others are opt-in (--workload) lines: S2 / BN are the deeper U-Net stages, X128 /
# X256 the resolution-scaling stress cases, which also time cuDNN dense SDPA on the
# same inputs.
WORKLOADS = {
    "S1": dict(S1, nside=64),
    "S1_bas64": dict(S1, bas=64, nside=64),
    "S1_bs128": dict(S1, bs=128, nside=64),
    "S2": dict(B=1, N=12288, Hq=16, Hk=4, D=64, bs=64, K=20, bas=1024, nside=32),
    "BN": dict(B=1, N=3072, Hq=20, Hk=5, D=64, bs=64, K=20, bas=1024, nside=16),
    "X128": dict(B=1, N=196608, Hq=12, Hk=3, D=64, bs=64, K=24, bas=1024, nside=128),
    "X256": dict(B=1, N=786432, Hq=12, Hk=3, D=64, bs=64, K=24, bas=1024, nside=256),
}
# dram__bytes_read.sum + dram__bytes_write.sum of one bsa_engine_kernel attend launch
# at S1, from an `ncu --set full --clock-control none -k regex:bsa_engine` capture of
# this script (--steps 3 --warmup 3 --no-e2e --no-cpu-baseline); updated with the kernel.
ATTEND_TRAFFIC_BYTES = {"S1": 127_683_328 + 48_043_008}
L2_BYTES = 126 * 2**20


def describe(name, c):
    return (f"{name} mosaic_attn_func forward, Nside {c['nside']}: N={c['N']}, {c['Hq']}/{c['Hk']} heads, "
            f"d{c['D']}, sparse block {c['bs']}, top-k {c['K']}, window {c['bas']}; one ensemble member per GPU")
PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}
MEMBERS = 24


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=200)
    p.add_argument("--warmup", type=int, default=10)
    p.add_argument("--impl", choices=["b200", "reference"], default="b200")
    p.add_argument("--workload", choices=sorted(WORKLOADS), default="S1")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--no-backward", action="store_true")
    p.add_argument("--no-block", action="store_true")
    p.add_argument("--no-interp", action="store_true")
    p.add_argument("--no-updown", action="store_true")
    p.add_argument("--no-ensemble", action="store_true")
    p.add_argument("--no-reference-gpu", action="store_true")
    p.add_argument("--no-model", action="store_true")
    p.add_argument("--no-rollout", action="store_true")
    return p.parse_args()


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        d = json.load(open(path))
        return d["hbm_gbs"], d["bf16_tflops"], "measured"
    return PEAKS_FALLBACK["hbm_gbs"], PEAKS_FALLBACK["bf16_tflops"], "fallback"


def flops_attend(c):
    """FLOP of kernel (c): QK^T and PV over K*bs selected + bas local keys, 2 FLOP/MAC."""
    return 4 * c["B"] * c["N"] * c["Hq"] * c["D"] * (c["K"] * c["bs"] + c["bas"])


def flops_backward(c):
    """FLOP of the selected-block attention backward: per (query row, head, selected key)
    S, dP and dQ (3 x 128) in the dQ kernel and S^T, dP^T, dV, dK (4 x 128) in the dK/dV
    kernel, 2 FLOP/MAC over head_dim 64."""
    return 896 * c["B"] * c["N"] * c["Hq"] * c["K"] * c["bs"]


def backward_leg(c, sets, stream, steps, warmup):
    """Device time of mosaic_sparse_attn's backward (ops.mosaic_attn_bwd) on the
    workload's selected branch, with the selection top-k made on each input set."""
    import mosaic_b200 as M
    from mosaic_b200 import ops as mops

    scale = c["D"] ** -0.5
    legs = []
    for x in sets[:4]:
        qc, kc, _ = M.block_pool(x["q"], x["k"], x["v"], c["bs"])
        idx = M.attn_topk(qc, kc, c["K"])
        out, lse = mops.mosaic_attn_fwd(x["q"], x["k"], x["v"], idx, c["bs"], scale)
        go = torch.randn_like(x["q"], dtype=torch.float32).bfloat16()
        legs.append((x, idx, out, lse, go))
    status = mops.status_buffer(sets[0]["q"].device)

    def step(i):
        x, idx, out, lse, go = legs[i % len(legs)]
        mops.mosaic_attn_bwd(x["q"], x["k"], x["v"], out, lse, go, scale, idx, c["bs"], status=status)

    for i in range(warmup):
        step(i)
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for i in range(steps):
        step(i)
    b.record(stream)
    torch.cuda.synchronize()
    if int(status.item()):
        raise RuntimeError(f"device status {int(status.item())} after the backward leg")
    return a.elapsed_time(b) / steps


def block_leg(c, sets, stream, steps, warmup):
    """The whole attention block of a Mosaic layer (primitives.MosaicAttention.forward) at
    the workload's stage dims (dim = 64 Hq): the fused path (mosaic_attn_qkv_proj ->
    mosaic_attn_func -> mosaic_attn_out_proj) timed stage by stage, and the reference
    module's eager sequence on the same GPU (cuBLAS Linear layers, torch RoPE and
    softmax, layout copies, the same attention op in the middle) for comparison."""
    import torch.nn.functional as F

    import mosaic_b200 as M
    from mosaic_b200 import attention as A
    from mosaic_b200.healpix import healpix_rope_tables

    B, N, Hq, Hk = c["B"], c["N"], c["Hq"], c["Hk"]
    dim = 64 * Hq
    dev = sets[0]["q"].device
    g = torch.Generator(device=dev).manual_seed(99)
    sd = dim ** -0.5
    w_q, w_k, w_v = ((torch.randn(h * 64, dim, generator=g, device=dev) * sd).bfloat16() for h in (Hq, Hk, Hk))
    w_g = (torch.randn(3 * Hq, dim, generator=g, device=dev) * sd).bfloat16()
    w_o = (torch.randn(dim, Hq * 64, generator=g, device=dev) * (Hq * 64) ** -0.5).bfloat16()
    w_cat = torch.cat([w_q, w_k, w_v, w_g])
    cos, sin = (t.to(dev) for t in healpix_rope_tables(c["nside"]))
    xs = [torch.randn(N, B, dim, generator=g, device=dev).bfloat16() for _ in range(4)]

    def fused(x, ev=None):
        if ev: ev[0].record(stream)
        q, k, v, gw = A.qkv_projection(x, w_cat, Hq, Hk, cos, sin)
        if ev: ev[1].record(stream)
        o = M.mosaic_attn_func(q, k, v, gw, c["bas"], c["bs"], c["K"], False)
        if ev: ev[2].record(stream)
        out = A.out_projection(o, w_o)
        if ev: ev[3].record(stream)
        return out

    cos2 = cos.unsqueeze(0).unsqueeze(2).repeat_interleave(2, dim=-1)
    sin2 = sin.unsqueeze(0).unsqueeze(2).repeat_interleave(2, dim=-1)

    def rope(x):
        xf = x.float()
        rot = torch.stack((-xf[..., 1::2], xf[..., 0::2]), dim=-1).flatten(-2)
        return (xf * cos2 + rot * sin2).to(x.dtype)

    def eager(x):
        q = F.linear(x, w_q).reshape(N, B, Hq, 64).permute(1, 0, 2, 3)
        k = F.linear(x, w_k).reshape(N, B, Hk, 64).permute(1, 0, 2, 3)
        v = F.linear(x, w_v).reshape(N, B, Hk, 64).permute(1, 0, 2, 3).contiguous()
        logits = F.linear(x, w_g).reshape(N, B, Hq, 3).permute(3, 1, 0, 2)
        gw = torch.softmax(logits.float(), dim=0).to(x.dtype)
        q, k = rope(q).contiguous(), rope(k).contiguous()
        o = M.mosaic_attn_func(q, k, v, gw.unsqueeze(-1), c["bas"], c["bs"], c["K"], False)
        return F.linear(o.permute(1, 0, 2, 3).reshape(N, B, Hq * 64), w_o)

    ref_out, out = eager(xs[0]), fused(xs[0])
    torch.cuda.synchronize()
    agree = float((ref_out.float() - out.float()).abs().max())
    for i in range(warmup):
        fused(xs[i % 4])
        eager(xs[i % 4])
    torch.cuda.synchronize()
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(steps)]
    for i in range(steps):
        fused(xs[i % 4], evs[i])
    torch.cuda.synchronize()
    st = [sum(e[j].elapsed_time(e[j + 1]) for e in evs) / steps for j in range(3)]
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for i in range(steps):
        eager(xs[i % 4])
    b.record(stream)
    torch.cuda.synchronize()
    eager_ms = a.elapsed_time(b) / steps
    M_ = B * N
    flop_in = 2 * M_ * dim * (w_cat.shape[0])
    flop_out = 2 * M_ * (Hq * 64) * dim
    return {"what": f"primitives.MosaicAttention.forward at dim {dim}: fused projection (RoPE, gates) -> "
                    "mosaic_attn_func -> output projection", "steps": steps,
            "ms": sum(st), "tokens_per_s": M_ / (sum(st) / 1000),
            "stages_us": {"qkv_proj": 1000 * st[0], "attention": 1000 * st[1], "out_proj": 1000 * st[2]},
            "qkv_proj_tflops": flop_in / (st[0] / 1000) / 1e12, "out_proj_tflops": flop_out / (st[2] / 1000) / 1e12,
            "eager_reference_sequence_ms": eager_ms, "fused_speedup_vs_eager": eager_ms / sum(st),
            "max_abs_vs_eager": agree}


def interp_leg(stream, steps, warmup, dim=768, heads=12, k=24):
    """primitives.CrossAttentionInterpolate.forward at the model's sizes (dim 768, 12 heads,
    24 neighbours, one ensemble member) in both directions between the 240 x 121 lat-lon
    grid and HEALPix nside 64: mosaic_row_rms + mosaic_linear (to_kv) ->
    mosaic_interp_attend_tiled (tables built once, as the module does at scheme set-up) ->
    mosaic_linear (to_o), stage by stage, beside the reference module's eager torch
    sequence on the same GPU (RMSNorm, Linear layers, gather, softmax). The untiled
    gather kernel (mosaic_interp_attend) is timed beside the tiled one."""
    import torch.nn.functional as F

    from mosaic_b200 import interp as I
    from mosaic_b200.healpix import get_healpix_grid

    dev = torch.device("cuda", torch.cuda.current_device())
    lon = torch.linspace(0, 360, 241)[:-1]
    lat = torch.linspace(-90, 90, 121)
    ll = torch.deg2rad(torch.stack(torch.meshgrid(lon, lat, indexing="ij"), -1).reshape(-1, 2)).to(dev)
    hp = torch.deg2rad(get_healpix_grid(64)).to(dev)
    g = torch.Generator(device=dev).manual_seed(7)
    w_q = torch.randn(dim, 3, generator=g, device=dev)
    w_kv = (torch.randn(2 * dim, dim, generator=g, device=dev) * dim ** -0.5).bfloat16()
    w_o = (torch.randn(dim, dim, generator=g, device=dev) * dim ** -0.5).bfloat16()
    res = {}
    for name, (pf, pt) in (("ll_to_hp", (ll, hp)), ("hp_to_ll", (hp, ll))):
        nb = I.knn_neighbors(pf, pt, k)
        rel = F.normalize(I.rad_to_xyz(pt).unsqueeze(1) - I.rad_to_xyz(pf)[nb], dim=-1).float()
        nb32 = nb.to(torch.int32)
        tiles = {key: (val.to(dev) if torch.is_tensor(val) else val) for key, val in I.build_tiles(nb, pt).items()}
        S_from, S_to = pf.shape[0], pt.shape[0]
        xs = [torch.randn(S_from, 1, dim, generator=g, device=dev).bfloat16() for _ in range(4)]
        eps = torch.finfo(torch.float32).eps  # torch.nn.RMSNorm's eps=None default

        def fused(x, ev=None):
            if ev: ev[0].record(stream)
            kv = I.linear(x, w_kv, I.row_rms(x, eps))
            if ev: ev[1].record(stream)
            o = I.interp_attend_tiled(kv, tiles, rel, w_q, heads, S_from)
            if ev: ev[2].record(stream)
            out = I.linear(o, w_o)
            if ev: ev[3].record(stream)
            return out

        def eager(x):
            q = F.linear(rel, w_q).reshape(S_to, k, 1, heads, dim // heads)
            xn = F.rms_norm(x, (dim,), eps=eps)
            kv = F.linear(xn, w_kv).reshape(S_from, 1, 2, heads, dim // heads).permute(2, 0, 1, 3, 4)
            kk, vv = kv[:, nb]
            a = torch.softmax((q * kk).sum(-1, keepdim=True).float() * (dim // heads) ** -0.5, dim=1).to(x.dtype)
            return F.linear((a * vv).sum(1).reshape(S_to, 1, dim), w_o)

        ref_out, out = eager(xs[0]), fused(xs[0])
        torch.cuda.synchronize()
        diff = float((ref_out.float() - out.float()).abs().max())
        for i in range(warmup):
            fused(xs[i % 4])
            eager(xs[i % 4])
        torch.cuda.synchronize()
        evs = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(steps)]
        for i in range(steps):
            fused(xs[i % 4], evs[i])
        torch.cuda.synchronize()
        st = [sum(e[j].elapsed_time(e[j + 1]) for e in evs) / steps for j in range(3)]
        a_, b_ = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a_.record(stream)
        for i in range(steps):
            eager(xs[i % 4])
        b_.record(stream)
        torch.cuda.synchronize()
        eager_ms = a_.elapsed_time(b_) / steps
        kv0 = I.linear(xs[0], w_kv, I.row_rms(xs[0], eps))
        a_.record(stream)
        for i in range(steps):
            I.interp_attend(kv0, nb32, rel, w_q, heads, S_from)
        b_.record(stream)
        torch.cuda.synchronize()
        untiled_us = 1000 * a_.elapsed_time(b_) / steps
        gather = S_to * k * 2 * dim * 2                              # k / v bytes the targets read
        hbm = S_from * 2 * dim * 2 + S_to * dim * 2 + S_to * k * 16   # kv once, out, neighbours + rel_pos
        res[name] = {"points_from": S_from, "points_to": S_to, "ms": sum(st),
                     "stages_us": {"rms_to_kv": 1000 * st[0], "attend": 1000 * st[1], "to_o": 1000 * st[2]},
                     "attend_untiled_us": untiled_us, "tiles": tiles["tile_targets"].numel() - 1,
                     "union_reuse": S_to * k / tiles["tile_points"].numel(),
                     "attend_gather_gbs": gather / (st[1] / 1000) / 1e9, "attend_hbm_gbs": hbm / (st[1] / 1000) / 1e9,
                     "eager_reference_sequence_ms": eager_ms, "fused_speedup_vs_eager": eager_ms / sum(st),
                     "max_abs_vs_eager": diff}
    res["what"] = ("primitives.CrossAttentionInterpolate.forward, dim 768, 12 heads, k 24, one member, "
                   "240 x 121 lat-lon <-> HEALPix nside 64")
    return res


def updown_leg(stream, steps, warmup, dims=(768, 1024), nsides=(64, 32)):
    """primitives.HEALPixDownsample (nside 64 -> 32, 768 -> 1024 channels) and
    HEALPixUpsample (32 -> 64, 1024 -> 768, with the skip connection) at the U-Net's first
    stage, one member: the fused modules (one tcgen05 GEMM with the bias / shortcut
    epilogue + the RMSNorm pass) beside the reference modules' eager sequence (rearrange,
    two cuBLAS Linear layers, adds, torch RMSNorm) on the same GPU, same bf16 weights."""
    import torch.nn.functional as F_
    from mosaic_b200 import updown as U

    dev = torch.device("cuda", torch.cuda.current_device())
    g = torch.Generator(device=dev).manual_seed(11)
    c_fine, c_coarse = dims
    nf, nc = nsides
    Fk = (nf // nc) ** 2
    n = 12 * nc * nc
    res = {}
    for kind in ("down", "up"):
        c_in, c_out = (c_fine, c_coarse) if kind == "down" else (c_coarse, c_fine)
        m = (U.HEALPixDownsample(c_in, c_out, nf, nc, False) if kind == "down"
             else U.HEALPixUpsample(c_in, c_out, nc, nf, False)).to(dev)
        m.proj_x.to(torch.bfloat16)
        m.proj_pos.to(torch.bfloat16)
        rows_in = n * Fk if kind == "down" else n
        xs = [torch.randn(rows_in, 1, c_in, generator=g, device=dev).bfloat16() for _ in range(4)]
        scs = [torch.randn(n * Fk, 1, c_out, generator=g, device=dev).bfloat16() for _ in range(4)]
        eps = torch.finfo(torch.float32).eps  # torch.nn.RMSNorm's eps=None default
        rel = m.rel_pos.bfloat16()

        def fused(i):
            return m(xs[i % 4]) if kind == "down" else m(xs[i % 4], scs[i % 4])

        def eager(i):
            x = xs[i % 4]
            if kind == "down":
                y = F_.linear(x.reshape(n, Fk, 1, c_in).permute(0, 2, 1, 3).reshape(n, 1, Fk * c_in), m.proj_x.weight)
                y = y + F_.linear(rel, m.proj_pos.weight).unsqueeze(1)
            else:
                y = F_.linear(x, m.proj_x.weight) + F_.linear(rel, m.proj_pos.weight).unsqueeze(1)
                y = y.reshape(n, 1, Fk, c_out).permute(0, 2, 1, 3).reshape(n * Fk, 1, c_out) + scs[i % 4]
            return F_.rms_norm(y, (c_out,), eps=eps)

        with torch.no_grad():
            diff = float((fused(0).float() - eager(0).float()).abs().max())
            ts = {}
            for label, fn in (("fused", fused), ("eager", eager)):
                for i in range(warmup):
                    fn(i)
                torch.cuda.synchronize()
                a_, b_ = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a_.record(stream)
                for i in range(steps):
                    fn(i)
                b_.record(stream)
                torch.cuda.synchronize()
                ts[label] = a_.elapsed_time(b_) / steps
        flop = 2 * n * (Fk * c_in if kind == "down" else c_in) * (c_out if kind == "down" else Fk * c_out)
        res[kind] = {"ms": ts["fused"], "gemm_tflops_incl_norm": flop / (ts["fused"] / 1000) / 1e12,
                     "eager_reference_sequence_ms": ts["eager"], "fused_speedup_vs_eager": ts["eager"] / ts["fused"],
                     "max_abs_vs_eager": diff, "flop": flop}
    res["what"] = (f"HEALPixDownsample nside {nf}->{nc} ({c_fine}->{c_coarse}) and HEALPixUpsample {nc}->{nf} "
                   f"({c_coarse}->{c_fine}, + shortcut), one member, no affine norm")
    return res


def bytes_pool(c):
    """Algorithmic HBM bytes of the pool kernel: read q, k, v once, write the pooled rows."""
    heads = c["Hq"] + 2 * c["Hk"]
    return c["B"] * c["N"] * heads * c["D"] * 2 + c["B"] * (c["N"] // c["bs"]) * heads * c["D"] * 2


# ----------------------------------------------------------------------------- clocks
class ClockSampler:
    """Polls SM clock and throttle reasons through NVML (read-only) while running."""

    REASONS = {
        "hw_slowdown": 0x8, "hw_thermal_slowdown": 0x40, "sw_thermal_slowdown": 0x20, "sw_power_cap": 0x4,
        "hw_power_brake_slowdown": 0x80,
    }

    def __init__(self, device_index):
        self.samples, self.reasons, self.max_mhz = [], set(), None
        self._stop = threading.Event()
        try:
            import pynvml

            pynvml.nvmlInit()
            uuid = str(torch.cuda.get_device_properties(device_index).uuid)
            self.h = None
            for i in range(pynvml.nvmlDeviceGetCount()):
                h = pynvml.nvmlDeviceGetHandleByIndex(i)
                u = pynvml.nvmlDeviceGetUUID(h)
                u = u.decode() if isinstance(u, bytes) else u
                if u.replace("GPU-", "") == uuid.replace("GPU-", ""):
                    self.h = h
            self.nvml = pynvml
            if self.h is not None:
                self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
        except Exception:
            self.h = None

    def _run(self):
        nv = self.nvml
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM))
                r = nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                for name, bit in self.REASONS.items():
                    if r & bit:
                        self.reasons.add(name)
            except Exception:
                pass
            time.sleep(0.01)

    def __enter__(self):
        if self.h is not None:
            self.t = threading.Thread(target=self._run, daemon=True)
            self.t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        if self.h is not None:
            self.t.join()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["unavailable"], "samples": 0}
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples)}


# ----------------------------------------------------------------------------- CPU legs
def cpu_sample(c, windows, reps, warm=1):
    """Times the oracle port of mosaic_attn_func on the host cores over a bounded sample:
    per rep, the sequence-global part once (pooling, coarse attention, top-k over all
    tokens: oracle.mosaic_attn_global) and the local + selected branches of the sampled
    windows (oracle.mosaic_attn_window). The full call is extrapolated as
    t_full = t_global + t_windows * (windows in the sequence / windows sampled), and the
    rate is B * N / t_full. Returns (tokens/s, cores, seconds spent, t_full seconds)."""
    from oracle import bsa_oracle as O

    torch.set_num_threads(os.cpu_count() or 1)
    x = O.make_inputs(c["B"], c["N"], c["Hq"], c["Hk"], seed=0, rope=False)
    q, k, v, w = x["q"], x["k"], x["v"], x["w"]

    def one():
        t0 = time.perf_counter()
        o_cmp, idx = O.mosaic_attn_global(q, k, v, c["bs"], c["K"])
        t1 = time.perf_counter()
        for win in windows:
            O.mosaic_attn_window(q, k, v, w, c["bas"], c["bs"], win, o_cmp, idx)
        return t1 - t0, time.perf_counter() - t1

    for _ in range(warm):
        one()
    tg, tw = zip(*[one() for _ in range(reps)])
    nw = c["N"] // c["bas"]
    t_full = statistics.mean(tg) + statistics.mean(tw) * nw / len(windows)
    return c["B"] * c["N"] / t_full, torch.get_num_threads(), sum(tg) + sum(tw), t_full


def cpu_sample_text(name, c, windows, reps, warm):
    return (f"oracle port (fp32 torch) of mosaic_attn_func on {name} inputs: per step the global part (pooling, "
            f"coarse attention, top-k over all {c['N']} tokens) once and the local + selected branches of "
            f"{len(windows)} of the {c['N'] // c['bas']} windows; full call = t_global + t_windows x "
            f"{c['N'] // c['bas']}/{len(windows)}, value = B*N / full call; {reps} timed step(s) after {warm} warm-up")


def sample_windows(c, count):
    """`count` local windows spread over the sequence (first and last included)."""
    nw = c["N"] // c["bas"]
    count = min(count, nw)
    return sorted({round(i * (nw - 1) / max(count - 1, 1)) for i in range(count)})


def reference_arm(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    name = args.workload
    c = WORKLOADS[name]
    windows = sample_windows(c, 4)
    value, cores, secs, t_full = cpu_sample(c, windows, reps=args.steps, warm=args.warmup)
    sample = cpu_sample_text(name, c, windows, args.steps, args.warmup)
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "impl": "reference", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000 * secs / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": describe(name, c) + " (CPU sample)", "B": c["B"], "N": c["N"]},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "kind": "port", "sample": sample,
                         "full_call_ms_extrapolated": 1000 * t_full},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------------------- B200 arm
class Stages:
    """The four kernels of mosaic_bsa_fwd, called one by one through the C ABI so
    that CUDA events can bracket each of them."""

    def __init__(self, lib, c, dev):
        from mosaic_b200.ops import _ptr
        self.lib, self.c, self._ptr = lib, c, _ptr
        B, N, Hq, Hk, D, bs, K = c["B"], c["N"], c["Hq"], c["Hk"], c["D"], c["bs"], c["K"]
        nb = N // bs
        e = lambda *s, dt=torch.bfloat16: torch.empty(*s, dtype=dt, device=dev)
        self.q_cmp, self.k_cmp, self.v_cmp = e(B, nb, Hq, D), e(B, nb, Hk, D), e(B, nb, Hk, D)
        self.o_cmp = e(B, nb, Hq, D)
        self.idx = e(B, nb, Hk, K, dt=torch.int64)
        self.out = e(B, N, Hq, D)
        self.status = torch.zeros(1, dtype=torch.int32, device=dev)
        self.ws = torch.empty(lib.mosaic_bsa_workspace_bytes(B, N, Hq, Hk, D, bs, K, 0), dtype=torch.uint8,
                              device=dev)

    def run_fused(self, x, stream):
        """One step through mosaic_bsa_fwd (what mosaic_attn_func calls)."""
        from mosaic_b200 import _lib
        c = self.c
        a = _lib.MosaicBsaArgs()
        a.q, a.k, a.v, a.gates = x["q"].data_ptr(), x["k"].data_ptr(), x["v"].data_ptr(), x["w"].data_ptr()
        a.out = self.out.data_ptr()
        a.block_indices = self.idx.data_ptr()
        a.workspace, a.workspace_bytes = self.ws.data_ptr(), self.ws.numel()
        a.status = self.status.data_ptr()
        a.batch, a.seq_len, a.num_q_heads, a.num_kv_heads, a.head_dim = c["B"], c["N"], c["Hq"], c["Hk"], c["D"]
        a.block_attn_size, a.sparse_block_size, a.sparse_block_count = c["bas"], c["bs"], c["K"]
        rc = self.lib.mosaic_bsa_fwd(ctypes.byref(a), ctypes.c_void_p(stream.cuda_stream))
        if rc:
            raise RuntimeError(f"mosaic_bsa_fwd failed (rc={rc})")

    def run(self, x, stream, events=None):
        p, c, L = self._ptr, self.c, self.lib
        B, N, Hq, Hk, D, bs, K, bas = (c[k] for k in ("B", "N", "Hq", "Hk", "D", "bs", "K", "bas"))
        nb = N // bs
        s = ctypes.c_void_p(stream.cuda_stream)
        null = ctypes.c_void_p(0)
        rec = (lambda i: events[i].record(stream)) if events else (lambda i: None)
        rec(0)
        dt = 0  # MOSAIC_DTYPE_BF16
        rc = L.mosaic_block_pool(p(x["q"]), p(x["k"]), p(x["v"]), null, null, null, null, p(self.q_cmp),
                                 p(self.k_cmp), p(self.v_cmp), B, N, Hq, Hk, D, bs, dt, s)
        rec(1)
        rc |= L.mosaic_cmp_attn_fwd(p(self.q_cmp), p(self.k_cmp), p(self.v_cmp), p(self.o_cmp), p(self.status),
                                    B, nb, Hq, Hk, D, 0.125, dt, s)
        rec(2)
        rc |= L.mosaic_attn_topk(p(self.q_cmp), p(self.k_cmp), p(self.idx), B, nb, Hq, Hk, D, K, dt, s)
        rec(3)
        rc |= L.mosaic_bsa_attend_fwd(p(x["q"]), p(x["k"]), p(x["v"]), p(self.idx), p(x["w"]), p(self.o_cmp),
                                      p(self.out), p(self.status), B, N, Hq, Hk, D, bas, bs, K, 0, 0.125, dt, s)
        rec(4)
        if rc:
            raise RuntimeError(f"mosaic_b200 stage launch failed (rc={rc})")


STAGE_NAMES = ["pool", "cmp_attn", "topk", "attend"]
LAUNCHES_PER_STEP = 4


def dense_sdpa(x, c, reps=3):
    """Times torch SDPA on the cuDNN backend (dense, non-causal) over the same q, k, v:
    the dense attention that block-sparse attention replaces. k and v are expanded to
    the query heads beforehand (outside the timing), so cuDNN runs plain MHA."""
    from torch.nn.attention import SDPBackend, sdpa_kernel
    import torch.nn.functional as F

    G = c["Hq"] // c["Hk"]
    q = x["q"].transpose(1, 2).contiguous()
    k = x["k"].repeat_interleave(G, dim=2).transpose(1, 2).contiguous()
    v = x["v"].repeat_interleave(G, dim=2).transpose(1, 2).contiguous()
    out = None
    for backend, name in ((SDPBackend.CUDNN_ATTENTION, "cudnn"), (SDPBackend.FLASH_ATTENTION, "flash")):
        try:
            with sdpa_kernel(backend):
                out = F.scaled_dot_product_attention(q, k, v)
                torch.cuda.synchronize()
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record()
                for _ in range(reps):
                    out = F.scaled_dot_product_attention(q, k, v)
                b.record()
                torch.cuda.synchronize()
            ms = a.elapsed_time(b) / reps
            flop = 4 * c["B"] * c["N"] * c["N"] * c["Hq"] * c["D"]
            del q, k, v, out
            return {"backend": name, "ms": ms, "tflops": flop / (ms / 1000) / 1e12, "reps": reps}
        except RuntimeError as e:  # backend not available for this shape: try the next one
            err = str(e).splitlines()[0][:120]
    return {"backend": None, "error": err}


def _timed(fn, stream, reps, warmup):
    """Mean device milliseconds of fn() over `reps` calls (CUDA events on `stream`)."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for _ in range(reps):
        fn()
    b.record(stream)
    torch.cuda.synchronize()
    return a.elapsed_time(b) / reps


def reference_gpu_leg(c, x, stream, reps, warmup):
    """The reference's own GPU code on the same B200 and inputs (baseline/reference.py):
    its Triton selected-block kernel (ops.mosaic_attn_fwd_kernel, every autotuner config
    valid for the block size, best one reported) against the selected-only mode of
    kernel (c) on the same block indices; its local branch (primitives.block_attention
    = flash_attn_func) against mosaic_block_attn_fwd; and its whole
    primitives.mosaic_attn_func against ours. Outputs are compared too."""
    from baseline import reference as R

    if not R.available():
        return {"unavailable": "baseline/_ref is empty (the reference checkout was absent when build() ran)"}
    import mosaic_b200 as M
    from mosaic_b200 import ops as mops

    ref = R.load(x["q"].device)
    B, N, Hq, D, bs, K, bas = (c[k] for k in ("B", "N", "Hq", "D", "bs", "K", "bas"))
    q, k, v = x["q"], x["k"], x["v"]
    w5 = x["w"].unsqueeze(-1)
    scale = D ** -0.5
    qc, kc, _ = M.block_pool(q, k, v, bs)
    idx = M.attn_topk(qc, kc, K)
    res = {"what": "reference GPU code (Triton kernel, flash-attn / torch ops) on the same B200 and inputs",
           "notes": ref.notes}
    cfg_ms = {}
    for cfg in ref.configs(bs):
        cfg_ms[json.dumps(cfg)] = _timed(lambda: ref.sparse_attn_fwd(q, k, v, idx, bs, scale, cfg), stream, reps,
                                         warmup)
    best = min(cfg_ms, key=cfg_ms.get)
    ref.config = json.loads(best)
    ours_sel = _timed(lambda: mops.mosaic_attn_fwd(q, k, v, idx, bs, scale), stream, reps, warmup)
    r_out, r_lse = ref.sparse_attn_fwd(q, k, v, idx, bs, scale)
    o_out, o_lse = mops.mosaic_attn_fwd(q, k, v, idx, bs, scale)
    d = (r_out.float() - o_out.float()).abs()
    flop_sel = 4 * B * N * Hq * D * K * bs
    res["selected"] = {
        "reference_triton_us": 1000 * cfg_ms[best], "reference_triton_config": ref.config,
        "reference_triton_us_by_config": {k_: 1000 * v_ for k_, v_ in cfg_ms.items()},
        "ours_us": 1000 * ours_sel, "speedup": cfg_ms[best] / ours_sel,
        "reference_triton_tflops": flop_sel / (cfg_ms[best] / 1000) / 1e12,
        "ours_tflops": flop_sel / (ours_sel / 1000) / 1e12,
        "max_abs_diff": float(d.max()), "mean_abs_diff": float(d.mean()),
        "lse_max_abs_diff": float((r_lse - o_lse).abs().max())}
    ref_loc = _timed(lambda: ref.primitives.block_attention(q, k, v, bas), stream, reps, warmup)
    ours_loc = _timed(lambda: M.block_attention(q, k, v, bas), stream, reps, warmup)
    d = (ref.primitives.block_attention(q, k, v, bas).float() - M.block_attention(q, k, v, bas).float()).abs()
    res["local"] = {"reference_us": 1000 * ref_loc, "ours_us": 1000 * ours_loc, "speedup": ref_loc / ours_loc,
                    "max_abs_diff": float(d.max()), "mean_abs_diff": float(d.mean())}
    ref_full = _timed(lambda: ref.primitives.mosaic_attn_func(q, k, v, w5, bas, bs, K, False), stream, reps, warmup)
    ours_full = _timed(lambda: M.mosaic_attn_func(q, k, v, w5, bas, bs, K, False), stream, reps, warmup)
    r_full = ref.primitives.mosaic_attn_func(q, k, v, w5, bas, bs, K, False).float()
    o_full, o_idx = M.mosaic_attn_func(q, k, v, w5, bas, bs, K, False, return_block_indices=True)
    d = (r_full - o_full.float()).abs()
    r_idx = ref.primitives.attn_topk(qc, kc, K)
    same_sel = (torch.sort(r_idx, -1).values == torch.sort(o_idx, -1).values).all(-1).float().mean()
    res["mosaic_attn_func"] = {"reference_ms": ref_full, "ours_ms": ours_full, "speedup": ref_full / ours_full,
                               "max_abs_diff": float(d.max()), "mean_abs_diff": float(d.mean()),
                               "rows_with_same_selection": float(same_sel)}
    res["reps"] = reps
    return res


def fp16_leg(c, sets, stream, steps, warmup):
    """The same op with fp16 activations (the reference rollout's dtype under fp16 autocast):
    mosaic_attn_func on fp16 copies of the input sets (pooling, top-k scores and attention
    operands in fp16), device time per call."""
    import mosaic_b200 as M

    xs = [{k: v.half() for k, v in x.items()} for x in sets[:4]]
    n = len(xs)  # fewer sets for the workloads whose inputs alone exceed L2
    ms = _timed_rot(lambda i: M.mosaic_attn_func(xs[i % n]["q"], xs[i % n]["k"], xs[i % n]["v"],
                                                 xs[i % n]["w"].unsqueeze(-1), c["bas"], c["bs"], c["K"], False),
                    stream, steps, warmup)
    return {"what": "mosaic_attn_func with fp16 q/k/v/gates (native fp16 kernels)", "ms": ms,
            "tokens_per_s": c["B"] * c["N"] / (ms / 1000), "steps": steps}


def rope_leg(c, sets, stream, steps, warmup):
    """Where Mosaic's 2D RoPE (primitives.py:132-135) is applied: (a) by the producer of q
    and k (the fused QKV-projection epilogue of MosaicAttention, so the op reads rotated
    q/k: the `value` path), against (b) inside the op (`rope_tables`: the pool kernel
    rotates un-rotated q/k on their way in and writes rotated copies that kernel (c)
    then reads). Device time of mosaic_attn_func per call for both, same inputs."""
    import mosaic_b200 as M
    from mosaic_b200.healpix import healpix_rope_tables

    cos, sin = (t.to(sets[0]["q"].device) for t in healpix_rope_tables(c["nside"]))
    args = (c["bas"], c["bs"], c["K"], False)

    def call(i, tables):
        x = sets[i % len(sets)]
        return M.mosaic_attn_func(x["q"], x["k"], x["v"], x["w"].unsqueeze(-1), *args, rope_tables=tables)

    pre = _timed_rot(lambda i: call(i, None), stream, steps, warmup)
    fused = _timed_rot(lambda i: call(i, (cos, sin)), stream, steps, warmup)
    B, N, Hq, Hk, D = c["B"], c["N"], c["Hq"], c["Hk"], c["D"]
    return {"what": "mosaic_attn_func on pre-rotated q/k (RoPE in the producer's epilogue) vs rope_tables "
                    "(RoPE in the pool kernel, rotated copies written to the workspace and re-read)",
            "prerotated_ms": pre, "rope_tables_ms": fused, "rope_tables_extra_ms": fused - pre,
            "rotated_copy_bytes": B * N * (Hq + Hk) * D * 2, "steps": steps}


def _timed_rot(fn, stream, reps, warmup):
    """Like _timed, with the call index passed to fn (rotating input sets)."""
    for i in range(warmup):
        fn(i)
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for i in range(reps):
        fn(i)
    b.record(stream)
    torch.cuda.synchronize()
    return a.elapsed_time(b) / reps


# One step of the Mosaic U-Net calls the block-sparse attention 14 times per member, with
# the reference presets (inference.py:71-88: 128-token blocks, window 1024, GQA 4): stage 1
# (nside 64, 12 heads, top-k 24) and stage 2 (nside 32, 16 heads, top-k 12) with 4 encoder
# + 2 decoder blocks each, the bottleneck (nside 16, 20 heads, top-k 4) with 2 blocks.
UNET_ATTENTION = [  # (label, nside, q heads, top-k, calls), in the order of one step
    ("enc1", 64, 12, 24, 4), ("enc2", 32, 16, 12, 4), ("bottleneck", 16, 20, 4, 2),
    ("dec2", 32, 16, 12, 2), ("dec1", 64, 12, 24, 2)]
FIELD_NUMEL = 240 * 121 * 82  # the model's output field per member (lat-lon grid x channels)


def ensemble_leg(dev, rank, world, dist, stream, steps, warmup):
    """One 24-member ensemble step of the attention work, sharded by member: this rank
    runs the 14 block-sparse attention calls of one U-Net step (UNET_ATTENTION) for its
    members (ensemble.member_range, batched along the attention batch as mosaic.py:308
    batches them), then `ensemble.gather_members` all-gathers the per-member output
    fields (NCCL all_gather_into_tensor; 240 x 121 x 82 fp32 per member, the model's
    output size, taken from the last attention output) to every rank. Step time =
    max over ranks of the device time of the whole step, gather included."""
    import mosaic_b200 as M
    from mosaic_b200 import ensemble as E

    lo, hi = E.member_range(MEMBERS, rank, world)
    m = hi - lo
    g = torch.Generator(device=dev).manual_seed(4321 + rank)
    stages = {}
    for label, nside, Hq, K, calls in UNET_ATTENTION:
        if nside in stages:
            continue
        N, Hk = 12 * nside * nside, Hq // 4
        stages[nside] = dict(
            q=torch.randn(m, N, Hq, 64, generator=g, device=dev).bfloat16(),
            k=torch.randn(m, N, Hk, 64, generator=g, device=dev).bfloat16(),
            v=torch.randn(m, N, Hk, 64, generator=g, device=dev).bfloat16(),
            w=torch.sigmoid(torch.randn(3, m, N, Hq, 1, generator=g, device=dev)).bfloat16())
    field = torch.empty(m, FIELD_NUMEL, dtype=torch.float32, device=dev)

    def step(ev=None):
        out = None
        for label, nside, Hq, K, calls in UNET_ATTENTION:
            s = stages[nside]
            for _ in range(calls):
                out = M.mosaic_attn_func(s["q"], s["k"], s["v"], s["w"], 1024, 128, K, False)
        field.copy_(out.reshape(m, -1)[:, :FIELD_NUMEL])
        if ev:
            ev[0].record(stream)
        full = E.gather_members(field, MEMBERS) if dist is not None else field
        if ev:
            ev[1].record(stream)
        return full

    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(2)] for _ in range(steps)]
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for i in range(steps):
        full = step(evs[i])
    b.record(stream)
    torch.cuda.synchronize()
    step_ms = a.elapsed_time(b) / steps
    gather_ms = sum(e[0].elapsed_time(e[1]) for e in evs) / steps
    if dist is not None:
        t = torch.tensor([step_ms, gather_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        step_ms, gather_ms = (float(x_) for x_ in t.tolist())
        dist.barrier()
    assert full.shape[0] == MEMBERS
    flop = sum(calls * 4 * (12 * ns * ns) * Hq * 64 * (K * 128 + 1024) for _, ns, Hq, K, calls in UNET_ATTENTION)
    return {"what": "one 24-member step of the U-Net's attention work: 14 mosaic_attn_func calls per member "
                    "(reference presets: 6 at nside 64 / 12 heads / top-k 24, 6 at nside 32 / 16 heads / top-k 12, "
                    "2 at nside 16 / 20 heads / top-k 4; blocks 128, window 1024), members batched per rank, then "
                    "an all-gather of 240x121x82 fp32 output fields per member (taken from the last attention "
                    "output); synthetic inputs; device time, max over ranks",
            "members": MEMBERS, "members_per_rank": m, "steps": steps, "step_ms": step_ms,
            "step_per_s": 1000.0 / step_ms, "gather_ms": gather_ms, "gather_share": gather_ms / step_ms,
            "gathered_bytes_per_rank": MEMBERS * FIELD_NUMEL * 4,
            "attention_flop_per_member": flop,
            "attention_tflops_per_gpu": flop * m / ((step_ms - gather_ms) / 1000) / 1e12,
            "attention_frac_of_peak": flop * m / ((step_ms - gather_ms) / 1000) / 1e12 / peaks()[1],
            "peak_source": peaks()[2] + " bf16_tflops (burst)"}


UNET_TFLOP_PER_MEMBER = 11.45  # FlopCounterMode on the reference model at the era5 preset, one member


def model_leg(dev, rank, world, dist, stream, steps, warmup):
    """One 24-member forward step of the whole Mosaic U-Net: the reference's own
    Transformer (mosaic.py, era5 preset, random weights, from baseline/_ref) with
    mosaic_b200's transformer block (attention block + fused FFN), interpolation and
    resampling modules rebound into it (baseline.reference.build_model), bf16. Members are sharded over the ranks (num_noise_samples =
    24 / N each, the model's own member batching, mosaic.py:300-308) and the output
    fields [1, members, 240, 121, 82] are all-gathered over NCCL inside the timed step.
    Also: the same step captured in one CUDA graph (forward only; replayed, then the
    gather), and on one GPU the model with the reference's own modules (flash-attn, its
    Triton kernel, torch ops) on the same weights and inputs, with the output difference."""
    from baseline import reference as R

    if not R.available():
        return {"unavailable": "baseline/_ref is empty (the reference checkout was absent when build() ran)"}
    from mosaic_b200 import ensemble as E

    ref = R.load(dev)
    lo, hi = E.member_range(MEMBERS, rank, world)
    m = hi - lo
    model = R.build_model(ref, dev, ours=True, dtype=torch.bfloat16, seed=0)
    g = torch.Generator(device=dev).manual_seed(5)
    x = torch.randn(1, 1, 2, R.GRID_LON, R.GRID_LAT, 82, generator=g, device=dev).bfloat16()
    dyt = torch.rand(1, 1, 2, generator=g, device=dev).bfloat16()
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(2)] for _ in range(steps)]

    def gather(out):
        return E.gather_members(out, MEMBERS, dim=1) if dist is not None else out

    res = {"what": "one 24-member forward step of the whole Mosaic U-Net (the reference's Transformer, era5 "
                   "preset, random weights, bf16) with mosaic_b200's attention, interpolation and resampling "
                   "modules; members sharded over ranks, output fields all-gathered over NCCL in the step",
           "members": MEMBERS, "members_per_rank": m, "steps": steps}
    with torch.no_grad():
        first = model(x, dyt, m)
        for _ in range(warmup):
            gather(model(x, dyt, m))
        torch.cuda.synchronize()
        if dist is not None:
            dist.barrier()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for i in range(steps):
            out = model(x, dyt, m)
            evs[i][0].record(stream)
            full = gather(out)
            evs[i][1].record(stream)
        b.record(stream)
        torch.cuda.synchronize()
        step_ms = a.elapsed_time(b) / steps
        gather_ms = sum(e[0].elapsed_time(e[1]) for e in evs) / steps
        assert full.shape[1] == MEMBERS
        # the forward captured in one CUDA graph (its noise generator registered, so every
        # replay draws new noise), replayed, then the gather
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            for _ in range(2):
                model(x, dyt, m)
        torch.cuda.current_stream(dev).wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        graph.register_generator_state(model.noise_generator.generator)
        with torch.cuda.graph(graph):
            g_out = model(x, dyt, m)
        for _ in range(warmup):
            graph.replay()
            gather(g_out)
        torch.cuda.synchronize()
        if dist is not None:
            dist.barrier()
        a.record(stream)
        for _ in range(steps):
            graph.replay()
            gather(g_out)
        b.record(stream)
        torch.cuda.synchronize()
        graph_ms = a.elapsed_time(b) / steps
        del graph
    if dist is not None:
        t = torch.tensor([step_ms, gather_ms, graph_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        step_ms, gather_ms, graph_ms = (float(v) for v in t.tolist())
        dist.barrier()
    res.update(step_ms=step_ms, step_per_s=1000.0 / step_ms, gather_ms=gather_ms, gather_share=gather_ms / step_ms,
               graph_step_ms=graph_ms, graph_step_per_s=1000.0 / graph_ms,
               tflop_per_step=UNET_TFLOP_PER_MEMBER * MEMBERS,
               achieved_tflops_per_gpu=UNET_TFLOP_PER_MEMBER * m / (step_ms / 1000),
               frac_of_peak=UNET_TFLOP_PER_MEMBER * m / (step_ms / 1000) / peaks()[1])
    if world == 1:
        ref_model = R.build_model(ref, dev, ours=False, dtype=torch.bfloat16, seed=0)
        with torch.no_grad():
            r_first = ref_model(x, dyt, m)  # same weights, same noise (both generators seeded 42, first draw)
            d = (r_first.float() - first.float())
            ref_ms = _timed(lambda: ref_model(x, dyt, m), stream, max(2, steps - 1), 1)
        res.update(reference_modules_step_ms=ref_ms, speedup_vs_reference_modules=ref_ms / step_ms,
                   rel_l2_vs_reference_modules=float(d.norm() / r_first.float().norm()),
                   max_abs_vs_reference_modules=float(d.abs().max()),
                   mean_abs_vs_reference_modules=float(d.abs().mean()), reference_notes=ref.notes)
        del ref_model
    del model
    torch.cuda.empty_cache()
    return res


ROLLOUT_STEPS = 4


def rollout_leg(dev, stream):
    """The reference's autoregressive rollout (inference.py:330-390: 24 members, fp16
    autocast over fp32 weights, state (de)normalised around each step) on its own U-Net
    (era5 preset, random weights, synthetic normalisation statistics and initial
    state), through mosaic_b200.rollout.unroll_direct: with mosaic_b200's modules and
    steps 2.. replayed from one CUDA graph, the same eagerly, and the reference's
    modules eagerly (the reference's loop). Device time of the whole rollout (CUDA
    events on the launching stream), after one untimed 2-step rollout of each."""
    import types

    from baseline import reference as R
    from mosaic_b200.rollout import unroll_direct

    if not R.available():
        return {"unavailable": "baseline/_ref is empty (the reference checkout was absent when build() ran)"}
    ref = R.load(dev)
    ours = R.build_model(ref, dev, ours=True, dtype=None, seed=0)
    g = torch.Generator(device=dev).manual_seed(3)
    ns = types.SimpleNamespace(state_mean=torch.randn(82, generator=g, device=dev) * 3,
                               state_std=torch.rand(82, generator=g, device=dev) + 0.5)
    x0 = ns.state_mean + ns.state_std * torch.randn(1, 2, R.GRID_LON, R.GRID_LAT, 82, generator=g, device=dev)
    dyt = torch.rand(1, 2, generator=g, device=dev)
    delta = torch.tensor([0.25, 1 / 365], device=dev)

    def timed(model, graph, steps):
        unroll_direct(model, x0, dyt, delta, ns, 2, MEMBERS, graph=graph)  # warm-up
        torch.cuda.synchronize()
        ev = []
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        unroll_direct(model, x0, dyt, delta, ns, steps, MEMBERS, graph=graph, step_events=ev)
        b.record(stream)
        torch.cuda.synchronize()
        per = {}
        for t, kind, e0, e1 in ev:
            per.setdefault(kind, []).append(e0.elapsed_time(e1))
        return a.elapsed_time(b), {k: sum(v) / len(v) for k, v in per.items()}

    T = ROLLOUT_STEPS
    graph_ms, g_steps = timed(ours, True, T)
    eager_ms, e_steps = timed(ours, False, T)
    del ours
    torch.cuda.empty_cache()
    ref_model = R.build_model(ref, dev, ours=False, dtype=None, seed=0)
    ref_ms, r_steps = timed(ref_model, False, T)
    del ref_model
    torch.cuda.empty_cache()
    return {"what": "unroll_direct (inference.py:330-390) of the reference's U-Net, 24 members, fp16 autocast "
                    "over fp32 weights, synthetic state and normalisation statistics; per-step times from CUDA "
                    "events around each step",
            "members": MEMBERS, "unroll_steps": T, "graph_replayed_steps": T - 2,
            "rollout_ms": graph_ms, "ms_per_step": g_steps["graph"], "graph_eager_steps_ms": g_steps["eager"],
            "eager_rollout_ms": eager_ms, "eager_ms_per_step": e_steps["eager"],
            "reference_modules_rollout_ms": ref_ms, "reference_modules_ms_per_step": r_steps["eager"],
            "speedup_vs_reference_modules": r_steps["eager"] / g_steps["graph"]}


def b200_arm(args):
    from mosaic_b200 import _lib
    import mosaic_b200 as M

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    lib = _lib.load()
    name = args.workload
    c = WORKLOADS[name]
    B, N, Hq, Hk, D = c["B"], c["N"], c["Hq"], c["Hk"], c["D"]

    # input sets per rank (member = rank), rotated so that a set is re-read only after
    # more than 2 x L2 of other inputs went through the cache
    set_bytes = B * N * (Hq + 2 * Hk) * D * 2 + 3 * B * N * Hq * 2
    nsets = max(2, min(32, -(-3 * L2_BYTES // set_bytes)))
    g = torch.Generator(device=dev).manual_seed(1234 + rank)
    sets = []
    for _ in range(nsets):
        sets.append(dict(
            q=torch.randn(B, N, Hq, D, generator=g, device=dev).bfloat16(),
            k=torch.randn(B, N, Hk, D, generator=g, device=dev).bfloat16(),
            v=torch.randn(B, N, Hk, D, generator=g, device=dev).bfloat16(),
            w=torch.sigmoid(torch.randn(3, B, N, Hq, generator=g, device=dev)).bfloat16()))
    st = Stages(lib, c, dev)
    stream = torch.cuda.current_stream(dev)

    def barrier():
        if dist is not None:
            dist.barrier()

    for i in range(args.warmup):
        st.run_fused(sets[i % nsets], stream)
    torch.cuda.synchronize()
    barrier()
    t_start, t_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        torch.cuda.synchronize()
        t_start.record(stream)
        for i in range(args.steps):
            st.run_fused(sets[i % nsets], stream)
        t_end.record(stream)
        torch.cuda.synchronize()
    barrier()
    ms = t_start.elapsed_time(t_end)
    # per-kernel attribution: the same kernels launched one entry point at a time
    events = [[torch.cuda.Event(enable_timing=True) for _ in range(5)] for _ in range(args.steps)]
    for i in range(args.steps):
        st.run(sets[i % nsets], stream, events[i])
    torch.cuda.synchronize()
    stage_ms = [sum(events[i][s].elapsed_time(events[i][s + 1]) for i in range(args.steps)) / args.steps
                for s in range(4)]
    status = int(st.status.item())
    if status:
        raise RuntimeError(f"device status {status} after the timed region")
    if dist is not None:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    value = world * B * N * args.steps / (ms / 1000.0)

    # e2e: public API with host buffers (pinned): every step copies its inputs in and
    # its output out; StreamedAttention overlaps step i's attention with the copy-in of
    # step i+1 and the copy-out of step i-1 (PCIe is full duplex)
    e2e = None
    if not args.no_e2e:
        from mosaic_b200.streaming import StreamedAttention

        host = [{k: v.cpu().pin_memory() for k, v in s_.items()} for s_ in sets[:2]]
        out_host = [torch.empty(B, N, Hq, D, dtype=torch.bfloat16).pin_memory() for _ in range(2)]
        h2d = sum(v.numel() * v.element_size() for v in host[0].values())
        d2h = out_host[0].numel() * out_host[0].element_size()
        pipe = StreamedAttention(dev, c["bas"], c["bs"], c["K"])

        def e2e_steps(n, start):
            for i in range(start, start + n):
                x = host[i % 2]
                pipe.submit(x["q"], x["k"], x["v"], x["w"], out_host[i % 2])
            pipe.join()

        n_e2e = max(3, min(args.steps, 50))
        e2e_steps(args.warmup, 0)
        torch.cuda.synchronize()
        barrier()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        e2e_steps(n_e2e, args.warmup)
        b.record(stream)
        torch.cuda.synchronize()
        barrier()
        e_ms = a.elapsed_time(b)
        if dist is not None:
            t = torch.tensor([e_ms], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            e_ms = float(t.item())
        pcie = (h2d + d2h) * n_e2e / (e_ms / 1000.0) / 1e9
        e2e = {"value": world * B * N * n_e2e / (e_ms / 1000.0), "unit": UNIT, "h2d_bytes_per_step": h2d,
               "d2h_bytes_per_step": d2h, "steps": n_e2e,
               "path": "mosaic_b200.streaming.StreamedAttention -> mosaic_attn_func, pinned host inputs/outputs",
               "host_copy_gbs_per_rank": pcie, "host_copy_gbs_all_ranks": pcie * world,
               "limiter": "host<->device copies (the device step takes a fraction of the copy time); with several "
                          "ranks all copies share the host's memory and PCIe root complex"}
        del host, out_host, pipe

    f16 = rope = None
    if rank == 0 and world == 1:
        f16 = fp16_leg(c, sets, stream, max(3, min(args.steps, 50)), max(3, args.warmup))
        if "nside" in c:
            rope = rope_leg(c, sets, stream, max(3, min(args.steps, 50)), max(3, args.warmup))
    ens = unet = None
    if not args.no_ensemble and name == "S1":
        ens = ensemble_leg(dev, rank, world, dist, stream, steps=max(2, min(args.steps, 4)), warmup=1)
    if not args.no_model and name == "S1":
        unet = model_leg(dev, rank, world, dist, stream, steps=3, warmup=1)
    roll = None
    if not args.no_model and not args.no_rollout and world == 1 and name == "S1":
        roll = rollout_leg(dev, stream)
    ref_gpu = None
    if not args.no_reference_gpu and rank == 0 and world == 1 and name in ("S1", "S1_bs128"):
        ref_gpu = reference_gpu_leg(c, sets[0], stream, reps=max(3, min(args.steps, 20)), warmup=2)

    sdpa = None
    if name.startswith("X") and rank == 0:
        sdpa = dense_sdpa(sets[0], c)
        if sdpa.get("ms"):
            sdpa["bsa_speedup"] = sdpa["ms"] / (ms / args.steps)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        windows = sample_windows(c, 8)
        reps = 3 if N <= 49152 else 1
        v_cpu, cores, secs, t_full = cpu_sample(c, windows, reps=reps)
        cpu = {"value": v_cpu, "unit": UNIT, "cores": cores, "kind": "port",
               "sample": cpu_sample_text(name, c, windows, reps, 1) + f", {secs:.1f} s of CPU work",
               "full_call_ms_extrapolated": 1000 * t_full}

    hbm, tf, src = peaks()
    bwd = None
    if not args.no_backward:
        n_bwd = max(3, min(args.steps, 50))
        bwd_ms = backward_leg(c, sets, stream, n_bwd, max(3, args.warmup))
        bwd = {"what": "mosaic_sparse_attn backward (ops.mosaic_attn_bwd: D, inverted block index, dQ and dK/dV "
                       "tcgen05 kernels) on this workload's selected branch, top-k selection of each input set",
               "ms": bwd_ms, "steps": n_bwd, "flop_per_step": flops_backward(c),
               "achieved_tflops": flops_backward(c) / (bwd_ms / 1000) / 1e12, "peak_tflops": tf,
               "frac": flops_backward(c) / (bwd_ms / 1000) / 1e12 / tf}
    blk = None
    if not args.no_block and world == 1:
        blk = block_leg(c, sets, stream, max(3, min(args.steps, 50)), max(3, args.warmup))
        blk["qkv_proj_frac"] = blk["qkv_proj_tflops"] / tf
        blk["out_proj_frac"] = blk["out_proj_tflops"] / tf
    itp = None
    if not args.no_interp and world == 1 and name == "S1":
        itp = interp_leg(stream, max(3, min(args.steps, 50)), max(3, args.warmup))
        for leg in ("ll_to_hp", "hp_to_ll"):
            itp[leg]["attend_hbm_frac"] = itp[leg]["attend_hbm_gbs"] / hbm
    ud = None
    if not args.no_updown and world == 1 and name == "S1":
        ud = updown_leg(stream, max(3, min(args.steps, 50)), max(3, args.warmup))
        for leg in ("down", "up"):
            ud[leg]["frac_of_peak"] = ud[leg]["gemm_tflops_incl_norm"] / tf
    t_att = stage_ms[3] / 1000.0
    achieved = flops_attend(c) / t_att / 1e12
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": describe(name, c),
                   "B_per_gpu": B, "N": N, "Hq": Hq, "Hk": Hk, "head_dim": D, "sparse_block": c["bs"],
                   "topk": c["K"], "window": c["bas"], "parallelism": f"members x{world}",
                   "l2": f"{nsets} rotating input sets of {set_bytes / 1e6:.0f} MB (L2 126 MB)"},
        "value_per_gpu": value / world,
        "roofline": {"bound": "tensor", "kernel": "bsa_engine_kernel (c: local + selected + gated combine)",
                     "achieved": achieved, "peak": tf, "unit": "TFLOP/s", "frac": achieved / tf,
                     "peak_source": src + " bf16_tflops (burst)", "traffic": ATTEND_TRAFFIC_BYTES.get(name),
                     "flop_per_launch": flops_attend(c)},
        "kernels_us": {n: 1000 * t for n, t in zip(STAGE_NAMES, stage_ms)},
        "pool_hbm": {"achieved_gbs": bytes_pool(c) / (stage_ms[0] / 1000) / 1e9, "peak_gbs": hbm,
                     "frac": bytes_pool(c) / (stage_ms[0] / 1000) / 1e9 / hbm},
        "gpu_launches": LAUNCHES_PER_STEP * args.steps,
        "kernels_note": "kernels_us from a second K-step loop of the same kernels launched one at a time; "
                        "in the timed loop top-k overlaps the coarse attention",
        "clocks": clk.summary(),
        "e2e": e2e,
        "cpu_baseline": cpu,
    }
    if f16 is not None:
        line["fp16"] = f16
    if rope is not None:
        line["rope_placement"] = rope
    if ens is not None:
        line["ensemble"] = ens
    if unet is not None:
        line["unet_step"] = unet
    if roll is not None:
        line["rollout"] = roll
    if ref_gpu is not None:
        line["reference_gpu"] = ref_gpu
    if sdpa is not None:
        line["dense_sdpa"] = sdpa
    if bwd is not None:
        line["backward"] = bwd
    if blk is not None:
        line["attention_block"] = blk
    if itp is not None:
        line["interpolation"] = itp
    if ud is not None:
        line["updown"] = ud
    if rank == 0:
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.destroy_process_group()


def main():
    args = parse()
    if args.impl == "reference":
        reference_arm(args)
    else:
        b200_arm(args)


if __name__ == "__main__":
    main()
