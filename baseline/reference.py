"""The reference implementation (maxxxzdn/mosaic) as the GPU speed bar on the same B200.

The reference is an unpackaged Python project: `pip install --target baseline/_ref`
refuses it (it has neither setup.py nor pyproject.toml). Its install here is
therefore a verbatim copy of the module files the attention path and the model
import (ops.py with the Triton kernels, primitives.py, utils.py, mosaic.py with the
U-Net) into baseline/_ref, which git ignores and which travels with the source tree
to the GPU box. `install(src_dir)` makes that copy; nothing of it is committed or
edited.

`load()` imports the copies. Two bindings are set at load time, both outside the
reference files:
  * `healpy` (absent from the image) is a stub module: only
    utils.get_healpix_grid uses it; the attention path never calls that, and
    `build_model` rebinds it to mosaic_b200.healpix's restatement;
  * the reference's Triton autotuner is bypassed: its config list includes
    q_tile_size = 128, which with 64-token blocks makes tiles_per_block zero and
    divides by it (ops.py:54-55), so every launch here goes to the kernel's JIT
    function (`mosaic_attn_fwd_kernel.fn`) with an explicit q_tile_size that
    divides the block size, over the autotuner's other choices (num_warps 4 / 8,
    num_stages 2 / 3), and `primitives.mosaic_sparse_attn` is rebound to that
    launch. The launch grid and arguments are those of ops.mosaic_attn_fwd
    (ops.py:137-176).
flash_attn_func (flash-attn 2.8.3 in the image) is used as the reference imports
it; if it cannot run on this GPU, `load()` rebinds primitives.flash_attn_func to
torch SDPA with the same semantics and says so in the returned notes.
"""
import os
import shutil
import sys
import types

HERE = os.path.dirname(os.path.abspath(__file__))
REF_DIR = os.path.join(HERE, "_ref")
FILES = ("ops.py", "primitives.py", "utils.py", "mosaic.py")


def install(src_dir):
    """Copy the reference's attention-path modules, unmodified, into baseline/_ref.
    Returns True when the copy is in place."""
    if not all(os.path.exists(os.path.join(src_dir, f)) for f in FILES):
        return available()
    os.makedirs(REF_DIR, exist_ok=True)
    for f in FILES:
        shutil.copyfile(os.path.join(src_dir, f), os.path.join(REF_DIR, f))
    return available()


def available():
    return all(os.path.exists(os.path.join(REF_DIR, f)) for f in FILES)


class Reference:
    """The loaded reference modules plus the autotuner-free launch of its forward kernel."""

    def __init__(self, ops, primitives, notes, mosaic=None):
        self.ops, self.primitives, self.notes, self.mosaic = ops, primitives, notes, mosaic
        self.config = dict(q_tile_size=64, num_warps=4, num_stages=2)

    def sparse_attn_fwd(self, q, k, v, block_indices, block_size, softmax_scale=None, config=None):
        """ops.mosaic_attn_fwd (ops.py:137-176) with the given kernel config: (output, lse)."""
        import torch
        import triton

        cfg = dict(self.config if config is None else config)
        B, N, Hk, D = k.shape
        Hq = q.shape[2]
        scale = D ** -0.5 if softmax_scale is None else softmax_scale
        if block_size % cfg["q_tile_size"] != 0:
            raise ValueError(f"q_tile_size {cfg['q_tile_size']} does not divide block size {block_size}")
        q, k, v, block_indices = (t.contiguous() for t in (q, k, v, block_indices))
        out = torch.empty(B, N, Hq, D, dtype=v.dtype, device=q.device)
        lse = torch.empty(B, N, Hq, dtype=torch.float32, device=q.device)
        grid = (triton.cdiv(N, cfg["q_tile_size"]), Hq // Hk, B * Hk)
        self.ops.mosaic_attn_fwd_kernel.fn[grid](
            q_ptr=q, k_ptr=k, v_ptr=v, output_ptr=out, lse_ptr=lse, block_indices_ptr=block_indices,
            softmax_scale=scale, seq_len=N, num_kv_heads=Hk, num_q_heads=Hq, q_heads_per_kv_head=Hq // Hk,
            feature_dim=D, kv_block_size=block_size, num_kv_blocks_per_q_block=block_indices.shape[-1],
            q_tile_size=cfg["q_tile_size"], num_warps=cfg["num_warps"], num_stages=cfg["num_stages"])
        return out, lse

    def configs(self, block_size):
        """The autotuner's configs (ops.py:7-17) that are valid for this block size."""
        return [dict(q_tile_size=t, num_warps=w, num_stages=s) for t in (64, 128) if block_size % t == 0
                for w in (4, 8) for s in (2, 3)]

    def mosaic_sparse_attn(self, q, k, v, block_indices, block_size, softmax_scale=None):
        """Stand-in for ops.mosaic_sparse_attn (ops.py:557-566) in the forward: same
        result (output cast to q's dtype, ops.py:538), launched without the autotuner."""
        out, _ = self.sparse_attn_fwd(q, k, v, block_indices, block_size, softmax_scale)
        return out.to(q.dtype)


def load(device=None):
    """Import the installed reference modules; returns a Reference (raises if absent)."""
    if not available():
        raise FileNotFoundError("baseline/_ref does not hold the reference modules")
    saved = {name: sys.modules.get(name) for name in ("ops", "utils", "primitives", "mosaic", "healpy")}
    sys.modules.setdefault("healpy", types.ModuleType("healpy"))
    sys.path.insert(0, REF_DIR)
    try:
        for name in ("ops", "utils", "primitives", "mosaic"):
            sys.modules.pop(name, None)
        import ops as ref_ops  # noqa: E402  (the reference's ops.py)
        import primitives as ref_prim  # noqa: E402  (the reference's primitives.py)
        import mosaic as ref_mosaic  # noqa: E402  (the reference's mosaic.py: the U-Net)
    finally:
        sys.path.remove(REF_DIR)
        for name, mod in saved.items():
            if mod is None:
                sys.modules.pop(name, None)
            else:
                sys.modules[name] = mod
    ref = Reference(ref_ops, ref_prim, [], ref_mosaic)
    ref_prim.mosaic_sparse_attn = ref.mosaic_sparse_attn
    if device is not None:
        _check_flash_attn(ref, device)
    return ref


def _sdpa_gqa(q, k, v):
    """flash_attn_func's semantics (non-causal, scale head_dim**-0.5, query head j reads
    kv head j // G) on torch SDPA; [B, L, H, D] layouts."""
    import torch.nn.functional as F

    G = q.shape[2] // k.shape[2]
    qt = q.transpose(1, 2)
    kt = k.repeat_interleave(G, dim=2).transpose(1, 2)
    vt = v.repeat_interleave(G, dim=2).transpose(1, 2)
    return F.scaled_dot_product_attention(qt, kt, vt).transpose(1, 2)


def _check_flash_attn(ref, device):
    import torch

    q = torch.randn(1, 128, 4, 64, device=device, dtype=torch.bfloat16)
    k = torch.randn(1, 128, 1, 64, device=device, dtype=torch.bfloat16)
    try:
        o = ref.primitives.flash_attn_func(q, k, k)
        torch.cuda.synchronize(device)
        if (o.float() - _sdpa_gqa(q, k, k).float()).abs().max().item() > 2e-2:
            raise RuntimeError("flash_attn_func disagrees with SDPA")
        ref.notes.append("flash_attn_func: flash-attn 2.8.3 as imported by the reference")
    except Exception as e:  # no kernel image for this GPU, or a wrong result
        ref.primitives.flash_attn_func = _sdpa_gqa
        ref.notes.append(f"flash_attn_func unavailable here ({str(e).splitlines()[0][:100]}); "
                         "torch SDPA with its semantics stands in")


# ----------------------------------------------------------------------------- the U-Net
def era5_config(mosaic):
    """The reference's `era5` model preset (inference.py:71-88 stage / bottleneck configs,
    inference.py:290-306 model config): 3 stages (nside 64 / 32 / 16, dims 768 / 1024 /
    1280, 12 / 16 / 20 heads, GQA 4, 128-token blocks, top-k 24 / 12 / 4, window 1024,
    depths 4+2 / 4+2 / 2), 82 variables x 2 history states + 3 static, 24 neighbours,
    noise 32, no affine RMSNorm."""
    S, Bn = mosaic.StageConfig, mosaic.BottleneckConfig
    stages = [S(nside=64, dim=768, num_heads=12, block_attn_size=1024, sparse_block_size=128, sparse_block_count=24,
                encoder_depth=4, decoder_depth=2, mlp_ratio=4.0, gqa_ratio=4),
              S(nside=32, dim=1024, num_heads=16, block_attn_size=1024, sparse_block_size=128,
                sparse_block_count=12, encoder_depth=4, decoder_depth=2, mlp_ratio=4.0, gqa_ratio=4)]
    bottleneck = Bn(nside=16, dim=1280, num_heads=20, block_attn_size=1024, sparse_block_size=128,
                    sparse_block_count=4, depth=2, mlp_ratio=4.0, gqa_ratio=4)
    return mosaic.ModelConfig(
        dim=768, num_heads=12, variables=[f"var{i}" for i in range(82)],
        static_variables=["geopotential_at_surface", "land_sea_mask", "soil_type"], k_neighbors=24,
        qk_norm=False, rope=True, rope_theta=10000, sparse_every=1, qkv_compress_ratio=1, num_history_steps=2,
        noise_dim=32, rmsnorm_elementwise_affine=False, cg_stage_cfgs=stages, bottleneck_cfg=bottleneck)


GRID_LON, GRID_LAT = 240, 121  # the 1.5-degree lat-lon grid


def build_model(ref, device, ours=True, dtype=None, seed=0):
    """The reference's Transformer (mosaic.py:136-336) with the era5 preset and random
    weights (torch.manual_seed(seed), the reference's own initialisers), its static
    fields ~ N(0, 1) on the 240 x 121 grid, on `device` in eval mode.

    ours=True rebinds, before construction, the names the model resolves at build time
    to mosaic_b200's modules: the block class mosaic.py imports from primitives
    (`_MosaicBlock`, whose attention is mosaic_b200.MosaicAttention and whose FFN is the
    fused mosaic_b200.MosaicSwiGLU), primitives.MosaicAttention,
    mosaic.CrossAttentionInterpolate, mosaic.HEALPixDownsample and
    mosaic.HEALPixUpsample (the names those classes are looked up by); ours=False restores the
    reference's own classes. Either way the HEALPix pixel centres come from
    mosaic_b200.healpix (the reference's utils.get_healpix_grid needs healpy, which is
    not installed here)."""
    import torch
    import mosaic_b200 as M
    from mosaic_b200.healpix import get_healpix_grid

    prim, mos = ref.primitives, ref.mosaic
    if not hasattr(ref, "_orig"):
        ref._orig = dict(MosaicAttention=prim.MosaicAttention, CrossAttentionInterpolate=mos.CrossAttentionInterpolate,
                         HEALPixDownsample=mos.HEALPixDownsample, HEALPixUpsample=mos.HEALPixUpsample,
                         _MosaicBlock=mos._MosaicBlock)
    prim.MosaicAttention = M.MosaicAttention if ours else ref._orig["MosaicAttention"]
    mos._MosaicBlock = M.MosaicBlock if ours else ref._orig["_MosaicBlock"]
    for name in ("CrossAttentionInterpolate", "HEALPixDownsample", "HEALPixUpsample"):
        setattr(mos, name, getattr(M, name) if ours else ref._orig[name])
    mos.get_healpix_grid = get_healpix_grid
    prim.get_healpix_grid = get_healpix_grid
    torch.manual_seed(seed)
    model = mos.Transformer(era5_config(mos))
    g = torch.Generator().manual_seed(seed + 1)
    lon = torch.linspace(0, 360, GRID_LON + 1)[:-1]
    lat = torch.linspace(-90, 90, GRID_LAT)
    model.initialize_static_vars(torch.randn(GRID_LON, GRID_LAT, 3, generator=g), lon, lat)
    model = model.to(device)
    model.initialize_interpolation(lon.to(device), lat.to(device))
    if dtype is not None:
        model = model.to(dtype)
    return model.eval()


def profile_step(members=2, ours=True, autocast=False):
    """One forward step of the era5 U-Net (`members` ensemble members) on cuda:0 after
    three warm-up steps, inside the NVTX range "unet_step", so that a profiler can take
    exactly that step's launches (ncu --nvtx --nvtx-include "unet_step/"). bf16 weights
    and inputs, or with `autocast` fp32 weights and inputs under fp16 autocast (the
    reference rollout's setting, inference.py:59,379)."""
    import contextlib

    import torch

    dev = torch.device("cuda:0")
    ref = load(dev)
    dt = None if autocast else torch.bfloat16
    model = build_model(ref, dev, ours=ours, dtype=dt, seed=0)
    g = torch.Generator(device=dev).manual_seed(5)
    x = torch.randn(1, 1, 2, GRID_LON, GRID_LAT, 82, generator=g, device=dev)
    dyt = torch.rand(1, 1, 2, generator=g, device=dev)
    if not autocast:
        x, dyt = x.bfloat16(), dyt.bfloat16()
    ctx = torch.autocast("cuda", dtype=torch.float16) if autocast else contextlib.nullcontext()
    with torch.no_grad(), ctx:
        for _ in range(3):
            model(x, dyt, members)
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_push("unet_step")
        out = model(x, dyt, members)
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_pop()
    return out


if __name__ == "__main__":
    # python -m baseline.reference [members] [ref] [autocast]: one profiled U-Net step (see profile_step)
    profile_step(int(sys.argv[1]) if len(sys.argv) > 1 else 2, ours="ref" not in sys.argv[2:],
                 autocast="autocast" in sys.argv[2:])
