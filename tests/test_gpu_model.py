"""The whole Mosaic U-Net with mosaic_b200 inside: the reference's own Transformer
(mosaic.py, era5 preset: three stages, 14 attention blocks, the two grid
interpolations, down/upsampling; random weights) built twice on the B200 in bf16 —
once with the reference's modules (flash-attn, its Triton kernel, torch ops) and once
with mosaic_b200's MosaicAttention, CrossAttentionInterpolate and
HEALPixDownsample/Upsample rebound into it — and the reference's state dict loaded
into the second. Skipped when baseline/_ref holds no reference copy.

* One forward step of 2 ensemble members on the same input: the two output fields
  [1, 2, 240, 121, 82] agree within max-abs 2e-2 / mean-abs 2e-3 (bf16 throughout, 14
  attention blocks deep; both models draw the same noise, their generators seeded 42).
* The step captured in one CUDA graph replays to the eager step's output bit for bit
  (same fixed noise; every mosaic_b200 kernel in the step reduces in a fixed order)."""
import pytest
import torch

from baseline import reference as R

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not R.available(), reason="baseline/_ref holds no reference copy")]

DEV = torch.device("cuda")


@pytest.fixture(scope="module")
def models():
    ref = R.load(DEV)
    ref_model = R.build_model(ref, DEV, ours=False, dtype=torch.bfloat16, seed=0)
    ours = R.build_model(ref, DEV, ours=True, dtype=torch.bfloat16, seed=0)
    ours.load_state_dict(ref_model.state_dict())
    g = torch.Generator(device=DEV).manual_seed(5)
    x = torch.randn(1, 1, 2, R.GRID_LON, R.GRID_LAT, 82, generator=g, device=DEV).bfloat16()
    dyt = torch.rand(1, 1, 2, generator=g, device=DEV).bfloat16()
    yield ref_model, ours, x, dyt
    del ref_model, ours
    torch.cuda.empty_cache()


def test_unet_step_with_mosaic_b200_modules_matches_reference_modules(models):
    ref_model, ours, x, dyt = models
    import mosaic_b200 as M

    assert isinstance(ours.encoder_stages[0].blocks[0].attention, M.MosaicAttention)
    assert isinstance(ours.interp_to_hp, M.CrossAttentionInterpolate)
    assert isinstance(ours.downsample_layers[0], M.HEALPixDownsample)
    with torch.no_grad():
        a = ref_model(x, dyt, 2)
        b = ours(x, dyt, 2)
    torch.cuda.synchronize()
    assert a.shape == b.shape == (1, 2, R.GRID_LON, R.GRID_LAT, 82)
    d = (a.float() - b.float()).abs()
    assert torch.isfinite(b.float()).all()
    assert d.max().item() <= 2e-2 and d.mean().item() <= 2e-3, (d.max().item(), d.mean().item())


def test_unet_step_replays_from_one_cuda_graph(models):
    _, ours, x, dyt = models
    with torch.no_grad():
        # one fixed noise draw for the eager step and the replays (the bench registers the
        # generator with the graph instead, so that every replay draws new noise)
        noise = ours.noise_generator(2, DEV, x.dtype).clone()
        ours.noise_generator.forward = lambda num_samples, device, dtype: noise
        try:
            side = torch.cuda.Stream(DEV)
            side.wait_stream(torch.cuda.current_stream(DEV))
            with torch.cuda.stream(side):
                for _ in range(2):
                    ours(x, dyt, 2)
            torch.cuda.current_stream(DEV).wait_stream(side)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                g_out = ours(x, dyt, 2)
            eager = ours(x, dyt, 2).clone()
            graph.replay()
            graph.replay()
            torch.cuda.synchronize()
            d = (g_out.float() - eager.float()).abs()
            assert torch.equal(g_out, eager), (d.max().item(), d.mean().item())
            del graph
        finally:
            del ours.noise_generator.forward
