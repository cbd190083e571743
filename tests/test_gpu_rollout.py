"""mosaic_b200.rollout.unroll_direct: the reference's autoregressive rollout
(inference.py:330-390) with the steps after the first replayed from one CUDA graph,
run on the reference's own U-Net (mosaic.py, era5 preset, random fp32 weights, fp16
autocast as in the reference's rollout) with mosaic_b200's modules rebound. Skipped
when baseline/_ref holds no reference copy.

* graph=True gives the same trajectory as graph=False, bit for bit: 4 steps, 2
  members, the model's own noise generator (the graph replays advance it as the
  eager calls do).
* Against the reference's modules (same weights, same noise, eager loop): every step's
  state, in normalised units, within max-abs 2e-2 / mean-abs 2e-3 (fp16 autocast in
  the reference's modules, bf16 inside mosaic_b200's fused projections; measured
  max 0.008 / mean 0.0012 at step 4)."""
import types

import pytest
import torch

from baseline import reference as R

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not R.available(), reason="baseline/_ref holds no reference copy")]

DEV = torch.device("cuda")
C, T, M = 82, 4, 2


@pytest.fixture(scope="module")
def setup():
    ref = R.load(DEV)
    ours = R.build_model(ref, DEV, ours=True, dtype=None, seed=0)
    ref_model = R.build_model(ref, DEV, ours=False, dtype=None, seed=0)
    ref_model.load_state_dict(ours.state_dict())
    g = torch.Generator(device=DEV).manual_seed(3)
    ns = types.SimpleNamespace(state_mean=torch.randn(C, generator=g, device=DEV) * 3,
                               state_std=torch.rand(C, generator=g, device=DEV) + 0.5)
    x0 = ns.state_mean + ns.state_std * torch.randn(1, 2, R.GRID_LON, R.GRID_LAT, C, generator=g, device=DEV)
    dyt = torch.rand(1, 2, generator=g, device=DEV)
    delta = torch.tensor([0.25, 1 / 365], device=DEV)
    yield ref_model, ours, ns, x0, dyt, delta
    del ref_model, ours
    torch.cuda.empty_cache()


def _run(model, setup, graph, step_events=None):
    from mosaic_b200.rollout import unroll_direct

    _, _, ns, x0, dyt, delta = setup
    model.noise_generator.generator = None  # re-seeded on the first draw
    return unroll_direct(model, x0, dyt, delta, ns, T, M, graph=graph, step_events=step_events)


def test_graph_rollout_matches_eager_rollout(setup):
    ours = setup[1]
    eager = _run(ours, setup, False)
    ev = []
    graphed = _run(ours, setup, True, ev)
    torch.cuda.synchronize()
    assert [(t, kind) for t, kind, _, _ in ev] == [(0, "eager"), (1, "eager"), (2, "graph"), (3, "graph")]
    assert all(e0.elapsed_time(e1) > 0 for _, _, e0, e1 in ev)
    assert graphed.shape == (1, M, 2 + T, R.GRID_LON, R.GRID_LAT, C)
    assert torch.isfinite(graphed).all()
    assert not torch.equal(graphed[:, 0, 2 + T - 1], graphed[:, 1, 2 + T - 1])  # members differ
    for t in range(2 + T):
        assert torch.equal(graphed[:, :, t], eager[:, :, t]), t


def test_rollout_with_mosaic_b200_modules_matches_reference_modules(setup):
    ref_model, ours, ns = setup[0], setup[1], setup[2]
    a = _run(ref_model, setup, False)
    b = _run(ours, setup, True)
    torch.cuda.synchronize()
    assert torch.equal(a[:, :, :2], b[:, :, :2])
    for t in range(2, 2 + T):
        d = ((a[:, :, t] - b[:, :, t]) / ns.state_std).abs()
        assert d.max().item() <= 2e-2 and d.mean().item() <= 2e-3, (t, d.max().item(), d.mean().item())
