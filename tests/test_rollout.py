"""Host logic of mosaic_b200.rollout.unroll_direct on CPU (graph=False): the
trajectory layout, the ensemble expansion on the first step, the history window and
the day/year time advance follow the reference's loop (inference.py:357-389), here
restated step by step against a toy model whose output depends on every input."""
import types

import torch

from mosaic_b200.rollout import unroll_direct


class Toy(torch.nn.Module):
    """model(norm_state [B, n, H, lon, lat, C], day_year_time [B, n, 2], s) ->
    [B, n * s, lon, lat, C], member-dependent through a per-call counter."""

    def __init__(self):
        super().__init__()
        self.calls = 0

    def forward(self, x, dyt, s):
        self.calls += 1
        b, n, h = x.shape[:3]
        y = x.mean(2) * 0.9 + x[:, :, -1] * 0.1 + dyt.sum(-1)[..., None, None, None] + 0.01 * self.calls
        y = y.repeat_interleave(s, dim=1)
        return y + 0.001 * torch.arange(n * s, dtype=y.dtype).view(1, -1, 1, 1, 1)


def reference_loop(model, x0, dyt0, delta, ns, T, M):
    # the reference's unroll_direct, restated (inference.py:357-389)
    B, H = x0.shape[:2]
    traj = torch.empty((B, M, T + H) + x0.shape[2:], dtype=x0.dtype)
    cur = x0.unsqueeze(1)
    dyt = dyt0.unsqueeze(1)
    traj[:, :, :H] = cur
    for t in range(T):
        ne = M if t == 0 else 1
        out = model((cur - ns.state_mean) / ns.state_std, dyt, ne)
        nxt = out * ns.state_std + ns.state_mean
        dyt = dyt + delta.unsqueeze(0).unsqueeze(0).expand(B, ne, -1)
        traj[:, :, t + H] = nxt
        cur = traj[:, :, t + 1:t + 1 + H]
    return traj


def test_unroll_direct_eager_matches_reference_loop():
    g = torch.Generator().manual_seed(0)
    C = 3
    ns = types.SimpleNamespace(state_mean=torch.randn(C, generator=g), state_std=torch.rand(C, generator=g) + 0.5)
    x0 = torch.randn(2, 3, 4, 5, C, generator=g)
    dyt = torch.rand(2, 2, generator=g)
    delta = torch.tensor([0.25, 0.01])
    want = reference_loop(Toy(), x0, dyt, delta, ns, 4, 3)
    got = unroll_direct(Toy(), x0, dyt, delta, ns, 4, 3, dtype=torch.bfloat16, graph=False)
    assert got.shape == (2, 3, 7, 4, 5, C)
    torch.testing.assert_close(got, want, rtol=0, atol=0)


def test_unroll_direct_zero_steps_and_graph_needs_cuda():
    x0 = torch.zeros(1, 2, 3, 3, 1)
    ns = types.SimpleNamespace(state_mean=torch.zeros(1), state_std=torch.ones(1))
    out = unroll_direct(Toy(), x0, torch.zeros(1, 2), torch.zeros(2), ns, 0, 4, graph=False)
    assert out.shape == (1, 4, 2, 3, 3, 1) and torch.equal(out, torch.zeros_like(out))
    try:
        unroll_direct(Toy(), x0, torch.zeros(1, 2), torch.zeros(2), ns, 2, 4, graph=True)
    except ValueError:
        pass
    else:
        raise AssertionError("graph=True on CPU must raise")
