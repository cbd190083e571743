"""Autoregressive rollout with every step after the first replayed from one CUDA graph.

`unroll_direct` keeps the reference's rollout contract (inference.py:330-390): same
arguments, same trajectory [B, members, history + steps, lon, lat, channels] in the
initial state's dtype, the ensemble expanded on the first step only, the model run
under autocast at `dtype`, the state (de)normalised with `norm_stats.state_mean /
state_std` around each step and the day/year time advanced by `day_year_delta` per
step. `model` is anything with the reference's call signature
`model(norm_state, day_year_time, num_noise_samples)`: the reference's WeatherModel or
Transformer, with mosaic_b200's modules rebound into it or not.

The difference is how the steps run. Step 0 expands [B, 1, ...] to the members, so
its shapes differ from every later step; it runs eagerly, and so does step 1, on a
side stream, as the warm-up that creates library handles, the model's noise generator
and the modules' cached weights before capture. From step 2 on, the shapes are fixed,
so one step — normalise, model, de-normalise, advance the time, shift the history
window by one state — is captured once into a CUDA graph over static buffers and
replayed; each replay's new state is then copied into the trajectory. Every CUDA
`torch.Generator` found on the model's modules (the reference's NoiseGenerator owns
one) is registered with the graph, so that each replay draws fresh noise as the eager
loop would. Autocast runs with its weight-cast cache off inside the capture, as CUDA
graphs require.
"""
import torch

__all__ = ["unroll_direct"]


def _generators(model):
    gens = []
    for mod in model.modules():
        g = getattr(mod, "generator", None)
        if isinstance(g, torch.Generator) and g.device.type == "cuda" and all(g is not h for h in gens):
            gens.append(g)
    return gens


@torch.no_grad()
def unroll_direct(model, initial_unnorm_state, day_year_time, day_year_delta, norm_stats, num_unroll_steps,
                  num_ensemble_members, dtype=torch.float16, graph=True, warmup_steps=1, step_events=None):
    """Forecast `num_unroll_steps` steps of `num_ensemble_members` members
    (inference.py:330-390).

    initial_unnorm_state: [B, history, lon, lat, channels] in physical units;
    day_year_time: [B, 2]; day_year_delta: [2]; norm_stats: an object with
    `state_mean` and `state_std` (broadcastable to the state). Returns the trajectory
    [B, members, history + num_unroll_steps, lon, lat, channels].

    graph=False runs every step eagerly (the reference's loop, step for step);
    graph=True replays steps 1 + warmup_steps .. num_unroll_steps - 1 from one CUDA
    graph. Both give the same trajectory when the model draws no noise or its
    generators are registered (graph replays advance them as eager calls do).

    step_events: a list to which (step, "eager" | "graph", start, end) is appended for
    every step, start and end being CUDA events recorded around the step on the stream
    that runs it (for timing; nothing is synchronised)."""
    if graph and initial_unnorm_state.device.type != "cuda":
        raise ValueError("unroll_direct(graph=True) runs on a CUDA device")
    B, H = initial_unnorm_state.shape[:2]
    M, T = num_ensemble_members, num_unroll_steps
    dev = initial_unnorm_state.device
    mean, std = norm_stats.state_mean, norm_stats.state_std
    traj = torch.empty((B, M, H + T) + tuple(initial_unnorm_state.shape[2:]), dtype=initial_unnorm_state.dtype,
                       device=dev)
    traj[:, :, :H] = initial_unnorm_state.unsqueeze(1)
    if T == 0:
        return traj

    def step(state, dyt, num_ens, cache=True):
        norm = (state - mean) / std
        with torch.autocast(dev.type, dtype=dtype, cache_enabled=cache):
            out = model(norm, dyt, num_ens)
        return out * std + mean

    def mark(t, kind, stream=None):
        if step_events is None:
            return None
        e = torch.cuda.Event(enable_timing=True)
        e.record(stream)
        return (t, kind, e)

    def done(m, stream=None):
        if m is not None:
            e = torch.cuda.Event(enable_timing=True)
            e.record(stream)
            step_events.append(m + (e,))

    def advance(dyt, num_ens):
        return dyt + day_year_delta.unsqueeze(0).unsqueeze(0).expand(B, num_ens, -1)

    # step 0: the ensemble is expanded here
    dyt = day_year_time.unsqueeze(1)
    m = mark(0, "eager")
    traj[:, :, H] = step(traj[:, :1, :H], dyt, M)
    dyt = advance(dyt, M)
    done(m)
    t = 1
    if not graph:
        for t in range(1, T):
            m = mark(t, "eager")
            traj[:, :, H + t] = step(traj[:, :, t:t + H], dyt, 1)
            dyt = advance(dyt, M)
            done(m)
        return traj

    # eager warm-up steps (real steps of the rollout) on a side stream
    cur = torch.cuda.current_stream(dev)
    side = torch.cuda.Stream(dev)
    side.wait_stream(cur)
    with torch.cuda.stream(side):
        while t < T and t < 1 + warmup_steps:
            m = mark(t, "eager", side)
            traj[:, :, H + t] = step(traj[:, :, t:t + H], dyt, 1, cache=False)
            dyt = advance(dyt, M)
            done(m, side)
            t += 1
    cur.wait_stream(side)
    if t >= T:
        return traj

    s_state = traj[:, :, t:t + H].clone()
    s_dyt = dyt.clone()
    delta = day_year_delta.to(s_dyt.dtype).view(1, 1, -1)
    g = torch.cuda.CUDAGraph()
    for gen in _generators(model):
        g.register_generator_state(gen)
    with torch.cuda.graph(g):
        s_next = step(s_state, s_dyt, 1, cache=False)
        s_dyt.add_(delta)
        s_state.copy_(torch.cat([s_state[:, :, 1:], s_next.unsqueeze(2).to(s_state.dtype)], dim=2))
    for t in range(t, T):
        m = mark(t, "graph")
        g.replay()
        traj[:, :, H + t].copy_(s_next)
        done(m)
    del g
    return traj
