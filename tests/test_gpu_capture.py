"""Graph capture around the op on the GPU: torch.compile traces through the
custom operator, and a captured CUDA graph replays to the eager result."""
import pytest
import torch

import mosaic_b200 as M
from oracle import bsa_oracle as O

pytestmark = pytest.mark.gpu


def host_batch(N, Hq, Hk, seed):
    x = O.make_inputs(1, N, Hq, Hk, seed=seed, rope=False)
    return {n: x[n].bfloat16() for n in ("q", "k", "v", "w")}


def test_compiled_graph_calls_the_library():
    """torch.compile traces around the op (an opaque custom op) and the compiled
    function returns what the eager call returns."""
    x = host_batch(3072, 4, 1, 7)
    q, k, v, w = (x[n].cuda() for n in ("q", "k", "v", "w"))

    def layer(q, k, v, w):
        return M.mosaic_attn_func(q * 1.0, k, v, w, 1024, 64, 8, False) + 0.0

    eager = layer(q, k, v, w)
    compiled = torch.compile(layer, backend="aot_eager", fullgraph=True)(q, k, v, w)
    assert torch.equal(eager, compiled)


def test_cuda_graph_replay():
    """The op can be captured in a CUDA graph (mode="reduce-overhead" captures the
    reference model this way) and replays to the eager result on new inputs."""
    a, b = host_batch(3072, 4, 1, 8), host_batch(3072, 4, 1, 9)
    dev = {n: a[n].cuda() for n in ("q", "k", "v", "w")}
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        M.mosaic_attn_func(dev["q"], dev["k"], dev["v"], dev["w"], 1024, 64, 8, False)  # warm-up
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        out = M.mosaic_attn_func(dev["q"], dev["k"], dev["v"], dev["w"], 1024, 64, 8, False)
    for x in (b, a):
        for n in dev:
            dev[n].copy_(x[n])
        g.replay()
        torch.cuda.synchronize()
        ref = M.mosaic_attn_func(x["q"].cuda(), x["k"].cuda(), x["v"].cuda(), x["w"].cuda(), 1024, 64, 8, False)
        assert torch.equal(out, ref)
