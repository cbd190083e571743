"""StreamedAttention (host batches with overlapped copies) returns exactly what
mosaic_attn_func returns on each batch in order, and keeps working when batch
shapes change between submissions."""
import pytest
import torch

import mosaic_b200 as M
from mosaic_b200.streaming import StreamedAttention
from oracle import bsa_oracle as O

pytestmark = pytest.mark.gpu


def host_batch(N, Hq, Hk, seed):
    x = O.make_inputs(1, N, Hq, Hk, seed=seed, rope=False)
    return {n: x[n].bfloat16().pin_memory() for n in ("q", "k", "v", "w")}


@pytest.mark.parametrize("depth", [2, 3])
def test_streamed_equals_sequential(depth):
    bas, bs, K = 1024, 64, 8
    batches = [host_batch(3072, 4, 1, seed) for seed in range(5)]
    outs = [torch.empty(1, 3072, 4, 64, dtype=torch.bfloat16).pin_memory() for _ in batches]
    pipe = StreamedAttention("cuda", bas, bs, K, depth=depth)
    for x, o in zip(batches, outs):
        pipe.submit(x["q"], x["k"], x["v"], x["w"], o)
    pipe.join()
    torch.cuda.synchronize()
    for x, o in zip(batches, outs):
        ref = M.mosaic_attn_func(x["q"].cuda(), x["k"].cuda(), x["v"].cuda(), x["w"].cuda(), bas, bs, K, False)
        assert torch.equal(o, ref.cpu())


def test_streamed_shape_change():
    bas, bs, K = 1024, 64, 4
    batches = [host_batch(3072, 4, 1, 1), host_batch(2048, 8, 2, 2), host_batch(3072, 4, 1, 3)]
    outs = [torch.empty(x["q"].shape, dtype=torch.bfloat16).pin_memory() for x in batches]
    pipe = StreamedAttention("cuda", bas, bs, K)
    for x, o in zip(batches, outs):
        pipe.submit(x["q"], x["k"], x["v"], x["w"], o)
    pipe.join()
    torch.cuda.synchronize()
    for x, o in zip(batches, outs):
        ref = M.mosaic_attn_func(x["q"].cuda(), x["k"].cuda(), x["v"].cuda(), x["w"].cuda(), bas, bs, K, False)
        assert torch.equal(o, ref.cpu())


def test_depth_must_allow_overlap():
    with pytest.raises(ValueError):
        StreamedAttention("cuda", 1024, 64, 8, depth=1)

