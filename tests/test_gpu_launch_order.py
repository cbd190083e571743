"""Ordering inside one forward call on the GPU. In mosaic_bsa_fwd, top-k starts
while the coarse attention still runs, and the attention kernel starts while top-k
still runs (programmatic stream serialization); each waits on the device before it
reads what the earlier kernels write. If a wait were missing or misplaced, a call
would read the block indices or the coarse-attention rows of the call queued before
it. These tests queue calls on inputs whose selections differ, back to back with no
host synchronisation between them, and check every output against the same call
made alone. The kernels are deterministic, so the outputs must be bit-identical."""
import pytest
import torch

import mosaic_b200 as M
from oracle import bsa_oracle as O

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _inputs(seed, N=12288, Hq=12, Hk=3):
    x = O.make_inputs(1, N, Hq, Hk, seed=seed, rope=False)
    return [x[k].to(DEV) for k in ("q", "k", "v", "w")]


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_back_to_back_calls_match_isolated_calls(dtype):
    sets = [[t.to(dtype) for t in _inputs(seed)] for seed in (31, 32, 33)]
    alone = []
    for q, k, v, w in sets:
        out, idx = M.mosaic_attn_func(q, k, v, w, 1024, 64, 24, False, return_block_indices=True)
        torch.cuda.synchronize()
        alone.append((out.clone(), idx.clone()))
    # the selections differ between the sets, so a stale read would show
    assert not torch.equal(alone[0][1], alone[1][1]) and not torch.equal(alone[1][1], alone[2][1])

    queued = []
    for r in range(12):
        q, k, v, w = sets[r % 3]
        queued.append(M.mosaic_attn_func(q, k, v, w, 1024, 64, 24, False, return_block_indices=True))
    torch.cuda.synchronize()
    for r, (out, idx) in enumerate(queued):
        ref_out, ref_idx = alone[r % 3]
        assert torch.equal(idx, ref_idx), f"call {r}: block indices differ from the isolated call"
        assert torch.equal(out, ref_out), f"call {r}: output differs from the isolated call"


def test_no_compression_and_reused_buffers():
    """no_compression (no coarse attention: top-k runs alone before the attention
    kernel) and calls that write into the same workspace one after another."""
    sets = [_inputs(seed) for seed in (41, 42)]
    alone = []
    for q, k, v, w in sets:
        alone.append(M.mosaic_attn_func(q, k, v, w, 1024, 64, 16, False, no_compression=True))
        torch.cuda.synchronize()
    queued = [M.mosaic_attn_func(*sets[r % 2], 1024, 64, 16, False, no_compression=True) for r in range(8)]
    torch.cuda.synchronize()
    for r, out in enumerate(queued):
        assert torch.equal(out, alone[r % 2]), f"call {r} differs from the isolated call"
