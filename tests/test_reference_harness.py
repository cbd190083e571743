"""The reference-arm harness (baseline/reference.py) on the CPU: the installed copy of
the reference imports, and the autotuner-free launch never offers a q tile that does
not divide the block size (the reference's autotuner would, ops.py:20-23,54-55)."""
import pytest

from baseline import reference as R

pytestmark = pytest.mark.skipif(not R.available(), reason="baseline/_ref holds no reference copy")


def test_reference_modules_import():
    ref = R.load()
    assert hasattr(ref.ops, "mosaic_attn_fwd_kernel")
    assert ref.primitives.mosaic_sparse_attn == ref.mosaic_sparse_attn
    assert callable(ref.primitives.mosaic_attn_func)


@pytest.mark.parametrize("bs", [64, 128, 256])
def test_configs_divide_the_block(bs):
    cfgs = R.load().configs(bs)
    assert cfgs and all(bs % c["q_tile_size"] == 0 for c in cfgs)
    assert {c["num_warps"] for c in cfgs} == {4, 8} and {c["num_stages"] for c in cfgs} == {2, 3}
