"""Device-side failure detection, exercised without faulting the GPU: a bounded
wait on a barrier that nothing arrives on must give up after its limit, record
MOSAIC_STATUS_TIMEOUT in the status word the host reads, and let the kernel (and
the CUDA context) carry on."""
import ctypes

import pytest
import torch

import mosaic_b200 as M
from mosaic_b200 import _lib
from mosaic_b200 import ops as mops
from oracle import bsa_oracle as O

pytestmark = pytest.mark.gpu


def test_bounded_wait_times_out_and_reports():
    lib = _lib.load()
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    result = torch.full((2,), -1, dtype=torch.int32, device="cuda")
    rc = lib.mosaic_selftest_wait_timeout(ctypes.c_void_p(status.data_ptr()), ctypes.c_void_p(result.data_ptr()),
                                          20000, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == _lib.MOSAIC_OK
    torch.cuda.synchronize()
    assert result.tolist() == [0, 1]
    assert status.item() & _lib.MOSAIC_STATUS_TIMEOUT
    with pytest.raises(RuntimeError):
        mops.check_status(status)
    # the context is still usable: a real forward right after runs and is correct
    x = O.make_inputs(1, 768, 4, 1, seed=30, rope=False)
    out = M.block_attention(x["q"].cuda(), x["k"].cuda(), x["v"].cuda(), 256)
    d = (out.float().cpu() - O.block_attention(x["q"], x["k"], x["v"], 256)).abs()
    assert d.max() < 2e-2


def test_selftest_rejects_bad_arguments():
    lib = _lib.load()
    assert lib.mosaic_selftest_wait_timeout(None, None, 10, None) == _lib.MOSAIC_ERR_INVALID_ARGUMENT
