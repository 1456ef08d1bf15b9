"""Failure detection on the GPU without a GPU fault: the bounded mbarrier wait that
every tensor-core kernel uses is made to wait on a phase nothing completes
(mhc_selftest_wait_timeout).  The kernel gives up, records MHC_ERR_TIMEOUT, and
returns; the host reads the status; the context keeps working."""
import pytest
import torch

import FlagOS_mhc as M
from FlagOS_mhc import _C
from oracle import mhc_oracle as O
from tests._util import TOL_BF16, rel_err
from tests.gen import post_inputs

pytestmark = pytest.mark.gpu


def test_bounded_wait_times_out_and_context_survives():
    L = _C.lib()
    assert L.mhc_device_status() == 0
    s = _C.stream_of(torch.empty(1, device="cuda"))
    assert L.mhc_selftest_wait_timeout(1 << 12, s) == 0
    assert L.mhc_device_status() == _C.MHC_ERR_TIMEOUT
    assert L.mhc_device_status() == 0          # read and cleared
    assert L.mhc_selftest_wait_timeout(0, s) == _C.MHC_ERR_INVALID_ARGUMENT
    # an operator right after still runs and is correct
    x, hr, ho, hp, _ = post_inputs(64, 4, 256, torch.bfloat16, seed=1)
    y = M.mhc_post(x.cuda(), hr.cuda(), ho.cuda(), hp.cuda())
    assert rel_err(y, O.post_fwd(x, hr, ho, hp, dtype=torch.float64)) <= TOL_BF16
    assert L.mhc_device_status() == 0
