"""Bounded device waits run out cleanly: an mbarrier wait (the TMA-fed kernels' kind) and a flag
wait (the multi-GPU transport's kind), each on something that never completes, with a 1 ms limit
through the library's own wait functions. The wait gives up, lyth_b200_device_error reports
LYTH_E_TIMEOUT once, and the next launch and the next status check are clean: the context stays
usable. No fault or trap is involved (the wait returns)."""
import numpy as np
import pytest
import torch

import lyth_b200 as lb
from oracle import oracle as orc

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("which", [0, 1])
def test_wait_runs_out_and_reports_timeout(cuda, which):
    assert lb.lib.lyth_b200_device_error() == lb.OK  # nothing pending from earlier tests
    s = torch.cuda.current_stream().cuda_stream
    assert lb.lib.lyth_b200_wait_selftest(which, 1000, s) == lb.OK
    torch.cuda.synchronize()
    assert lb.lib.lyth_b200_device_error() == lb.E_TIMEOUT
    assert lb.lib.lyth_b200_device_error() == lb.OK  # reported once, then cleared
    # the context is still usable: a kernel runs and is bit-exact
    n = 4099
    x, y = orc.uniform(1, n), orc.uniform(2, n)
    xd, yd = torch.from_numpy(x).to(cuda), torch.from_numpy(y).to(cuda)
    lb.saxpy(2.5, xd, yd)
    assert np.array_equal(yd.cpu().numpy().view(np.uint32), orc.saxpy(2.5, x, y).view(np.uint32))
    assert lb.lib.lyth_b200_device_error() == lb.OK


def test_wait_selftest_refuses_bad_arguments(cuda):
    s = torch.cuda.current_stream().cuda_stream
    assert lb.lib.lyth_b200_wait_selftest(2, 1000, s) == lb.E_INVALID
    assert lb.lib.lyth_b200_wait_selftest(0, 0, s) == lb.E_INVALID
    assert lb.lib.lyth_b200_wait_selftest(0, 3_000_000, s) == lb.E_INVALID
