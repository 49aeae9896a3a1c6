"""The kernels' bounded waits give up cleanly (the failure path, made to happen on purpose).

Every mbarrier wait in the attention and GEMM kernels is bounded by SM clock cycles; one
that runs out sets the CTA's abort flag and the wait-timeout bit of the device status word,
and the kernel drains and returns. ``hb_selftest_wait_timeout`` runs that same wait with a
short limit on a barrier phase nothing completes (a flag no thread sets), so the limit runs
out: the call must return, report the wait as failed with the abort flag set, raise
HB_STATUS_WAIT_TIMEOUT, and leave the context usable for the next launch.
"""

import pytest
import torch

from helios_b200 import _native

pytestmark = pytest.mark.gpu


def test_bounded_wait_times_out_sets_status_and_returns():
    lib = _native.load()
    _native.device_status()  # start from a clear status word
    result = torch.full((2,), -1, dtype=torch.int32, device="cuda")
    rc = lib.hb_selftest_wait_timeout(1_000_000, result.data_ptr(), torch.cuda.current_stream().cuda_stream)
    _native.check(rc, "hb_selftest_wait_timeout")
    status = _native.device_status()
    assert result.tolist() == [0, 1]
    assert status & 1, _native.describe_status(status)  # HB_STATUS_WAIT_TIMEOUT
    # The context still works: an ordinary launch and a clear status afterwards.
    x = torch.arange(8, device="cuda", dtype=torch.float32)
    assert float((x * 2).sum()) == 56.0
    assert _native.device_status() == 0


def test_wait_limit_is_checked_on_the_host():
    lib = _native.load()
    result = torch.zeros(2, dtype=torch.int32, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    assert lib.hb_selftest_wait_timeout(0, result.data_ptr(), stream) == _native.HB_ERR_INVALID
    assert lib.hb_selftest_wait_timeout(1 << 40, result.data_ptr(), stream) == _native.HB_ERR_INVALID
