"""The timeout path of the bounded device waits, exercised without faulting a
GPU: q2b_watchdog_selftest launches one thread that waits, with a short limit,
on a barrier nothing completes.  The wait gives up, the kernel returns, and
the code it recorded surfaces on the host -- through q2b_device_status (which
clears it) and through the per-step WatchdogMonitor poll the training path
uses -- while later launches keep working."""
import ctypes

import pytest
import torch

from cloverlm_b200 import _lib
from cloverlm_b200.quant import NVFP4QuantMode, quant_fp4

pytestmark = pytest.mark.gpu

SELFTEST_CODE = 6


def _selftest(cycles=20000):
    stream = torch.cuda.current_stream()
    _lib.call("q2b_watchdog_selftest", cycles, ctypes.c_void_p(stream.cuda_stream))


def test_wait_that_runs_out_reports_and_clears():
    assert _lib.device_status() == 0
    x = torch.randn(256, 512, device="cuda").to(torch.bfloat16)
    before = quant_fp4(x, scale_override=1.0, mode=NVFP4QuantMode.FOUR_SIX)
    _selftest()
    assert _lib.device_status() == SELFTEST_CODE
    assert _lib.device_status() == 0  # read clears it
    after = quant_fp4(x, scale_override=1.0, mode=NVFP4QuantMode.FOUR_SIX)
    assert torch.equal(before.fp4, after.fp4)
    assert torch.equal(before.micro_scales.view(torch.uint8), after.micro_scales.view(torch.uint8))
    assert _lib.device_status() == 0


def test_monitor_raises_on_the_training_path():
    mon = _lib.WatchdogMonitor(torch.device("cuda", torch.cuda.current_device()))
    mon.poll()
    mon.check_now()  # nothing tripped
    _selftest()
    mon.poll()
    with pytest.raises(_lib.WatchdogTimeout, match="code 6"):
        mon.check_now()
    assert _lib.device_status() == SELFTEST_CODE


def test_selftest_rejects_bad_limits():
    with pytest.raises(ValueError, match="wait_cycles"):
        _selftest(10)
