"""Failure detection on the GPU without a fault: a bounded device-side wait that runs out.

Every tensor-core kernel of the library waits on mbarriers through the same bounded wait
(tc::mbar_wait).  bl_wait_selftest runs that wait in a one-thread kernel with a short
limit on a phase that nothing completes (a flag that nothing sets): the wait must give up,
record its code in the device status word and let the kernel return, after which the
context must still run the library's kernels.  With the phase completed the status must
stay clear.
"""

import time

import pytest
import torch

pytestmark = pytest.mark.gpu

SELFTEST_CODE = 0x7F01


def _selftest(arrive, limit_ns):
    from boltz_lumi_b200 import _lib

    _lib.call("bl_wait_selftest", int(arrive), int(limit_ns), torch.cuda.current_stream().cuda_stream)


def test_completed_wait_leaves_status_clear():
    from boltz_lumi_b200 import _lib

    assert _lib.device_status(reset=True) == 0
    _selftest(arrive=True, limit_ns=1_000_000)
    assert _lib.device_status(reset=True) == 0


def test_wait_that_runs_out_reports_and_returns():
    from boltz_lumi_b200 import _lib, kernels

    assert _lib.device_status(reset=True) == 0
    t0 = time.perf_counter()
    _selftest(arrive=False, limit_ns=2_000_000)  # 2 ms
    status = _lib.device_status(reset=False)  # synchronises: the kernel has returned
    elapsed = time.perf_counter() - t0
    assert status == SELFTEST_CODE, hex(status)
    assert elapsed < 5.0, elapsed
    assert _lib.device_status(reset=True) == SELFTEST_CODE
    assert _lib.device_status(reset=False) == 0
    # The context is still usable: a library kernel runs and is correct afterwards.
    x = torch.randn(64, 128, device="cuda")
    w = torch.rand(128, device="cuda") + 0.5
    b = torch.randn(128, device="cuda")
    with torch.inference_mode():
        y = kernels.layer_norm(x, w, b, 1e-5, out_dtype=torch.float32)
    expected = torch.nn.functional.layer_norm(x, (128,), w, b, 1e-5)
    assert torch.allclose(y, expected, atol=1e-5)
    assert _lib.device_status(reset=True) == 0


def test_selftest_rejects_bad_limits():
    from boltz_lumi_b200 import _lib

    with pytest.raises(RuntimeError, match="bl_wait_selftest"):
        _lib.call("bl_wait_selftest", 0, 0, None)
    with pytest.raises(RuntimeError, match="bl_wait_selftest"):
        _lib.call("bl_wait_selftest", 0, 3_000_000_000, None)
