"""Shared test configuration: the ``gpu`` marker and parity helpers."""

import os
import sys
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(autouse=True)
def _device_status_clean(request):
    """After every GPU test, every bounded device-side wait must have completed."""
    yield
    if request.node.get_closest_marker("gpu") and torch.cuda.is_available():
        from boltz_lumi_b200 import _lib

        assert _lib.device_status(reset=True) == 0, "a bounded device-side wait timed out"


def report(actual, expected):
    """Error summary in the reference tests' vocabulary (test_operator_additions.py:26-40)."""
    a = actual.detach().double().cpu()
    e = expected.detach().double().cpu()
    err = (a - e).abs()
    norm = e.norm().item()
    return dict(
        max_absolute_error=err.max().item() if err.numel() else 0.0,
        relative_l2_error=(a - e).norm().item() / norm if norm else None,
        failing_values=int((a != e).sum()),
    )


def record_parity(case, info):
    """Append a case's measured errors to the JSON-lines file named by BL_PARITY_LOG (if set),
    so a GPU run leaves the per-op error table behind."""
    path = os.environ.get("BL_PARITY_LOG")
    if not path:
        return
    import json

    with open(path, "a") as f:
        f.write(json.dumps({"case": case, **{k: v for k, v in info.items()}}) + "\n")


def assert_close(actual, expected, atol, rtol=0.0, rel_l2=None):
    """max |a - e| <= atol + rtol |e| elementwise, optional relative-L2 bound."""
    a = actual.detach().double().cpu()
    e = expected.detach().double().cpu()
    assert a.shape == e.shape, (a.shape, e.shape)
    assert torch.isfinite(a).all(), "non-finite output"
    bad = (a - e).abs() > atol + rtol * e.abs()
    info = report(actual, expected)
    info.update(atol=atol, rtol=rtol, over_tolerance=int(bad.sum()))
    assert not bad.any(), info
    if rel_l2 is not None and info["relative_l2_error"] is not None:
        assert info["relative_l2_error"] <= rel_l2, info
    return info
