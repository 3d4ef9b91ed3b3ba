import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if REPO not in sys.path:
    sys.path.insert(0, REPO)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (B200, sm_100a) device")


@pytest.fixture(scope="session")
def cuda():
    """Device fixture for -m gpu tests: fails (never skips) without a GPU, so a
    broken GPU box cannot pass the suite silently."""
    import torch
    assert torch.cuda.is_available(), "gpu-marked test needs a CUDA device"
    major, _ = torch.cuda.get_device_capability(0)
    assert major >= 10, "kernels are built for sm_100a (B200)"
    import tabinfer_b200  # noqa: F401  (loads libtabinfer_b200.so, raises if missing)
    return torch.device("cuda", 0)


@pytest.fixture(autouse=True)
def _no_device_wait_timeouts(request):
    """After every GPU test: the device error word that bounded in-kernel waits
    set must still be clear (a timed-out wait would otherwise only show up as
    missing output)."""
    yield
    if request.node.get_closest_marker("gpu") is None:
        return
    import torch
    if not torch.cuda.is_available():
        return
    import tabinfer_b200 as tb
    code = tb.default_context(0).device_error()
    assert code == 0, "a bounded device-side wait timed out (code 0x%x)" % code


@pytest.fixture(scope="session")
def golden():
    import numpy as np
    d = os.path.join(REPO, "tests", "golden")
    return {"tern": dict(np.load(os.path.join(d, "ternary_packs.npz"))),
            "int4": dict(np.load(os.path.join(d, "int4_js.npz")))}
