import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "minimax-h3-swift_b200")
for p in (ROOT, PKG):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


def has_gpu():
    try:
        import torch

        return torch.cuda.is_available() and torch.cuda.get_device_capability(0)[0] == 10
    except Exception:
        return False


@pytest.fixture(scope="session")
def gpu():
    if not has_gpu():
        pytest.fail("this test needs a B200 GPU (run with -m 'not gpu' on CPU)")
    import torch

    return torch.device("cuda:0")


@pytest.fixture(autouse=True)
def _device_status_clean(request):
    """After every GPU test: the kernels' device status word must be clean
    (a bounded wait that gave up records H3C_ERR_TIMEOUT there; the calls
    themselves are asynchronous and cannot report it)."""
    yield
    if request.node.get_closest_marker("gpu") is None or "no_status_check" in request.keywords:
        return
    if not has_gpu():
        return
    import torch

    from h3attention import Runtime

    for d in range(torch.cuda.device_count()):
        if d in Runtime._by_device:
            torch.cuda.synchronize(d)
            Runtime._by_device[d].device_status()
