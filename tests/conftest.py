import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200)")
    config.addinivalue_line("markers", "slow: long-running")


@pytest.fixture(scope="session")
def oracle_lib():
    from oracle import oracle

    oracle.build()
    return oracle


@pytest.fixture(autouse=True)
def _device_status_stays_clear(request):
    """Every GPU test ends with the device status word clear: no kernel's
    bounded staging wait gave up (a give-up leaves games unstepped)."""
    yield
    if request.node.get_closest_marker("gpu") is None:
        return
    import torch

    if not torch.cuda.is_available():
        return
    from nanorts_b200.runtime import check_device

    torch.cuda.synchronize()
    check_device(torch.cuda.current_device())
