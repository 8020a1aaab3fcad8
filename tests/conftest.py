import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "vllm-exl3_b200")
ORACLE = os.path.join(ROOT, "oracle")
GOLDEN = os.path.join(ROOT, "tests", "golden")
for p in (PKG, ORACLE):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200); run with -m gpu")


def cuda_ok() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.fixture(scope="session")
def cuda():
    if not cuda_ok():
        pytest.skip("CUDA GPU required")
    import torch
    return torch.device("cuda", 0)


@pytest.fixture(scope="session")
def native(cuda):
    """The drop-in module on a GPU box; the CUDA library must load (no fallback)."""
    import vllm_exl3_c
    from exl3_b200 import _native
    _native.load()
    return vllm_exl3_c


@pytest.fixture(autouse=True)
def _device_status_clean(request):
    """GPU tests: the shared workspace's device status word must stay 0 (a
    kernel that skipped work or gave up a bounded wait records a code there
    and would otherwise pass unnoticed).  Tests that provoke a code clear it."""
    if request.node.get_closest_marker("gpu") is None or not cuda_ok():
        yield
        return
    import vllm_exl3_c
    vllm_exl3_c.device_status(clear=True)
    yield
    st = vllm_exl3_c.device_status(clear=True)
    assert st == 0, f"device status word {st} after the test"
