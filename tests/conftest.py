import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (ROOT, os.path.join(ROOT, "flash-evict-prefill_b200")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


def pytest_collection_modifyitems(config, items):
    import torch
    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="CUDA GPU required")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session", autouse=True)
def _short_watchdog():
    """Device-side waits in these tests last microseconds; a 0.5 s watchdog
    makes a kernel that waits on something that never happens report a
    timeout quickly instead of after the 2 s default per wait."""
    import torch
    if torch.cuda.is_available():
        from flash_evict import _lib
        _lib.load().fe_set_watchdog_ns(500_000_000)
    yield


@pytest.fixture(autouse=True)
def _device_status(request):
    """After every GPU test: no kernel may have raised the device status word
    (watchdog timeout); tests that raise it on purpose clear it themselves."""
    yield
    if "gpu" in request.node.keywords:
        import torch
        if torch.cuda.is_available():
            from flash_evict import _lib
            status = _lib.device_status(torch.cuda.current_device(), clear=True)
            assert status == 0, f"device status word raised: {status}"


def pytest_terminal_summary(terminalreporter):
    from common import PARITY_FIGURES
    if PARITY_FIGURES:
        terminalreporter.write_sep("-", "parity figures (GPU vs float64 oracle)")
        for line in PARITY_FIGURES:
            terminalreporter.write_line(line)
