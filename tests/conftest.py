import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = Path(__file__).resolve().parent / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU; run with -m gpu")


@pytest.fixture(autouse=True)
def _no_failed_device_check(request):
    """With the checked library loaded (CUTEX_B200_CHECKED=1): after every GPU test,
    no device-side index check may have failed (tests/test_gpu_device_checks.py)."""

    yield
    if os.environ.get("CUTEX_B200_CHECKED") != "1" or request.node.get_closest_marker("gpu") is None:
        return
    import torch

    from cutex_b200 import _lib

    if not torch.cuda.is_available():
        return
    site, value = _lib.check_record(torch.cuda.current_stream().cuda_stream)
    assert site == 0, f"device-side check 0x{site:x} failed (value {value})"
