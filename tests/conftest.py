import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100) GPU; run with -m gpu")


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    major, minor = torch.cuda.get_device_capability(0)
    if (major, minor) != (10, 0):
        pytest.skip(f"needs sm_100, found sm_{major}{minor}")
    from demon_b200 import _build
    _build.build()
    return torch.device("cuda", 0)
