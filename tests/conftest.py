import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
for p in (ROOT, ROOT / "tests", ROOT / "tests" / "golden"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200) and libaoakv.so")


@pytest.fixture(scope="session")
def cuda():
    """Skips when no GPU is visible; on a GPU box the library must load."""
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import aoa_kv_b200
    aoa_kv_b200._lib.load()
    return torch.device("cuda:0")
