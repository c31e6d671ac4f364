import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "tests"))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 GPU (run with -m gpu on a B200)")
    config.addinivalue_line("markers", "slow: full-size cases that take more than a few seconds")


@pytest.fixture(scope="session")
def cuda():
    """The CUDA device the gpu tests run on, with libcairn_b200.so loaded (never a fallback)."""
    import torch

    import cairn_b200

    if not torch.cuda.is_available():
        pytest.fail("a gpu test ran without a CUDA device")
    cairn_b200.lib()
    torch.cuda.set_device(0)
    return torch.device("cuda", 0)
