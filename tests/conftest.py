import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = Path(__file__).resolve().parent / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def golden_dir() -> Path:
    return GOLDEN


def load_golden(name: str):
    import torch

    return torch.load(GOLDEN / f"{name}.pt", weights_only=False)


os.environ.setdefault("OMP_NUM_THREADS", str(os.cpu_count() or 1))
