import os
import sys
from pathlib import Path

import pytest
import torch

REPO = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(REPO))
sys.path.insert(0, str(REPO / "iris-3b-metal_b200"))
GOLDEN = REPO / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (sm_100a) device")
    torch.set_num_threads(min(8, os.cpu_count() or 1))


def golden(name: str):
    return torch.load(GOLDEN / f"{name}.pt", weights_only=False)


requires_gpu = pytest.mark.gpu
