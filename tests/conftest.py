import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
SRC = ROOT / "blackwell-inference-server_b200"
for p in (str(ROOT), str(SRC), str(ROOT / "tests" / "golden")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (B200, sm_100a) device")


@pytest.fixture(scope="session")
def golden():
    import json

    import numpy as np

    gdir = ROOT / "tests" / "golden"
    data = np.load(gdir / "golden.npz")
    index = json.loads((gdir / "golden_index.json").read_text())
    return data, index


@pytest.fixture(scope="session")
def cuda_dev():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("GPU test selected but no CUDA device is visible")
    return torch.device("cuda:0")
