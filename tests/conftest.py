import os
import sys
from pathlib import Path

import numpy as np
import pytest

REPO = Path(__file__).resolve().parents[1]
GOLDEN = REPO / "tests" / "golden"
if str(REPO) not in sys.path:
    sys.path.insert(0, str(REPO))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


def load_golden(name):
    from flowedge_b200.checkpoint import read_safetensors

    tensors, metadata = read_safetensors(GOLDEN / f"{name}.safetensors")
    data = dict(np.load(GOLDEN / f"{name}.npz"))
    return tensors, metadata, data


@pytest.fixture
def golden():
    return load_golden
