import pathlib
import sys

import pytest

ROOT = pathlib.Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "tests" / "golden"))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); run with -m gpu")


@pytest.fixture(scope="session")
def golden():
    import json

    import numpy as np
    d = ROOT / "tests" / "golden"
    return np.load(d / "golden.npz"), json.loads((d / "golden_meta.json").read_text())


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from siliconfer_b200 import _lib
    _lib.load()
    return torch.device("cuda", 0)
