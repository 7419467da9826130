import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

MODEL_DIR = os.environ.get("MYLLM_MODEL_DIR", "/tmp/myllm_b200_models")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200)")


@pytest.fixture(scope="session")
def model_dir():
    os.makedirs(MODEL_DIR, exist_ok=True)
    return MODEL_DIR


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from myllm_b200 import _native
    _native.lib()  # loud failure if the extension is missing
    return torch.device("cuda:0")
