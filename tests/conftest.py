import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200) and the built libsemx.so")


def pytest_collection_modifyitems(config, items):
    # GPU tests fail loudly (not skip) when a GPU run is requested without a GPU, so a
    # CPU-only environment can never report the GPU tier as green.
    pass


@pytest.fixture(scope="session")
def golden():
    import torch

    def load(name):
        return torch.load(ROOT / "tests" / "golden" / f"{name}.pt", weights_only=True)

    return load
