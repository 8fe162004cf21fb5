import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
for p in (ROOT, ROOT / "lizard-reproduction_b200", ROOT / "oracle", ROOT / "tests" / "golden"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))

GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (run on the B200 box)")


@pytest.fixture(scope="session")
def built_lib():
    """Path of liblizard_cuda.so, building it first when it is missing."""
    sys.path.insert(0, str(ROOT / "lizard-reproduction_b200" / "csrc"))
    import build  # lizard-reproduction_b200/csrc/build.py
    return build.build()


def load_golden(name):
    import torch
    return torch.load(GOLDEN / f"{name}.pt", weights_only=False)
