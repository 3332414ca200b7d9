import os
import subprocess
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if REPO not in sys.path:
    sys.path.insert(0, REPO)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


def _built(path):
    return os.path.exists(os.path.join(REPO, path))


@pytest.fixture(scope="session", autouse=True)
def _build_native():
    """Builds the oracle and the library in tree if they are missing (no-op on the GPU box,
    where the prebuilt files travel with the repository)."""
    if not _built("oracle/liboracle.so"):
        subprocess.run(["make", "-s", "-C", os.path.join(REPO, "oracle")], check=True)
    if not _built("l2domain_b200/lib/libl2d.so"):
        subprocess.run(["make", "-s", "-C", os.path.join(REPO, "l2domain_b200", "csrc")], check=True)
    yield


def has_gpu():
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False
