import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")
    config.addinivalue_line("markers", "slow: long-running")


def _cuda_available() -> bool:
    try:
        import torch

        return torch.cuda.is_available()
    except Exception:
        return False


def pytest_collection_modifyitems(config, items):
    if _cuda_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device in this environment")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session")
def port():
    from oracle import Port

    return Port()


@pytest.fixture(scope="session")
def ref():
    from oracle import Ref, ref_path

    if ref_path() is None:
        pytest.skip("oracle/_ref not built here")
    try:
        return Ref()
    except OSError as e:  # built on a CPU this host cannot run
        pytest.skip(f"oracle/_ref cannot be loaded here: {e}")
