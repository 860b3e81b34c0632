import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PACKAGE_ROOT = os.path.join(REPO, "ictc-o3-hp-ascend_b200")
for path in (PACKAGE_ROOT, REPO):
    if path not in sys.path:
        sys.path.insert(0, path)

GOLDEN = os.path.join(REPO, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200) and libictc_cuda.so")
    config.addinivalue_line("markers", "multigpu: starts one NCCL rank process per GPU on several GPUs")


def pytest_collection_modifyitems(config, items):
    """Tests that start rank processes on several GPUs run after all the others (they
    are the slowest and need the most of the box), keeping the collection order
    otherwise."""
    items.sort(key=lambda item: item.get_closest_marker("multigpu") is not None)


def golden(name):
    import numpy as np
    return dict(np.load(os.path.join(GOLDEN, name)))


@pytest.fixture(scope="session")
def cuda_device():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("GPU test selected but no CUDA device is visible")
    return torch.device("cuda", 0)
