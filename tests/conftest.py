import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and the built extension")


def golden(name):
    import numpy as np

    return np.load(os.path.join(GOLDEN, name))


@pytest.fixture(scope="session")
def tsne_golden():
    return golden("tsne_small.npz")


@pytest.fixture(scope="session")
def umap_golden():
    return golden("umap_small.npz")


@pytest.fixture(scope="session")
def umap_scalar_golden():
    return golden("umap_scalar.npz")


@pytest.fixture(scope="session")
def umap_device_golden():
    return golden("umap_device_small.npz")
