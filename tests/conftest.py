import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (REPO, os.path.join(REPO, "opus-lab-notebooks_b200")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def golden_kmeans():
    import numpy as np
    return dict(np.load(os.path.join(REPO, "tests", "golden", "kmeans_golden.npz")))


@pytest.fixture(scope="session")
def golden_decode():
    import numpy as np
    return dict(np.load(os.path.join(REPO, "tests", "golden", "decode_golden.npz")))
