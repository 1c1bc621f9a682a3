import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "tests", "golden"))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a); run with -m gpu")


def pytest_runtest_setup(item):
    if item.get_closest_marker("gpu") is not None:
        import torch
        if not torch.cuda.is_available():
            pytest.fail("GPU test selected but no CUDA device is visible", pytrace=False)


@pytest.fixture(scope="session")
def golden():
    import numpy as np
    d = os.path.join(ROOT, "tests", "golden")
    return dict(codec=np.load(os.path.join(d, "codec_cases.npz")), config1=np.load(os.path.join(d, "config1.npz")))
