"""Shared test set-up.

Markers: `gpu` tests need a CUDA device and run the product path (the
libepb200.so engine) against the CPU oracle; everything else runs on CPU.
"""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (ROOT, os.path.join(ROOT, "oracle")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); runs the CUDA engine")


@pytest.fixture(scope="session")
def oracle():
    """The CPU oracle module (built on demand)."""
    import build_oracle as obuild
    obuild.build_oracle()
    import oracle as o
    return o


@pytest.fixture(scope="session")
def golden_density():
    import numpy as np
    return np.load(os.path.join(ROOT, "tests", "golden", "density_ref.npz"))


@pytest.fixture(scope="session")
def golden_dct():
    import numpy as np
    return np.load(os.path.join(ROOT, "tests", "golden", "dct_ref.npz"))


@pytest.fixture(scope="session")
def cuda_device():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("gpu test selected but torch.cuda.is_available() is False")
    from dreamplacett_framework_b200 import build
    build.build()
    return torch.device("cuda", 0)
