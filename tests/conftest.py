import os
import sys

import numpy as np
import pytest

ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), ".."))
for p in (ROOT, os.path.join(ROOT, "sme-ai-ops_b200")):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a compute-capability-10.x CUDA device")
    config.addinivalue_line("markers", "slow: takes more than a few seconds")


@pytest.fixture(scope="session")
def oracle():
    from oracle import oracle as O
    O.build()
    O.lib()
    return O


@pytest.fixture(scope="session")
def golden():
    def load(name):
        return dict(np.load(os.path.join(GOLDEN, name)))
    return load


@pytest.fixture(scope="session")
def cuda():
    """The CUDA device; GPU tests fail (not skip) when it is missing, so a
    silent CPU-only run cannot pass for a GPU run."""
    import torch
    import smeai_b200 as S
    assert torch.cuda.is_available(), "GPU test run without a CUDA device"
    S.lib()
    assert S.device_ready(), f"no compute-capability-10.x device: {S.last_error()}"
    return torch.device("cuda:0")
