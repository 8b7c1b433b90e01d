import json
import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if REPO not in sys.path:
    sys.path.insert(0, REPO)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and libhct_b200.so")


@pytest.fixture(scope="session")
def golden():
    with open(os.path.join(REPO, "tests", "golden", "golden.json")) as f:
        return json.load(f)


@pytest.fixture(scope="session")
def orc():
    import oracle

    oracle.lib()
    return oracle


@pytest.fixture(scope="session")
def hb():
    """The product package on a GPU; fails loudly if the CUDA library is absent."""
    import torch

    if not torch.cuda.is_available():
        pytest.fail("GPU test collected on a machine without CUDA")
    import haagenti_b200

    haagenti_b200._lib.load()
    return haagenti_b200


@pytest.fixture(scope="session")
def dev():
    import torch

    return torch.device("cuda", 0)
