import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); parity tests through the C-ABI")


@pytest.fixture(scope="session")
def oracle():
    from oracle import oracle as O
    if not os.path.exists(O.ORACLE_SO):
        O.build()
    return O.Oracle()


@pytest.fixture(scope="session")
def reference():
    from oracle import oracle as O
    if not os.path.exists(O.REF_SO):
        pytest.skip("reference CPU library (oracle/_ref) not built here")
    return O.Reference()


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("gpu-marked test run without a CUDA device")
    return torch.device("cuda", 0)
