import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line(
        "markers", "gpu: needs a CUDA device (B200); parity tests proper")


@pytest.fixture(scope="session")
def port():
    from oracle import pyoracle

    if not os.path.exists(pyoracle.PORT_SO):
        pyoracle.build_port()
    return pyoracle.Port()


@pytest.fixture(scope="session")
def ref():
    from oracle import pyoracle

    if not pyoracle.ref_available():
        pytest.skip("oracle/_ref (compiled reference) not built here")
    return pyoracle.Ref()


@pytest.fixture(scope="session")
def cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from opendressi_b200 import _native

    _native.load()
    return torch.device("cuda:0")
