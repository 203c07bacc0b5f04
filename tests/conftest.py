import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 GPU (B200)")


@pytest.fixture(scope="session")
def built_library():
    from nvcr_b200.build import build

    return build()


@pytest.fixture(scope="session")
def oracle():
    from oracle.oracle import Oracle, build

    build(reference=True)
    return Oracle()


@pytest.fixture(scope="session")
def reference():
    from oracle.oracle import Reference, build

    build(reference=True)
    if not Reference.available():
        pytest.skip("the reference CPU executor (oracle/_ref) is not built here")
    return Reference()


@pytest.fixture(scope="session")
def fx_oracle():
    from oracle.fx import FxOracle
    from oracle.oracle import build

    build(reference=True)
    return FxOracle()


@pytest.fixture(scope="session")
def fx_reference():
    from oracle.fx import FxReference
    from oracle.oracle import Reference, build

    build(reference=True)
    if not Reference.available():
        pytest.skip("the reference CPU executor (oracle/_ref) is not built here")
    return FxReference()


@pytest.fixture(scope="session")
def cuda(built_library):
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    torch.cuda.init()
    return torch.device("cuda:0")
