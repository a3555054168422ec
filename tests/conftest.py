import pathlib
import sys

import pytest

ROOT = pathlib.Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 GPU (runs the sm_100a kernels)")


@pytest.fixture(scope="session")
def pkg():
    import __graft_entry__

    return __graft_entry__.load_package()


@pytest.fixture(scope="session")
def orc():
    from oracle import moe_oracle

    return moe_oracle
