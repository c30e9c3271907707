import os
import subprocess
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (os.path.join(REPO, "oracle"), os.path.join(REPO, "sa3.cpp_b200"), REPO):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) and the built sa3k library")


@pytest.fixture(scope="session", autouse=True)
def _built_oracle():
    """The C oracle (test infrastructure) is rebuilt if missing; the reference part is optional."""
    if not os.path.exists(os.path.join(REPO, "oracle", "liboracle.so")):
        subprocess.run(["make", "-C", os.path.join(REPO, "oracle")], check=True, capture_output=True)


@pytest.fixture(scope="session")
def sa3k_lib():
    import build as sa3k_build  # sa3.cpp_b200/build.py (incremental)
    sa3k_build.build()
    import sa3k
    return sa3k.lib()


@pytest.fixture(scope="session")
def ctx(sa3k_lib):
    import torch
    import sa3k
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    c = sa3k.Context(0)
    yield c
    c.sync()
    c.close()
