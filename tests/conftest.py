import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (ROOT, os.path.join(ROOT, "oracle"), os.path.join(ROOT, "tests")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and libdiskllm_cuda.so")
    config.addinivalue_line("markers", "slow: long-running")


@pytest.fixture(scope="session")
def have_reference():
    import oracle

    if not oracle.have_reference():
        pytest.skip("oracle/_ref not built (reference sources unavailable)")
    return True
