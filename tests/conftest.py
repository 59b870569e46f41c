import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100) GPU")
    config.addinivalue_line("markers", "slow: long-running")


@pytest.fixture(scope="session")
def oracle():
    from oracle.oracle_py import Oracle

    return Oracle()


@pytest.fixture(scope="session")
def reference():
    from oracle.oracle_py import REF_SO, Reference

    if not os.path.exists(REF_SO):
        pytest.skip("reference library not built (needs the reference sources at build time)")
    return Reference()


@pytest.fixture(scope="session")
def ctx():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from clusterlm_b200.runtime import Context

    c = Context(0)
    yield c
    c.close()
