"""Shared pytest setup.  Tests marked `gpu` need an sm_100 GPU (run with -m gpu on a B200 box);
everything else runs on the CPU (-m "not gpu")."""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 (B200) GPU; the CUDA path has no CPU fallback")


@pytest.fixture(scope="session")
def pf():
    """The product package with its CUDA library loaded (fails loudly if missing)."""
    import ptxforge_b200
    ptxforge_b200.load_library()
    return ptxforge_b200


@pytest.fixture(scope="session")
def oracle_mod():
    import oracle
    oracle.lib()
    return oracle


@pytest.fixture(scope="session")
def ctx(pf):
    """One context on cuda:0 for the GPU tests."""
    c = pf.Context(0)
    yield c
    c.close()
