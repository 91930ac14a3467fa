import os
import subprocess
import sys

import pytest

TESTS = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(TESTS)
PKG = os.path.join(REPO, "ane-lm_b200")
for p in (TESTS, PKG, REPO):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def _cuda_available() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


def pytest_collection_modifyitems(config, items):
    if _cuda_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device in this environment")
    for it in items:
        if "gpu" in it.keywords:
            it.add_marker(skip)


@pytest.fixture(scope="session")
def oracle():
    from oracle_lib import Oracle
    return Oracle()


@pytest.fixture(scope="session")
def ref():
    from oracle_lib import load_ref
    lib = load_ref()
    if lib is None:
        pytest.skip("reference build oracle/_ref absent (no reference tree on this machine)")
    return lib


@pytest.fixture(scope="session")
def ane():
    """The CUDA backend; builds libane_cuda.so if it is missing."""
    so = os.path.join(PKG, "libane_cuda.so")
    if not os.path.exists(so):
        subprocess.run(["make", "-s", "-j8", "-C", PKG], check=True)
    import ane_lm_cuda
    ane_lm_cuda.lib()
    return ane_lm_cuda
