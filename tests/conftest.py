"""Shared test setup: the `gpu` marker, import paths and the checker libs."""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "deepseek-v4-flash-0731-in-c_b200")
for p in (os.path.join(ROOT, "oracle"), os.path.join(ROOT, "tests", "golden"), PKG):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


@pytest.fixture(scope="session")
def orc():
    from oracle import Oracle
    return Oracle()


@pytest.fixture(scope="session")
def ref():
    from oracle import Ref, REF_SO
    if not os.path.exists(REF_SO):
        pytest.skip("reference library oracle/_ref/libdsv4_ref.so not built here")
    return Ref()


@pytest.fixture(scope="session")
def cuda():
    """The product library; GPU tests fail (not skip) when it is missing."""
    import torch
    if not torch.cuda.is_available():
        pytest.fail("GPU test run without a CUDA device")
    import dsv4cuda
    dsv4cuda.set_abort_on_error(False)
    dsv4cuda.init(0)
    yield dsv4cuda
    # no kernel of the session may have given up on a bounded wait
    assert dsv4cuda.device_error() == 0
