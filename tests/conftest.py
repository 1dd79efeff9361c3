"""Shared fixtures.  GPU tests are marked ``gpu``; they need a B200 and fail (not skip) when
the device cannot be opened, so a GPU run can never pass by silently skipping."""
import importlib
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

PACKAGE = "magnetar-provider-cuda_b200"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 device (sm_100a)")


def load_package():
    return importlib.import_module(PACKAGE)


@pytest.fixture(scope="session")
def mpc():
    return load_package()


@pytest.fixture(scope="session")
def oracle():
    from oracle import oracle as orc
    orc.build()
    return orc


@pytest.fixture(scope="session")
def kernels(mpc):
    k = mpc.CudaKernels(0)  # raises when there is no usable device
    yield k
    k.close()


@pytest.fixture()
def executor(mpc, kernels):
    ex = mpc.CudaExecutor(kernels)
    yield ex
    ex.close()
