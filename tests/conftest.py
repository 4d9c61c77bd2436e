"""Shared pytest setup: the `gpu` marker, import paths, and fixtures.

GPU tests (marked `gpu`) run on a B200 through the C ABI of libvrs; the
rest run anywhere and cover the oracle, the golden fixtures, the host logic
and the library's exported symbols.
"""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (os.path.join(ROOT, "vector-rs_b200", "python"), os.path.join(ROOT, "oracle"), ROOT):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200) and libvrs")


@pytest.fixture(scope="session")
def orc():
    import oracle
    oracle.build()
    return oracle


def _build_lib():
    import importlib.util
    spec = importlib.util.spec_from_file_location(
        "vrs_build", os.path.join(ROOT, "vector-rs_b200", "build.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod.build()


@pytest.fixture(scope="session")
def vc():
    import vector_cuda
    if not os.path.exists(vector_cuda.LIB_PATH):
        _build_lib()
    vector_cuda.lib()
    return vector_cuda


@pytest.fixture(scope="session")
def gpu(vc):
    n = vc.CudaDeviceContext.device_count()
    if n < 1:
        pytest.fail("GPU test requested but no CUDA device is visible")
    return n
