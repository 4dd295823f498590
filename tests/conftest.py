"""Shared fixtures. `-m gpu` tests need a CUDA GPU and call the library through its C ABI; everything else runs on
the CPU (the oracle against the reference and gguf-py, the tables, the host logic, the ABI's exports)."""
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "trench-gguf_b200")
ORACLE = os.path.join(ROOT, "oracle")
for p in (PKG, ORACLE):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (runs the sm_100a library through its C ABI)")


@pytest.fixture(scope="session")
def tables():
    path = os.path.join(PKG, "gpuq_tables.bin")
    if not os.path.exists(path):
        subprocess.check_call([sys.executable, os.path.join(PKG, "gen_tables.py"), path])
    return path


@pytest.fixture(scope="session")
def oracle(tables):
    import oracle as orc
    if not orc.available("oracle"):
        subprocess.check_call(["make", "-s", "-C", ORACLE, "oracle"])
    return orc.Checker("oracle", tables)


@pytest.fixture(scope="session")
def reference(tables):
    import oracle as orc
    if not orc.available("reference"):
        pytest.skip("reference host build absent (oracle/_ref: built where the reference sources are)")
    return orc.Checker("reference", tables)


@pytest.fixture(scope="session")
def gpuq(tables):
    import gpuq as g
    return g.Gpuq(device=int(os.environ.get("GPUQ_DEVICE", "0")), tables=tables)


@pytest.fixture(scope="session")
def selftest_inputs():
    import workloads
    return workloads.selftest(rows=64, cols=2304)
