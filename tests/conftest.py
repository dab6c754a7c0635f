"""Shared fixtures.  `gpu`-marked tests need a B200; everything else runs on
the CPU (the driver runs `pytest -m "not gpu"` without a GPU)."""
import importlib
import os
import shutil
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (sm_100a)")
    config.addinivalue_line("markers", "slow: long-running CPU test")


def _ensure_oracle():
    lib = os.path.join(ROOT, "oracle", "liboracle.so")
    if not os.path.exists(lib):
        subprocess.run(["make", "-s", "-C", os.path.join(ROOT, "oracle"), "liboracle.so"], check=True)


def _ensure_library():
    """Builds libsplsage.so (nvcc cross-compiles for sm_100a without a GPU)
    when a fresh checkout has none; the ABI tests inspect the built file."""
    lib = os.path.join(ROOT, "sota-papers-lab_b200", "libsplsage.so")
    if not os.path.exists(lib) and shutil.which("nvcc"):
        subprocess.run(["make", "-s", "-C", os.path.join(ROOT, "sota-papers-lab_b200", "csrc")], check=True)


_ensure_oracle()
_ensure_library()


@pytest.fixture(scope="session")
def oracle():
    from oracle import oracle as o
    return o


@pytest.fixture(scope="session")
def sage():
    """The product's Python mirror of the spl_nn::sage API (over libsplsage.so)."""
    return importlib.import_module("sota-papers-lab_b200")
