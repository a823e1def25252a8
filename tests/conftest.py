"""Shared fixtures.

* ``pkg``      — the product package (directory miraclereasoning-cpu_b200/).
* ``backend``  — a CUDABackend on cuda:0 (GPU tests only; they are marked
  ``gpu`` and fail loudly, never fall back, if the library or device is missing).

The CPU oracle (oracle/) is imported directly by the tests that check against it.
"""
import importlib
import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parents[1]
for path in (REPO, REPO / "tests", REPO / "tests" / "golden"):
    if str(path) not in sys.path:
        sys.path.insert(0, str(path))

PACKAGE = "miraclereasoning-cpu_b200"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (B200) device and the built libmiracle_cuda.so")


def load_package():
    return importlib.import_module(PACKAGE)


def submodule(name):
    return importlib.import_module(f"{PACKAGE}.{name}")


@pytest.fixture(scope="session")
def pkg():
    return load_package()


@pytest.fixture(scope="session")
def backend(pkg):
    return submodule("backend").CUDABackend()
