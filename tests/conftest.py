"""Shared fixtures.

`m3` is the product binding (m3.c_b200/m3cuda.py over libm3cuda.so);
`oracle` is the CPU checker module (oracle/oracle.py); `ref` is the
reference's own CPU provider (oracle/_ref/libm3ref.so) bound to the m3.h API.
GPU tests are marked `gpu` and call the product through its C ABI.
"""

from __future__ import annotations

import importlib.util
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PACKAGE_DIR = os.path.join(ROOT, "m3.c_b200")
ORACLE_DIR = os.path.join(ROOT, "oracle")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200)")


def _load(name: str, path: str):
    if name in sys.modules:
        return sys.modules[name]
    spec = importlib.util.spec_from_file_location(name, path)
    module = importlib.util.module_from_spec(spec)
    sys.modules[name] = module
    spec.loader.exec_module(module)
    return module


def load_m3():
    return _load("m3cuda", os.path.join(PACKAGE_DIR, "m3cuda.py"))


def load_oracle():
    return _load("m3_oracle_py", os.path.join(ORACLE_DIR, "oracle.py"))


@pytest.fixture(scope="session")
def m3():
    module = load_m3()
    module.load()
    return module


@pytest.fixture(scope="session")
def oracle():
    module = load_oracle()
    module.restatement()
    return module


@pytest.fixture(scope="session")
def ref(m3, oracle):
    if not oracle.reference_available():
        pytest.skip("reference CPU library was not built")
    return m3.bind(oracle.reference(), cuda=False)


@pytest.fixture(scope="session")
def gpu(m3):
    if m3.load().m3_cuda_device_count() == 0:
        pytest.fail("a gpu-marked test needs a CUDA device")
    return True
