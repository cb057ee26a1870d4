"""Shared fixtures. `gpu` tests need a CUDA device and run the CUDA path through the C ABI;
everything else runs on CPU (oracle pinning, host logic, library exports)."""
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "oracle"))

import __graft_entry__  # noqa: E402

PKG = __graft_entry__.load_package()
from xqwen35_b200.packer import synthetic  # noqa: E402
import oracle as ORACLE  # noqa: E402

GOLDEN = os.path.join(ROOT, "tests", "golden")
PKG_CACHE = os.environ.get("XQ_TEST_PACKAGES", os.path.join(os.environ.get("TMPDIR", "/tmp"), "xq_test_packages"))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and the built libxqwen35.so")


def cuda_available() -> bool:
    try:
        import torch

        return torch.cuda.is_available()
    except Exception:
        return False


def pytest_collection_modifyitems(config, items):
    if cuda_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for it in items:
        if "gpu" in it.keywords:
            it.add_marker(skip)


def package(name: str, seed: int = 0, quant: str = "sym") -> str:
    d = os.path.join(PKG_CACHE, f"{name}_s{seed}_{quant}")
    synthetic.make_package(d, synthetic.preset(name), seed=seed, quant=quant)
    return d


@pytest.fixture(scope="session")
def pkg():
    return PKG


@pytest.fixture(scope="session")
def oracle():
    if not os.path.exists(ORACLE.PORT_LIB):
        ORACLE.build()
    return ORACLE


@pytest.fixture(scope="session")
def small_pkg():
    return package("small", seed=7)


def rel_err(a, b) -> float:
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.abs(a - b).max() / max(1e-30, np.abs(b).max()))
