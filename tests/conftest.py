"""Shared fixtures.  GPU tests carry @pytest.mark.gpu; everything else runs
on a CPU-only machine."""
from __future__ import annotations

import importlib.util
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
PKG_DIR = ROOT / "mini-llama_b200"
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def load_package():
    """Import mini-llama_b200/ (hyphenated directory) as `mini_llama_b200`."""
    if "mini_llama_b200" in sys.modules:
        return sys.modules["mini_llama_b200"]
    spec = importlib.util.spec_from_file_location(
        "mini_llama_b200", PKG_DIR / "__init__.py", submodule_search_locations=[str(PKG_DIR)])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["mini_llama_b200"] = mod
    spec.loader.exec_module(mod)
    return mod


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200); run with -m gpu")


@pytest.fixture(scope="session")
def pkg():
    return load_package()


@pytest.fixture(scope="session")
def oracle():
    from oracle.oracle import Oracle
    return Oracle()


@pytest.fixture(scope="session")
def reference():
    from oracle.oracle import Reference
    if not Reference.available("scalar"):
        pytest.skip("reference checker oracle/_ref not built here")
    return Reference("scalar")


def rel_l2_rows(y: np.ndarray, ref: np.ndarray) -> np.ndarray:
    """Relative L2 error of each output vector (row of y), the tolerance
    metric of the contract: ||y - ref|| / ||ref|| per row."""
    y2 = np.atleast_2d(np.asarray(y, dtype=np.float64))
    r2 = np.atleast_2d(np.asarray(ref, dtype=np.float64))
    num = np.linalg.norm(y2 - r2, axis=1)
    den = np.linalg.norm(r2, axis=1)
    return num / np.maximum(den, 1e-30)
