"""Shared test setup.

* `gpu` marker: tests that need a B200 (run with -m gpu on a GPU box).
* The package directory name contains dashes, so it is loaded by path and
  registered as the module `hf_llm_b200`.
* `oracle` is the CPU oracle (oracle/), built on first use.
"""
from __future__ import annotations

import importlib.util
import sys
from pathlib import Path

import numpy as np
import pytest

REPO = Path(__file__).resolve().parent.parent
PKG_DIR = REPO / "huggingface-local-llm-ui_b200"


def load_pkg():
    name = "hf_llm_b200"
    if name in sys.modules:
        return sys.modules[name]
    spec = importlib.util.spec_from_file_location(name, PKG_DIR / "__init__.py",
                                                  submodule_search_locations=[str(PKG_DIR)])
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def load_oracle():
    if str(REPO / "oracle") not in sys.path:
        sys.path.insert(0, str(REPO / "oracle"))
    import oracle as orc  # noqa: E402
    orc.build()
    return orc


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (sm_100a) device")


@pytest.fixture(scope="session")
def pkg():
    return load_pkg()


@pytest.fixture(scope="session")
def orc():
    return load_oracle()


@pytest.fixture(scope="session")
def engine(pkg):
    """CudaEngine on device 0.  On a GPU run the library must load: a
    missing or unbuildable libb2q fails the test, it never falls back."""
    from hf_llm_b200 import build
    build.build()
    from hf_llm_b200.engine import CudaEngine
    return CudaEngine.global_(0)


def rel_l2(a, b) -> float:
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    den = np.linalg.norm(b)
    return float(np.linalg.norm(a - b) / (den if den > 0 else 1.0))
