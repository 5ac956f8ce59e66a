"""Shared test set-up.

* `gpu` marker: tests that need a CUDA device (run with `-m gpu` on a B200).
* Paths: the repo root (for the `oracle` checker package) and the library's
  Python front end (`hrm-text-cuda_b200/hrm_layer_ops`).
* The product library and the oracle are (re)built before the tests run: make
  is incremental, so a source edited since the last build is never tested
  through a stale library.
"""

import os
import subprocess
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "hrm-text-cuda_b200")
for p in (ROOT, PKG):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (sm_100a B200)")


def _ensure_built():
    subprocess.run(["make", "-C", PKG, "-s", "-j8"], check=True)
    subprocess.run(["make", "-C", os.path.join(ROOT, "oracle"), "-s", "liboracle.so"], check=True)


_ensure_built()


@pytest.fixture(scope="session")
def oracle():
    from oracle import Oracle

    return Oracle()


@pytest.fixture(scope="session")
def rng():
    return np.random.default_rng(0)


@pytest.fixture(scope="session")
def cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("a gpu-marked test ran without a CUDA device")
    return torch.device("cuda", 0)
