"""Shared pytest setup.

Markers:
  gpu  -- needs a CUDA device (run with `-m gpu` on a B200 box).  Everything
          else runs on the CPU: the oracle pins, host-side logic, and the
          C-ABI load/export checks.
"""
from __future__ import annotations

import os
import subprocess
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: test needs a CUDA device (B200)")


def _ensure_oracle():
    import oracle

    if not os.path.exists(oracle.LIB_PATH):
        subprocess.run(["make", "-s", "-C", os.path.join(ROOT, "oracle")], check=True)
    return oracle


@pytest.fixture(scope="session")
def O():
    """The CPU oracle (oracle/liboracle.so)."""
    return _ensure_oracle()


@pytest.fixture(scope="session")
def golden():
    return dict(np.load(os.path.join(ROOT, "tests", "golden", "reference_vectors.npz")))


@pytest.fixture(scope="session")
def K():
    """The product library (kunlunk200_lib_b200), loaded from its in-tree build."""
    import kunlunk200_lib_b200 as lib

    if not os.path.exists(lib.LIB_PATH):
        from kunlunk200_lib_b200 import build

        build.build()
    lib.lib()
    return lib


@pytest.fixture(scope="session")
def gpu(K):
    """Skip-free GPU gate: a `-m gpu` run on a machine without a device fails loudly."""
    n = K.device_count()
    assert n > 0, "no CUDA device visible to libkunlunk200"
    K.select(0)
    return 0
