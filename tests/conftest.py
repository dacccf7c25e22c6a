"""Shared test setup: import paths and the ``gpu`` marker.

``-m "not gpu"`` tests run anywhere (oracle vs golden vectors, host logic, the C ABI
loads and exports its symbols). ``-m gpu`` tests need a CUDA device and call the
kernels through libb200.so.
"""

import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "ml-switcheroo-compiler_b200")
for p in (ROOT, PKG):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and libb200.so")


def load_golden(case: str):
    d = np.load(os.path.join(GOLDEN, case + ".npz"))
    ins = {k[4:]: d[k] for k in d.files if k.startswith("in__")}
    outs = {k[5:]: d[k] for k in d.files if k.startswith("out__")}
    return ins, outs


@pytest.fixture(scope="session")
def cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("CUDA device required for -m gpu tests (no CPU fallback exists)")
    import b200._lib as L
    from b200.build import build

    build()
    L.load()
    return torch.device("cuda", 0)
