"""Shared fixtures.  `-m "not gpu"` runs on any host; `-m gpu` needs a B200."""
from __future__ import annotations

import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (run on the B200 box)")
    config.addinivalue_line("markers", "slow: full-size model cases")


@pytest.fixture(scope="session")
def gpt2b():
    """The product package with its library built (incremental)."""
    from cuda_gpt2_inference_b200 import build
    build.build()
    import cuda_gpt2_inference_b200 as pkg
    pkg.lib()
    return pkg


@pytest.fixture(scope="session")
def orc():
    import oracle
    oracle.orc()
    return oracle


@pytest.fixture(scope="session")
def golden():
    return np.load(os.path.join(GOLDEN, "ref_cpu_loops.npz"))


@pytest.fixture(scope="session")
def cuda(gpt2b):
    import torch
    if not torch.cuda.is_available():
        pytest.fail("a gpu-marked test ran without a CUDA device")
    torch.cuda.set_device(0)
    return torch.device("cuda:0")


def rel_err(got, ref) -> float:
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    return float(np.abs(got - ref).max() / max(1e-30, np.abs(ref).max()))


def cosine(a, b) -> float:
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    return float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b) + 1e-300))
