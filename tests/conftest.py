"""Shared pytest setup: import paths, the gpu marker, common fixtures."""
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for sub in ("oracle", "qwen-mobile-agent_b200", "tests"):
    p = os.path.join(ROOT, sub)
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def oracle():
    import oracle as O
    O.lib()
    return O


@pytest.fixture(scope="session")
def ref_lib(oracle):
    if not oracle.ref_available():
        pytest.skip("reference oracle (oracle/_ref) not built")
    R = oracle.ref()
    R.qr_init(1)
    return R


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import qma_cuda as Q
    Q.init(0)
    return Q


@pytest.fixture
def rng():
    return np.random.default_rng(1234)
