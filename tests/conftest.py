import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (ROOT, os.path.join(ROOT, "oracle")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


def has_gpu() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.fixture(scope="session")
def ref_oracle():
    import oracle
    if not oracle.ref_available():
        pytest.skip("oracle/_ref not built (reference tree absent when it was built)")
    return oracle.RefOracle()


@pytest.fixture(scope="session")
def port_oracle():
    import oracle
    return oracle.PortOracle()


@pytest.fixture(scope="session")
def cuda_lib():
    """The CUDA library, loaded on a GPU session; GPU tests fail (not skip) without it."""
    from spinn_b200 import lib, runtime
    L = lib.lib()
    runtime.init(0)
    return L


def rel_l2(a, b) -> float:
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    d = np.linalg.norm(b)
    return float(np.linalg.norm(a - b) / (d if d > 0 else 1.0))
