import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200); runs through libsmallmind_cuda.so")


@pytest.fixture(scope="session")
def O():
    from oracle import oracle
    oracle.lib()
    return oracle


@pytest.fixture(scope="session")
def ctx():
    import smallmind_b200 as sm
    c = sm.CudaContext(0)
    yield c
    c.close()


def rel_err(y, ref):
    """max |y - ref| / max(max|ref|, rms(ref)) — the GEMV/GEMM tolerance measure."""
    import numpy as np
    y = np.asarray(y, np.float64)
    ref = np.asarray(ref, np.float64)
    scale = max(np.abs(ref).max(), np.sqrt(np.mean(ref * ref)), 1e-30)
    return float(np.abs(y - ref).max() / scale)


def cosine(a, b):
    import numpy as np
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    return float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b)))
