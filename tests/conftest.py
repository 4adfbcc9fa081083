import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for sub in ("qwen3-iree_b200", "oracle"):
    p = os.path.join(ROOT, sub)
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (sm_100) device; runs on the B200 box")


@pytest.fixture(scope="session")
def O():
    import oracle

    oracle.lib()
    return oracle


@pytest.fixture(scope="session")
def q3():
    import q3b200

    q3b200.lib()
    return q3b200


@pytest.fixture(scope="session")
def gpu(q3):
    n = q3.device_count()
    assert n > 0, "GPU tests need a CUDA device"
    q3.set_device(0)
    return q3


@pytest.fixture(scope="session")
def model_weights(q3):
    from q3b200.weights import synthetic_weights

    return synthetic_weights(seed=0)


def bits(a):
    return np.ascontiguousarray(a).view(np.uint16)


def rel_l2(a, b):
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))
