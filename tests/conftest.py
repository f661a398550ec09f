import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (runs on the B200 box)")
    config.addinivalue_line("markers", "slow: larger cases")


def cuda_available() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


def pytest_collection_modifyitems(config, items):
    if cuda_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


def mixture(n, d, n_centres, sigma, nq, qsigma=0.05, seed=0, normalize=True):
    """Seeded Gaussian-mixture rows and perturbed-row queries (benchmark config shapes)."""
    rng = np.random.default_rng(seed)
    cent = rng.standard_normal((n_centres, d)).astype(np.float32)
    X = cent[rng.integers(0, n_centres, n)] + np.float32(sigma) * rng.standard_normal((n, d)).astype(np.float32)
    if normalize:
        X /= np.linalg.norm(X, axis=1, keepdims=True)
    src = rng.integers(0, n, nq)
    Q = X[src] + np.float32(qsigma) * rng.standard_normal((nq, d)).astype(np.float32)
    if normalize:
        Q /= np.linalg.norm(Q, axis=1, keepdims=True)
    return np.ascontiguousarray(X, np.float32), np.ascontiguousarray(Q, np.float32)


@pytest.fixture(scope="session")
def oracle():
    from oracle import oracle as O
    O.lib()
    return O
