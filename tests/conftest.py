import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(ROOT, 'tests', 'golden')
sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line('markers', 'gpu: needs a CUDA device (B200, sm_100a)')


def golden(name):
    return np.load(os.path.join(GOLDEN, name))


def rel(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


@pytest.fixture(scope='session')
def foam_small():
    return golden('foam_small.npz')


@pytest.fixture(scope='session')
def march_small():
    return golden('march_small.npz')


def cuda(x, dtype=None):
    import torch
    t = torch.as_tensor(np.ascontiguousarray(x))
    if dtype is not None:
        t = t.to(dtype)
    return t.cuda().contiguous()


def bits(x):
    """float32 array -> int32 view (bitwise comparisons)."""
    return np.ascontiguousarray(np.asarray(x, dtype=np.float32)).view(np.int32)


def split(flat, off):
    return [flat[off[i]:off[i + 1]] for i in range(len(off) - 1)]


def small_inputs(z, keys=('raw', 'dA', 'cA', 'sh', 'o', 'd', 'start', 'near', 'far')):
    """Golden fixture arrays as CUDA tensors (int32 for start, float32 otherwise)."""
    import torch
    out = {}
    for k in keys:
        out[k] = cuda(z[k], torch.int32 if k == 'start' else torch.float32)
    return out
