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


TIE_RTOL = 1e-4  # a threshold decision counts as a near-tie when the quantity is this close (relative)


def tie_distance(rec, n, t_thresh, w_thresh):
    """How close one ray's compositing came to a threshold decision, from its records rec (S, 8) (t, site,
    sigma, ...) of n samples, composited in float64 as the renderer does (foam.cu:370-389): the smallest
    relative distance, over its segments, of the segment weight w = T alpha to w_thresh (which decides
    whether the segment is coloured) and of the transmittance after the segment to t_thresh (which ends
    the ray)."""
    t = np.asarray(rec[:n, 0], np.float64)
    sig = np.asarray(rec[:n, 2], np.float64)
    if n < 2:
        return np.inf
    alpha = 1.0 - np.exp(-0.5 * (sig[:-1] + sig[1:]) * (t[1:] - t[:-1]))
    T_after = np.cumprod(1.0 - alpha)
    T_before = np.concatenate([[1.0], T_after[:-1]])
    w = T_before * alpha
    dist = np.inf
    if w_thresh > 0:
        dist = min(dist, float(np.min(np.abs(w - w_thresh))) / w_thresh)
    if t_thresh > 0:
        dist = min(dist, float(np.min(np.abs(T_after - t_thresh))) / t_thresh)
    return dist


def audit_stats(stats, ref_stats, ref_rec, t_thresh, w_thresh, rtol=TIE_RTOL):
    """Rays whose per-ray stats differ between two renderers must be documented near-ties: a segment
    weight within rtol of w_thresh or a transmittance within rtol of t_thresh (from the second renderer's
    records, which must hold the whole ray). -> boolean mask of the rays whose stats agree; raises with the
    unexplained rays otherwise."""
    stats, ref_stats = np.asarray(stats), np.asarray(ref_stats)
    same = (stats == ref_stats).all(1)
    bad = []
    K = ref_rec.shape[1]
    for r in np.flatnonzero(~same):
        n = int(ref_stats[r, 0])
        if n > K:
            bad.append((int(r), 'records do not hold the ray'))
            continue
        dist = tie_distance(ref_rec[r], n, t_thresh, w_thresh)
        if not dist <= rtol:
            bad.append((int(r), f'closest threshold distance {dist:.2e}'))
    assert not bad, f'stats differ on rays that are not near-ties: {bad[:8]}'
    return same
