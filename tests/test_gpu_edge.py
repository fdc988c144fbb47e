"""Edge cases of the CUDA path: empty batches, rays missing the sites' hull, long walks, errors raised
with the reference's messages, and the loop-cap status word."""

import numpy as np
import pytest
import torch

from conftest import bits, cuda, rel, small_inputs
from oracle import oracle

pytestmark = pytest.mark.gpu


def _ext():
    from voronoi_gauss_b200 import ext
    return ext


def _graph(z):
    ext = _ext()
    return ext.Graph(cuda(z['points']), cuda(z['offsets']), cuda(z['adj']))


def test_empty_batch(foam_small):
    z = foam_small
    ext = _ext()
    g, x = _graph(z), small_inputs(z)
    e = {k: x[k][:0] for k in ('o', 'd', 'start', 'near', 'far')}
    fx = ext.foam_extension()
    rgb, T, depth, stats, rec = fx.foam_forward(g.points, g.offsets, g.adj, x['raw'], x['dA'], x['cA'], x['sh'], 3,
                                                e['o'], e['d'], e['start'], e['near'], e['far'], 1e-4, 1e-4, 256)
    assert rgb.shape == (0, 3) and stats.shape == (0, 3) and rec.shape == (0, 256, 8)
    grads = fx.foam_backward(g.points, g.offsets, g.adj, x['raw'], x['dA'], x['cA'], x['sh'], 3, e['o'], e['d'],
                             e['start'], e['near'], e['far'], 1e-4, 1e-4, rgb, T, rgb, T, rec, stats)
    for gr, p in zip(grads, (x['raw'], x['dA'], x['cA'], x['sh'])):
        assert gr.shape == p.shape and float(gr.abs().max()) == 0.0
    mx = ext.march_extension()
    out = mx.march_forward(g.points, g.offsets, g.adj, x['raw'], x['dA'], x['cA'], x['sh'], 3, e['o'], e['d'],
                           e['start'], e['near'], e['near'], e['far'], 0.05, 4, 1e-4, 1e-4)
    assert out[0].shape == (0, 3)
    grads = mx.march_backward(g.points, g.offsets, g.adj, x['raw'], x['dA'], x['cA'], x['sh'], 3, e['o'], e['d'],
                              e['start'], e['near'], e['near'], e['far'], 0.05, 4, 1e-4, 1e-4, out[0], out[1], out[0],
                              out[1])
    assert float(grads[0].abs().max()) == 0.0


def _odd_rays(z):
    """Rays from outside the hull pointing away from it, and rays starting from a far-away site."""
    rng = np.random.default_rng(9)
    B = 48
    o = rng.uniform(-3, 3, (B, 3)).astype(np.float32)
    o[:16] = np.array([4.0, 0.5, -0.3], np.float32) + rng.uniform(-0.2, 0.2, (16, 3)).astype(np.float32)
    d = rng.normal(size=(B, 3)).astype(np.float32)
    d[:16] = np.array([1.0, 0.1, 0.0], np.float32)  # away from the sites
    d /= np.linalg.norm(d, axis=1, keepdims=True)
    near = np.full(B, 0.02, np.float32)
    far = np.full(B, 6.0, np.float32)
    start = rng.integers(0, len(z['points']), B).astype(np.int32)  # arbitrary, often far: long walks
    return o, d, start, near, far


def test_rays_missing_hull_and_long_walks(foam_small):
    z = foam_small
    ext = _ext()
    g, x = _graph(z), small_inputs(z)
    o, d, start, near, far = _odd_rays(z)
    params = [x[k].clone().requires_grad_() for k in ('raw', 'dA', 'cA', 'sh')]
    fg, T, depth, stats = ext.foam(g, *params, 3, cuda(o), cuda(d), cuda(start), cuda(near), cuda(far),
                                   t_thresh=1e-4, w_thresh=1e-4, record_cap=32)
    g_rgb = np.ones((len(o), 3), np.float32)
    g_T = np.ones(len(o), np.float32)
    (fg.sum() + T.sum()).backward()
    args = (z['points'], z['offsets'], z['adj'], z['raw'], z['dA'], z['cA'], z['sh'], 3, o, d, start, near, far, 1e-4,
            1e-4)
    r = oracle.foam_forward(*args, 32)
    assert (stats.cpu().numpy() == r[3]).all()
    assert (stats.cpu().numpy()[:, 0] >= 2).all()
    assert np.abs(fg.detach().cpu().numpy() - r[0]).max() <= 1e-4
    og = oracle.foam_backward(*args, r[0], r[1], g_rgb, g_T, r[4], r[3])
    for p, want in zip(params, og):
        assert rel(p.grad.cpu().numpy(), want) <= 1e-3


def test_records_are_reference_format(foam_small):
    """rec (B, K, 8) = (t, site bits, sigma, C rgb, m_min, 1 / sum of weights): sites are original ids,
    t is non-decreasing, the first site is the walk's result and consecutive sites are neighbours."""
    z = foam_small
    ext = _ext()
    g, x = _graph(z), small_inputs(z)
    rgb, T, depth, stats, rec = ext.foam_extension().foam_forward(
        g.points, g.offsets, g.adj, x['raw'], x['dA'], x['cA'], x['sh'], 3, x['o'], x['d'], x['start'], x['near'],
        x['far'], 1e-4, 1e-4, 256)
    stats, rec = stats.cpu().numpy(), rec.cpu().numpy()
    off, adj = z['offsets'], z['adj']
    for r in range(len(stats)):
        s = stats[r, 0]
        cells = bits(rec[r, :s, 1])
        assert (np.diff(rec[r, :s, 0]) >= 0).all()
        for a, b in zip(cells[:-1], cells[1:]):
            assert a == b or b in adj[off[a]:off[a + 1]]
        # 1 / sum of colour weights: 0 for samples whose colour was never needed (foam.cu:285), as in the
        # reference; every endpoint of a coloured segment has one
        coloured = rec[r, :s, 7] > 0
        assert (rec[r, :s, 7] >= 0).all()
        if stats[r, 1] > 0:
            assert coloured.sum() >= stats[r, 1] + 1 or coloured.sum() == s


def test_bad_arguments_raise_reference_errors(foam_small):
    z = foam_small
    ext = _ext()
    g, x = _graph(z), small_inputs(z)
    fx = ext.foam_extension()
    base = [g.points, g.offsets, g.adj, x['raw'], x['dA'], x['cA'], x['sh'], 3, x['o'], x['d'], x['start'], x['near'],
            x['far'], 1e-4, 1e-4, 0]
    cases = [(3, x['raw'].double(), 'raw has the wrong dtype'), (3, x['raw'].cpu(), 'raw must be a CUDA tensor'),
             (4, x['dA'].t().contiguous().t(), 'dA must be contiguous'), (6, x['sh'][:, :9].contiguous(),
                                                                          'sh must be (N, 16, 3)'),
             (10, x['start'].float(), 'start has the wrong dtype'), (7, 4, 'sh_deg must be in 0..3')]
    for i, val, msg in cases:
        args = list(base)
        args[i] = val
        with pytest.raises(RuntimeError, match=msg.replace('(', r'\(').replace(')', r'\)')):
            fx.foam_forward(*args)
    with pytest.raises(RuntimeError, match='record_cap'):
        fx.foam_forward(*base[:-1], -1)


def test_status_word_clear_after_normal_renders(foam_small):
    from voronoi_gauss_b200 import _lib
    import ctypes
    z = foam_small
    ext = _ext()
    _lib.call('vg_status_reset')
    g, x = _graph(z), small_inputs(z)
    ext.foam(g, x['raw'], x['dA'], x['cA'], x['sh'], 3, x['o'], x['d'], x['start'], x['near'], x['far'])
    bits_ = ctypes.c_int(-1)
    _lib.call('vg_status', ctypes.addressof(bits_))
    assert bits_.value == 0


def test_forward_is_deterministic(foam_small):
    z = foam_small
    ext = _ext()
    g, x = _graph(z), small_inputs(z)
    a = ext.foam_extension().foam_forward(g.points, g.offsets, g.adj, x['raw'], x['dA'], x['cA'], x['sh'], 3, x['o'],
                                          x['d'], x['start'], x['near'], x['far'], 1e-4, 1e-4, 64)
    b = ext.foam_extension().foam_forward(g.points, g.offsets, g.adj, x['raw'], x['dA'], x['cA'], x['sh'], 3, x['o'],
                                          x['d'], x['start'], x['near'], x['far'], 1e-4, 1e-4, 64)
    for u, v in zip(a[:4], b[:4]):
        assert torch.equal(u, v)
    s = a[3][:, 0].clamp(max=64)
    valid = torch.arange(64, device=s.device)[None, :] < s[:, None]
    assert torch.equal(a[4][valid], b[4][valid])  # records beyond a ray's samples are unspecified
