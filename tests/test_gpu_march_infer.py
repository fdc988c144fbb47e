"""CUDA fixed-step marcher and inference renderer against the CPU oracle and the reference's golden
vectors (test_march.py / test_foam.py:120-132 settings)."""

import numpy as np
import pytest
import torch

from conftest import cuda, rel, small_inputs
from oracle import oracle

pytestmark = pytest.mark.gpu

IMG_TOL = 1e-4
GRAD_TOL = 1e-3


def _ext():
    from voronoi_gauss_b200 import ext
    return ext


def test_march_matches_oracle_and_reference(march_small):
    z = march_small
    ext = _ext()
    g = ext.Graph(cuda(z['points']), cuda(z['offsets']), cuda(z['adj']))
    x = small_inputs(z, ('raw', 'dA', 'cA', 'sh', 'o', 'd', 'start', 'near', 'mid', 'far'))
    params = [x[k].clone().requires_grad_() for k in ('raw', 'dA', 'cA', 'sh')]
    dt, n_bg = float(z['dt']), int(z['n_bg'])
    fg, T, depth, stats = ext.march(g, *params, 3, x['o'], x['d'], x['start'], x['near'], x['mid'], x['far'], dt,
                                    n_bg, t_thresh=0.0, w_thresh=-1.0)
    ((fg * cuda(z['g_rgb'])).sum() + (T * cuda(z['g_T'])).sum()).backward()
    args = (z['points'], z['offsets'], z['adj'], z['raw'], z['dA'], z['cA'], z['sh'], 3, z['o'], z['d'], z['start'],
            z['near'], z['mid'], z['far'], dt, n_bg, 0.0, -1.0)
    o_rgb, o_T, o_depth, o_stats = oracle.march_forward(*args)
    assert (stats.cpu().numpy() == o_stats).all()
    assert np.abs(fg.detach().cpu().numpy() - o_rgb).max() <= IMG_TOL
    assert np.abs(T.detach().cpu().numpy() - o_T).max() <= IMG_TOL
    assert np.abs(depth.cpu().numpy() - o_depth).max() <= IMG_TOL
    assert np.abs(fg.detach().cpu().numpy() - z['ref_fg']).max() <= IMG_TOL
    og = oracle.march_backward(*args, o_rgb, o_T, z['g_rgb'], z['g_T'])
    for name, p, want in zip(('raw', 'dA', 'cA', 'sh'), params, og):
        assert rel(p.grad.cpu().numpy(), want) <= GRAD_TOL, f'{name} vs oracle'
        assert rel(p.grad.cpu().numpy(), z[f'ref_g_{name}']) <= GRAD_TOL, f'{name} vs reference'


@pytest.mark.parametrize('t_thresh,w_thresh', [(1e-4, 1e-4), (1e-2, 1e-3)])
def test_march_thresholds_match_oracle(march_small, t_thresh, w_thresh):
    z = march_small
    ext = _ext()
    g = ext.Graph(cuda(z['points']), cuda(z['offsets']), cuda(z['adj']))
    x = small_inputs(z, ('raw', 'dA', 'cA', 'sh', 'o', 'd', 'start', 'near', 'mid', 'far'))
    dt, n_bg = 0.02, 4
    out = ext.march_extension().march_forward(g.points, g.offsets, g.adj, x['raw'], x['dA'], x['cA'], x['sh'], 3,
                                              x['o'], x['d'], x['start'], x['near'], x['mid'], x['far'], dt, n_bg,
                                              t_thresh, w_thresh)
    ref = oracle.march_forward(z['points'], z['offsets'], z['adj'], z['raw'], z['dA'], z['cA'], z['sh'], 3, z['o'],
                               z['d'], z['start'], z['near'], z['mid'], z['far'], dt, n_bg, t_thresh, w_thresh)
    assert (out[3].cpu().numpy() == ref[3]).all()
    for a, b in zip(out[:3], ref[:3]):
        assert np.abs(a.cpu().numpy() - b).max() <= IMG_TOL


PACKS = ['plain', 'morton', 'eps', 'eps_morton']


def _pack(z, tag):
    sh = z[f'pack_{tag}_sh']
    return dict(points=cuda(z[f'pack_{tag}_points']), offsets=cuda(z[f'pack_{tag}_offsets']),
                nbr=cuda(z[f'pack_{tag}_nbr']), edge=cuda(z[f'pack_{tag}_edge']), attr=cuda(z[f'pack_{tag}_attr']),
                sh=cuda(sh, torch.float16 if sh.dtype == np.float16 else torch.float32),
                orig=cuda(z[f'pack_{tag}_orig'], torch.int32))


@pytest.mark.parametrize('tag', PACKS)
@pytest.mark.parametrize('mode', [0, 1, 2])
@pytest.mark.parametrize('stage', [0, 1, 2])
@pytest.mark.parametrize('exact_stats', [True, False])
def test_foam_infer_matches_oracle(foam_small, tag, mode, stage, exact_stats):
    """Per ray (exact_stats: every stats column as the reference kernel counts it) and with deferred,
    cell-major colours (the default): stats columns 0-3 equal to the oracle's, column 4 the SH colours
    of the cell-major pass, and the image bit-identical to the per-ray kernel's."""
    z = foam_small
    ext = _ext()
    p = _pack(z, tag)
    rng = np.random.default_rng(4)
    attr = z[f'pack_{tag}_attr'].copy()
    attr[:, 16:19] = rng.uniform(0, 1, (len(attr), 3))  # baked colours
    p['attr'] = cuda(attr)
    start = z['start'] if tag in ('plain', 'eps') else np.argsort(z[f'pack_{tag}_orig'])[z['start']]
    start = start.astype(np.int32)
    cap_np = np.where(np.arange(len(start)) % 3 == 0, 5, 1 << 30).astype(np.int32)
    color_cut = 2 * np.log(1e3) if tag.startswith('eps') else float('inf')
    x = small_inputs(z, ('o', 'd', 'near', 'far'))
    args = (p['points'], p['offsets'], p['nbr'], p['edge'], p['attr'], p['sh'], 3, x['o'], x['d'], cuda(start),
            x['near'], x['far'], 0.0, -1.0, color_cut, mode, stage, cuda(cap_np), p['orig'])
    out = ext.foam_infer_extension().foam_infer(*args, exact_stats=exact_stats)
    ref = oracle.foam_infer(z[f'pack_{tag}_points'], z[f'pack_{tag}_offsets'], z[f'pack_{tag}_nbr'],
                            z[f'pack_{tag}_edge'], attr, z[f'pack_{tag}_sh'], 3, z['o'], z['d'], start, z['near'],
                            z['far'], 0.0, -1.0, color_cut, mode, stage, cap_np, z[f'pack_{tag}_orig'])
    cols = 5 if exact_stats or stage < 2 else 4
    assert (out[3].cpu().numpy()[:, :cols] == ref[3][:, :cols]).all()
    for a, b in zip(out[:3], ref[:3]):
        assert np.abs(a.cpu().numpy() - b).max() <= IMG_TOL
    if not exact_stats:
        per_ray = ext.foam_infer_extension().foam_infer(*args, exact_stats=True)
        for a, b in zip(out[:3], per_ray[:3]):
            assert torch.equal(a, b), 'deferred colours changed the image'


def test_foam_infer_exact_equals_training_kernel(foam_small):
    """foam_infer, exact options, Morton order: the training kernel's image (test_foam.py:120-132)."""
    z = foam_small
    ext = _ext()
    x = small_inputs(z)
    g = ext.Graph(cuda(z['points']), cuda(z['offsets']), cuda(z['adj']))
    with torch.no_grad():
        train = ext.foam(g, x['raw'], x['dA'], x['cA'], x['sh'], 3, x['o'], x['d'], x['start'], x['near'], x['far'],
                         t_thresh=0.0, w_thresh=-1.0)[0]
    for tag in ('plain', 'morton'):
        p = _pack(z, tag)
        start = z['start'] if tag == 'plain' else np.argsort(z[f'pack_{tag}_orig'])[z['start']]
        for mode in (0, 2):
            out = ext.foam_infer_extension().foam_infer(
                p['points'], p['offsets'], p['nbr'], p['edge'], p['attr'], p['sh'], 3, x['o'], x['d'],
                cuda(start.astype(np.int32)), x['near'], x['far'], 0.0, -1.0, float('inf'), mode, 2,
                torch.empty(0, dtype=torch.int32, device='cuda'), p['orig'])
            assert float((out[0] - train).abs().max()) <= IMG_TOL
