"""Pins the CPU oracle's NeRF-sampler field functions (vgf.cu:51-335 restated in oracle/vg_oracle.c)
against tests/golden/field_small.npz, made by the reference's own float64 code (test_grad.py): the
greedy walk must reach the exact nearest site of every sample (barring distance ties), and the
density / colour values and gradients must match the float64 autograd reference."""

import numpy as np
import pytest

from conftest import golden, rel
from oracle import oracle

VAL_TOL = 1e-5   # relative error (norm over all samples) of fp32 field values vs float64
GRAD_TOL = 1e-3  # relative error of gradients (norm over all sites)


@pytest.fixture(scope='module')
def fz():
    return golden('field_small.npz')


def _graph(z):
    return z['points'], z['offsets'], z['adj']


def test_walk_reaches_exact_nearest_sites(fz):
    z = fz
    site, steps = oracle.walk(*_graph(z), z['o'], z['d'], z['z'], z['start'])
    got = site.reshape(-1)
    nn, dist = z['nn_site'][:, 0], z['nn_dist']
    tie = np.abs(dist[:, 1] - dist[:, 0]) <= 1e-6 * np.maximum(dist[:, 0], 1e-12)
    assert (got[~tie] == nn[~tie]).all()
    assert steps.sum() > 0 and (steps >= 0).all()


def test_walk_empty_and_single_sample(fz):
    z = fz
    site, steps = oracle.walk(*_graph(z), z['o'][:3], z['d'][:3], np.zeros((3, 0), np.float32), z['start'][:3])
    assert site.shape == (3, 0) and (steps == 0).all()
    site, _ = oracle.walk(*_graph(z), z['o'][:5], z['d'][:5], z['z'][:5, :1], z['start'][:5])
    assert (site[:, 0] == oracle.walk(*_graph(z), z['o'][:5], z['d'][:5], z['z'][:5], z['start'][:5])[0][:, 0]).all()


def test_density_and_color_values(fz):
    z = fz
    sigma = oracle.density_forward(*_graph(z), z['raw'], z['ls'], z['quat'], z['x'], z['site'])
    assert rel(sigma, z['ref_sigma']) < VAL_TOL
    rgb = oracle.color_forward(*_graph(z), z['cls'], z['cquat'], z['sh'], 3, z['x'], z['dirs'], z['site'])
    assert rel(rgb, z['ref_rgb']) < VAL_TOL


def test_density_scale_mult_widens_the_gaussians(fz):
    z = fz
    s1 = oracle.density_forward(*_graph(z), z['raw'], z['ls'], z['quat'], z['x'], z['site'])
    s2 = oracle.density_forward(*_graph(z), z['raw'], z['ls'] + np.log(2.0), z['quat'], z['x'], z['site'])
    s3 = oracle.density_forward(*_graph(z), z['raw'], z['ls'], z['quat'], z['x'], z['site'], scale_mult=2.0)
    assert rel(s3, s2) < 1e-5 and rel(s3, s1) > 1e-2


def test_field_gradients(fz):
    z = fz
    g_raw, g_ls, g_q = oracle.density_backward(*_graph(z), z['raw'], z['ls'], z['quat'], z['x'], z['site'],
                                               z['g_sigma'])
    assert rel(g_raw, z['ref_g_raw']) < GRAD_TOL
    assert rel(g_ls, z['ref_g_ls']) < GRAD_TOL
    assert rel(g_q, z['ref_g_quat']) < GRAD_TOL
    rgb = oracle.color_forward(*_graph(z), z['cls'], z['cquat'], z['sh'], 3, z['x'], z['dirs'], z['site'])
    g_cls, g_cq, g_sh = oracle.color_backward(*_graph(z), z['cls'], z['cquat'], z['sh'], 3, z['x'], z['dirs'],
                                              z['site'], rgb, z['g_rgb'])
    assert rel(g_cls, z['ref_g_cls']) < GRAD_TOL
    assert rel(g_cq, z['ref_g_cquat']) < GRAD_TOL
    assert rel(g_sh, z['ref_g_sh']) < GRAD_TOL
