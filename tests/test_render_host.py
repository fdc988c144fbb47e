"""The proposal sampler's host arithmetic (render.py:16-74) against the reference's own functions.

`tests/golden/render_host.npz` holds the reference's render.ray_bounds / s_to_t / composite /
sample_pdf / resample outputs on 256 seeded rays (made by make_golden.py). These are plain float32
torch functions on both sides, run here on the CPU, so every output must be bit-identical.
"""

import os

import numpy as np
import torch

from voronoi_gauss_b200 import render

GOLD = np.load(os.path.join(os.path.dirname(__file__), 'golden', 'render_host.npz'))


def t(name):
    return torch.from_numpy(GOLD[name])


def test_ray_bounds():
    near, mid, far = render.ray_bounds(t('o'), t('d'), 0.02, 4.0)
    assert torch.equal(near, t('near')) and torch.equal(mid, t('mid')) and torch.equal(far, t('far'))
    assert bool((far > mid).all()) and bool((mid > near).all())


def test_s_to_t_monotone_and_exact():
    tt = render.s_to_t(t('s'), t('near'), t('mid'), t('far'))
    assert torch.equal(tt, t('t'))
    assert bool((tt[:, 1:] >= tt[:, :-1]).all())
    # s = 0, 1/2, 1 land on near, mid, far
    ends = render.s_to_t(torch.tensor([[0.0, 0.5, 1.0]]).expand(len(tt), 3), t('near'), t('mid'), t('far'))
    assert torch.allclose(ends[:, 0], t('near')) and torch.allclose(ends[:, 1], t('mid'))
    assert torch.allclose(ends[:, 2], t('far'), rtol=1e-5)


def test_composite():
    w, T = render.composite(t('sigma'), t('t'), t('far'))
    assert torch.equal(w, t('w')) and torch.equal(T, t('T'))
    # weights and the final transmittance partition the ray (up to the 1e-10 guard)
    assert torch.allclose(w.sum(1) + T, torch.ones_like(T), atol=1e-5)


def test_sample_pdf_and_resample():
    S = t('bins').shape[1] - 1
    x = render.sample_pdf(t('bins'), t('w')[:, :S], 48, det=True)
    assert torch.equal(x, t('pdf_det'))
    s_new = render.resample(t('s'), t('w'), 64, det=True)
    assert torch.equal(s_new, t('s_new'))
    assert bool((s_new >= 0).all()) and bool((s_new <= 1).all())
    assert bool((s_new[:, 1:] >= s_new[:, :-1]).all())


def test_sample_pdf_random_draws_stay_in_bins():
    torch.manual_seed(0)
    bins = t('bins')
    x = render.sample_pdf(bins, t('w')[:, :bins.shape[1] - 1], 32, det=False)
    assert bool((x >= bins[:, :1]).all()) and bool((x <= bins[:, -1:]).all())
