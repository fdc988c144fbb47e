"""Pins the CPU oracle (oracle/vg_oracle.c) against the golden vectors made by the reference's own
float64 code (tests/golden/make_golden.py): cell sequences, sample parameters, images and gradients.
The oracle is what the GPU parity tests compare the CUDA kernels with."""

import numpy as np
import pytest

from conftest import golden, rel
from oracle import oracle

F32_TOL = 1e-4   # fp32 kernel arithmetic vs float64 reference, absolute, images / transmittance
GRAD_TOL = 1e-3  # relative error of gradients (norm over all sites)


def split(flat, off):
    return [flat[off[i]:off[i + 1]] for i in range(len(off) - 1)]


def run_foam(z, record_cap, threads=1):
    out = oracle.foam_forward(z['points'], z['offsets'], z['adj'], z['raw'], z['dA'], z['cA'], z['sh'], 3, z['o'],
                              z['d'], z['start'], z['near'], z['far'], 0.0, -1.0, record_cap, n_threads=threads)
    return out


def test_foam_cells_and_samples_match_reference_trace(foam_small):
    z = foam_small
    rgb, T, depth, stats, rec = run_foam(z, 256)
    ts = split(z['ref_t'], z['ref_t_off'])
    cells = split(z['ref_cells'], z['ref_t_off'])
    assert (stats[:, 0] == [len(t) for t in ts]).all()
    for r in range(len(ts)):
        s = stats[r, 0]
        got_cells = rec[r, :s, 1].view(np.int32)
        assert (got_cells == cells[r]).all(), f'ray {r}: cell sequence differs'
        np.testing.assert_allclose(rec[r, :s, 0], ts[r], atol=1e-5, rtol=0)


def test_foam_images_match_reference(foam_small):
    z = foam_small
    rgb, T, depth, stats, rec = run_foam(z, 0)
    assert np.abs(rgb - z['ref_fg']).max() <= F32_TOL
    assert np.abs(T - z['ref_T']).max() <= F32_TOL
    assert stats[:, 1].tolist() == (stats[:, 0] - 1).tolist()  # w_thresh = -1: every segment coloured


@pytest.mark.parametrize('record_cap', [256, 0, 6])
def test_foam_gradients_match_reference(foam_small, record_cap):
    """Replay of every ray (256), re-trace of every ray (0) and a mix (6), as test_foam.py:114-118."""
    z = foam_small
    rgb, T, depth, stats, rec = run_foam(z, record_cap)
    g = oracle.foam_backward(z['points'], z['offsets'], z['adj'], z['raw'], z['dA'], z['cA'], z['sh'], 3, z['o'],
                             z['d'], z['start'], z['near'], z['far'], 0.0, -1.0, rgb, T, z['g_rgb'], z['g_T'], rec,
                             stats)
    for name, got in zip(('raw', 'dA', 'cA', 'sh'), g):
        assert rel(got, z[f'ref_g_{name}']) <= GRAD_TOL, name


def test_foam_threads_agree(foam_small):
    z = foam_small
    a = run_foam(z, 16, threads=1)
    b = run_foam(z, 16, threads=4)
    for x, y in zip(a, b):
        assert np.array_equal(x, y)


def test_foam_config1_rays():
    """64 rays of the config-1 scene (10k uniform sites, sh_deg 1) against the reference's float64
    trace, compositing and gradients."""
    from voronoi_gauss_b200 import scenes
    z = golden('foam_config1.npz')
    g = scenes.build_graph(1, cache=True)
    assert len(g['points']) == int(z['n_sites']) and len(g['adj']) == int(z['n_adj'])
    prm = scenes.make_params(1, g['points'].astype(np.float64))
    dA = oracle.conic_forward(prm['d_log_scale'], prm['d_quat'])
    cA = oracle.conic_forward(prm['c_log_scale'], prm['c_quat'])
    rgb, T, depth, stats, rec = oracle.foam_forward(g['points'], g['offsets'], g['adj'], prm['raw'], dA, cA,
                                                    prm['sh'], 1, z['o'], z['d'], z['start'], z['near'], z['far'],
                                                    0.0, -1.0, 512)
    ts = split(z['ref_t'], z['ref_t_off'])
    cells = split(z['ref_cells'], z['ref_t_off'])
    for r in range(len(ts)):
        s = stats[r, 0]
        assert s == len(ts[r])
        assert (rec[r, :s, 1].view(np.int32) == cells[r]).all()
    assert np.abs(rgb - z['ref_fg']).max() <= F32_TOL
    assert np.abs(T - z['ref_T']).max() <= F32_TOL
    gr = oracle.foam_backward(g['points'], g['offsets'], g['adj'], prm['raw'], dA, cA, prm['sh'], 1, z['o'], z['d'],
                              z['start'], z['near'], z['far'], 0.0, -1.0, rgb, T, z['g_rgb'], z['g_T'], rec, stats)
    n = len(g['points'])
    for name, got in zip(('raw', 'dA', 'cA', 'sh'), gr):
        rows, vals = z[f'ref_g_{name}_rows'], z[f'ref_g_{name}_vals']
        want = np.zeros((n,) + vals.shape[1:], np.float64)
        want[rows] = vals
        if name == 'sh':
            assert np.abs(got[:, 4:]).max() == 0.0  # bands beyond sh_deg 1 get no gradient
            got = got[:, :4]
        assert rel(got, want) <= GRAD_TOL, name


def test_march_matches_reference(march_small):
    z = march_small
    args = (z['points'], z['offsets'], z['adj'], z['raw'], z['dA'], z['cA'], z['sh'], 3, z['o'], z['d'],
            z['start'], z['near'], z['mid'], z['far'], float(z['dt']), int(z['n_bg']))
    rgb, T, depth, stats = oracle.march_forward(*args, 0.0, -1.0)
    n_ref = np.diff(z['ref_sites_off'])
    assert (stats[:, 0] == n_ref).all()
    assert np.abs(rgb - z['ref_fg']).max() <= F32_TOL
    assert np.abs(T - z['ref_T']).max() <= F32_TOL
    g = oracle.march_backward(*args, 0.0, -1.0, rgb, T, z['g_rgb'], z['g_T'])
    for name, got in zip(('raw', 'dA', 'cA', 'sh'), g):
        assert rel(got, z[f'ref_g_{name}']) <= GRAD_TOL, name


@pytest.mark.parametrize('floor', [0.0, 0.01])
def test_conic_matches_reference(floor):
    z = golden('conic.npz')
    A = oracle.conic_forward(z['ls'], z['quat'], floor)
    assert rel(A, z[f'A_{floor}']) <= 1e-5
    g_ls, g_q = oracle.conic_backward(z['ls'], z['quat'], floor, z['gA'])
    # The reference kernel (vgf.cu:402) applies d iv / d ls without the clamp's zero derivative, unlike
    # its torch twin; rows whose log-scale is clamped are compared for the quaternion only.
    inside = (np.abs(z['ls']) < 20).all(1)
    assert rel(g_ls[inside], z[f'g_ls_{floor}'][inside]) <= 1e-4
    assert rel(g_q, z[f'g_quat_{floor}']) <= 1e-4


@pytest.mark.parametrize('tag', ['plain', 'morton'])
@pytest.mark.parametrize('mode', [0, 2])
def test_foam_infer_exact_modes_match_reference(foam_small, tag, mode):
    """foam_infer on the reference's own pack layouts, exact options (no cut-offs), lazy and fused
    colours: same image as the float64 training-path reference (test_foam.py:120-132)."""
    z = foam_small
    start = z['start'] if tag == 'plain' else np.argsort(z[f'pack_{tag}_orig'])[z['start']]
    rgb, T, depth, stats = oracle.foam_infer(
        z[f'pack_{tag}_points'], z[f'pack_{tag}_offsets'], z[f'pack_{tag}_nbr'], z[f'pack_{tag}_edge'],
        z[f'pack_{tag}_attr'], z[f'pack_{tag}_sh'], 3, z['o'], z['d'], start, z['near'], z['far'], 0.0, -1.0,
        float('inf'), mode, 2, None, z[f'pack_{tag}_orig'])
    assert np.abs(rgb - z['ref_fg']).max() <= F32_TOL
    assert np.abs(T - z['ref_T']).max() <= F32_TOL
    ts = split(z['ref_t'], z['ref_t_off'])
    assert (stats[:, 0] == [len(t) for t in ts]).all()


def test_foam_infer_cutoffs_close(foam_small):
    """eps_density 1e-3 + fp16 SH + Morton order: an approximation, close to the exact image."""
    z = foam_small
    tag = 'eps_morton'
    start = np.argsort(z[f'pack_{tag}_orig'])[z['start']]
    rgb, T, depth, stats = oracle.foam_infer(
        z[f'pack_{tag}_points'], z[f'pack_{tag}_offsets'], z[f'pack_{tag}_nbr'], z[f'pack_{tag}_edge'],
        z[f'pack_{tag}_attr'], z[f'pack_{tag}_sh'], 3, z['o'], z['d'], start, z['near'], z['far'], 0.0, -1.0,
        2 * np.log(1e3), 2, 2, None, z[f'pack_{tag}_orig'])
    assert np.isfinite(rgb).all() and (T >= 0).all() and (T <= 1).all()
    assert (stats[:, 3] <= stats[:, 0] * 64).all()
