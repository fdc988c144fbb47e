"""CUDA interaction-point renderer (libvgb200 through the drop-in ext module) against the CPU oracle and
the golden vectors of the reference's float64 code: cell sequences and sample parameters bit for bit,
images within 1e-4, gradients within 1e-3 relative."""

import numpy as np
import pytest
import torch

from conftest import audit_stats, bits, cuda, golden, rel, small_inputs, split
from oracle import oracle

pytestmark = pytest.mark.gpu

IMG_TOL = 1e-4   # max |rgb / T / depth - oracle|
GRAD_TOL = 1e-3  # relative error of gradients
TIE_IMG_TOL = 1e-3  # rays at a documented near-tie of t_thresh / w_thresh (one segment of weight ~1e-4 apart)


def _ext():
    from voronoi_gauss_b200 import ext
    return ext


def graph_of(z):
    ext = _ext()
    return ext.Graph(cuda(z['points'], torch.float32), cuda(z['offsets'], torch.int32), cuda(z['adj'], torch.int32))


def test_foam_forward_matches_oracle_bitwise_cells(foam_small):
    z = foam_small
    ext = _ext()
    g, x = graph_of(z), small_inputs(z)
    rgb, T, depth, stats, rec = ext.foam_extension().foam_forward(
        g.points, g.offsets, g.adj, x['raw'], x['dA'], x['cA'], x['sh'], 3, x['o'], x['d'], x['start'], x['near'],
        x['far'], 0.0, -1.0, 256)
    o_rgb, o_T, o_depth, o_stats, o_rec = oracle.foam_forward(
        z['points'], z['offsets'], z['adj'], z['raw'], z['dA'], z['cA'], z['sh'], 3, z['o'], z['d'], z['start'],
        z['near'], z['far'], 0.0, -1.0, 256)
    stats, rec = stats.cpu().numpy(), rec.cpu().numpy()
    assert (stats == o_stats).all()
    ts, cells = split(z['ref_t'], z['ref_t_off']), split(z['ref_cells'], z['ref_t_off'])
    for r in range(len(stats)):
        s = stats[r, 0]
        assert (bits(rec[r, :s, 1]) == bits(o_rec[r, :s, 1])).all(), f'ray {r}: cells differ from the oracle'
        assert (bits(rec[r, :s, 0]) == bits(o_rec[r, :s, 0])).all(), f'ray {r}: sample t differs from the oracle'
        assert (bits(rec[r, :s, 1]) == cells[r]).all(), f'ray {r}: cells differ from the reference trace'
        np.testing.assert_allclose(rec[r, :s, 2], o_rec[r, :s, 2], rtol=1e-5, atol=1e-6)  # sigma
        np.testing.assert_allclose(rec[r, :s, 3:6], o_rec[r, :s, 3:6], atol=1e-5)  # colour of the sample
    assert np.abs(rgb.cpu().numpy() - o_rgb).max() <= IMG_TOL
    assert np.abs(T.cpu().numpy() - o_T).max() <= IMG_TOL
    assert np.abs(depth.cpu().numpy() - o_depth).max() <= IMG_TOL
    assert np.abs(rgb.cpu().numpy() - z['ref_fg']).max() <= IMG_TOL


@pytest.mark.parametrize('record_cap', [256, 0, 6, 2])
def test_foam_gradients_match_oracle_and_reference(foam_small, record_cap):
    """Replay (256), re-trace (0), mixed (6) and nearly-all re-traced (2), as test_foam.py:114-118."""
    z = foam_small
    ext = _ext()
    g, x = graph_of(z), small_inputs(z)
    params = [x[k].clone().requires_grad_() for k in ('raw', 'dA', 'cA', 'sh')]
    fg, T, _, stats = ext.foam(g, *params, 3, x['o'], x['d'], x['start'], x['near'], x['far'], t_thresh=0.0,
                               w_thresh=-1.0, record_cap=record_cap)
    ((fg * cuda(z['g_rgb'])).sum() + (T * cuda(z['g_T'])).sum()).backward()
    o_rgb, o_T, _, o_stats, o_rec = oracle.foam_forward(
        z['points'], z['offsets'], z['adj'], z['raw'], z['dA'], z['cA'], z['sh'], 3, z['o'], z['d'], z['start'],
        z['near'], z['far'], 0.0, -1.0, 256)
    og = oracle.foam_backward(z['points'], z['offsets'], z['adj'], z['raw'], z['dA'], z['cA'], z['sh'], 3, z['o'],
                              z['d'], z['start'], z['near'], z['far'], 0.0, -1.0, o_rgb, o_T, z['g_rgb'], z['g_T'],
                              o_rec, o_stats)
    for name, p, want in zip(('raw', 'dA', 'cA', 'sh'), params, og):
        got = p.grad.cpu().numpy()
        assert rel(got, want) <= GRAD_TOL, f'{name} vs oracle'
        assert rel(got, z[f'ref_g_{name}']) <= GRAD_TOL, f'{name} vs reference'


@pytest.mark.parametrize('sh_deg', [0, 1, 2])
def test_foam_lower_sh_degrees(foam_small, sh_deg):
    z = foam_small
    ext = _ext()
    g, x = graph_of(z), small_inputs(z)
    params = [x[k].clone().requires_grad_() for k in ('raw', 'dA', 'cA', 'sh')]
    fg, T, _, stats = ext.foam(g, *params, sh_deg, x['o'], x['d'], x['start'], x['near'], x['far'], t_thresh=0.0,
                               w_thresh=-1.0, record_cap=64)
    ((fg * cuda(z['g_rgb'])).sum() + (T * cuda(z['g_T'])).sum()).backward()
    o_rgb, o_T, _, o_stats, o_rec = oracle.foam_forward(
        z['points'], z['offsets'], z['adj'], z['raw'], z['dA'], z['cA'], z['sh'], sh_deg, z['o'], z['d'], z['start'],
        z['near'], z['far'], 0.0, -1.0, 64)
    assert np.abs(fg.detach().cpu().numpy() - o_rgb).max() <= IMG_TOL
    og = oracle.foam_backward(z['points'], z['offsets'], z['adj'], z['raw'], z['dA'], z['cA'], z['sh'], sh_deg,
                              z['o'], z['d'], z['start'], z['near'], z['far'], 0.0, -1.0, o_rgb, o_T, z['g_rgb'],
                              z['g_T'], o_rec, o_stats)
    for name, p, want in zip(('raw', 'dA', 'cA', 'sh'), params, og):
        assert rel(p.grad.cpu().numpy(), want) <= GRAD_TOL, name
    nb = (sh_deg + 1) ** 2
    assert float(params[3].grad[:, nb:].abs().max()) == 0.0


def _config1(n_rays_per_cam=4096, cams=4):
    from voronoi_gauss_b200 import render, scenes, sites
    gr = scenes.build_graph(1)
    prm = scenes.make_params(1, gr['points'].astype(np.float64))
    order = scenes.tile_order(64, 64)
    os_, ds_, starts = [], [], []
    for i in range(cams):
        centre, c2w = scenes.orbit_camera(i, cams)
        o, d = scenes.camera_rays(centre, c2w, 64, 64, 50.0, order=order)
        os_.append(o[:n_rays_per_cam]), ds_.append(d[:n_rays_per_cam])
        starts.append(np.full(len(o[:n_rays_per_cam]), sites.nearest_sites(gr['points'], centre[None])[0], np.int32))
    o, d = torch.cat(os_), torch.cat(ds_)
    near, _, far = render.ray_bounds(o, d, 0.02, 4.0)
    return gr, prm, o.numpy(), d.numpy(), np.concatenate(starts), near.numpy(), far.numpy()


def test_foam_config1_full_image_matches_oracle():
    """Config 1 (10k sites, 4 cameras x 64 x 64 rays, default thresholds 1e-4): stats, records and
    images against the oracle; gradients within 1e-3."""
    ext = _ext()
    gr, prm, o, d, start, near, far = _config1()
    g = ext.Graph(cuda(gr['points']), cuda(gr['offsets']), cuda(gr['adj']))
    ls, q, cls, cq = (cuda(prm[k]) for k in ('d_log_scale', 'd_quat', 'c_log_scale', 'c_quat'))
    dA, cA = ext.conic(ls, q), ext.conic(cls, cq)
    o_dA = oracle.conic_forward(prm['d_log_scale'], prm['d_quat'])
    o_cA = oracle.conic_forward(prm['c_log_scale'], prm['c_quat'])
    assert rel(dA.cpu().numpy(), o_dA) <= 1e-6 and rel(cA.cpu().numpy(), o_cA) <= 1e-6
    raw, sh = cuda(prm['raw']).requires_grad_(), cuda(prm['sh']).requires_grad_()
    dA_, cA_ = dA.detach().clone().requires_grad_(), cA.detach().clone().requires_grad_()
    B = len(o)
    gen = torch.Generator().manual_seed(3)
    g_rgb, g_T = torch.randn(B, 3, generator=gen), torch.randn(B, generator=gen)
    rgb, T, depth, stats = ext.foam(g, raw, dA_, cA_, sh, 1, cuda(o), cuda(d), cuda(start), cuda(near), cuda(far))
    ((rgb * g_rgb.cuda()).sum() + (T * g_T.cuda()).sum()).backward()
    nt = max(1, min(32, __import__('os').cpu_count() or 1))
    args = (gr['points'], gr['offsets'], gr['adj'], prm['raw'], dA.cpu().numpy(), cA.cpu().numpy(), prm['sh'], 1, o, d,
            start, near, far, 1e-4, 1e-4)
    o_rgb, o_T, o_depth, o_stats, o_rec = oracle.foam_forward(*args, 256, n_threads=nt)
    # the oracle's expf and the GPU's __expf round differently, so a ray whose compositing passes within a
    # hair of t_thresh or w_thresh may stop or colour one segment apart: every such ray must be a near-tie
    same = audit_stats(stats.cpu().numpy(), o_stats, o_rec, 1e-4, 1e-4)
    rgb_d, T_d = np.abs(rgb.detach().cpu().numpy() - o_rgb), np.abs(T.detach().cpu().numpy() - o_T)
    assert rgb_d[same].max() <= IMG_TOL and T_d[same].max() <= IMG_TOL
    # a near-tie moves at most one segment of weight ~1e-4 (or a tail of transmittance ~1e-4)
    assert rgb_d.max() <= TIE_IMG_TOL and T_d.max() <= TIE_IMG_TOL
    og = oracle.foam_backward(*args, o_rgb, o_T, g_rgb.numpy(), g_T.numpy(), o_rec, o_stats, n_threads=nt)
    for name, p, want in zip(('raw', 'dA', 'cA', 'sh'), (raw, dA_, cA_, sh), og):
        assert rel(p.grad.cpu().numpy(), want) <= GRAD_TOL, name


def test_foam_no_grad_path_equals_training_forward(foam_small):
    """ext.foam without gradients (record_cap 0, ext.py:213-215) renders the same image."""
    z = foam_small
    ext = _ext()
    g, x = graph_of(z), small_inputs(z)
    args = (g, x['raw'], x['dA'], x['cA'], x['sh'], 3, x['o'], x['d'], x['start'], x['near'], x['far'])
    with torch.no_grad():
        a = ext.foam(*args)
    b = ext.foam_extension().foam_forward(g.points, g.offsets, g.adj, x['raw'], x['dA'], x['cA'], x['sh'], 3, x['o'],
                                          x['d'], x['start'], x['near'], x['far'], 1e-4, 1e-4, 256)
    for u, v in zip(a, b[:4]):
        assert torch.equal(u, v)


def test_conic_matches_oracle_and_reference():
    ext = _ext()
    z = golden('conic.npz')
    for floor in (0.0, 0.01):
        ls, q = cuda(z['ls']).requires_grad_(), cuda(z['quat']).requires_grad_()
        A = ext.conic(ls, q, floor)
        (A * cuda(z['gA'])).sum().backward()
        assert rel(A.detach().cpu().numpy(), oracle.conic_forward(z['ls'], z['quat'], floor)) <= 1e-6
        assert rel(A.detach().cpu().numpy(), z[f'A_{floor}']) <= 1e-5
        o_gls, o_gq = oracle.conic_backward(z['ls'], z['quat'], floor, z['gA'])
        assert rel(ls.grad.cpu().numpy(), o_gls) <= 1e-5
        assert rel(q.grad.cpu().numpy(), o_gq) <= 1e-5
        inside = (np.abs(z['ls']) < 20).all(1)
        assert rel(ls.grad.cpu().numpy()[inside], z[f'g_ls_{floor}'][inside]) <= 1e-4
        assert rel(q.grad.cpu().numpy(), z[f'g_quat_{floor}']) <= 1e-4


@pytest.mark.parametrize('record_cap', [256, 24])
def test_counted_backward_matches_counting_backward(record_cap):
    """The forward's kept per-cell sample counts (foam_forward(..., counts=)) replace the backward's
    counting pass: they sum to the recorded samples of the rays that fit their records (rays with more
    samples are re-traced and left out), and the gradients equal those of the backward that counts the
    records itself (up to the order of float atomics)."""
    ext = _ext()
    gr, prm, o, d, start, near, far = _config1()
    g = ext.Graph(cuda(gr['points']), cuda(gr['offsets']), cuda(gr['adj']))
    dA = ext.conic(cuda(prm['d_log_scale']), cuda(prm['d_quat']))
    cA = ext.conic(cuda(prm['c_log_scale']), cuda(prm['c_quat']))
    raw, sh = cuda(prm['raw']), cuda(prm['sh'])
    rays = [cuda(x) for x in (o, d, start, near, far)]
    args = (g.points, g.offsets, g.adj, raw, dA, cA, sh, 1, *rays, 1e-4, 1e-4)
    B = len(o)
    counts = torch.empty(ext.sample_counts_size(len(gr['points']), B, record_cap), dtype=torch.int32, device='cuda')
    fx = ext.foam_extension()
    rgb, T, _, stats, rec = fx.foam_forward(*args, record_cap, counts=counts)
    S = stats[:, 0].long()
    fits = S <= record_cap
    assert int(counts.long().sum()) == int(S[fits].sum())
    if record_cap == 24:
        assert int((~fits).sum()) > 0  # some rays overflow their records
    gen = torch.Generator().manual_seed(5)
    g_rgb, g_T = torch.randn(B, 3, generator=gen).cuda(), torch.randn(B, generator=gen).cuda()
    kept = fx.foam_backward(*args, rgb, T, g_rgb, g_T, rec, stats, counts=counts)
    counted = fx.foam_backward(*args, rgb, T, g_rgb, g_T, rec, stats)
    for name, a, b in zip(('raw', 'dA', 'cA', 'sh'), kept, counted):
        assert rel(a.cpu().numpy(), b.cpu().numpy()) <= 1e-5, name



def test_counted_backward_with_foreign_counts_sets_status():
    """Per-cell counts that do not belong to the records given to the counted backward never make it write
    outside its buffers: all-zero counts leave every recorded sample without a place in its cell's bucket
    (its item is dropped), and counts whose buckets overflow the item buffer drop the whole pass; both set
    status bit 8 and the call returns with finite gradients. The forward's own counts set no such bit."""
    import ctypes

    from voronoi_gauss_b200 import _lib
    ext = _ext()
    gr, prm, o, d, start, near, far = _config1()
    g = ext.Graph(cuda(gr['points']), cuda(gr['offsets']), cuda(gr['adj']))
    dA = ext.conic(cuda(prm['d_log_scale']), cuda(prm['d_quat']))
    cA = ext.conic(cuda(prm['c_log_scale']), cuda(prm['c_quat']))
    raw, sh = cuda(prm['raw']), cuda(prm['sh'])
    rays = [cuda(x) for x in (o, d, start, near, far)]
    args = (g.points, g.offsets, g.adj, raw, dA, cA, sh, 1, *rays, 1e-4, 1e-4)
    B, K = len(o), 256
    counts = torch.empty(ext.sample_counts_size(len(gr['points']), B, K), dtype=torch.int32, device='cuda')
    fx = ext.foam_extension()
    rgb, T, _, stats, rec = fx.foam_forward(*args, K, counts=counts)
    gen = torch.Generator().manual_seed(7)
    g_rgb, g_T = torch.randn(B, 3, generator=gen).cuda(), torch.randn(B, generator=gen).cuda()

    def status_after(cnt):
        _lib.call('vg_status_reset')
        grads = fx.foam_backward(*args, rgb, T, g_rgb, g_T, rec, stats, counts=cnt)
        torch.cuda.synchronize()
        assert all(bool(torch.isfinite(x).all()) for x in grads)
        bits_ = ctypes.c_int(-1)
        _lib.call('vg_status', ctypes.addressof(bits_))
        return bits_.value

    assert status_after(torch.zeros_like(counts)) & 8
    assert status_after(torch.full_like(counts, 1 << 24)) & 8
    assert not status_after(counts) & 8
