"""The NeRF-sampler field kernels (Graph.walk, ext.density, ext.color and their extension-level
functions, vgf.cu:438-533) on the GPU against the CPU oracle (pinned to the reference's float64 code by
test_oracle_field.py) and against the reference's own CUDA kernels (oracle/_ref/vgf_ext, skipped when
not built): walked sites and steps bit for bit, field values within 1e-4 and gradients within 1e-3
relative (norm over all entries)."""

import ctypes

import numpy as np
import pytest
import torch

from conftest import cuda, golden, rel
from oracle import oracle

pytestmark = pytest.mark.gpu

VAL_TOL = 1e-4   # relative error of field values (fp32 kernels, __expf, conic form of the quadratic)
GRAD_TOL = 1e-3  # relative error of gradients


@pytest.fixture(scope='module')
def fz():
    return golden('field_small.npz')


def _ext():
    from voronoi_gauss_b200 import ext
    return ext


def _graph(z):
    return _ext().Graph(cuda(z['points']), cuda(z['offsets']), cuda(z['adj']))


def _g(z):
    return z['points'], z['offsets'], z['adj']


def _f(z, k):
    return cuda(z[k], torch.float32)


def _status():
    from voronoi_gauss_b200 import _lib
    bits = ctypes.c_int(0)
    _lib.call('vg_status', ctypes.addressof(bits))
    return bits.value


def test_walk_matches_oracle_bit_exact(fz):
    z = fz
    g = _graph(z)
    site, steps = g.walk(_f(z, 'o'), _f(z, 'd'), _f(z, 'z'), cuda(z['start'], torch.int32))
    r_site, r_steps = oracle.walk(*_g(z), z['o'], z['d'], z['z'], z['start'])
    assert (site.cpu().numpy() == r_site).all()
    assert (steps.cpu().numpy() == r_steps).all()


def test_walk_empty_inputs(fz):
    z = fz
    g = _graph(z)
    site, steps = g.walk(_f(z, 'o')[:4], _f(z, 'd')[:4], torch.zeros(4, 0, device='cuda'),
                         cuda(z['start'][:4], torch.int32))
    assert site.shape == (4, 0) and (steps == 0).all()
    site, steps = g.walk(_f(z, 'o')[:0], _f(z, 'd')[:0], torch.zeros(0, 5, device='cuda'),
                         cuda(z['start'][:0], torch.int32))
    assert site.shape == (0, 5) and steps.numel() == 0


def test_density_forward_and_scale_mult(fz):
    z = fz
    ext = _ext()
    args = (_f(z, 'raw'), _f(z, 'ls'), _f(z, 'quat'), _f(z, 'x'), cuda(z['site'], torch.int32))
    g = _graph(z)
    for mult in (1.0, 2.0, 4.0):
        s = ext.extension().density_forward(g.points, g.offsets, g.adj, *args, mult)
        r = oracle.density_forward(*_g(z), z['raw'], z['ls'], z['quat'], z['x'], z['site'], scale_mult=mult)
        assert rel(s.cpu().numpy(), r) < VAL_TOL
    assert rel(ext.density(g, *args).cpu().numpy(), z['ref_sigma']) < VAL_TOL


@pytest.mark.parametrize('deg', [0, 1, 2, 3])
def test_color_forward(fz, deg):
    z = fz
    g = _graph(z)
    rgb = _ext().color(g, _f(z, 'cls'), _f(z, 'cquat'), _f(z, 'sh'), _f(z, 'x'), _f(z, 'dirs'),
                       cuda(z['site'], torch.int32), deg)
    r = oracle.color_forward(*_g(z), z['cls'], z['cquat'], z['sh'], deg, z['x'], z['dirs'], z['site'])
    assert rel(rgb.cpu().numpy(), r) < VAL_TOL
    if deg == 3:
        assert rel(rgb.cpu().numpy(), z['ref_rgb']) < VAL_TOL


def test_field_gradients_through_autograd(fz):
    z = fz
    g = _graph(z)
    ext = _ext()
    params = [_f(z, k).requires_grad_() for k in ('raw', 'ls', 'quat', 'cls', 'cquat', 'sh')]
    raw, ls, q, cls, cq, sh = params
    x, dirs, site = _f(z, 'x'), _f(z, 'dirs'), cuda(z['site'], torch.int32)
    sigma = ext.density(g, raw, ls, q, x, site)
    rgb = ext.color(g, cls, cq, sh, x, dirs, site, 3)
    ((sigma * _f(z, 'g_sigma')).sum() + (rgb * _f(z, 'g_rgb')).sum()).backward()
    o_raw, o_ls, o_q = oracle.density_backward(*_g(z), z['raw'], z['ls'], z['quat'], z['x'], z['site'], z['g_sigma'])
    o_rgb = oracle.color_forward(*_g(z), z['cls'], z['cquat'], z['sh'], 3, z['x'], z['dirs'], z['site'])
    o_cls, o_cq, o_sh = oracle.color_backward(*_g(z), z['cls'], z['cquat'], z['sh'], 3, z['x'], z['dirs'], z['site'],
                                              o_rgb, z['g_rgb'])
    for p, o, k in zip(params, (o_raw, o_ls, o_q, o_cls, o_cq, o_sh), ('raw', 'ls', 'quat', 'cls', 'cquat', 'sh')):
        gp = p.grad.cpu().numpy()
        assert rel(gp, o) < GRAD_TOL, k
        assert rel(gp, z[f'ref_g_{k}']) < GRAD_TOL, k


def test_color_backward_low_degree_zeroes_unused_bands(fz):
    z = fz
    g = _graph(z)
    ext = _ext()
    args = [_f(z, k) for k in ('cls', 'cquat', 'sh')]
    x, dirs, site = _f(z, 'x'), _f(z, 'dirs'), cuda(z['site'], torch.int32)
    rgb = ext.extension().color_forward(g.points, g.offsets, g.adj, *args, 1, x, dirs, site)
    g_ls, g_q, g_sh = ext.extension().color_backward(g.points, g.offsets, g.adj, *args, 1, x, dirs, site, rgb,
                                                     _f(z, 'g_rgb'))
    o = oracle.color_backward(*_g(z), z['cls'], z['cquat'], z['sh'], 1, z['x'], z['dirs'], z['site'],
                              rgb.cpu().numpy(), z['g_rgb'])
    assert (g_sh[:, 4:] == 0).all()
    for a, b in zip((g_ls, g_q, g_sh), o):
        assert rel(a.cpu().numpy(), b) < GRAD_TOL


def test_empty_samples_give_empty_values_and_zero_gradients(fz):
    z = fz
    g = _graph(z)
    fe = _ext().extension()
    x0, s0 = torch.zeros(0, 3, device='cuda'), torch.zeros(0, dtype=torch.int32, device='cuda')
    args = (_f(z, 'raw'), _f(z, 'ls'), _f(z, 'quat'))
    assert fe.density_forward(g.points, g.offsets, g.adj, *args, x0, s0, 1.0).numel() == 0
    grads = fe.density_backward(g.points, g.offsets, g.adj, *args, x0, s0, torch.zeros(0, device='cuda'))
    assert all(float(t.abs().max()) == 0.0 for t in grads)
    cargs = (_f(z, 'cls'), _f(z, 'cquat'), _f(z, 'sh'))
    assert fe.color_forward(g.points, g.offsets, g.adj, *cargs, 3, x0, x0, s0).shape == (0, 3)
    grads = fe.color_backward(g.points, g.offsets, g.adj, *cargs, 3, x0, x0, s0, x0, x0)
    assert all(float(t.abs().max()) == 0.0 for t in grads)


def test_out_of_range_sites_are_skipped_and_flagged(fz):
    z = fz
    from voronoi_gauss_b200 import _lib
    g = _graph(z)
    fe = _ext().extension()
    site = cuda(z['site'][:8], torch.int32).clone()
    site[3] = len(z['points'])
    site[5] = -1
    torch.cuda.synchronize()
    _lib.call('vg_status_reset')
    s = fe.density_forward(g.points, g.offsets, g.adj, _f(z, 'raw'), _f(z, 'ls'), _f(z, 'quat'), _f(z, 'x')[:8], site,
                           1.0)
    assert _status() & 4
    s = s.cpu().numpy()
    assert s[3] == 0 and s[5] == 0 and (s[[0, 1, 2, 4, 6, 7]] > 0).all()
    _lib.call('vg_status_reset')
    start = cuda(z['start'][:4], torch.int32).clone()
    start[1] = 1 << 30
    site, steps = g.walk(_f(z, 'o')[:4], _f(z, 'd')[:4], _f(z, 'z')[:4], start)
    assert _status() & 4
    assert (site[1] == -1).all() and int(steps[1]) == 0 and (site[0] >= 0).all()
    _lib.call('vg_status_reset')


def test_bad_arguments_raise(fz):
    z = fz
    g = _graph(z)
    fe = _ext().extension()
    with pytest.raises(RuntimeError, match='wrong dtype'):
        fe.density_forward(g.points, g.offsets, g.adj, _f(z, 'raw'), _f(z, 'ls'), _f(z, 'quat'), _f(z, 'x'),
                           cuda(z['site']).long(), 1.0)
    with pytest.raises(RuntimeError, match='must be a CUDA tensor'):
        fe.color_forward(g.points, g.offsets, g.adj, _f(z, 'cls'), _f(z, 'cquat'), torch.as_tensor(z['sh']), 3,
                         _f(z, 'x'), _f(z, 'dirs'), cuda(z['site'], torch.int32))
    with pytest.raises(RuntimeError, match='z must be'):
        fe.walk(g.points, g.offsets, g.adj, _f(z, 'o'), _f(z, 'd'), _f(z, 'z').reshape(-1),
                cuda(z['start'], torch.int32))


# ------------------------------------------------------------------ against the reference kernels

def _ref():
    from oracle import ref_build
    if not ref_build.available('vgf_ext'):
        pytest.skip('oracle/_ref/vgf_ext not built')
    return ref_build.load_reference('vgf_ext')


@pytest.fixture(scope='module')
def scene10k():
    """10k uniform sites (config-1 distribution), 2048 rays of 96 sorted samples, per-site parameters."""
    from voronoi_gauss_b200 import sites
    rng = np.random.default_rng(0)
    pts, _, offsets, adj = sites.delaunay_graph(rng.uniform(-1, 1, (10000, 3)))
    n = len(pts)
    gen = torch.Generator().manual_seed(1)
    B, S = 2048, 96
    o = torch.tensor(rng.uniform(-1.1, 1.1, (B, 3)), dtype=torch.float32)
    d = torch.nn.functional.normalize(torch.randn(B, 3, generator=gen), dim=-1)
    zz = torch.sort(torch.rand(B, S, generator=gen) * 2.0, 1)[0]
    start = sites.nearest_sites(pts, o.numpy()).astype(np.int32)
    p = {'raw': torch.randn(n, generator=gen) * 0.5, 'ls': torch.randn(n, 3, generator=gen) * 0.3 - 3.0,
         'quat': torch.randn(n, 4, generator=gen), 'cls': torch.randn(n, 3, generator=gen) * 0.3 - 3.0,
         'cquat': torch.randn(n, 4, generator=gen), 'sh': torch.randn(n, 16, 3, generator=gen) * 0.3}
    dev = {k: v.cuda().contiguous() for k, v in p.items()}
    return dict(points=cuda(pts.astype(np.float32)), offsets=cuda(offsets, torch.int32), adj=cuda(adj, torch.int32),
                o=o.cuda(), d=d.cuda(), z=zz.cuda(), start=cuda(start, torch.int32), **dev)


def test_walk_matches_reference_kernel(scene10k):
    R = _ref()
    s = scene10k
    g = _ext().Graph(s['points'], s['offsets'], s['adj'])
    site, steps = g.walk(s['o'], s['d'], s['z'], s['start'])
    r_site, r_steps = R.walk(s['points'], s['offsets'], s['adj'], s['o'], s['d'], s['z'], s['start'])
    assert torch.equal(site, r_site)
    assert torch.equal(steps, r_steps)


def test_fields_match_reference_kernels(scene10k):
    R = _ref()
    s = scene10k
    ext = _ext()
    g = ext.Graph(s['points'], s['offsets'], s['adj'])
    site, _ = g.walk(s['o'], s['d'], s['z'], s['start'])
    x = (s['o'][:, None] + s['d'][:, None] * s['z'][..., None]).reshape(-1, 3).contiguous()
    site = site.reshape(-1).contiguous()
    dirs = s['d'][:, None].expand(-1, s['z'].size(1), 3).reshape(-1, 3).contiguous()
    P = (s['points'], s['offsets'], s['adj'])
    fe = ext.extension()
    for mult in (1.0, 4.0):
        a = fe.density_forward(*P, s['raw'], s['ls'], s['quat'], x, site, mult)
        b = R.density_forward(*P, s['raw'], s['ls'], s['quat'], x, site, mult)
        assert rel(a.cpu().numpy(), b.cpu().numpy()) < VAL_TOL
    gen = torch.Generator(device='cuda').manual_seed(2)
    gs = torch.randn(x.size(0), device='cuda', generator=gen)
    for a, b in zip(fe.density_backward(*P, s['raw'], s['ls'], s['quat'], x, site, gs),
                    R.density_backward(*P, s['raw'], s['ls'], s['quat'], x, site, gs)):
        assert rel(a.cpu().numpy(), b.cpu().numpy()) < GRAD_TOL
    rgb = fe.color_forward(*P, s['cls'], s['cquat'], s['sh'], 3, x, dirs, site)
    r_rgb = R.color_forward(*P, s['cls'], s['cquat'], s['sh'], 3, x, dirs, site)
    assert rel(rgb.cpu().numpy(), r_rgb.cpu().numpy()) < VAL_TOL
    assert float((rgb - r_rgb).abs().max()) < 1e-4
    g_rgb = torch.randn(x.size(0), 3, device='cuda', generator=gen)
    for a, b in zip(fe.color_backward(*P, s['cls'], s['cquat'], s['sh'], 3, x, dirs, site, rgb, g_rgb),
                    R.color_backward(*P, s['cls'], s['cquat'], s['sh'], 3, x, dirs, site, r_rgb, g_rgb)):
        assert rel(a.cpu().numpy(), b.cpu().numpy()) < GRAD_TOL


def test_render_rays_matches_reference_kernels(scene10k, monkeypatch):
    """The proposal-sampler renderer end to end (render.render_rays, deterministic samples), once on this
    build's kernels and once with the reference's kernels substituted for walk / density / colour."""
    R = _ref()
    s = scene10k
    ext = _ext()
    from voronoi_gauss_b200 import render
    from voronoi_gauss_b200.model import VoronoiGaussField
    params = {'raw': s['raw'], 'd_log_scale': s['ls'], 'd_quat': s['quat'], 'c_log_scale': s['cls'],
              'c_quat': s['cquat'], 'sh': s['sh'], 'sh_deg': 3}
    model = VoronoiGaussField.from_params(s['points'], s['offsets'], s['adj'], params)
    o, d, start = s['o'][:512], s['d'][:512], s['start'][:512]
    out = render.render_rays(model, o, d, start, perturb=False)
    ((out['rgb'] ** 2).sum()).backward()
    mine = out['rgb'].detach(), [p.grad.clone() for p in (model.raw, model.d_log_scale, model.c_log_scale, model.sh_dc)]
    model.zero_grad()

    class RefField:
        walk = staticmethod(R.walk)
        density_forward = staticmethod(R.density_forward)
        density_backward = staticmethod(R.density_backward)
        color_forward = staticmethod(R.color_forward)
        color_backward = staticmethod(R.color_backward)

    monkeypatch.setattr(ext, 'extension', lambda: RefField)
    out = render.render_rays(model, o, d, start, perturb=False)
    ((out['rgb'] ** 2).sum()).backward()
    ref = out['rgb'].detach(), [p.grad for p in (model.raw, model.d_log_scale, model.c_log_scale, model.sh_dc)]
    assert float((mine[0] - ref[0]).abs().max()) < 1e-4
    for a, b in zip(mine[1], ref[1]):
        assert rel(a.cpu().numpy(), b.cpu().numpy()) < GRAD_TOL


def test_backward_paths_agree(fz):
    """The per-sample scatter (workspace sized for no samples) and the cell-major scatter (workspace
    sized for the samples, the default of ext) give the same gradients."""
    from voronoi_gauss_b200 import _lib
    z = fz
    g = _graph(z)
    pk = g.pack
    fe = _ext().extension()
    x, dirs, site = _f(z, 'x'), _f(z, 'dirs'), cuda(z['site'], torch.int32)
    m = x.size(0)
    raw, ls, q, cls, cq, sh = (_f(z, k) for k in ('raw', 'ls', 'quat', 'cls', 'cquat', 'sh'))
    gs, grgb = _f(z, 'g_sigma'), _f(z, 'g_rgb')
    stream = torch.cuda.current_stream().cuda_stream
    small = _lib.lib().vg_field_workspace_bytes(pk.n, 0, 1, 0)
    assert small < _lib.lib().vg_field_workspace_bytes(pk.n, 0, 1, m)
    ws = torch.empty(small, dtype=torch.uint8, device='cuda')
    per = [torch.empty_like(raw), torch.empty_like(ls), torch.empty_like(q)]
    _lib.call('vg_density_backward', pk.ptr, pk.n, pk.m, raw.data_ptr(), ls.data_ptr(), q.data_ptr(), x.data_ptr(),
              site.data_ptr(), m, gs.data_ptr(), *(t.data_ptr() for t in per), ws.data_ptr(), small, stream)
    cm = fe.density_backward(g.points, g.offsets, g.adj, raw, ls, q, x, site, gs)
    for a, b in zip(per, cm):
        assert rel(a.cpu().numpy(), b.cpu().numpy()) < GRAD_TOL
    rgb = fe.color_forward(g.points, g.offsets, g.adj, cls, cq, sh, 3, x, dirs, site)
    small = _lib.lib().vg_field_workspace_bytes(pk.n, 3, 3, 0)
    ws = torch.empty(small, dtype=torch.uint8, device='cuda')
    per = [torch.empty_like(cls), torch.empty_like(cq), torch.empty_like(sh)]
    _lib.call('vg_color_backward', pk.ptr, pk.n, pk.m, cls.data_ptr(), cq.data_ptr(), sh.data_ptr(), 3, x.data_ptr(),
              dirs.data_ptr(), site.data_ptr(), m, rgb.data_ptr(), grgb.data_ptr(), *(t.data_ptr() for t in per),
              ws.data_ptr(), small, stream)
    cm = fe.color_backward(g.points, g.offsets, g.adj, cls, cq, sh, 3, x, dirs, site, rgb, grgb)
    for a, b in zip(per, cm):
        assert rel(a.cpu().numpy(), b.cpu().numpy()) < GRAD_TOL
