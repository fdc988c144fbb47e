"""Generates the golden fixtures in this directory from the reference's own CPU code.

Run where the reference checkout is available (VG_REFERENCE, or a `reference` directory beside the
repository, as oracle/ref_build.reference_root finds it); the GPU box
and the tests only read the committed .npz files. Every fixture stores its inputs and the outputs of
the reference's float64 restatements:

* foam_small.npz   - test_foam.py's scene (300 sites, rng(2)), 64 rays, thresholds disabled:
                     test_foam.trace cell sequences (test_foam.py:18-37), float64 compositing and
                     autograd gradients of raw / dA / cA / sh (test_foam.py:76-104); the reference
                     pack_foam layouts (render.py:179-225) for four option sets, with ext.conic
                     replaced by its torch twin ext.conic_reference (ext.py:139-149) because the
                     CUDA conic cannot run here; render.morton_order (render.py:168-176).
* march_small.npz  - test_march.py's scene (rng(1)), dt 0.05, n_bg 8, conic floor 0.01: samples()
                     + exact nearest sites + float64 compositing and gradients (test_march.py:14-88).
* conic.npz        - ext.conic_reference in float64 and its autograd gradients.
* sh_basis.npz     - render.sh_basis for degrees 0..3 (render.py:143-165).
* foam_config1.npz - 64 rays of an orbit camera over the config-1 scene (10k uniform sites), float64
                     trace + compositing + sparse gradients.
* ckpt_small.pth   - a checkpoint written in train.py's format (train.py:168-170) from the reference's
                     own VoronoiGaussField (model.py:19-59), 300 sites, randomised parameters.
* render_host.npz  - the proposal sampler's host arithmetic on 256 seeded rays: render.ray_bounds,
                     s_to_t, composite, sample_pdf (stratified and the bin edges of resample) and
                     resample (render.py:16-74), float32 as the reference computes them.
* camera_rays.npz  - colmap.ColmapScene.rays (colmap.py:129-134) of every pixel of a 37x23 image, the
                     intrinsics and camera-to-world matrix built as ColmapScene.__init__ does
                     (colmap.py:104-114) from a SIMPLE_PINHOLE camera (fov 50 deg) and a seeded pose,
                     and bench_infer.tile_order (bench_infer.py:37-41) of the image.
* model_init.npz   - the initial parameters of the reference's VoronoiGaussField (model.py:23-39) for
                     200 seeded sites (init_alpha 0.2, spacings including 0), in state_dict order.
* field_small.npz  - test_grad.py's setup (400 uniform sites, rng(0)): exact nearest sites (cKDTree) of
                     sorted ray samples for the walk, and the float64 density / colour fields with
                     their autograd gradients (test_grad.py:45-125).
"""

import os
import sys
from types import SimpleNamespace

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
from oracle.ref_build import reference_root  # noqa: E402

REF = reference_root()
if REF is None:
    raise SystemExit('reference checkout not found: set VG_REFERENCE to its directory')
sys.path.insert(0, REF)

import ext as ref_ext  # noqa: E402
import render as ref_render  # noqa: E402
import sites as ref_sites  # noqa: E402
import test_foam  # noqa: E402
import test_grad  # noqa: E402
import test_march  # noqa: E402
from scipy.spatial import cKDTree  # noqa: E402

torch.set_default_dtype(torch.float32)


def ragged(seqs, dtype):
    off = np.zeros(len(seqs) + 1, dtype=np.int64)
    off[1:] = np.cumsum([len(s) for s in seqs])
    return np.concatenate(seqs).astype(dtype), off


def composite64(sigma, delta, colour):
    """float64 front-to-back compositing of segments with optical depths tau = sigma * delta and colours
    `colour`: opacity a_k = 1 - exp(-tau_k), transmittance the running product of 1 - a (exactly 0 once a
    segment is opaque), weight_k = a_k prod_{j<k} (1 - a_j). -> (foreground colour, final transmittance)."""
    opacity = 1 - torch.exp(-sigma * delta)
    through = torch.cumprod(torch.nn.functional.pad(1 - opacity, (1, 0), value=1.0), 0)
    return ((opacity * through[:-1])[:, None] * colour).sum(0), through[-1]


def mixture_colour(P, cA, X, mask, basis, sh):
    """float64 colour at the points X: the neighbourhood's max(SH + 1/2, 0) blended with the normalised
    weights exp(-m_k / 2) of the colour Mahalanobis distances (masked to each point's neighbourhood)."""
    logits = (-0.5 * test_march.mahalanobis6(P, cA, X)).masked_fill(~mask, -float('inf'))
    site_colour = (torch.einsum('j,njc->nc', basis, sh) + 0.5).clamp_min(0)
    return torch.softmax(logits, 1) @ site_colour


def foam_reference(pts, offsets, adj, raw, dA, cA, sh, o, d, near, far, g_rgb, g_T, cells0=None, sh_deg=3):
    """float64 trace + compositing + gradients, as test_foam.py:76-104; only the first (sh_deg + 1)^2 SH
    bands are used, as the kernels do (foam.cu:143-153)."""
    n = len(pts)
    tree = cKDTree(pts)
    P = torch.tensor(pts, dtype=torch.float64)
    ref = [torch.tensor(np.asarray(t), dtype=torch.float64).requires_grad_() for t in (raw, dA, cA, sh)]
    rraw, rdA, rcA, rsh = ref
    o64, d64 = np.asarray(o, np.float64), np.asarray(d, np.float64)
    fg_ref, T_ref, ts, cells = [], [], [], []
    for r in range(len(o64)):
        x0 = o64[r] + float(near[r]) * d64[r]
        start_cell = tree.query(x0)[1] if cells0 is None else cells0[r]
        t, cl = test_foam.trace(pts, offsets, adj, o64[r], d64[r], float(near[r]), float(far[r]), start_cell)
        ts.append(t)
        cells.append(cl)
        X = torch.from_numpy(o64[r] + np.outer(t, d64[r]))
        mask = test_grad.neighborhood_mask(offsets, adj, torch.tensor(cl), n)
        sigma = (torch.exp(rraw)[None] * torch.exp(-0.5 * test_march.mahalanobis6(P, rdA, X)) * mask).sum(1)
        basis = test_grad.sh_basis(torch.tensor(d64[r])) * (torch.arange(16) < (sh_deg + 1) ** 2)
        C = mixture_colour(P, rcA, X, mask, basis, rsh)
        # trapezoid rule between consecutive samples (foam.cu:1-16)
        fg, T = composite64(0.5 * (sigma[1:] + sigma[:-1]), torch.tensor(t[1:] - t[:-1]), 0.5 * (C[1:] + C[:-1]))
        fg_ref.append(fg)
        T_ref.append(T)
    fg_ref = torch.stack(fg_ref)
    T_ref = torch.stack(T_ref)
    ((fg_ref * torch.tensor(g_rgb, dtype=torch.float64)).sum() +
     (T_ref * torch.tensor(g_T, dtype=torch.float64)).sum()).backward()
    t_flat, t_off = ragged(ts, np.float64)
    c_flat, _ = ragged(cells, np.int32)
    return dict(ref_fg=fg_ref.detach().numpy(), ref_T=T_ref.detach().numpy(), ref_t=t_flat, ref_t_off=t_off,
                ref_cells=c_flat, ref_g_raw=rraw.grad.numpy(), ref_g_dA=rdA.grad.numpy(),
                ref_g_cA=rcA.grad.numpy(), ref_g_sh=rsh.grad.numpy())


def small_scene(seed):
    """Scene and parameters of test_foam.py:41-60 / test_march.py:35-49 (CPU generator)."""
    torch.manual_seed(0)
    rng = np.random.default_rng(seed)
    pts, _, offsets, adj = ref_sites.delaunay_graph(rng.uniform(-0.9, 0.9, (300, 3)))
    n = len(pts)
    raw = torch.randn(n) * 0.5 + 1.0
    ls = torch.randn(n, 3) * 0.3 - 1.8
    q = torch.randn(n, 4)
    cls = torch.randn(n, 3) * 0.3 - 1.8
    cq = torch.randn(n, 4)
    sh = torch.randn(n, 16, 3) * 0.3
    return rng, pts, offsets, adj, raw, ls, q, cls, cq, sh


def make_foam_small():
    rng, pts, offsets, adj, raw, ls, q, cls, cq, sh = small_scene(2)
    B = 64
    o = torch.tensor(rng.uniform(-0.5, 0.5, (B, 3)), dtype=torch.float32)
    d = torch.nn.functional.normalize(torch.randn(B, 3), dim=-1)
    start = torch.tensor(cKDTree(pts).query(o.numpy())[1], dtype=torch.int32)
    near, _, far = ref_render.ray_bounds(o, d, 0.02, 2.0)
    g_rgb, g_T = torch.randn(B, 3), torch.randn(B)
    dA, cA = ref_ext.conic_reference(ls, q), ref_ext.conic_reference(cls, cq)
    out = dict(points=pts.astype(np.float32), offsets=offsets, adj=adj, raw=raw.numpy(), ls=ls.numpy(),
               quat=q.numpy(), cls=cls.numpy(), cquat=cq.numpy(), dA=dA.numpy(), cA=cA.numpy(), sh=sh.numpy(),
               o=o.numpy(), d=d.numpy(), start=start.numpy(), near=near.numpy(), far=far.numpy(),
               g_rgb=g_rgb.numpy(), g_T=g_T.numpy(), sh_deg=3, far_radius=2.0)
    out.update(foam_reference(pts.astype(np.float32).astype(np.float64), offsets, adj, raw.numpy(), dA.numpy(),
                              cA.numpy(), sh.numpy(), o.numpy(), d.numpy(), near.numpy(), far.numpy(),
                              g_rgb.numpy(), g_T.numpy()))
    # reference inference packs (ext.conic -> its torch twin, since CUDA is not available here)
    graph = SimpleNamespace(points=torch.tensor(pts, dtype=torch.float32), offsets=torch.tensor(offsets),
                            adj=torch.tensor(adj))
    model = SimpleNamespace(graph=graph, raw=raw, d_log_scale=ls, d_quat=q, c_log_scale=cls, c_quat=cq,
                            sh=lambda: sh, sh_deg=3)
    saved = ref_ext.conic
    ref_ext.conic = ref_ext.conic_reference
    try:
        for tag, kw in (('plain', {}), ('morton', dict(reorder=True)),
                        ('eps', dict(eps_density=1e-3, sh_half=True)),
                        ('eps_morton', dict(eps_density=1e-3, sh_half=True, reorder=True, scale_floor=0.01))):
            pk = ref_render.pack_foam(model, **kw)
            for key in ('points', 'offsets', 'nbr', 'edge', 'attr', 'orig'):
                out[f'pack_{tag}_{key}'] = pk[key].numpy()
            out[f'pack_{tag}_sh'] = pk['sh'].numpy()
        out['morton_perm'] = ref_render.morton_order(graph.points).numpy()
    finally:
        ref_ext.conic = saved
    np.savez_compressed(os.path.join(HERE, 'foam_small.npz'), **out)


def make_march_small():
    rng, pts, offsets, adj, raw, ls, q, cls, cq, sh = small_scene(1)
    n = len(pts)
    dA, cA = ref_ext.conic_reference(ls, q, 0.01), ref_ext.conic_reference(cls, cq, 0.01)
    B, dt, n_bg = 64, 0.05, 8
    o = torch.tensor(rng.uniform(-0.5, 0.5, (B, 3)), dtype=torch.float32)
    d = torch.nn.functional.normalize(torch.randn(B, 3), dim=-1)
    start = torch.tensor(cKDTree(pts).query(o.numpy())[1], dtype=torch.int32)
    near, mid, far = ref_render.ray_bounds(o, d, 0.02, 2.0)
    g_rgb, g_T = torch.randn(B, 3), torch.randn(B)
    P = torch.tensor(pts.astype(np.float32), dtype=torch.float64)
    ref = [t.double().requires_grad_() for t in (raw, dA, cA, sh)]
    rraw, rdA, rcA, rsh = ref
    tree = cKDTree(pts.astype(np.float32).astype(np.float64))
    fg_ref, T_ref, sites_all = [], [], []
    for r in range(B):
        t, delta = test_march.samples(near[r].item(), mid[r].item(), far[r].item(), dt, n_bg)
        O, D = o[r].double(), d[r].double()
        X = O + torch.outer(torch.tensor(t), D)
        _, nearest = tree.query(X.numpy())
        site = torch.from_numpy(nearest)
        sites_all.append(site.numpy().astype(np.int32))
        mask = test_grad.neighborhood_mask(offsets, adj, site, n)
        sigma = (torch.exp(rraw)[None] * torch.exp(-0.5 * test_march.mahalanobis6(P, rdA, X)) * mask).sum(1)
        # one segment per fixed step, coloured at its midpoint (march.cu:221-262)
        fg, T = composite64(sigma, torch.tensor(delta), mixture_colour(P, rcA, X, mask, test_grad.sh_basis(D), rsh))
        fg_ref.append(fg)
        T_ref.append(T)
    fg_ref = torch.stack(fg_ref)
    T_ref = torch.stack(T_ref)
    ((fg_ref * g_rgb.double()).sum() + (T_ref * g_T.double()).sum()).backward()
    s_flat, s_off = ragged(sites_all, np.int32)
    np.savez_compressed(
        os.path.join(HERE, 'march_small.npz'), points=pts.astype(np.float32), offsets=offsets, adj=adj,
        raw=raw.numpy(), dA=dA.numpy(), cA=cA.numpy(), sh=sh.numpy(), o=o.numpy(), d=d.numpy(),
        start=start.numpy(), near=near.numpy(), mid=mid.numpy(), far=far.numpy(), g_rgb=g_rgb.numpy(),
        g_T=g_T.numpy(), dt=dt, n_bg=n_bg, sh_deg=3, ref_fg=fg_ref.detach().numpy(), ref_T=T_ref.detach().numpy(),
        ref_sites=s_flat, ref_sites_off=s_off, ref_g_raw=rraw.grad.numpy(), ref_g_dA=rdA.grad.numpy(),
        ref_g_cA=rcA.grad.numpy(), ref_g_sh=rsh.grad.numpy())


def make_conic():
    g = torch.Generator().manual_seed(5)
    n = 512
    ls = torch.randn(n, 3, generator=g) * 0.8 - 1.5
    ls[:4] = torch.tensor([[25.0, -25.0, 0.0]])  # clamp branch
    q = torch.randn(n, 4, generator=g)
    gA = torch.randn(n, 6, generator=g)
    out = dict(ls=ls.numpy(), quat=q.numpy(), gA=gA.numpy())
    for floor in (0.0, 0.01):
        L, Q = ls.double().requires_grad_(), q.double().requires_grad_()
        A = ref_ext.conic_reference(L, Q, floor)
        (A * gA.double()).sum().backward()
        out[f'A_{floor}'] = A.detach().numpy()
        out[f'g_ls_{floor}'] = L.grad.numpy()
        out[f'g_quat_{floor}'] = Q.grad.numpy()
    np.savez_compressed(os.path.join(HERE, 'conic.npz'), **out)


def make_sh_basis():
    g = torch.Generator().manual_seed(7)
    dirs = torch.nn.functional.normalize(torch.randn(256, 3, generator=g, dtype=torch.float64), dim=-1)
    out = {'dirs': dirs.numpy()}
    for deg in range(4):
        out[f'b{deg}'] = ref_render.sh_basis(dirs, deg).numpy()
    np.savez_compressed(os.path.join(HERE, 'sh_basis.npz'), **out)


def make_foam_config1():
    from voronoi_gauss_b200 import scenes
    pts0 = np.random.default_rng(0).uniform(-1, 1, (10000, 3))
    pts, _, offsets, adj = ref_sites.delaunay_graph(pts0)
    prm = scenes.make_params(1, pts)
    dA = ref_ext.conic_reference(prm['d_log_scale'], prm['d_quat'])
    cA = ref_ext.conic_reference(prm['c_log_scale'], prm['c_quat'])
    centre, c2w = scenes.orbit_camera(0, 4)
    o, d = scenes.camera_rays(centre, c2w, 64, 64, 50.0, order=scenes.tile_order(64, 64))
    sel = np.arange(0, 64 * 64, 64)  # 64 rays spread over the image
    o, d = o[sel].contiguous(), d[sel].contiguous()
    near, _, far = ref_render.ray_bounds(o, d, 0.02, 4.0)
    start = np.full(len(o), ref_sites.nearest_sites(pts, centre[None])[0], dtype=np.int32)
    g = torch.Generator().manual_seed(11)
    g_rgb, g_T = torch.randn(len(o), 3, generator=g), torch.randn(len(o), generator=g)
    p32 = pts.astype(np.float32)
    # starting cell: nearest site of x(near) (what the walk from the camera site reaches)
    x0 = o.double().numpy() + near.double().numpy()[:, None] * d.double().numpy()
    cells0 = cKDTree(p32.astype(np.float64)).query(x0)[1]
    ref = foam_reference(p32.astype(np.float64), offsets, adj, prm['raw'].numpy(), dA.numpy(), cA.numpy(),
                         prm['sh'].numpy(), o.numpy(), d.numpy(), near.numpy(), far.numpy(), g_rgb.numpy(),
                         g_T.numpy(), cells0=cells0, sh_deg=1)
    ref['ref_g_sh'] = ref['ref_g_sh'][:, :4]
    sparse = {}
    for key in ('ref_g_raw', 'ref_g_dA', 'ref_g_cA', 'ref_g_sh'):
        gk = ref.pop(key)
        rows = np.nonzero(np.abs(gk.reshape(len(gk), -1)).sum(1))[0].astype(np.int32)
        sparse[key + '_rows'] = rows
        sparse[key + '_vals'] = gk[rows].astype(np.float32)
    np.savez_compressed(os.path.join(HERE, 'foam_config1.npz'), sel=sel, start=start, o=o.numpy(), d=d.numpy(),
                        near=near.numpy(), far=far.numpy(), g_rgb=g_rgb.numpy(), g_T=g_T.numpy(),
                        n_sites=len(pts), n_adj=len(adj), **ref, **sparse)


def make_field_small():
    rng = np.random.default_rng(0)
    pts, _, offsets, adj = ref_sites.delaunay_graph(rng.uniform(-1, 1, (400, 3)))
    n = len(pts)
    p32 = pts.astype(np.float32)
    tree = cKDTree(p32.astype(np.float64))
    g = torch.Generator().manual_seed(3)
    # walk: rays from random origins, sorted samples (test_grad.py:62-72)
    B, S = 500, 40
    o = torch.tensor(rng.uniform(-1.2, 1.2, (B, 3)), dtype=torch.float32)
    d = torch.nn.functional.normalize(torch.randn(B, 3, generator=g), dim=-1)
    z = torch.sort(torch.rand(B, S, generator=g) * 2.5, 1)[0]
    start = tree.query(o.double().numpy())[1].astype(np.int32)
    x_walk = (o[:, None].double() + d[:, None].double() * z[..., None].double()).reshape(-1, 3).numpy()
    nn_dist, nn_site = tree.query(x_walk, k=2)
    # fields (test_grad.py:74-125)
    m = 3000
    x = torch.tensor(rng.uniform(-1, 1, (m, 3)), dtype=torch.float32)
    site = torch.tensor(tree.query(x.double().numpy())[1], dtype=torch.int32)
    raw = torch.randn(n, generator=g) * 0.5
    ls = torch.randn(n, 3, generator=g) * 0.3 - 1.2
    q = torch.randn(n, 4, generator=g)
    cls = torch.randn(n, 3, generator=g) * 0.3 - 1.2
    cq = torch.randn(n, 4, generator=g)
    sh = torch.randn(n, 16, 3, generator=g) * 0.3
    dirs = torch.randn(m, 3, generator=g)
    g_sigma = torch.randn(m, generator=g)
    g_rgb = torch.randn(m, 3, generator=g)
    P = torch.tensor(p32, dtype=torch.float64)
    ref = [p.double().requires_grad_() for p in (raw, ls, q, cls, cq, sh)]
    rraw, rls, rq, rcls, rcq, rsh = ref
    X = x.double()
    mask = test_grad.neighborhood_mask(offsets, adj, site, n)
    md = test_grad.mahalanobis(P, rls, rq, X)
    sigma_ref = (torch.exp(rraw)[None] * torch.exp(-0.5 * md) * mask).sum(1)
    mc = test_grad.mahalanobis(P, rcls, rcq, X).masked_fill(~mask, float('inf'))
    a = torch.softmax(-0.5 * mc, 1)
    D = torch.nn.functional.normalize(dirs.double(), dim=-1)
    ck = (torch.einsum('mj,njc->mnc', test_grad.sh_basis(D), rsh) + 0.5).clamp_min(0)
    rgb_ref = (a[..., None] * ck).sum(1)
    ((sigma_ref * g_sigma.double()).sum() + (rgb_ref * g_rgb.double()).sum()).backward()
    np.savez_compressed(
        os.path.join(HERE, 'field_small.npz'), points=p32, offsets=offsets, adj=adj, o=o.numpy(), d=d.numpy(),
        z=z.numpy(), start=start, nn_site=nn_site.astype(np.int32), nn_dist=nn_dist, x=x.numpy(),
        site=site.numpy(), raw=raw.numpy(), ls=ls.numpy(), quat=q.numpy(), cls=cls.numpy(), cquat=cq.numpy(),
        sh=sh.numpy(), dirs=dirs.numpy(), g_sigma=g_sigma.numpy(), g_rgb=g_rgb.numpy(), sh_deg=3,
        ref_sigma=sigma_ref.detach().numpy(), ref_rgb=rgb_ref.detach().numpy(),
        **{f'ref_g_{k}': r.grad.numpy() for k, r in zip(('raw', 'ls', 'quat', 'cls', 'cquat', 'sh'), ref)})


def make_ckpt_small():
    import model as ref_model
    rng, pts, offsets, adj, *_ = small_scene(4)
    n = len(pts)
    P = torch.tensor(pts, dtype=torch.float32)
    m = ref_model.VoronoiGaussField(P, torch.tensor(offsets), torch.tensor(adj), torch.rand(n, 3),
                                    torch.full((n,), 0.05))
    g = torch.Generator().manual_seed(9)
    with torch.no_grad():
        for p in m.parameters():
            p.add_(torch.randn(p.shape, generator=g) * 0.1)
    m.sh_deg = 2
    torch.save({'state': m.state_dict(), 'points': m.graph.points, 'offsets': m.graph.offsets, 'adj': m.graph.adj,
                'sh_deg': m.sh_deg, 'normalization': {'scale': 1.0}, 'args': {'iters': 0}},
               os.path.join(HERE, 'ckpt_small.pth'))


def make_render_host():
    g = torch.Generator().manual_seed(11)
    B, S = 256, 64
    o = torch.randn(B, 3, generator=g) * 1.5
    d = torch.nn.functional.normalize(torch.randn(B, 3, generator=g), dim=-1)
    near, mid, far = ref_render.ray_bounds(o, d, 0.02, 4.0)
    s = torch.linspace(0, 1, S + 1)[:-1].expand(B, S) + torch.rand(B, S, generator=g) / S
    t = ref_render.s_to_t(s, near, mid, far)
    sigma = torch.rand(B, S, generator=g) * 20 * (torch.rand(B, S, generator=g) < 0.3)
    w, T = ref_render.composite(sigma, t, far)
    bins = torch.sort(torch.rand(B, S + 1, generator=g), 1)[0]
    pdf_det = ref_render.sample_pdf(bins, w[:, :S], 48, det=True)
    s_new = ref_render.resample(s, w, 64, det=True)
    out = {k: v.numpy() for k, v in dict(o=o, d=d, near=near, mid=mid, far=far, s=s, t=t, sigma=sigma, w=w, T=T,
                                          bins=bins, pdf_det=pdf_det, s_new=s_new).items()}
    np.savez_compressed(os.path.join(HERE, 'render_host.npz'), **out)


def make_camera_rays():
    import math
    import colmap as ref_colmap
    torch.Tensor.cuda = lambda self, *a, **k: self  # tile_order ends with .cuda(); keep it on the CPU
    import bench_infer as ref_bench_infer
    W, H, fov = 37, 23, 50.0
    f = 0.5 * W / math.tan(math.radians(fov) / 2.0)
    fx, fy, cx, cy = ref_colmap.intrinsics(0, [f, W / 2.0, H / 2.0])
    K = np.array([[fx, 0, cx], [0, fy, cy], [0, 0, 1]])
    rng = np.random.default_rng(12)
    R, _ = np.linalg.qr(rng.normal(size=(3, 3)))
    R *= np.sign(np.linalg.det(R))
    c2w = np.eye(4)
    c2w[:3, :3] = R
    c2w[:3, 3] = rng.normal(size=3) * 2.0
    cam = SimpleNamespace(K=torch.tensor(K[None], dtype=torch.float32),
                          c2w=torch.tensor(c2w[None], dtype=torch.float32))
    cam.K_inv = torch.linalg.inv(cam.K)
    cam.centers = cam.c2w[:, :3, 3]
    py, px = torch.meshgrid(torch.arange(H).float(), torch.arange(W).float(), indexing='ij')
    img = torch.zeros(H * W, dtype=torch.long)
    o, d = ref_colmap.ColmapScene.rays(cam, img, px.reshape(-1), py.reshape(-1))
    order = ref_bench_infer.tile_order(H, W)
    np.savez_compressed(os.path.join(HERE, 'camera_rays.npz'), W=W, H=H, fov=fov, centre=c2w[:3, 3], rot=R,
                        o=o.expand(H * W, 3).numpy(), d=d.numpy(), order=order.numpy())


def make_model_init():
    import model as ref_model
    g = torch.Generator().manual_seed(0)
    n = 200
    pts, colors = torch.rand(n, 3, generator=g), torch.rand(n, 3, generator=g) * 1.4 - 0.2
    spacing = torch.rand(n, generator=g) * 0.05
    spacing[3] = 0.0
    m = ref_model.VoronoiGaussField(pts, torch.zeros(n + 1, dtype=torch.int32), torch.zeros(0, dtype=torch.int32),
                                    colors, spacing, init_alpha=0.2, sh_deg=2)
    state = {f'state_{k}': v.numpy() for k, v in m.state_dict().items()}
    np.savez_compressed(os.path.join(HERE, 'model_init.npz'), points=pts.numpy(), colors=colors.numpy(),
                        spacing=spacing.numpy(), keys=np.array(list(m.state_dict())), **state)


MAKERS = {'sh_basis': make_sh_basis, 'conic': make_conic, 'foam_small': make_foam_small,
          'march_small': make_march_small, 'foam_config1': make_foam_config1, 'field_small': make_field_small,
          'ckpt_small': make_ckpt_small, 'render_host': make_render_host,
          'camera_rays': make_camera_rays, 'model_init': make_model_init}

if __name__ == '__main__':
    # python make_golden.py [name ...]: only the named fixtures (default all)
    for name in sys.argv[1:] or list(MAKERS):
        MAKERS[name]()
    print('fixtures written to', HERE)

