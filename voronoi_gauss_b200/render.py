"""Host-side callers of the hot path, with the reference's signatures (voronoi-gauss render.py).

* ``sphere_exit``, ``ray_bounds`` (render.py:16-25): near = const, mid = exit of the unit ball,
  far = exit of the far_radius ball (at least mid + 1e-3).
* ``render_rays_foam`` (render.py:127-140): conics of both Gaussians, ``ext.foam``, background composite
  ``fg + T sigmoid(bg_logit)``.
* ``render_rays_uniform`` (render.py:109-124): the same with ``ext.march`` and a conic floor of dt / 2.
* ``sh_basis``, ``morton_order``, ``pack_foam``, ``bake_colors``, ``render_rays_foam_infer``
  (render.py:143-257): the inference layout and its renderer.
* ``s_to_t``, ``sample_pdf``, ``composite``, ``proposal_weights``, ``resample``, ``render_rays``
  (render.py:28-106): the NeRF-style proposal sampler over the field kernels (``Graph.walk``,
  ``ext.density``, ``ext.color``): 64 stratified samples in a normalised ray coordinate s (linear in t
  inside the unit ball, linear in disparity beyond), two gradient-free proposal passes with widened
  density Gaussians, then the merged samples walked to their sites and rendered with gradients.
* ``render_image`` (render.py:260-266).
"""

from __future__ import annotations

import math

import torch

from . import ext


def sphere_exit(o, d, radius):
    b = (o * d).sum(-1)
    c = (o * o).sum(-1) - radius * radius
    return -b + (b * b - c).clamp_min(0).sqrt()


def ray_bounds(o, d, near, far_radius):
    t_mid = sphere_exit(o, d, 1.0).clamp_min(near + 1e-3)
    t_far = torch.maximum(sphere_exit(o, d, far_radius), t_mid + 1e-3)
    return torch.full_like(t_mid, near), t_mid, t_far


def s_to_t(s, t_near, t_mid, t_far):
    """Ray depth of the normalised coordinate s in [0, 1] (render.py:28-33): s < 1/2 maps linearly onto
    [near, mid], s >= 1/2 linearly in disparity onto [mid, far]."""
    t_near, t_mid, t_far = t_near[:, None], t_mid[:, None], t_far[:, None]
    inside = t_near + (t_mid - t_near) * (2 * s).clamp(max=1)
    u = (2 * s - 1).clamp(min=0)
    beyond = 1.0 / (1.0 / t_mid + u * (1.0 / t_far - 1.0 / t_mid))
    return torch.where(s < 0.5, inside, beyond)


def sample_pdf(bins, weights, n, det=True):
    """n samples per row from the piecewise-constant density of `weights` over `bins` (render.py:36-50):
    inverse-CDF sampling at stratified midpoints (det) or uniform draws."""
    w = weights + 1e-5
    cdf = torch.cumsum(w / w.sum(-1, keepdim=True), -1)
    cdf = torch.cat([torch.zeros_like(cdf[:, :1]), cdf], -1)
    if det:
        u = torch.linspace(0.5 / n, 1 - 0.5 / n, n, device=bins.device).expand(len(bins), n).contiguous()
    else:
        u = torch.rand(len(bins), n, device=bins.device)
    hi = torch.searchsorted(cdf, u, right=True)
    lo = (hi - 1).clamp_min(0)
    hi = hi.clamp_max(cdf.shape[-1] - 1)
    c0, c1 = cdf.gather(1, lo), cdf.gather(1, hi)
    b0, b1 = bins.gather(1, lo), bins.gather(1, hi)
    span = c1 - c0
    span = torch.where(span < 1e-5, torch.ones_like(span), span)
    return b0 + (u - c0) / span * (b1 - b0)


def composite(sigma, t, t_far):
    """Front-to-back weights of point samples (render.py:53-57): the last interval runs to t_far;
    returns (weights (B, S), final transmittance (B))."""
    delta = torch.cat([t[:, 1:] - t[:, :-1], (t_far[:, None] - t[:, -1:]).clamp_min(0)], 1)
    alpha = 1.0 - torch.exp(-sigma * delta)
    trans = torch.cumprod(torch.cat([torch.ones_like(alpha[:, :1]), 1.0 - alpha + 1e-10], 1), 1)
    return alpha * trans[:, :-1], trans[:, -1]


def proposal_weights(model, o, d, s, bounds, start, scale_mult):
    """Compositing weights of samples s under the density widened by scale_mult, without gradients
    (render.py:60-68)."""
    t = s_to_t(s, *bounds)
    site, _ = model.walk(o, d, t, start)
    x = (o[:, None] + d[:, None] * t[..., None]).reshape(-1, 3)
    with torch.no_grad():
        sigma = ext.density(model.graph, model.raw, model.d_log_scale, model.d_quat, x, site.reshape(-1),
                            scale_mult).view_as(t)
    w, _ = composite(sigma, t, bounds[2])
    return w


def resample(s, w, n, det):
    """n new samples drawn from the weights w of the sorted samples s (render.py:71-74)."""
    mid = 0.5 * (s[:, 1:] + s[:, :-1])
    bins = torch.cat([torch.zeros_like(s[:, :1]), mid, torch.ones_like(s[:, :1])], 1)
    return sample_pdf(bins, w, n, det)


def render_rays(model, o, d, start, n_coarse=64, n_fine=(64, 64), proposal_mult=(4.0, 2.0), near=0.02,
                far_radius=4.0, perturb=True, min_weight=1e-4):
    """NeRF-style rendering (render.py:77-106): o, d (B, 3) rays, start (B,) the site containing each
    origin -> dict with rgb (B, 3), acc, depth and sampler statistics. Colours are evaluated only for the
    samples with weight > min_weight."""
    B = len(o)
    bounds = ray_bounds(o, d, near, far_radius)
    s = torch.linspace(0, 1, n_coarse + 1, device=o.device)[:-1].expand(B, n_coarse)
    s = s + (torch.rand_like(s) if perturb else 0.5) / n_coarse
    with torch.no_grad():
        for n, mult in zip(n_fine, proposal_mult):
            w = proposal_weights(model, o, d, s, bounds, start, mult)
            s, _ = torch.sort(torch.cat([s, resample(s, w, n, det=not perturb)], 1), 1)
        t = s_to_t(s, *bounds)
        site, steps = model.walk(o, d, t, start)
    S = t.shape[1]
    x = (o[:, None] + d[:, None] * t[..., None]).reshape(-1, 3)
    site = site.reshape(-1)
    sigma = ext.density(model.graph, model.raw, model.d_log_scale, model.d_quat, x, site).view(B, S)
    w, t_final = composite(sigma, t, bounds[2])
    active = (w.detach() > min_weight).reshape(-1).nonzero().squeeze(1)
    dirs = d[:, None].expand(B, S, 3).reshape(-1, 3)
    c = ext.color(model.graph, model.c_log_scale, model.c_quat, model.sh(), x[active], dirs[active], site[active],
                  model.sh_deg)
    rgb_s = torch.zeros(B * S, 3, device=o.device, dtype=c.dtype).index_put((active,), c).view(B, S, 3)
    rgb = (w[..., None] * rgb_s).sum(1) + t_final[:, None] * torch.sigmoid(model.bg_logit)
    return {'rgb': rgb, 'acc': 1.0 - t_final, 'depth': (w * t).sum(1), 'walk_steps': steps.float().mean() / S,
            'active': len(active) / (B * S)}


def render_rays_uniform(model, o, d, start, dt=1 / 512, n_bg=64, near=0.02, far_radius=4.0, t_thresh=1e-4,
                        w_thresh=1e-4, scale_floor=None, perturb=False):
    """Fixed steps dt inside the unit ball, n_bg steps uniform in disparity beyond it, early termination at
    T < t_thresh, in one fused kernel; scale_floor (default dt / 2) is added in quadrature to every scale."""
    near_t, mid_t, far_t = ray_bounds(o, d, near, far_radius)
    floor = 0.5 * dt if scale_floor is None else scale_floor
    dA = ext.conic(model.d_log_scale, model.d_quat, floor)
    cA = ext.conic(model.c_log_scale, model.c_quat, floor)
    fg, T, depth, stats = ext.march(model.graph, model.raw, dA, cA, model.sh(), model.sh_deg, o, d, start, near_t,
                                    mid_t, far_t, dt, n_bg, t_thresh, w_thresh)
    rgb = fg + T[:, None] * torch.sigmoid(model.bg_logit)
    stats = stats.float()
    return {'rgb': rgb, 'acc': 1.0 - T, 'depth': depth, 'samples': stats[:, 0].mean(),
            'active': (stats[:, 1].sum() / stats[:, 0].sum()).item(),
            'walk_steps': stats[:, 2].sum() / stats[:, 0].sum()}


def render_rays_foam(model, o, d, start, near=0.02, far_radius=4.0, t_thresh=1e-4, w_thresh=1e-4, scale_floor=0.0,
                     perturb=False):
    """Samples at the interaction points of each ray with the Voronoi faces (plus x(near) and x(far)), segments
    composited with the trapezoid rule in one fused kernel."""
    near_t, _, far_t = ray_bounds(o, d, near, far_radius)
    dA = ext.conic(model.d_log_scale, model.d_quat, scale_floor)
    cA = ext.conic(model.c_log_scale, model.c_quat, scale_floor)
    fg, T, depth, stats = ext.foam(model.graph, model.raw, dA, cA, model.sh(), model.sh_deg, o, d, start, near_t,
                                   far_t, t_thresh, w_thresh)
    rgb = fg + T[:, None] * torch.sigmoid(model.bg_logit)
    stats = stats.float()
    segments = (stats[:, 0] - 1).sum().clamp_min(1)
    return {'rgb': rgb, 'acc': 1.0 - T, 'depth': depth, 'samples': stats[:, 0].mean(),
            'active': (stats[:, 1].sum() / segments).item(), 'walk_steps': stats[:, 2].mean()}


def sh_basis(d, deg):
    """Real SH basis (B, 16) of unit directions d (B, 3), the kernels' constants and signs."""
    x, y, z = d.unbind(-1)
    b = torch.zeros(len(d), 16, device=d.device, dtype=d.dtype)
    b[:, 0] = 0.28209479177387814
    if deg >= 1:
        b[:, 1], b[:, 2], b[:, 3] = -0.4886025119029199 * y, 0.4886025119029199 * z, -0.4886025119029199 * x
    if deg >= 2:
        xx, yy, zz = x * x, y * y, z * z
        b[:, 4] = 1.0925484305920792 * x * y
        b[:, 5] = -1.0925484305920792 * y * z
        b[:, 6] = 0.31539156525252005 * (2 * zz - xx - yy)
        b[:, 7] = -1.0925484305920792 * x * z
        b[:, 8] = 0.5462742152960396 * (xx - yy)
    if deg >= 3:
        b[:, 9] = -0.5900435899266435 * y * (3 * xx - yy)
        b[:, 10] = 2.890611442640554 * x * y * z
        b[:, 11] = -0.4570457994644658 * y * (4 * zz - xx - yy)
        b[:, 12] = 0.3731763325901154 * z * (2 * zz - 3 * xx - 3 * yy)
        b[:, 13] = -0.4570457994644658 * x * (4 * zz - xx - yy)
        b[:, 14] = 1.445305721320277 * z * (xx - yy)
        b[:, 15] = -0.5900435899266435 * x * (xx - 3 * yy)
    return b


def morton_order(points, bits=10):
    """Permutation sorting the points along a Z-order curve of their bounding box (render.py:168-176); equal
    codes keep index order."""
    lo, hi = points.amin(0), points.amax(0)
    q = ((points - lo) / (hi - lo).clamp_min(1e-12) * (2 ** bits - 1)).long()
    code = torch.zeros(len(points), dtype=torch.long, device=points.device)
    for b in range(bits):
        for a in range(3):
            code |= ((q[:, a] >> b) & 1) << (3 * b + a)
    return torch.argsort(code, stable=True)


@torch.no_grad()
def pack_foam(model, scale_floor=0.0, eps_density=0.0, sh_half=False, reorder=False):
    """Records of the inference renderer (render.py:179-225), built on the device by vg_infer_pack:
    self-first neighbourhoods (offsets (N + 1), nbr (E)) with one float4 per edge = (p_j, half2(r2_j,
    lam_j)); r2 the squared distance beyond which rho_j G_j < eps_density (inf when eps_density = 0), lam
    the smallest eigenvalue of the colour conic, both rounded to the safe side; attr (N, 20) = (density
    conic, min(raw, 30), 0, colour conic, 0, 0, baked rgb, 0); sh (N, 16, 3) fp32 or fp16. reorder renumbers
    the sites along a Z-order curve (perm: new -> old, inv: old -> new; orig = perm breaks ties as before
    the renumbering)."""
    from . import _lib
    g = model.graph
    n, m = len(g.points), len(g.adj)
    dev = g.points.device
    if dev.type != 'cuda':
        raise RuntimeError('pack_foam needs the scene on a CUDA device')
    f = [t.detach().float().contiguous() for t in (model.raw, model.d_log_scale, model.d_quat, model.c_log_scale,
                                                    model.c_quat, model.sh())]
    points = torch.empty(n, 4, device=dev)
    offsets = torch.empty(n + 1, dtype=torch.int32, device=dev)
    nbr = torch.empty(n + m, dtype=torch.int32, device=dev)
    edge = torch.empty(n + m, 4, device=dev)
    attr = torch.empty(n, 20, device=dev)
    sh = torch.empty(n, 16, 3, dtype=torch.float16 if sh_half else torch.float32, device=dev)
    sh32 = torch.empty(n, 16, 3, device=dev)
    orig = torch.empty(n if reorder else 0, dtype=torch.int32, device=dev)
    nbytes = _lib.lib().vg_infer_pack_workspace_bytes(n)
    ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    pk = g.pack if reorder else None
    with torch.cuda.device(dev):
        _lib.call('vg_infer_pack', pk.ptr if pk is not None else None, n, m, g.points.data_ptr(),
                  g.offsets.data_ptr(), g.adj.data_ptr() if m else None, *(t.data_ptr() for t in f),
                  float(scale_floor), float(eps_density), int(sh_half), int(reorder), points.data_ptr(),
                  offsets.data_ptr(), nbr.data_ptr(), edge.data_ptr(), attr.data_ptr(), sh.data_ptr(),
                  sh32.data_ptr(), orig.data_ptr() if reorder else None, ws.data_ptr(), nbytes,
                  torch.cuda.current_stream(dev).cuda_stream)
    perm = inv = None
    if reorder:
        perm = orig.long()
        inv = torch.empty_like(perm)
        inv[perm] = torch.arange(n, device=dev)
    return {'points': points, 'offsets': offsets, 'nbr': nbr, 'edge': edge, 'attr': attr, 'sh': sh, 'sh32': sh32,
            'perm': perm, 'inv': inv, 'orig': orig, 'baked_center': None}


@torch.no_grad()
def bake_colors(model, pack, center):
    """Site colours max(SH_k(d_k) + 1/2, 0) for the direction d_k from the camera centre to site k
    (render.py:228-235), written into pack['attr'][:, 16:19] on the device (vg_bake_colors)."""
    from . import _lib
    c = [float(v) for v in center.reshape(-1).tolist()]
    n = len(pack['points'])
    dev = pack['points'].device
    with torch.cuda.device(dev):
        _lib.call('vg_bake_colors', pack['points'].data_ptr(), pack['sh32'].data_ptr(), int(model.sh_deg), n, *c,
                  pack['attr'].data_ptr(), torch.cuda.current_stream(dev).cuda_stream)
    pack['baked_center'] = center


@torch.no_grad()
def render_rays_foam_infer(model, pack, o, d, start, near=0.02, far_radius=4.0, t_thresh=1e-4, w_thresh=1e-4,
                           colors='exact', eps_color=0.0, stage=2, cap=None):
    """Inference version of render_rays_foam (render.py:238-257): colors 'exact' (lazy second pass for the
    segments with weight > w_thresh), 'fused' (blended in the density pass) or 'baked' (bake_colors). Per-ray
    stats (B, 5): samples, coloured segments, walk steps, density Gaussians evaluated, SH evaluated."""
    near_t, _, far_t = ray_bounds(o, d, near, far_radius)
    cap = torch.empty(0, dtype=torch.int32, device=o.device) if cap is None else cap.int().contiguous()
    if pack['inv'] is not None:
        start = pack['inv'][start.long()]
    color_cut = 2 * math.log(1 / eps_color) if eps_color > 0 else float('inf')
    fg, T, depth, stats = ext.foam_infer_extension().foam_infer(
        pack['points'], pack['offsets'], pack['nbr'], pack['edge'], pack['attr'], pack['sh'], model.sh_deg,
        o.float().contiguous(), d.float().contiguous(), start.int().contiguous(), near_t.contiguous(),
        far_t.contiguous(), float(t_thresh), float(w_thresh), color_cut, {'exact': 0, 'baked': 1, 'fused': 2}[colors],
        int(stage), cap, pack['orig'])
    rgb = fg + T[:, None] * torch.sigmoid(model.bg_logit)
    return {'rgb': rgb, 'acc': 1.0 - T, 'depth': depth, 'stats': stats}


@torch.no_grad()
def render_image(model, scene, i, start, chunk=8192, renderer=render_rays, **kw):
    """Renders image i of a scene with .image_rays(i) -> (o, d, gt) and .H, .W (render.py:260-266)."""
    o, d, gt = scene.image_rays(i)
    start = torch.full((len(o),), int(start), dtype=torch.int32, device=o.device)
    out = [renderer(model, o[j:j + chunk], d[j:j + chunk], start[j:j + chunk], perturb=False, **kw)['rgb']
           for j in range(0, len(o), chunk)]
    return torch.cat(out).view(scene.H, scene.W, 3).clamp(0, 1), gt
