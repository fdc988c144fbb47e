"""Host-side callers of the hot path, with the reference's signatures (voronoi-gauss render.py).

* ``sphere_exit``, ``ray_bounds`` (render.py:16-25): near = const, mid = exit of the unit ball,
  far = exit of the far_radius ball (at least mid + 1e-3).
* ``s_to_t``, ``sample_pdf``, ``composite``, ``proposal_weights``, ``resample``, ``render_rays``
  (render.py:28-106): the NeRF-style proposal sampler over the field kernels (``Graph.walk``,
  ``ext.density``, ``ext.color``): 64 stratified samples in a normalised ray coordinate s (linear in t
  inside the unit ball, linear in disparity beyond), two gradient-free proposal passes with widened
  density Gaussians, then the merged samples walked to their sites and rendered with gradients.
* ``render_rays_uniform`` (render.py:109-124) and ``render_rays_foam`` (render.py:127-140): conics of
  both Gaussians, the fused ``ext.march`` / ``ext.foam`` renderers, background composite
  ``fg + T sigmoid(bg_logit)``.
* ``sh_basis``, ``morton_order``, ``pack_foam``, ``bake_colors``, ``render_rays_foam_infer``
  (render.py:143-257): the inference layout (built on the device) and its renderer.
* ``render_image`` (render.py:260-266).

The sampler arithmetic is written so that every float32 operation matches the reference's, in value and
order: the sample positions decide which Voronoi cells the walk visits, so they are bit-identical.
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F

from . import ext

_GAP = 1e-3  # minimum distances near -> mid -> far


# ------------------------------------------------------------------------------- ray coordinates

def sphere_exit(o, d, radius):
    """Distance along unit d from o to where the ray leaves the origin-centred ball of `radius`: the larger
    root of |o + t d|^2 = radius^2, with the discriminant clamped at 0 for rays that miss the ball."""
    half_b = (o * d).sum(-1)
    c = (o * o).sum(-1) - radius * radius
    return torch.sqrt(torch.clamp(half_b * half_b - c, min=0)) - half_b


def ray_bounds(o, d, near, far_radius):
    """(near, mid, far) per ray: the constant near plane, mid where the ray leaves the unit ball (at least
    1e-3 beyond near), far where it leaves the far_radius ball (at least 1e-3 beyond mid)."""
    mid = torch.clamp(sphere_exit(o, d, 1.0), min=near + _GAP)
    far = torch.max(sphere_exit(o, d, far_radius), mid + _GAP)
    return mid.new_full(mid.shape, near), mid, far


def s_to_t(s, t_near, t_mid, t_far):
    """Ray depth of the normalised coordinate s in [0, 1]: the first half maps linearly in t onto
    [near, mid], the second half linearly in 1/t onto [mid, far]."""
    near, mid, far = (b.unsqueeze(1) for b in (t_near, t_mid, t_far))
    two_s = 2 * s
    inside = near + (mid - near) * torch.clamp(two_s, max=1)
    inv_mid = 1.0 / mid
    beyond = 1.0 / (inv_mid + torch.clamp(two_s - 1, min=0) * (1.0 / far - inv_mid))
    return torch.where(s < 0.5, inside, beyond)


def _points(o, d, t):
    """Sample positions o + t d of every (ray, sample), flattened to (B S, 3)."""
    return (o.unsqueeze(1) + d.unsqueeze(1) * t.unsqueeze(2)).reshape(-1, 3)


# ------------------------------------------------------------------------------- proposal sampler

def sample_pdf(bins, weights, n, det=True):
    """n draws per row from the piecewise-constant density that `weights` (plus 1e-5) put on the intervals
    of `bins`, by inverting its CDF at the n stratified midpoints (det) or at uniform random points."""
    w = weights + 1e-5
    cdf = F.pad(torch.cumsum(w / w.sum(-1, keepdim=True), -1), (1, 0))
    rows, last = len(bins), cdf.shape[-1] - 1
    if det:
        u = torch.linspace(0.5 / n, 1 - 0.5 / n, n, device=bins.device).expand(rows, n).contiguous()
    else:
        u = torch.rand(rows, n, device=bins.device)
    right = torch.searchsorted(cdf, u, right=True)
    lo, hi = torch.clamp(right - 1, min=0), torch.clamp(right, max=last)
    c_lo, c_hi = cdf.gather(1, lo), cdf.gather(1, hi)
    span = c_hi - c_lo
    span = torch.where(span < 1e-5, torch.ones_like(span), span)
    x_lo = bins.gather(1, lo)
    return x_lo + (u - c_lo) / span * (bins.gather(1, hi) - x_lo)


def composite(sigma, t, t_far):
    """Front-to-back weights of point samples: sample k stands for [t_k, t_k+1) (the last one up to t_far,
    empty past it), alpha_k = 1 - exp(-sigma_k dt_k), w_k = alpha_k prod_{j<k} (1 - alpha_j + 1e-10).
    -> (weights (B, S), transmittance after the last sample (B,))."""
    ends = torch.cat([t[:, 1:], torch.max(t_far.unsqueeze(1), t[:, -1:])], 1)
    alpha = 1.0 - torch.exp(-sigma * (ends - t))
    trans = torch.cumprod(F.pad(1.0 - alpha + 1e-10, (1, 0), value=1.0), 1)
    return alpha * trans[:, :-1], trans[:, -1]


def _sigma(model, x, site, scale_mult=1.0):
    return ext.density(model.graph, model.raw, model.d_log_scale, model.d_quat, x, site, scale_mult)


def proposal_weights(model, o, d, s, bounds, start, scale_mult):
    """Compositing weights of the samples s under the density widened by scale_mult, without gradients."""
    t = s_to_t(s, *bounds)
    site, _ = model.walk(o, d, t, start)
    with torch.no_grad():
        sigma = _sigma(model, _points(o, d, t), site.reshape(-1), scale_mult).view_as(t)
    return composite(sigma, t, bounds[2])[0]


def resample(s, w, n, det):
    """n new values of s drawn from the weights w of the sorted samples s, over bins that split [0, 1] at
    the midpoints between consecutive samples."""
    mids = 0.5 * (s[:, 1:] + s[:, :-1])
    return sample_pdf(F.pad(F.pad(mids, (1, 0), value=0.0), (0, 1), value=1.0), w, n, det)


def _refine(model, o, d, s, bounds, start, n_fine, proposal_mult, det):
    """The gradient-free proposal passes: each adds n draws from the widened-density weights of the
    current samples and keeps the merged set sorted."""
    for n, mult in zip(n_fine, proposal_mult):
        drawn = resample(s, proposal_weights(model, o, d, s, bounds, start, mult), n, det)
        s = torch.sort(torch.cat([s, drawn], 1), 1)[0]
    return s


def render_rays(model, o, d, start, n_coarse=64, n_fine=(64, 64), proposal_mult=(4.0, 2.0), near=0.02,
                far_radius=4.0, perturb=True, min_weight=1e-4):
    """NeRF-style rendering (render.py:77-106): o, d (B, 3) rays, start (B,) the site containing each
    origin -> dict with rgb (B, 3), acc, depth and sampler statistics (walk_steps per sample, active
    fraction). Colours are evaluated only for the samples with weight > min_weight."""
    B = len(o)
    bounds = ray_bounds(o, d, near, far_radius)
    grid = torch.linspace(0, 1, n_coarse + 1, device=o.device)[:-1].expand(B, n_coarse)
    s = grid + (torch.rand_like(grid) if perturb else 0.5) / n_coarse
    with torch.no_grad():
        s = _refine(model, o, d, s, bounds, start, n_fine, proposal_mult, not perturb)
        t = s_to_t(s, *bounds)
        site, steps = model.walk(o, d, t, start)
    S = t.shape[1]
    x, site = _points(o, d, t), site.reshape(-1)
    w, t_last = composite(_sigma(model, x, site).view(B, S), t, bounds[2])
    lit = torch.nonzero((w.detach() > min_weight).reshape(-1)).squeeze(1)
    dirs = d.unsqueeze(1).expand(B, S, 3).reshape(-1, 3)
    c = ext.color(model.graph, model.c_log_scale, model.c_quat, model.sh(), x[lit], dirs[lit], site[lit],
                  model.sh_deg)
    sample_rgb = c.new_zeros(B * S, 3).index_put((lit,), c).view(B, S, 3)
    rgb = _over_background(model, (w.unsqueeze(-1) * sample_rgb).sum(1), t_last)
    return {'rgb': rgb, 'acc': 1.0 - t_last, 'depth': (w * t).sum(1), 'walk_steps': steps.float().mean() / S,
            'active': len(lit) / (B * S)}


# ------------------------------------------------------------------------------- fused renderers

def _over_background(model, fg, T):
    """fg + T sigmoid(bg_logit): the learned background behind what the rays leave unabsorbed."""
    return fg + T.unsqueeze(1) * torch.sigmoid(model.bg_logit)


def _conics(model, floor):
    return (ext.conic(model.d_log_scale, model.d_quat, floor), ext.conic(model.c_log_scale, model.c_quat, floor))


def render_rays_uniform(model, o, d, start, dt=1 / 512, n_bg=64, near=0.02, far_radius=4.0, t_thresh=1e-4,
                        w_thresh=1e-4, scale_floor=None, perturb=False):
    """Fixed steps dt inside the unit ball, n_bg steps uniform in disparity beyond it, early termination at
    T < t_thresh, in one fused kernel; scale_floor (default dt / 2) is added in quadrature to every scale.
    Statistics per marched sample: active (coloured) fraction and walk steps."""
    bounds = ray_bounds(o, d, near, far_radius)
    dA, cA = _conics(model, 0.5 * dt if scale_floor is None else scale_floor)
    fg, T, depth, stats = ext.march(model.graph, model.raw, dA, cA, model.sh(), model.sh_deg, o, d, start, *bounds,
                                    dt, n_bg, t_thresh, w_thresh)
    samples, coloured, walks = stats.float().unbind(1)
    return {'rgb': _over_background(model, fg, T), 'acc': 1.0 - T, 'depth': depth, 'samples': samples.mean(),
            'active': (coloured.sum() / samples.sum()).item(), 'walk_steps': walks.sum() / samples.sum()}


def render_rays_foam(model, o, d, start, near=0.02, far_radius=4.0, t_thresh=1e-4, w_thresh=1e-4, scale_floor=0.0,
                     perturb=False):
    """Samples at the interaction points of each ray with the Voronoi faces (plus x(near) and x(far)), segments
    composited with the trapezoid rule in one fused kernel. Statistics: samples per ray, coloured fraction of
    the segments, walk steps to x(near) per ray."""
    t_near, _, t_far = ray_bounds(o, d, near, far_radius)
    dA, cA = _conics(model, scale_floor)
    fg, T, depth, stats = ext.foam(model.graph, model.raw, dA, cA, model.sh(), model.sh_deg, o, d, start, t_near,
                                   t_far, t_thresh, w_thresh)
    samples, coloured, walks = stats.float().unbind(1)
    segments = torch.clamp((samples - 1).sum(), min=1)
    return {'rgb': _over_background(model, fg, T), 'acc': 1.0 - T, 'depth': depth, 'samples': samples.mean(),
            'active': (coloured.sum() / segments).item(), 'walk_steps': walks.mean()}


# ------------------------------------------------------------------------------- inference layout

# Real SH basis up to degree 3 (render.py:143-165; the kernels' constants and signs): band l has the
# normalisation constants below, the Cartesian polynomials are those of the standard real basis.
_SH_C = (0.28209479177387814, 0.4886025119029199, 1.0925484305920792, 0.31539156525252005, 0.5462742152960396,
         0.5900435899266435, 2.890611442640554, 0.4570457994644658, 0.3731763325901154, 1.445305721320277)


def sh_basis(d, deg):
    """Real SH basis (B, 16) of unit directions d (B, 3); the functions above degree `deg` are zero."""
    c = _SH_C
    x, y, z = d.unbind(-1)
    cols = [torch.full_like(x, c[0])]
    if deg >= 1:
        cols += [-c[1] * y, c[1] * z, -c[1] * x]
    if deg >= 2:
        xx, yy, zz = x * x, y * y, z * z
        cols += [c[2] * x * y, -c[2] * y * z, c[3] * (2 * zz - xx - yy), -c[2] * x * z, c[4] * (xx - yy)]
    if deg >= 3:
        cols += [-c[5] * y * (3 * xx - yy), c[6] * x * y * z, -c[7] * y * (4 * zz - xx - yy),
                 c[8] * z * (2 * zz - 3 * xx - 3 * yy), -c[7] * x * (4 * zz - xx - yy), c[9] * z * (xx - yy),
                 -c[5] * x * (xx - 3 * yy)]
    cols += [torch.zeros_like(x)] * (16 - len(cols))
    return torch.stack(cols, -1)


def morton_order(points, bits=10):
    """Permutation sorting the points along a Z-order curve of their bounding box (render.py:168-176):
    each coordinate quantised to `bits` bits over the box, bit b of axis a placed at bit 3 b + a of the
    code; equal codes keep index order."""
    lo, hi = points.amin(0), points.amax(0)
    q = ((points - lo) / (hi - lo).clamp_min(1e-12) * (2 ** bits - 1)).long()
    level = torch.arange(bits, device=points.device)
    axis = torch.arange(3, device=points.device)
    digits = (q.unsqueeze(2) >> level) & 1                        # (N, 3, bits)
    code = (digits << (3 * level + axis.unsqueeze(1))).sum((1, 2))
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
    trace = ext.trace_records(nbr, edge, attr, n)  # the deferred renderer's per-edge records
    return {'points': points, 'offsets': offsets, 'nbr': nbr, 'edge': edge, 'attr': attr, 'sh': sh, 'sh32': sh32,
            'perm': perm, 'inv': inv, 'orig': orig, 'baked_center': None, 'trace': trace}


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
                           colors='exact', eps_color=0.0, stage=2, cap=None, exact_stats=False):
    """Inference version of render_rays_foam (render.py:238-257): colors 'exact' (lazy second pass for the
    segments with weight > w_thresh), 'fused' (blended in the density pass) or 'baked' (bake_colors), the
    neighbours below eps_color of the normalised colour weight skipped. Per-ray stats (B, 5): samples,
    coloured segments, walk steps, density Gaussians evaluated, SH evaluated (colours are deferred to a
    cell-major pass, whose SH count is reported; exact_stats=True renders per ray with the reference's
    per-ray colour cache and its SH count, same image)."""
    mode = {'exact': 0, 'baked': 1, 'fused': 2}[colors]
    t_near, _, t_far = ray_bounds(o, d, near, far_radius)
    if cap is None:
        cap = torch.empty(0, dtype=torch.int32, device=o.device)
    if pack['inv'] is not None:  # start sites in the renumbered order of the pack
        start = pack['inv'][start.long()]
    # a neighbour whose colour weight exp(-(m - m_min) / 2) is below eps_color is skipped:
    # m - m_min > 2 ln(1 / eps_color)
    skip_beyond = 2 * math.log(1 / eps_color) if eps_color > 0 else float('inf')
    layout = [pack[k] for k in ('points', 'offsets', 'nbr', 'edge', 'attr', 'sh')]
    rays = [o.float().contiguous(), d.float().contiguous(), start.int().contiguous(), t_near.contiguous(),
            t_far.contiguous()]
    fg, T, depth, stats = ext.foam_infer_extension().foam_infer(*layout, model.sh_deg, *rays, float(t_thresh),
                                                                float(w_thresh), skip_beyond, mode, int(stage),
                                                                cap.int().contiguous(), pack['orig'],
                                                                exact_stats=exact_stats, trace=pack.get('trace'))
    return {'rgb': _over_background(model, fg, T), 'acc': 1.0 - T, 'depth': depth, 'stats': stats}


@torch.no_grad()
def render_image(model, scene, i, start, chunk=8192, renderer=render_rays, **kw):
    """Image i of a scene with .image_rays(i) -> (o, d, gt) and .H, .W (render.py:260-266), rendered in
    chunks of rays from the start site `start`. -> (rgb (H, W, 3) in [0, 1], gt)."""
    o, d, gt = scene.image_rays(i)
    first = torch.full((len(o),), int(start), dtype=torch.int32, device=o.device)
    parts = []
    for a in range(0, len(o), chunk):
        b = a + chunk
        parts.append(renderer(model, o[a:b], d[a:b], first[a:b], perturb=False, **kw)['rgb'])
    return torch.cat(parts).view(scene.H, scene.W, 3).clamp(0, 1), gt
