"""Seeded synthetic scenes and orbit cameras for the five benchmark configurations.

The reference trains on Mip-NeRF 360 / Deep Blending COLMAP scenes, which are not available; these
generators stand in for them with the shapes, sizes and value distributions of the configurations:

1. tiny: 10k sites uniform in [-1, 1]^3 (seed 0), sh_deg 1, 4 orbit cameras at 64x64.
2. inference: 1M sites from a mixture of 64 anisotropic Gaussians, sh_deg 3, 800x800, 100 cameras.
3. training: 3M sites, 70 % within 0.01 of a union of 32 spheres and 30 % uniform, 1920x1080.
4. 8-GPU training: the same distribution with 8M sites, 3840x2160.
5. march: the config-2 scene, 256 steps of 2/256 through the unit ball, 1920x1080.

Per-site parameters follow the reference model's parameterisation (model.py:19-39): raw (density
log-rho, used as exp(min(raw, 30))), density and colour log-scales (N, 3) and quaternions (N, 4), and
SH (N, 16, 3) with the unused bands zero. Cameras are pinhole, looking at the origin from an orbit of
radius 3, with rays built by the formula of colmap.py:129-134 (pixel centre + 0.5, normalised d).
Scenes are cached as .npz files keyed by configuration and seed.
"""

from __future__ import annotations

import math
import os

import numpy as np
import torch

from . import sites

C0 = 0.28209479177387814

CONFIGS = {
    1: dict(name='tiny-10k', n=10_000, kind='uniform', sh_deg=1, W=64, H=64, n_cams=4, fov=50.0),
    2: dict(name='mixture-1M', n=1_000_000, kind='mixture', sh_deg=3, W=800, H=800, n_cams=100, fov=50.0),
    3: dict(name='surface-3M', n=3_000_000, kind='surface', sh_deg=3, W=1920, H=1080, n_cams=1, fov=50.0),
    4: dict(name='surface-8M', n=8_000_000, kind='surface', sh_deg=3, W=3840, H=2160, n_cams=1, fov=50.0),
    5: dict(name='mixture-1M-march', n=1_000_000, kind='mixture', sh_deg=3, W=1920, H=1080, n_cams=1,
            fov=50.0),
}


def _random_rotations(rng, n):
    """n rotation matrices of uniformly random unit quaternions (w, x, y, z), built from the quaternion's
    pairwise products."""
    q = rng.normal(size=(n, 4))
    q /= np.linalg.norm(q, axis=1, keepdims=True)
    w, x, y, z = q.T
    xx, yy, zz, xy, xz, yz, wx, wy, wz = x * x, y * y, z * z, x * y, x * z, y * z, w * x, w * y, w * z
    rows = (1 - 2 * (yy + zz), 2 * (xy - wz), 2 * (xz + wy),
            2 * (xy + wz), 1 - 2 * (xx + zz), 2 * (yz - wx),
            2 * (xz - wy), 2 * (yz + wx), 1 - 2 * (xx + yy))
    return np.stack(rows, -1).reshape(n, 3, 3)


def uniform_points(n, seed=0):
    return np.random.default_rng(seed).uniform(-1, 1, (n, 3))


def mixture_points(n, seed=0, clusters=64):
    """64 anisotropic Gaussian clusters (centres U[-0.8, 0.8]^3, per-axis sigma U[0.05, 0.3], random
    rotation), rejection-sampled to [-1, 1]^3."""
    rng = np.random.default_rng(seed)
    centres = rng.uniform(-0.8, 0.8, (clusters, 3))
    sig = rng.uniform(0.05, 0.3, (clusters, 3))
    rot = _random_rotations(rng, clusters)
    out, have = [], 0
    while have < n:
        m = int((n - have) * 1.3) + 1024
        c = rng.integers(0, clusters, m)
        z = rng.normal(size=(m, 3)) * sig[c]
        p = np.einsum('mij,mj->mi', rot[c], z) + centres[c]
        p = p[(np.abs(p) <= 1.0).all(1)]
        out.append(p)
        have += len(p)
    return np.concatenate(out)[:n]


def surface_points(n, seed=0, spheres=32, surface_frac=0.7, offset=0.01):
    """70 % of the sites on the surface of a union of 32 spheres (centres U[-0.6, 0.6]^3, radii
    U[0.1, 0.4]; sphere points not inside another sphere) moved by U(0, 0.01) along a random
    direction, 30 % uniform in [-1, 1]^3."""
    rng = np.random.default_rng(seed)
    centres = rng.uniform(-0.6, 0.6, (spheres, 3))
    radii = rng.uniform(0.1, 0.4, spheres)
    n_surf = int(round(n * surface_frac))
    area = radii ** 2
    out, have = [], 0
    while have < n_surf:
        m = int((n_surf - have) * 1.6) + 1024
        s = rng.choice(spheres, m, p=area / area.sum())
        u = rng.normal(size=(m, 3))
        u /= np.linalg.norm(u, axis=1, keepdims=True)
        p = centres[s] + radii[s, None] * u
        inside = np.zeros(m, dtype=bool)
        for k in range(spheres):
            dk = np.linalg.norm(p - centres[k], axis=1)
            inside |= (dk < radii[k] - 1e-9) & (s != k)
        p = p[~inside]
        out.append(p)
        have += len(p)
    surf = np.concatenate(out)[:n_surf]
    dirs = rng.normal(size=(n_surf, 3))
    dirs /= np.linalg.norm(dirs, axis=1, keepdims=True)
    surf = surf + dirs * rng.uniform(0.0, offset, (n_surf, 1))
    uni = rng.uniform(-1, 1, (n - n_surf, 3))
    pts = np.concatenate([surf, uni])
    return pts[rng.permutation(len(pts))]


def make_points(cfg, seed=0, n=None):
    c = CONFIGS[cfg]
    n = c['n'] if n is None else n
    if c['kind'] == 'uniform':
        return uniform_points(n, seed)
    if c['kind'] == 'mixture':
        return mixture_points(n, seed)
    return surface_points(n, seed)


def cache_dir():
    d = os.environ.get('VG_SCENE_CACHE') or os.path.join(os.environ.get('TMPDIR', '/tmp'), 'vgb200_scenes')
    os.makedirs(d, exist_ok=True)
    return d


def build_graph(cfg, seed=0, n=None, cache=True):
    """-> dict(points (N, 3) float32, offsets (N + 1) int32, adj (M) int32) for a configuration."""
    c = CONFIGS[cfg]
    n = c['n'] if n is None else n
    path = os.path.join(cache_dir(), f'graph_c{cfg}_n{n}_s{seed}.npz')
    if cache and os.path.exists(path):
        z = np.load(path)
        return {k: z[k] for k in ('points', 'offsets', 'adj')}
    pts = make_points(cfg, seed, n)
    p, _, off, adj = sites.delaunay_graph(pts)
    g = {'points': p.astype(np.float32), 'offsets': off.astype(np.int32), 'adj': adj.astype(np.int32)}
    if cache:
        tmp = path + f'.{os.getpid()}.tmp.npz'
        np.savez(tmp, **g)
        os.replace(tmp, path)
    return g


def _gen(seed):
    g = torch.Generator()
    g.manual_seed(seed)
    return g


def make_params(cfg, points, seed=0):
    """Per-site parameters (CPU float32 tensors) in the reference model's layout.

    Config 1: raw = log(softplus(N(0, 1))), log-scales N(-3, 0.3) repeated x3, identity quaternions,
    SH bands 0-1 ~ N(0, 0.3). Configs 2-5: the reference constructor's spacing-based initialisation
    (model.py:23-39: rho s sqrt(2 pi) = -ln(1 - 0.1), scale = spacing), base colour N(0.5, 0.2)
    stored as sh_dc = (c - 0.5) / C0, higher bands N(0, 0.05)."""
    c = CONFIGS[cfg]
    n = len(points)
    base = 1000 * seed
    q = torch.zeros(n, 4)
    q[:, 0] = 1.0
    sh = torch.zeros(n, 16, 3)
    if cfg == 1:
        raw = torch.log(torch.nn.functional.softplus(torch.randn(n, generator=_gen(base + 1))))
        ls = (torch.randn(n, generator=_gen(base + 2)) * 0.3 - 3.0)[:, None].repeat(1, 3)
        cls = (torch.randn(n, generator=_gen(base + 3)) * 0.3 - 3.0)[:, None].repeat(1, 3)
        sh[:, :4] = torch.randn(n, 4, 3, generator=_gen(base + 4)) * 0.3
    else:
        s = torch.from_numpy(sites.neighbor_spacing(np.asarray(points, dtype=np.float64))).float()
        s = s.clamp_min(1e-4)
        rho = -math.log(1.0 - 0.1) / (s * math.sqrt(2.0 * math.pi))
        raw = rho.log()
        ls = s.log()[:, None].repeat(1, 3)
        cls = ls.clone()
        col = torch.randn(n, 3, generator=_gen(base + 5)) * 0.2 + 0.5
        sh[:, 0] = (col - 0.5) / C0
        sh[:, 1:] = torch.randn(n, 15, 3, generator=_gen(base + 6)) * 0.05
    return {'raw': raw.contiguous(), 'd_log_scale': ls.contiguous(), 'd_quat': q.clone(),
            'c_log_scale': cls.contiguous(), 'c_quat': q.clone(), 'sh': sh.contiguous(),
            'sh_deg': c['sh_deg']}


# --------------------------------------------------------------------------------- cameras

def orbit_camera(i, n_cams, radius=3.0, elevation_deg=15.0):
    """Camera centre and camera-to-world rotation (columns: right, down, forward; OpenCV / COLMAP
    convention) looking at the origin."""
    theta = 2.0 * math.pi * i / max(n_cams, 1)
    phi = math.radians(elevation_deg)
    centre = radius * np.array([math.cos(phi) * math.cos(theta), math.cos(phi) * math.sin(theta), math.sin(phi)])
    fwd = -centre / np.linalg.norm(centre)
    up = np.array([0.0, 0.0, 1.0])
    right = np.cross(fwd, up)
    right /= np.linalg.norm(right)
    down = np.cross(fwd, right)
    return centre, np.stack([right, down, fwd], 1)


def march_bounds(o, d):
    """(near, mid, far) of the fixed-step workload (config 5): near where the ray enters the unit ball,
    mid where it leaves it, far = mid + 1e-3 (with n_bg = 0 nothing is marched beyond mid); rays that
    miss the ball get near = mid = 0.02 and no samples."""
    b = (o * d).sum(-1)
    c = (o * o).sum(-1) - 1.0
    disc = b * b - c
    root = torch.sqrt(torch.clamp(disc, min=0.0))
    hit = disc > 0
    near = torch.where(hit, torch.clamp(-b - root, min=0.02), torch.full_like(b, 0.02))
    mid = torch.where(hit, torch.maximum(-b + root, near), near)
    return near.contiguous(), mid.contiguous(), (mid + 1e-3).contiguous()


def tile_order(H, W, th=4, tw=8):
    """Pixel permutation grouping 32 consecutive rays into th x tw tiles (bench_infer.py:37-41)."""
    y, x = np.meshgrid(np.arange(H), np.arange(W), indexing='ij')
    key = ((y // th) * ((W + tw - 1) // tw) + x // tw) * (th * tw) + (y % th) * tw + x % tw
    return np.argsort(key.ravel(), kind='stable')


def camera_rays_device(centre, c2w, W, H, fov_deg=50.0, device='cuda', tile=(4, 8)):
    """camera_rays generated on the device by vg_camera_rays, directly in tile[0] x tile[1] pixel-tile
    order (the order of tile_order(H, W, *tile); tile None: row-major). -> o, d (W H, 3) float32."""
    from . import _lib
    f = 0.5 * W / math.tan(math.radians(fov_deg) / 2.0)
    K = np.array([[f, 0.0, W / 2.0], [0.0, f, H / 2.0], [0.0, 0.0, 1.0]])
    k_inv = np.ascontiguousarray(np.linalg.inv(K), np.float32)
    k_inv[1, 0] = k_inv[2, 0] = k_inv[2, 1] = 0.0
    k_inv[2, 2] = 1.0
    rot = np.ascontiguousarray(np.asarray(c2w, np.float64), np.float32)
    ctr = np.ascontiguousarray(np.asarray(centre, np.float64), np.float32)
    dev = torch.device(device)
    o = torch.empty(W * H, 3, device=dev)
    d = torch.empty(W * H, 3, device=dev)
    th, tw = tile if tile is not None else (0, 0)
    with torch.cuda.device(dev):
        _lib.call('vg_camera_rays', k_inv.ctypes.data, rot.ctypes.data, ctr.ctypes.data, int(W), int(H), int(th),
                  int(tw), o.data_ptr(), d.data_ptr(), torch.cuda.current_stream(dev).cuda_stream)
    return o, d


def camera_rays(centre, c2w, W, H, fov_deg=50.0, device='cpu', order=None):
    """Pinhole rays of every pixel (colmap.py:129-134): d = c2w K^-1 (px + 0.5, py + 0.5, 1),
    normalised. -> o (P, 3), d (P, 3) float32, in `order` (a pixel permutation) if given."""
    f = 0.5 * W / math.tan(math.radians(fov_deg) / 2.0)
    K = torch.tensor([[f, 0.0, W / 2.0], [0.0, f, H / 2.0], [0.0, 0.0, 1.0]], dtype=torch.float32, device=device)
    R = torch.tensor(c2w, dtype=torch.float32, device=device)
    py, px = torch.meshgrid(torch.arange(H, device=device).float(), torch.arange(W, device=device).float(),
                            indexing='ij')
    p = torch.stack([px.reshape(-1) + 0.5, py.reshape(-1) + 0.5, torch.ones(H * W, device=device)], -1)
    if order is not None:
        p = p[torch.as_tensor(order, device=device)]
    d = p @ torch.linalg.inv(K).T
    d = d @ R.T
    d = d / d.norm(dim=-1, keepdim=True)
    o = torch.tensor(centre, dtype=torch.float32, device=device).expand_as(d).contiguous()
    return o, d.contiguous()
