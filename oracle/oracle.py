"""TEST INFRASTRUCTURE ONLY — ctypes front end of the CPU checker (oracle/vg_oracle.c).

Used by tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg to check and time the
product; the product itself never imports this module. Inputs/outputs are numpy arrays (or CPU
torch tensors) in the reference layouts; signatures follow the reference extension functions
(foam.cu:505-533, march.cu:383-410, vgf.cu:438-561, foam_infer.cu:376-380).
"""

from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, '_build', 'libvgoracle.so')
_lib = None


def build():
    subprocess.run(['make', '-s', '-C', HERE], check=True)


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        _lib = ctypes.CDLL(LIB_PATH)
        i64, i32, f32, P = ctypes.c_int64, ctypes.c_int, ctypes.c_float, ctypes.c_void_p
        _lib.vgo_foam_forward.argtypes = [P, P, P, i64, P, P, P, P, i32, P, P, P, P, P, i64, f32, f32, i32,
                                          P, P, P, P, P, i32]
        _lib.vgo_foam_backward.argtypes = [P, P, P, i64, P, P, P, P, i32, P, P, P, P, P, i64, f32, f32,
                                           P, P, P, P, P, i32, P, P, P, P, P, i32]
        _lib.vgo_march_forward.argtypes = [P, P, P, i64, P, P, P, P, i32, P, P, P, P, P, P, i64, f32, i32, f32,
                                           f32, P, P, P, P, i32]
        _lib.vgo_march_backward.argtypes = [P, P, P, i64, P, P, P, P, i32, P, P, P, P, P, P, i64, f32, i32, f32,
                                            f32, P, P, P, P, P, P, P, P, i32]
        _lib.vgo_conic_forward.argtypes = [P, P, i64, f32, P]
        _lib.vgo_conic_backward.argtypes = [P, P, i64, f32, P, P, P]
        _lib.vgo_foam_infer.argtypes = [P, P, P, P, P, P, i32, i32, i64, P, P, P, P, P, i64, f32, f32, f32,
                                        i32, i32, P, P, P, P, P, P, i32]
        f64 = ctypes.c_double
        _lib.vgo_walk.argtypes = [P, P, P, i64, P, P, P, P, i64, i32, P, P]
        _lib.vgo_density_forward.argtypes = [P, P, P, i64, P, P, P, P, P, i64, f64, P]
        _lib.vgo_density_backward.argtypes = [P, P, P, i64, P, P, P, P, P, i64, P, P, P, P]
        _lib.vgo_color_forward.argtypes = [P, P, P, i64, P, P, P, i32, P, P, P, i64, P]
        _lib.vgo_color_backward.argtypes = [P, P, P, i64, P, P, P, i32, P, P, P, i64, P, P, P, P, P]
        for f in ('vgo_foam_forward', 'vgo_foam_backward', 'vgo_march_forward', 'vgo_march_backward',
                  'vgo_foam_infer', 'vgo_walk', 'vgo_density_forward', 'vgo_density_backward', 'vgo_color_forward',
                  'vgo_color_backward'):
            getattr(_lib, f).restype = ctypes.c_int
    return _lib


def _np(x, dtype):
    if hasattr(x, 'detach'):
        x = x.detach().cpu().numpy()
    return np.ascontiguousarray(np.asarray(x), dtype=dtype)


def _p(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def default_threads():
    return os.cpu_count() or 1


def foam_forward(points, offsets, adj, raw, dA, cA, sh, sh_deg, o, d, start, near, far, t_thresh=1e-4,
                 w_thresh=1e-4, record_cap=0, n_threads=1):
    """-> rgb (B, 3), T (B), depth (B), stats (B, 3) int32, rec (B, K, 8) float32 (foam.cu:505-526)."""
    f, i = np.float32, np.int32
    args = [_np(points, f), _np(offsets, i), _np(adj, i), _np(raw, f), _np(dA, f), _np(cA, f), _np(sh, f)]
    rays = [_np(o, f), _np(d, f), _np(start, i), _np(near, f), _np(far, f)]
    B = len(rays[0])
    K = int(record_cap)
    rgb, T, depth = np.zeros((B, 3), f), np.zeros(B, f), np.zeros(B, f)
    stats = np.zeros((B, 3), i)
    rec = np.zeros((B if K > 0 else 0, max(K, 0), 8), f)
    rc = lib().vgo_foam_forward(*map(_p, args[:3]), len(args[0]), *map(_p, args[3:]), int(sh_deg),
                                *map(_p, rays), B, float(t_thresh), float(w_thresh), K, _p(rgb), _p(T), _p(depth),
                                _p(stats), _p(rec) if K > 0 else None, int(n_threads))
    if rc:
        raise RuntimeError(f'oracle foam_forward failed ({rc})')
    return rgb, T, depth, stats, rec


def foam_backward(points, offsets, adj, raw, dA, cA, sh, sh_deg, o, d, start, near, far, t_thresh, w_thresh,
                  rgb, T, g_rgb, g_T, rec, stats, n_threads=1):
    """-> g_raw (N), g_dA (N, 6), g_cA (N, 6), g_sh (N, 16, 3) (foam.cu:528-558)."""
    f, i = np.float32, np.int32
    args = [_np(points, f), _np(offsets, i), _np(adj, i), _np(raw, f), _np(dA, f), _np(cA, f), _np(sh, f)]
    rays = [_np(o, f), _np(d, f), _np(start, i), _np(near, f), _np(far, f)]
    B = len(rays[0])
    n = len(args[0])
    rec = _np(rec, f)
    K = rec.shape[1] if rec.size > 0 else 0
    g = [np.zeros(n, f), np.zeros((n, 6), f), np.zeros((n, 6), f), np.zeros((n, 16, 3), f)]
    ins = [_np(rgb, f), _np(T, f), _np(g_rgb, f), _np(g_T, f)]
    rc = lib().vgo_foam_backward(*map(_p, args[:3]), n, *map(_p, args[3:]), int(sh_deg), *map(_p, rays), B,
                                 float(t_thresh), float(w_thresh), *map(_p, ins), _p(rec) if K > 0 else None, K,
                                 _p(_np(stats, i)), *map(_p, g), int(n_threads))
    if rc:
        raise RuntimeError(f'oracle foam_backward failed ({rc})')
    return g


def march_forward(points, offsets, adj, raw, dA, cA, sh, sh_deg, o, d, start, near, mid, far, dt, n_bg,
                  t_thresh=1e-4, w_thresh=1e-4, n_threads=1):
    """-> rgb (B, 3), T (B), depth (B), stats (B, 3) int32 (march.cu:383-403)."""
    f, i = np.float32, np.int32
    args = [_np(points, f), _np(offsets, i), _np(adj, i), _np(raw, f), _np(dA, f), _np(cA, f), _np(sh, f)]
    rays = [_np(o, f), _np(d, f), _np(start, i), _np(near, f), _np(mid, f), _np(far, f)]
    B = len(rays[0])
    rgb, T, depth = np.zeros((B, 3), f), np.zeros(B, f), np.zeros(B, f)
    stats = np.zeros((B, 3), i)
    rc = lib().vgo_march_forward(*map(_p, args[:3]), len(args[0]), *map(_p, args[3:]), int(sh_deg),
                                 *map(_p, rays), B, float(dt), int(n_bg), float(t_thresh), float(w_thresh),
                                 _p(rgb), _p(T), _p(depth), _p(stats), int(n_threads))
    if rc:
        raise RuntimeError(f'oracle march_forward failed ({rc})')
    return rgb, T, depth, stats


def march_backward(points, offsets, adj, raw, dA, cA, sh, sh_deg, o, d, start, near, mid, far, dt, n_bg,
                   t_thresh, w_thresh, rgb, T, g_rgb, g_T, n_threads=1):
    """-> g_raw, g_dA, g_cA, g_sh (march.cu:405-429)."""
    f, i = np.float32, np.int32
    args = [_np(points, f), _np(offsets, i), _np(adj, i), _np(raw, f), _np(dA, f), _np(cA, f), _np(sh, f)]
    rays = [_np(o, f), _np(d, f), _np(start, i), _np(near, f), _np(mid, f), _np(far, f)]
    B = len(rays[0])
    n = len(args[0])
    g = [np.zeros(n, f), np.zeros((n, 6), f), np.zeros((n, 6), f), np.zeros((n, 16, 3), f)]
    ins = [_np(rgb, f), _np(T, f), _np(g_rgb, f), _np(g_T, f)]
    rc = lib().vgo_march_backward(*map(_p, args[:3]), n, *map(_p, args[3:]), int(sh_deg), *map(_p, rays), B,
                                  float(dt), int(n_bg), float(t_thresh), float(w_thresh), *map(_p, ins), *map(_p, g),
                                  int(n_threads))
    if rc:
        raise RuntimeError(f'oracle march_backward failed ({rc})')
    return g


def conic_forward(log_scale, quat, floor=0.0):
    ls, q = _np(log_scale, np.float32), _np(quat, np.float32)
    A = np.zeros((len(q), 6), np.float32)
    lib().vgo_conic_forward(_p(ls), _p(q), len(q), float(floor), _p(A))
    return A


def conic_backward(log_scale, quat, floor, gA):
    ls, q, g = _np(log_scale, np.float32), _np(quat, np.float32), _np(gA, np.float32)
    g_ls, g_q = np.zeros_like(ls), np.zeros_like(q)
    lib().vgo_conic_backward(_p(ls), _p(q), len(q), float(floor), _p(g), _p(g_ls), _p(g_q))
    return g_ls, g_q


def foam_infer(points, offsets, nbr, edge, attr, sh, sh_deg, o, d, start, near, far, t_thresh, w_thresh,
               color_cut, color_mode, stage, cap=None, orig=None, n_threads=1):
    """-> rgb (B, 3), T (B), depth (B), stats (B, 5) (foam_infer.cu:376-435)."""
    f, i = np.float32, np.int32
    pts, off, nb, ed, at = _np(points, f), _np(offsets, i), _np(nbr, i), _np(edge, f), _np(attr, f)
    sh_half = 0
    sh_arr = None
    if sh is not None and (not hasattr(sh, 'numel') or sh.numel() > 0):
        a = sh.detach().cpu().numpy() if hasattr(sh, 'detach') else np.asarray(sh)
        if a.dtype == np.float16:
            sh_arr, sh_half = np.ascontiguousarray(a).view(np.uint16), 1
        else:
            sh_arr = np.ascontiguousarray(a, dtype=f)
    rays = [_np(o, f), _np(d, f), _np(start, i), _np(near, f), _np(far, f)]
    B = len(rays[0])
    n = len(pts)
    cap_a = _np(cap, i) if cap is not None and len(cap) == B else None
    orig_a = _np(orig, i) if orig is not None and len(orig) == n else None
    rgb, T, depth = np.zeros((B, 3), f), np.zeros(B, f), np.zeros(B, f)
    stats = np.zeros((B, 5), i)
    rc = lib().vgo_foam_infer(_p(pts), _p(off), _p(nb), _p(ed), _p(at), _p(sh_arr), sh_half, int(sh_deg), n,
                              *map(_p, rays), B, float(t_thresh), float(w_thresh), float(color_cut), int(color_mode),
                              int(stage), _p(cap_a), _p(orig_a), _p(rgb), _p(T), _p(depth), _p(stats),
                              int(n_threads))
    if rc:
        raise RuntimeError(f'oracle foam_infer failed ({rc})')
    return rgb, T, depth, stats


# ------------------------------------------------------------------- NeRF-sampler field kernels

def _graph(points, offsets, adj):
    return _np(points, np.float32), _np(offsets, np.int32), _np(adj, np.int32)


def walk(points, offsets, adj, o, d, z, start):
    """-> site (B, S) int32, steps (B) int32 (vgf.cu:438-456)."""
    g = _graph(points, offsets, adj)
    o, d, z, start = _np(o, np.float32), _np(d, np.float32), _np(z, np.float32), _np(start, np.int32)
    B, S = z.shape
    site, steps = np.zeros((B, S), np.int32), np.zeros(B, np.int32)
    lib().vgo_walk(*map(_p, g), len(g[0]), _p(o), _p(d), _p(z), _p(start), B, S, _p(site), _p(steps))
    return site, steps


def density_forward(points, offsets, adj, raw, log_scale, quat, x, site, scale_mult=1.0):
    """-> sigma (M) (vgf.cu:458-475)."""
    g = _graph(points, offsets, adj)
    f = [_np(a, np.float32) for a in (raw, log_scale, quat, x)]
    site = _np(site, np.int32)
    sigma = np.zeros(len(site), np.float32)
    lib().vgo_density_forward(*map(_p, g), len(g[0]), *map(_p, f), _p(site), len(site), float(scale_mult),
                              _p(sigma))
    return sigma


def density_backward(points, offsets, adj, raw, log_scale, quat, x, site, grad_sigma):
    """-> g_raw (N), g_ls (N, 3), g_quat (N, 4) (vgf.cu:477-492)."""
    g = _graph(points, offsets, adj)
    f = [_np(a, np.float32) for a in (raw, log_scale, quat, x)]
    site, gs = _np(site, np.int32), _np(grad_sigma, np.float32)
    n = len(g[0])
    g_raw, g_ls, g_quat = np.zeros(n, np.float32), np.zeros((n, 3), np.float32), np.zeros((n, 4), np.float32)
    lib().vgo_density_backward(*map(_p, g), n, *map(_p, f), _p(site), len(site), _p(gs), _p(g_raw), _p(g_ls),
                               _p(g_quat))
    return g_raw, g_ls, g_quat


def color_forward(points, offsets, adj, log_scale, quat, sh, sh_deg, x, dirs, site):
    """-> rgb (M, 3) (vgf.cu:494-513)."""
    g = _graph(points, offsets, adj)
    ls, q, sh = _np(log_scale, np.float32), _np(quat, np.float32), _np(sh, np.float32)
    x, dirs, site = _np(x, np.float32), _np(dirs, np.float32), _np(site, np.int32)
    rgb = np.zeros((len(site), 3), np.float32)
    lib().vgo_color_forward(*map(_p, g), len(g[0]), _p(ls), _p(q), _p(sh), int(sh_deg), _p(x), _p(dirs), _p(site),
                            len(site), _p(rgb))
    return rgb


def color_backward(points, offsets, adj, log_scale, quat, sh, sh_deg, x, dirs, site, rgb, grad_rgb):
    """-> g_ls (N, 3), g_quat (N, 4), g_sh (N, 16, 3) (vgf.cu:515-533)."""
    g = _graph(points, offsets, adj)
    ls, q, sh = _np(log_scale, np.float32), _np(quat, np.float32), _np(sh, np.float32)
    x, dirs, site = _np(x, np.float32), _np(dirs, np.float32), _np(site, np.int32)
    rgb, grad_rgb = _np(rgb, np.float32), _np(grad_rgb, np.float32)
    n = len(g[0])
    g_ls, g_quat, g_sh = np.zeros((n, 3), np.float32), np.zeros((n, 4), np.float32), np.zeros((n, 16, 3), np.float32)
    lib().vgo_color_backward(*map(_p, g), n, _p(ls), _p(q), _p(sh), int(sh_deg), _p(x), _p(dirs), _p(site), len(site),
                             _p(rgb), _p(grad_rgb), _p(g_ls), _p(g_quat), _p(g_sh))
    return g_ls, g_quat, g_sh
