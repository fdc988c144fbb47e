"""Drop-in replacement of the reference's extension module (voronoi-gauss ext.py) on libvgb200.

Same public surface and contracts as ext.py:30-216:

* ``Graph(points, offsets, adj)``: fixed sites and their CSR Delaunay adjacency on the GPU
  (ext.py:46-52). The packed, Morton-ordered neighbourhoods used by the kernels are built on first use
  and cached on the Graph.
* ``foam(graph, raw, dA, cA, sh, sh_deg, o, d, start, near, far, t_thresh, w_thresh, record_cap)``
  -> (rgb, T, depth, stats), autograd through raw / dA / cA / sh (ext.py:185-216);
  ``march(...)`` (ext.py:152-182); ``conic(log_scale, quat, floor)`` (ext.py:120-136) and its torch twin
  ``conic_reference`` (ext.py:139-149); the NeRF-sampler fields ``density(...)`` / ``color(...)``
  (ext.py:61-117) and ``Graph.walk`` (ext.py:54-58).
* ``foam_extension()``, ``march_extension()``, ``extension()``, ``foam_infer_extension()`` return objects
  with the reference's extension-level functions and signatures (foam.cu:560-565, march.cu:431-434,
  vgf.cu:563-571, foam_infer.cu:437-440): tensors in, freshly allocated tensors out,
  ``RuntimeError`` on a bad argument (the reference's TORCH_CHECK).

Every call runs on the input's device and on torch's current stream of that device, asynchronously.
"""

from __future__ import annotations

import weakref

import torch

from . import _lib

__all__ = ['Graph', 'foam', 'march', 'conic', 'conic_reference', 'density', 'color', 'extension', 'march_extension',
           'foam_extension', 'foam_infer_extension', 'GraphPack', 'graph_pack', 'nearest_sites']


def _ptr(t):
    return None if t is None or t.numel() == 0 else t.data_ptr()


def _stream(dev):
    return torch.cuda.current_stream(dev).cuda_stream


def _check(x, name, dtype):
    """The reference's CHECK_INPUT (foam.cu:34-37)."""
    if not x.is_cuda:
        raise RuntimeError(f'{name} must be a CUDA tensor')
    if not x.is_contiguous():
        raise RuntimeError(f'{name} must be contiguous')
    if x.dtype != dtype:
        raise RuntimeError(f'{name} has the wrong dtype')


# ----------------------------------------------------------------------------------- graph packs

class GraphPack:
    """Packed scene graph (vg_graph_pack) of (points, offsets, adj) on their device."""

    def __init__(self, points, offsets, adj):
        _check(points, 'points', torch.float32)
        _check(offsets, 'offsets', torch.int32)
        _check(adj, 'adj', torch.int32)
        if points.dim() != 2 or points.size(1) != 3:
            raise RuntimeError('points must be (N, 3)')
        if offsets.numel() != points.size(0) + 1:
            raise RuntimeError('offsets must be (N + 1)')
        self.n, self.m = points.size(0), adj.numel()
        self.device = points.device
        nbytes = _lib.lib().vg_graph_pack_bytes(self.n, self.m)
        self.buf = torch.empty(nbytes, dtype=torch.uint8, device=self.device)
        with torch.cuda.device(self.device):
            _lib.call('vg_graph_pack', points.data_ptr(), offsets.data_ptr(), _ptr(adj), self.n, self.m,
                      self.buf.data_ptr(), nbytes, _stream(self.device))
        self._src = tuple(weakref.ref(t) for t in (points, offsets, adj))
        self._ver = tuple(t._version for t in (points, offsets, adj))

    def matches(self, points, offsets, adj):
        for ref, ver, t in zip(self._src, self._ver, (points, offsets, adj)):
            if ref() is not t or t._version != ver:
                return False
        return True

    @property
    def ptr(self):
        return self.buf.data_ptr()


_PACKS: list = []


def graph_pack(points, offsets, adj):
    """Cached GraphPack of these exact tensors (rebuilt when one of them is modified in place)."""
    for p in _PACKS:
        if p.matches(points, offsets, adj):
            return p
    p = GraphPack(points, offsets, adj)
    _PACKS.insert(0, p)
    del _PACKS[4:]
    return p


class Graph:
    """Fixed sites and their Delaunay adjacency (CSR, int32) on the GPU (ext.py:46-58)."""

    def __init__(self, points, offsets, adj):
        self.points, self.offsets, self.adj = points.float().contiguous(), offsets.int().contiguous(), \
            adj.int().contiguous()
        self._pack = None

    @property
    def pack(self):
        if self._pack is None or not self._pack.matches(self.points, self.offsets, self.adj):
            self._pack = graph_pack(self.points, self.offsets, self.adj)
        return self._pack

    def walk(self, o, d, z, start):
        """Nearest site of every sample o + z d; z (B, S) sorted along each ray, start (B,) a site near o
        (ext.py:54-58). Returns (site (B, S) int32, steps (B) int32)."""
        o, d, start = _rays(o, d, start)
        site, steps = extension().walk(self.points, self.offsets, self.adj, o, d, z.float().contiguous(), start)
        return site, steps


def nearest_sites(graph, queries):
    """Original id of the site nearest to each query point (Q, 3) on the device (greedy walks on the
    packed graph; the reference does this on the host with a k-d tree, sites.py:38-39). -> (Q,) int32."""
    q = queries.detach().float().contiguous()
    _check(q, 'queries', torch.float32)
    if q.dim() != 2 or q.size(1) != 3:
        raise RuntimeError('queries must be (Q, 3)')
    out = torch.empty(q.size(0), dtype=torch.int32, device=q.device)
    if q.size(0):
        pk = graph.pack
        with torch.cuda.device(q.device):
            _lib.call('vg_nearest_sites', pk.ptr, pk.n, pk.m, q.data_ptr(), q.size(0), out.data_ptr(),
                      _stream(q.device))
    return out


# ------------------------------------------------------------------------- extension-level functions

def _scene_checks(points, offsets, adj, raw, dA, cA, sh):
    for x, name, dt in ((points, 'points', torch.float32), (offsets, 'offsets', torch.int32),
                        (adj, 'adj', torch.int32), (raw, 'raw', torch.float32), (dA, 'dA', torch.float32),
                        (cA, 'cA', torch.float32), (sh, 'sh', torch.float32)):
        _check(x, name, dt)
    n = points.size(0)
    if sh.dim() != 3 or sh.size(1) != 16 or sh.size(2) != 3:
        raise RuntimeError('sh must be (N, 16, 3)')
    if dA.dim() != 2 or cA.dim() != 2 or dA.size(1) != 6 or cA.size(1) != 6:
        raise RuntimeError('conics must be (N, 6)')
    if raw.numel() != n or dA.size(0) != n or cA.size(0) != n or sh.size(0) != n:
        raise RuntimeError('per-site tensors must have N rows')


def _ray_checks(**rays):
    for name, x in rays.items():
        _check(x, name, torch.int32 if name == 'start' else torch.float32)
    B = rays['o'].size(0)
    if rays['o'].shape != (B, 3) or rays['d'].shape != (B, 3):
        raise RuntimeError('o and d must be (B, 3)')
    for name, x in rays.items():
        if name not in ('o', 'd') and x.numel() != B:
            raise RuntimeError(f'{name} must be (B)')
    return B


def _workspace(n, sh_deg, backward, dev, n_rays=0, record_cap=0):
    nbytes = _lib.lib().vg_foam_workspace_bytes(n, int(sh_deg), int(n_rays), int(record_cap), int(backward))
    return torch.empty(max(nbytes, 256), dtype=torch.uint8, device=dev), nbytes


def sample_counts_size(n_sites, n_rays, record_cap):
    """int32 entries of the per-cell sample counts that foam_forward(..., counts=) keeps for the backward."""
    return _lib.lib().vg_foam_counts_bytes(int(n_sites), int(n_rays), int(record_cap)) // 4


def _sh_deg(sh_deg):
    if not 0 <= int(sh_deg) <= 3:
        raise RuntimeError('sh_deg must be in 0..3')
    return int(sh_deg)


class FoamExtension:
    """foam_forward / foam_backward with the reference's signatures (foam.cu:505-558)."""

    @staticmethod
    def foam_forward(points, offsets, adj, raw, dA, cA, sh, sh_deg, o, d, start, near, far, t_thresh, w_thresh,
                     record_cap, counts=None):
        """counts (optional, int32 of sample_counts_size entries): also keep the per-cell sample counts of the
        records for foam_backward(..., counts=) (vg_foam_forward_counted)."""
        _scene_checks(points, offsets, adj, raw, dA, cA, sh)
        B = _ray_checks(o=o, d=d, start=start, near=near, far=far)
        sh_deg, K = _sh_deg(sh_deg), int(record_cap)
        if K < 0:
            raise RuntimeError('record_cap must be >= 0')
        dev = o.device
        rgb = torch.empty(B, 3, device=dev)
        T = torch.empty(B, device=dev)
        depth = torch.empty(B, device=dev)
        stats = torch.empty(B, 3, dtype=torch.int32, device=dev)
        rec = torch.empty(B if K > 0 else 0, K, 8, device=dev)
        if B == 0:
            return [rgb, T, depth, stats, rec]
        pk = graph_pack(points, offsets, adj)
        ws, nbytes = _workspace(pk.n, sh_deg, 0, dev, B, K)
        args = [pk.ptr, pk.n, pk.m, raw.data_ptr(), dA.data_ptr(), cA.data_ptr(), sh.data_ptr(), sh_deg, o.data_ptr(),
                d.data_ptr(), start.data_ptr(), near.data_ptr(), far.data_ptr(), B, float(t_thresh), float(w_thresh),
                K, rgb.data_ptr(), T.data_ptr(), depth.data_ptr(), stats.data_ptr(), _ptr(rec)]
        with torch.cuda.device(dev):
            if counts is not None and K > 0:
                if counts.dtype != torch.int32 or not counts.is_contiguous() or \
                        counts.numel() < sample_counts_size(pk.n, B, K):
                    raise RuntimeError('counts must be a contiguous int32 tensor of sample_counts_size entries')
                _lib.call('vg_foam_forward_counted', *args, counts.data_ptr(), ws.data_ptr(), nbytes, _stream(dev))
            else:
                _lib.call('vg_foam_forward', *args, ws.data_ptr(), nbytes, _stream(dev))
        return [rgb, T, depth, stats, rec]

    @staticmethod
    def foam_backward(points, offsets, adj, raw, dA, cA, sh, sh_deg, o, d, start, near, far, t_thresh, w_thresh,
                      rgb, T, g_rgb, g_T, rec, stats, counts=None):
        """counts: the per-cell sample counts kept by foam_forward(..., counts=) for these records
        (vg_foam_backward_counted), so the records are not counted again."""
        _scene_checks(points, offsets, adj, raw, dA, cA, sh)
        B = _ray_checks(o=o, d=d, start=start, near=near, far=far)
        for x, name, dt in ((rgb, 'rgb', torch.float32), (T, 'T', torch.float32), (g_rgb, 'g_rgb', torch.float32),
                            (g_T, 'g_T', torch.float32), (rec, 'rec', torch.float32),
                            (stats, 'stats', torch.int32)):
            _check(x, name, dt)
        replay = rec.numel() > 0
        if replay and (rec.dim() != 3 or rec.size(0) != B or rec.size(2) != 8):
            raise RuntimeError('rec must be (B, K, 8)')
        sh_deg = _sh_deg(sh_deg)
        dev = o.device
        g_raw, g_dA, g_cA, g_sh = (torch.empty_like(x) for x in (raw, dA, cA, sh))
        pk = graph_pack(points, offsets, adj)
        ws, nbytes = _workspace(pk.n, sh_deg, 1, dev, B, rec.size(1) if replay else 0)
        head = [pk.ptr, pk.n, pk.m, raw.data_ptr(), dA.data_ptr(), cA.data_ptr(), sh.data_ptr(), sh_deg, _ptr(o),
                _ptr(d), _ptr(start), _ptr(near), _ptr(far), B, float(t_thresh), float(w_thresh), _ptr(rgb), _ptr(T),
                _ptr(g_rgb), _ptr(g_T), _ptr(rec) if replay else None, rec.size(1) if replay else 0, _ptr(stats)]
        tail = [g_raw.data_ptr(), g_dA.data_ptr(), g_cA.data_ptr(), g_sh.data_ptr(), ws.data_ptr(), nbytes, _stream(dev)]
        with torch.cuda.device(dev):
            if counts is not None and replay:
                if counts.numel() < sample_counts_size(pk.n, B, rec.size(1)):
                    raise RuntimeError('counts does not match the records')
                _lib.call('vg_foam_backward_counted', *head, counts.data_ptr(), *tail)
            else:
                _lib.call('vg_foam_backward', *head, *tail)
        return [g_raw, g_dA, g_cA, g_sh]


class MarchExtension:
    """march_forward / march_backward with the reference's signatures (march.cu:383-429)."""

    @staticmethod
    def march_forward(points, offsets, adj, raw, dA, cA, sh, sh_deg, o, d, start, near, mid, far, dt, n_bg, t_thresh,
                      w_thresh):
        _scene_checks(points, offsets, adj, raw, dA, cA, sh)
        B = _ray_checks(o=o, d=d, start=start, near=near, mid=mid, far=far)
        sh_deg = _sh_deg(sh_deg)
        dev = o.device
        rgb = torch.empty(B, 3, device=dev)
        T = torch.empty(B, device=dev)
        depth = torch.empty(B, device=dev)
        stats = torch.empty(B, 3, dtype=torch.int32, device=dev)
        if B == 0:
            return [rgb, T, depth, stats]
        pk = graph_pack(points, offsets, adj)
        ws, nbytes = _workspace(pk.n, sh_deg, False, dev)
        with torch.cuda.device(dev):
            _lib.call('vg_march_forward', pk.ptr, pk.n, pk.m, raw.data_ptr(), dA.data_ptr(), cA.data_ptr(),
                      sh.data_ptr(), sh_deg, o.data_ptr(), d.data_ptr(), start.data_ptr(), near.data_ptr(),
                      mid.data_ptr(), far.data_ptr(), B, float(dt), int(n_bg), float(t_thresh), float(w_thresh),
                      rgb.data_ptr(), T.data_ptr(), depth.data_ptr(), stats.data_ptr(), ws.data_ptr(), nbytes,
                      _stream(dev))
        return [rgb, T, depth, stats]

    @staticmethod
    def march_backward(points, offsets, adj, raw, dA, cA, sh, sh_deg, o, d, start, near, mid, far, dt, n_bg, t_thresh,
                       w_thresh, rgb, T, g_rgb, g_T):
        _scene_checks(points, offsets, adj, raw, dA, cA, sh)
        B = _ray_checks(o=o, d=d, start=start, near=near, mid=mid, far=far)
        for x, name in ((rgb, 'rgb'), (T, 'T'), (g_rgb, 'g_rgb'), (g_T, 'g_T')):
            _check(x, name, torch.float32)
        sh_deg = _sh_deg(sh_deg)
        dev = o.device
        g_raw, g_dA, g_cA, g_sh = (torch.empty_like(x) for x in (raw, dA, cA, sh))
        pk = graph_pack(points, offsets, adj)
        ws, nbytes = _workspace(pk.n, sh_deg, 3, dev, B)
        with torch.cuda.device(dev):
            _lib.call('vg_march_backward', pk.ptr, pk.n, pk.m, raw.data_ptr(), dA.data_ptr(), cA.data_ptr(),
                      sh.data_ptr(), sh_deg, _ptr(o), _ptr(d), _ptr(start), _ptr(near), _ptr(mid), _ptr(far), B,
                      float(dt), int(n_bg), float(t_thresh), float(w_thresh), _ptr(rgb), _ptr(T), _ptr(g_rgb),
                      _ptr(g_T), g_raw.data_ptr(), g_dA.data_ptr(), g_cA.data_ptr(), g_sh.data_ptr(), ws.data_ptr(),
                      nbytes, _stream(dev))
        return [g_raw, g_dA, g_cA, g_sh]


class FieldExtension:
    """The functions of the reference's vgf.cu module (vgf.cu:438-571): the NeRF-sampler walk, density
    and colour fields with their gradients, and the conics."""

    @staticmethod
    def walk(points, offsets, adj, o, d, z, start):
        for x, name, dt in ((points, 'points', torch.float32), (offsets, 'offsets', torch.int32),
                            (adj, 'adj', torch.int32), (o, 'o', torch.float32), (d, 'd', torch.float32),
                            (z, 'z', torch.float32), (start, 'start', torch.int32)):
            _check(x, name, dt)
        if z.dim() != 2:
            raise RuntimeError('z must be (B, S)')
        B, S = z.size(0), z.size(1)
        if o.shape != (B, 3) or d.shape != (B, 3) or start.numel() != B:
            raise RuntimeError('o, d must be (B, 3) and start (B)')
        site = torch.empty(B, S, dtype=torch.int32, device=z.device)
        steps = torch.empty(B, dtype=torch.int32, device=z.device)
        if B == 0:
            return [site, steps]
        pk = graph_pack(points, offsets, adj)
        with torch.cuda.device(z.device):
            _lib.call('vg_walk', pk.ptr, pk.n, pk.m, o.data_ptr(), d.data_ptr(), _ptr(z), start.data_ptr(), B, S,
                      _ptr(site), steps.data_ptr(), _stream(z.device))
        return [site, steps]

    @staticmethod
    def _field_checks(points, offsets, adj, log_scale, quat, x, site, **extra):
        for t, name, dt in ((points, 'points', torch.float32), (offsets, 'offsets', torch.int32),
                            (adj, 'adj', torch.int32), (log_scale, 'log_scale', torch.float32),
                            (quat, 'quat', torch.float32), (x, 'x', torch.float32), (site, 'site', torch.int32)):
            _check(t, name, dt)
        for name, t in extra.items():
            _check(t, name, torch.float32)
        n, m = points.size(0), x.size(0)
        if log_scale.shape != (n, 3) or quat.shape != (n, 4):
            raise RuntimeError('log_scale must be (N, 3) and quat (N, 4)')
        if x.dim() != 2 or x.size(1) != 3 or site.numel() != m:
            raise RuntimeError('x must be (M, 3) and site (M)')
        return m

    @staticmethod
    def _ws(n, sh_deg, kind, dev, m=0):
        nbytes = _lib.lib().vg_field_workspace_bytes(n, int(sh_deg), kind, int(m))
        return torch.empty(max(nbytes, 256), dtype=torch.uint8, device=dev), nbytes

    @classmethod
    def density_forward(cls, points, offsets, adj, raw, log_scale, quat, x, site, scale_mult):
        m = cls._field_checks(points, offsets, adj, log_scale, quat, x, site, raw=raw)
        if raw.numel() != points.size(0):
            raise RuntimeError('raw must be (N)')
        sigma = torch.empty(m, device=x.device)
        if m == 0:
            return sigma
        pk = graph_pack(points, offsets, adj)
        ws, nbytes = cls._ws(pk.n, 0, 0, x.device)
        with torch.cuda.device(x.device):
            _lib.call('vg_density_forward', pk.ptr, pk.n, pk.m, raw.data_ptr(), log_scale.data_ptr(),
                      quat.data_ptr(), x.data_ptr(), site.data_ptr(), m, float(scale_mult), sigma.data_ptr(),
                      ws.data_ptr(), nbytes, _stream(x.device))
        return sigma

    @classmethod
    def density_backward(cls, points, offsets, adj, raw, log_scale, quat, x, site, grad_sigma):
        m = cls._field_checks(points, offsets, adj, log_scale, quat, x, site, raw=raw, grad_sigma=grad_sigma)
        if raw.numel() != points.size(0) or grad_sigma.numel() != m:
            raise RuntimeError('raw must be (N) and grad_sigma (M)')
        g_raw, g_ls, g_quat = torch.empty_like(raw), torch.empty_like(log_scale), torch.empty_like(quat)
        pk = graph_pack(points, offsets, adj)
        ws, nbytes = cls._ws(pk.n, 0, 1, x.device, m)
        with torch.cuda.device(x.device):
            _lib.call('vg_density_backward', pk.ptr, pk.n, pk.m, raw.data_ptr(), log_scale.data_ptr(),
                      quat.data_ptr(), _ptr(x), _ptr(site), m, _ptr(grad_sigma), g_raw.data_ptr(), g_ls.data_ptr(),
                      g_quat.data_ptr(), ws.data_ptr(), nbytes, _stream(x.device))
        return [g_raw, g_ls, g_quat]

    @classmethod
    def color_forward(cls, points, offsets, adj, log_scale, quat, sh, sh_deg, x, dirs, site):
        m = cls._field_checks(points, offsets, adj, log_scale, quat, x, site, sh=sh, dirs=dirs)
        if sh.dim() != 3 or sh.size(1) != 16 or sh.size(2) != 3:
            raise RuntimeError('sh must be (N, 16, 3)')
        if dirs.shape != (m, 3):
            raise RuntimeError('dirs must be (M, 3)')
        sh_deg = _sh_deg(sh_deg)
        rgb = torch.empty(m, 3, device=x.device)
        if m == 0:
            return rgb
        pk = graph_pack(points, offsets, adj)
        ws, nbytes = cls._ws(pk.n, sh_deg, 2, x.device)
        with torch.cuda.device(x.device):
            _lib.call('vg_color_forward', pk.ptr, pk.n, pk.m, log_scale.data_ptr(), quat.data_ptr(), sh.data_ptr(),
                      sh_deg, x.data_ptr(), dirs.data_ptr(), site.data_ptr(), m, rgb.data_ptr(), ws.data_ptr(),
                      nbytes, _stream(x.device))
        return rgb

    @classmethod
    def color_backward(cls, points, offsets, adj, log_scale, quat, sh, sh_deg, x, dirs, site, rgb, grad_rgb):
        m = cls._field_checks(points, offsets, adj, log_scale, quat, x, site, sh=sh, dirs=dirs, rgb=rgb,
                              grad_rgb=grad_rgb)
        if sh.dim() != 3 or sh.size(1) != 16 or sh.size(2) != 3:
            raise RuntimeError('sh must be (N, 16, 3)')
        if dirs.shape != (m, 3) or rgb.shape != (m, 3) or grad_rgb.shape != (m, 3):
            raise RuntimeError('dirs, rgb and grad_rgb must be (M, 3)')
        sh_deg = _sh_deg(sh_deg)
        g_ls, g_quat, g_sh = torch.empty_like(log_scale), torch.empty_like(quat), torch.empty_like(sh)
        pk = graph_pack(points, offsets, adj)
        ws, nbytes = cls._ws(pk.n, sh_deg, 3, x.device, m)
        with torch.cuda.device(x.device):
            _lib.call('vg_color_backward', pk.ptr, pk.n, pk.m, log_scale.data_ptr(), quat.data_ptr(), sh.data_ptr(),
                      sh_deg, _ptr(x), _ptr(dirs), _ptr(site), m, _ptr(rgb), _ptr(grad_rgb), g_ls.data_ptr(),
                      g_quat.data_ptr(), g_sh.data_ptr(), ws.data_ptr(), nbytes, _stream(x.device))
        return [g_ls, g_quat, g_sh]

    @staticmethod
    def conic_forward(log_scale, quat, floor):
        _check(log_scale, 'log_scale', torch.float32)
        _check(quat, 'quat', torch.float32)
        n = quat.size(0)
        A = torch.empty(n, 6, device=quat.device)
        if n:
            with torch.cuda.device(quat.device):
                _lib.call('vg_conic_forward', log_scale.data_ptr(), quat.data_ptr(), n, float(floor), A.data_ptr(),
                          _stream(quat.device))
        return A

    @staticmethod
    def conic_backward(log_scale, quat, floor, gA):
        _check(log_scale, 'log_scale', torch.float32)
        _check(quat, 'quat', torch.float32)
        _check(gA, 'gA', torch.float32)
        n = quat.size(0)
        g_ls, g_quat = torch.empty_like(log_scale), torch.empty_like(quat)
        if n:
            with torch.cuda.device(quat.device):
                _lib.call('vg_conic_backward', log_scale.data_ptr(), quat.data_ptr(), n, float(floor), gA.data_ptr(),
                          g_ls.data_ptr(), g_quat.data_ptr(), _stream(quat.device))
        return [g_ls, g_quat]


_TRACE_CACHE = {}  # trace records of recent inference layouts (see trace_records)
_TRACE_CACHE_SIZE = 4


def trace_records(nbr, edge, attr, n_sites):
    """Trace records (E, 12) of an inference layout for the deferred renderer (vg_infer_trace_records).
    They depend only on nbr, edge and attr (columns 0-7), so they are built once per layout and reused.
    An entry is valid while the very tensor objects it was built from are alive and unmodified: it holds
    weak references to them and their in-place version counters (a new layout that reuses freed memory
    is a different object, so it never matches a stale entry)."""
    import weakref
    entry = _TRACE_CACHE.get(id(edge))
    if entry is not None:
        refs, versions, rec = entry
        live = tuple(r() for r in refs)
        if (live[0] is nbr and live[1] is edge and live[2] is attr and
                versions == (nbr._version, edge._version, attr._version) and rec.size(0) == nbr.numel()):
            return rec
        del _TRACE_CACHE[id(edge)]
    rec = torch.empty(nbr.numel(), 12, device=edge.device)
    with torch.cuda.device(edge.device):
        _lib.call('vg_infer_trace_records', nbr.data_ptr(), edge.data_ptr(), attr.data_ptr(), n_sites, nbr.numel(),
                  rec.data_ptr(), _stream(edge.device))
    while len(_TRACE_CACHE) >= _TRACE_CACHE_SIZE:
        _TRACE_CACHE.pop(next(iter(_TRACE_CACHE)))
    _TRACE_CACHE[id(edge)] = (tuple(weakref.ref(t) for t in (nbr, edge, attr)),
                              (nbr._version, edge._version, attr._version), rec)
    return rec


class FoamInferExtension:
    """foam_infer with the reference's signature (foam_infer.cu:376-435).

    At stage 2 the colours are deferred to a cell-major pass (vg_foam_infer_deferred): the same rgb, T,
    depth and stats columns 0-3 bit for bit, with stats column 4 counting the SH colours that pass
    evaluated. exact_stats=True renders per ray instead (vg_foam_infer), whose column 4 counts the misses
    of a per-ray colour cache like the reference kernel's. trace: the layout's trace records
    (trace_records), built and cached here when not given."""

    @staticmethod
    def foam_infer(points, offsets, nbr, edge, attr, sh, sh_deg, o, d, start, near, far, t_thresh, w_thresh,
                   color_cut, color_mode, stage, cap, orig, exact_stats=False, trace=None):
        for x, name, dt in ((points, 'points', torch.float32), (offsets, 'offsets', torch.int32),
                            (nbr, 'nbr', torch.int32), (edge, 'edge', torch.float32), (attr, 'attr', torch.float32),
                            (cap, 'cap', torch.int32), (orig, 'orig', torch.int32)):
            _check(x, name, dt)
        B = _ray_checks(o=o, d=d, start=start, near=near, far=far)
        if not (sh.is_cuda and sh.is_contiguous()):
            raise RuntimeError('sh must be a contiguous CUDA tensor')
        half = sh.dtype == torch.float16
        if not (half or sh.dtype == torch.float32):
            raise RuntimeError('sh must be float32 or float16')
        n = points.size(0)
        if points.dim() != 2 or points.size(1) != 4:
            raise RuntimeError('points must be (N, 4)')
        if offsets.numel() != n + 1:
            raise RuntimeError('offsets must be (N + 1)')
        if edge.dim() != 2 or edge.size(1) != 4 or edge.size(0) != nbr.numel():
            raise RuntimeError('edge must be (E, 4)')
        if attr.dim() != 2 or attr.size(1) != 20 or attr.size(0) != n:
            raise RuntimeError('attr must be (N, 20)')
        color_mode, stage = int(color_mode), int(stage)
        if not 0 <= color_mode <= 2:
            raise RuntimeError('color_mode must be 0 (lazy), 1 (baked) or 2 (fused)')
        baked = color_mode == 1
        if not baked and not (sh.dim() == 3 and sh.size(0) == n and sh.size(1) == 16 and sh.size(2) == 3):
            raise RuntimeError('sh must be (N, 16, 3)')
        if not 0 <= stage <= 2:
            raise RuntimeError('stage must be 0, 1 or 2')
        dev = o.device
        rgb = torch.empty(B, 3, device=dev)
        T = torch.empty(B, device=dev)
        depth = torch.empty(B, device=dev)
        stats = torch.empty(B, 5, dtype=torch.int32, device=dev)
        if B == 0:
            return [rgb, T, depth, stats]
        head = [points.data_ptr(), offsets.data_ptr(), nbr.data_ptr(), edge.data_ptr(), attr.data_ptr(),
                None if baked else _ptr(sh), int(half), _sh_deg(sh_deg), n, nbr.numel(), o.data_ptr(), d.data_ptr(),
                start.data_ptr(), near.data_ptr(), far.data_ptr(), B, float(t_thresh), float(w_thresh),
                float(color_cut), color_mode, stage, _ptr(cap) if cap.numel() == B else None,
                _ptr(orig) if orig.numel() == n else None]
        outs = [rgb.data_ptr(), T.data_ptr(), depth.data_ptr(), stats.data_ptr()]
        with torch.cuda.device(dev):
            if stage == 2 and not exact_stats:
                if trace is None:
                    trace = trace_records(nbr, edge, attr, n)
                elif trace.shape != (nbr.numel(), 12) or trace.dtype != torch.float32 or not trace.is_contiguous():
                    raise RuntimeError('trace must be the (E, 12) float32 trace records of the layout')
                nbytes = _lib.lib().vg_foam_infer_workspace_bytes(n, B)
                ws = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=dev)
                _lib.call('vg_foam_infer_deferred', *head, trace.data_ptr(), *outs, ws.data_ptr(), nbytes, _stream(dev))
            else:
                _lib.call('vg_foam_infer', *head, *outs, _stream(dev))
        return [rgb, T, depth, stats]


_FOAM, _MARCH, _FIELD, _INFER = FoamExtension(), MarchExtension(), FieldExtension(), FoamInferExtension()


def extension():
    return _FIELD


def march_extension():
    return _MARCH


def foam_extension():
    return _FOAM


def foam_infer_extension():
    return _INFER


# ---------------------------------------------------------------------------------------- autograd
#
# One autograd node type (_OpNode) serves every differentiable op. An op object carries the
# non-differentiable context of one call (graph, rays, settings) and knows four things: how to run the
# extension's forward on the differentiable tensors, which tensors its backward needs, which outputs
# carry no gradient, and how to turn output gradients into input gradients. The contracts are those of
# the reference's autograd functions (ext.py:61-216): the same saved tensors, the same non-differentiable
# outputs (depth, stats), gradients for the same inputs, and the same no-gradient shortcuts (the foam
# forward keeps no records then).


def _wants_grad(tensors):
    return torch.is_grad_enabled() and any(t.requires_grad for t in tensors)


def _dense(*tensors):
    return [t.contiguous() for t in tensors]


def _grad_or_zeros(g, like):
    return torch.zeros_like(like) if g is None else g.contiguous()


class _OpNode(torch.autograd.Function):
    @staticmethod
    def forward(ctx, op, *inputs):
        outputs = op.run(*inputs)
        ctx.op, ctx.n_inputs = op, len(inputs)
        ctx.save_for_backward(*inputs, *op.needs(outputs))
        frozen = op.frozen(outputs)
        if frozen:
            ctx.mark_non_differentiable(*frozen)
        return op.visible(outputs)

    @staticmethod
    def backward(ctx, *grads):
        saved = ctx.saved_tensors
        n = ctx.n_inputs
        return (None, *ctx.op.grads(saved[:n], saved[n:], grads))


class _Op:
    """Defaults: the backward needs only the inputs, every output is differentiable and visible."""

    def needs(self, outputs):
        return ()

    def frozen(self, outputs):
        return ()

    def visible(self, outputs):
        return outputs


class _ConicOp(_Op):
    def __init__(self, floor):
        self.floor = floor

    def run(self, log_scale, quat):
        return extension().conic_forward(log_scale, quat, self.floor)

    def grads(self, inputs, kept, grads):
        log_scale, quat = inputs
        g_ls, g_quat = extension().conic_backward(log_scale, quat, self.floor, grads[0].contiguous())
        return g_ls, g_quat


class _DensityOp(_Op):
    def __init__(self, graph, x, site):
        self.graph, self.x, self.site = graph, x, site

    def run(self, raw, log_scale, quat):
        g = self.graph
        return extension().density_forward(g.points, g.offsets, g.adj, raw, log_scale, quat, self.x, self.site, 1.0)

    def needs(self, sigma):
        return self.x, self.site

    def grads(self, inputs, kept, grads):
        g = self.graph
        x, site = kept
        return extension().density_backward(g.points, g.offsets, g.adj, *inputs, x, site, grads[0].contiguous())


class _ColorOp(_Op):
    def __init__(self, graph, x, dirs, site, sh_deg):
        self.graph, self.x, self.dirs, self.site, self.sh_deg = graph, x, dirs, site, sh_deg

    def run(self, log_scale, quat, sh):
        g = self.graph
        return extension().color_forward(g.points, g.offsets, g.adj, log_scale, quat, sh, self.sh_deg, self.x,
                                         self.dirs, self.site)

    def needs(self, rgb):
        return self.x, self.dirs, self.site, rgb

    def grads(self, inputs, kept, grads):
        g = self.graph
        x, dirs, site, rgb = kept
        log_scale, quat, sh = inputs
        return extension().color_backward(g.points, g.offsets, g.adj, log_scale, quat, sh, self.sh_deg, x, dirs, site,
                                          rgb, grads[0].contiguous())


class _RenderOp(_Op):
    """Shared by foam and march: the scene tensors (raw, dA, cA, sh) are the differentiable inputs, the
    rays travel with the op; outputs (rgb, T, depth, stats[, rec]), of which depth and stats carry no
    gradient and rec (foam only) stays hidden."""

    def __init__(self, graph, rays, sh_deg, settings):
        self.graph, self.rays, self.sh_deg, self.settings = graph, rays, sh_deg, settings

    def frozen(self, outputs):
        return outputs[2], outputs[3]

    def visible(self, outputs):
        return tuple(outputs[:4])

    def scene(self):
        g = self.graph
        return g.points, g.offsets, g.adj


class _FoamOp(_RenderOp):
    def __init__(self, graph, rays, sh_deg, t_thresh, w_thresh, record_cap):
        super().__init__(graph, rays, sh_deg, (t_thresh, w_thresh))
        self.record_cap = record_cap

    def run(self, raw, dA, cA, sh, record_cap=None):
        cap = self.record_cap if record_cap is None else record_cap
        B = self.rays[0].size(0)
        # a recording (training) forward also keeps the per-cell sample counts of its records, which its
        # backward reads instead of counting the records again
        counts = None
        if cap > 0 and B > 0:
            counts = torch.empty(sample_counts_size(self.graph.points.size(0), B, cap), dtype=torch.int32,
                                 device=raw.device)
        out = foam_extension().foam_forward(*self.scene(), raw, dA, cA, sh, self.sh_deg, *self.rays, *self.settings,
                                            cap, counts=counts)
        return [*out, counts if counts is not None else out[3].new_empty(0)]

    def needs(self, outputs):
        rgb, T, _, stats, rec, counts = outputs
        return (rgb, T, rec, stats, counts, *self.rays)

    def grads(self, inputs, kept, grads):
        rgb, T, rec, stats, counts, *rays = kept
        return foam_extension().foam_backward(*self.scene(), *inputs, self.sh_deg, *rays, *self.settings, rgb, T,
                                              _grad_or_zeros(grads[0], rgb), _grad_or_zeros(grads[1], T), rec,
                                              stats, counts=counts if counts.numel() else None)


class _MarchOp(_RenderOp):
    def run(self, raw, dA, cA, sh):
        return march_extension().march_forward(*self.scene(), raw, dA, cA, sh, self.sh_deg, *self.rays,
                                               *self.settings)

    def needs(self, outputs):
        rgb, T = outputs[0], outputs[1]
        return (rgb, T, *self.rays)

    def grads(self, inputs, kept, grads):
        rgb, T, *rays = kept
        return march_extension().march_backward(*self.scene(), *inputs, self.sh_deg, *rays, *self.settings, rgb, T,
                                                _grad_or_zeros(grads[0], rgb), _grad_or_zeros(grads[1], T))


def _rays(o, d, start, *bounds):
    """Ray tensors in the extension's dtypes: float32 o, d and bounds, int32 start sites."""
    return (o.float().contiguous(), d.float().contiguous(), start.int().contiguous(),
            *(b.float().contiguous() for b in bounds))


def conic(log_scale, quat, floor=0.0):
    """(N, 6) inverse covariances (xx, xy, xz, yy, yz, zz) of R diag(s^2 + floor^2) R^T (ext.py:134-136)."""
    return _OpNode.apply(_ConicOp(float(floor)), *_dense(log_scale, quat))


def conic_reference(log_scale, quat, floor=0.0):
    """Plain torch version of conic, for tests (ext.py:139-149): the rotation of the normalised
    quaternion (w, x, y, z) from its pairwise products, then R diag(1 / (s^2 + floor^2)) R^T."""
    u = quat / quat.norm(dim=-1, keepdim=True).clamp_min(1e-12)
    w, x, y, z = u.unbind(-1)
    xx, yy, zz = x * x, y * y, z * z
    xy, xz, yz = x * y, x * z, y * z
    wx, wy, wz = w * x, w * y, w * z
    R = torch.stack((1 - 2 * (yy + zz), 2 * (xy - wz), 2 * (xz + wy),
                     2 * (xy + wz), 1 - 2 * (xx + zz), 2 * (yz - wx),
                     2 * (xz - wy), 2 * (yz + wx), 1 - 2 * (xx + yy)), -1).view(-1, 3, 3)
    variance = torch.exp(2 * log_scale.clamp(-20, 20)) + floor * floor
    A = (R * (1.0 / variance)[:, None, :]) @ R.transpose(1, 2)
    return A[:, (0, 0, 0, 1, 1, 2), (0, 1, 2, 1, 2, 2)].contiguous()


def density(graph, raw, log_scale, quat, x, site, scale_mult=1.0):
    """sigma(x) = sum over the Voronoi neighbourhood of site of exp(raw_k) G_k(x) (ext.py:78-87).
    scale_mult widens the Gaussians (proposal passes): then, as without autograd, no graph is recorded."""
    x, site = x.detach().float().contiguous(), site.int().contiguous()
    params = _dense(raw, log_scale, quat)
    if scale_mult == 1.0 and _wants_grad(params):
        return _OpNode.apply(_DensityOp(graph, x, site), *params)
    return extension().density_forward(graph.points, graph.offsets, graph.adj, *(p.detach() for p in params), x, site,
                                       float(scale_mult))


def color(graph, log_scale, quat, sh, x, dirs, site, sh_deg=3):
    """C(x, d) = sum_k H_k(x) c_k(d) / sum_k H_k(x) over the Voronoi neighbourhood of site; sh (N, 16, 3)
    (ext.py:109-117)."""
    op = _ColorOp(graph, x.detach().float().contiguous(), dirs.detach().float().contiguous(), site.int().contiguous(),
                  int(sh_deg))
    params = _dense(log_scale, quat, sh)
    if _wants_grad(params):
        return _OpNode.apply(op, *params)
    return op.run(*(p.detach() for p in params))


def march(graph, raw, dA, cA, sh, sh_deg, o, d, start, near, mid, far, dt, n_bg, t_thresh=1e-4, w_thresh=1e-4):
    """Fixed-step rendering (ext.py:172-182): midpoints of dt steps from near to mid, then n_bg steps evenly
    spaced in 1/t out to far. Returns the foreground colour (B, 3), the remaining transmittance (B,), the
    depth (B,) and int32 counts per ray (B, 3): samples marched, samples coloured, walk steps."""
    op = _MarchOp(graph, _rays(o, d, start, near, mid, far), int(sh_deg),
                  (float(dt), int(n_bg), float(t_thresh), float(w_thresh)))
    params = _dense(raw, dA, cA, sh)
    if _wants_grad(params):
        return _OpNode.apply(op, *params)
    return op.run(*(p.detach() for p in params))


def foam(graph, raw, dA, cA, sh, sh_deg, o, d, start, near, far, t_thresh=1e-4, w_thresh=1e-4, record_cap=256):
    """Renders the rays at their crossings with the Voronoi faces (ext.py:205-216). Returns the foreground
    colour (B, 3) without background, the transmittance left after the last segment (B,), the depth (B,) and
    int32 counts per ray (B, 3): samples, coloured segments, walk steps to x(near). When gradients are
    needed, the first record_cap samples of every ray are recorded for the backward pass; rays with more
    samples, and all rays when record_cap is 0, are traced again there."""
    op = _FoamOp(graph, _rays(o, d, start, near, far), int(sh_deg), float(t_thresh), float(w_thresh),
                 int(record_cap))
    params = _dense(raw, dA, cA, sh)
    if _wants_grad(params):
        return _OpNode.apply(op, *params)
    return op.run(*(p.detach() for p in params), record_cap=0)[:4]
