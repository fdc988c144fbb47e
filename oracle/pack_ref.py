"""TEST INFRASTRUCTURE ONLY — torch restatement of the reference's inference packing (render.py:168-235:
morton_order, pack_foam, bake_colors), the checker of the device packing (vg_infer_pack /
vg_bake_colors). Pinned to the layouts the reference's own render.py produced (tests/golden/
foam_small.npz, tests/test_pack_host.py). Runs on CPU or GPU tensors; `conic` is the conic function to
use (the product's ext.conic on the GPU, ext.conic_reference on the CPU). The product never imports it.

Layout (render.py:179-225): points (N, 4) = (p, 0); a self-first CSR (offsets (N + 1), nbr (N + M)) whose
run for cell i is i followed by its Delaunay neighbours in adjacency order; edge (N + M, 4) = (p_j, the
bits of half2(r2_j, lam_j)); attr (N, 20) = (dA[6], min(raw, 30), 0, cA[6], 0 x 6); sh (N, 16, 3) fp32 or
fp16. With reorder, sites are renumbered along the Morton curve (perm: new -> old) and orig = perm.
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F

_SAFE_UP, _SAFE_DOWN = 1 + 2 ** -9, 1 - 2 ** -9  # rounding margins of the fp16 cut values
_LAM_MAX = 65000.0                                # below the largest finite fp16


def _spread_bits(v):
    """Moves bit k of a 10-bit integer to bit 3 k (two zero bits between consecutive bits)."""
    v = v & 0x3FF
    v = (v | (v << 16)) & 0x030000FF
    v = (v | (v << 8)) & 0x0300F00F
    v = (v | (v << 4)) & 0x030C30C3
    return (v | (v << 2)) & 0x09249249


def morton_order(points, bits=10):
    """Z-order permutation over the points' bounding box (render.py:168-176): 10-bit quantisation per
    axis, x in the lowest interleaved bit; stable for equal codes."""
    assert bits <= 10
    lo, hi = points.amin(0), points.amax(0)
    q = ((points - lo) / (hi - lo).clamp_min(1e-12) * (2 ** bits - 1)).long()
    code = _spread_bits(q[:, 0]) | (_spread_bits(q[:, 1]) << 1) | (_spread_bits(q[:, 2]) << 2)
    return torch.argsort(code, stable=True)


def _largest_variance(log_scale, floor2):
    """max over the three axes of s^2 + floor^2, s = exp(clamp(log_scale, -20, 20))."""
    return (torch.exp(2 * log_scale.clamp(-20, 20)) + floor2).amax(-1)


def _cuts(model, raw, scale_floor, eps_density):
    """Per-site half2 (r2, lam) as one float32 word: r2 the squared distance beyond which the site's density
    is below eps_density (inf when eps_density = 0), lam a lower bound of the colour conic's eigenvalues."""
    floor2 = scale_floor ** 2
    if eps_density > 0:
        excess = (raw - math.log(eps_density)).clamp_min(0)
        r2 = 2 * _largest_variance(model.d_log_scale, floor2) * excess * _SAFE_UP
    else:
        r2 = torch.full_like(raw, float('inf'))
    lam = ((1.0 / _largest_variance(model.c_log_scale, floor2)) * _SAFE_DOWN).clamp(max=_LAM_MAX)
    return torch.stack([r2, lam], -1).half().view(torch.float32).squeeze(-1)


def _self_first(offsets, adj):
    """Self-first CSR of (offsets, adj): run i = [i, adj[offsets[i]:offsets[i + 1]]]."""
    n = len(offsets) - 1
    ids = torch.arange(n, device=adj.device)
    owner = torch.repeat_interleave(ids, offsets[1:] - offsets[:-1])
    # a stable sort by owning cell keeps every cell's own id (listed first) ahead of its neighbours
    order = torch.argsort(torch.cat([ids, owner]), stable=True)
    return offsets + torch.arange(n + 1, device=adj.device), torch.cat([ids, adj])[order]


@torch.no_grad()
def pack_foam(model, conic, scale_floor=0.0, eps_density=0.0, sh_half=False, reorder=False):
    """render.py:179-225 restated with torch gathers (same outputs as the device packing)."""
    g = model.graph
    n = len(g.points)
    dev = g.points.device
    raw = model.raw.clamp(max=30.0)
    cut = _cuts(model, raw, scale_floor, eps_density)
    offsets, nbr = _self_first(g.offsets.long(), g.adj.long())
    edge = torch.cat([g.points[nbr], cut[nbr].unsqueeze(1)], 1)
    points = F.pad(g.points, (0, 1))
    attr = torch.zeros(n, 20, device=dev, dtype=raw.dtype)
    attr[:, 0:6] = conic(model.d_log_scale, model.d_quat, scale_floor)
    attr[:, 6] = raw
    attr[:, 8:14] = conic(model.c_log_scale, model.c_quat, scale_floor)
    sh = model.sh().contiguous()
    perm = inv = None
    if reorder:
        perm = morton_order(g.points)
        inv = torch.empty_like(perm)
        inv[perm] = torch.arange(n, device=dev)
        run = (offsets[1:] - offsets[:-1])[perm]
        new_offsets = F.pad(torch.cumsum(run, 0), (1, 0))
        # slot e of new cell i holds slot offsets[perm[i]] + (e - new_offsets[i]) of the old layout
        shift = torch.repeat_interleave(offsets[:-1][perm] - new_offsets[:-1], run)
        src = shift + torch.arange(len(nbr), device=dev)
        offsets, nbr, edge = new_offsets, inv[nbr[src]], edge[src]
        points, attr, sh = points[perm], attr[perm], sh[perm]
    sh = sh.contiguous()
    return {'points': points.contiguous(), 'offsets': offsets.int().contiguous(), 'nbr': nbr.int().contiguous(),
            'edge': edge.contiguous(), 'attr': attr.contiguous(), 'sh': sh.half() if sh_half else sh, 'sh32': sh,
            'perm': perm, 'inv': inv,
            'orig': (perm if reorder else torch.empty(0, device=dev)).int().contiguous()}


# The real SH basis by band (render.py:143-165): (index, constant, polynomial) with the constants and
# signs of the reference's kernels.
_BASIS = (
    (1, -0.4886025119029199, lambda x, y, z, xx, yy, zz: y),
    (2, 0.4886025119029199, lambda x, y, z, xx, yy, zz: z),
    (3, -0.4886025119029199, lambda x, y, z, xx, yy, zz: x),
    (4, 1.0925484305920792, lambda x, y, z, xx, yy, zz: x * y),
    (5, -1.0925484305920792, lambda x, y, z, xx, yy, zz: y * z),
    (6, 0.31539156525252005, lambda x, y, z, xx, yy, zz: 2 * zz - xx - yy),
    (7, -1.0925484305920792, lambda x, y, z, xx, yy, zz: x * z),
    (8, 0.5462742152960396, lambda x, y, z, xx, yy, zz: xx - yy),
    (9, -0.5900435899266435, lambda x, y, z, xx, yy, zz: y * (3 * xx - yy)),
    (10, 2.890611442640554, lambda x, y, z, xx, yy, zz: x * y * z),
    (11, -0.4570457994644658, lambda x, y, z, xx, yy, zz: y * (4 * zz - xx - yy)),
    (12, 0.3731763325901154, lambda x, y, z, xx, yy, zz: z * (2 * zz - 3 * xx - 3 * yy)),
    (13, -0.4570457994644658, lambda x, y, z, xx, yy, zz: x * (4 * zz - xx - yy)),
    (14, 1.445305721320277, lambda x, y, z, xx, yy, zz: z * (xx - yy)),
    (15, -0.5900435899266435, lambda x, y, z, xx, yy, zz: x * (xx - 3 * yy)),
)


def sh_basis(d, deg):
    """(B, 16) real SH basis of unit directions d; functions above degree `deg` are zero."""
    x, y, z = d.unbind(-1)
    xx, yy, zz = x * x, y * y, z * z
    b = torch.zeros(len(d), 16, device=d.device, dtype=d.dtype)
    b[:, 0] = 0.28209479177387814
    for k, c, poly in _BASIS[:(deg + 1) ** 2 - 1]:
        b[:, k] = c * poly(x, y, z, xx, yy, zz)
    return b


@torch.no_grad()
def baked_colors(points4, sh32, sh_deg, center):
    """render.py:228-235: max(SH_k(d_k) + 1/2, 0), d_k the unit direction from `center` to site k."""
    dirs = F.normalize(points4[:, :3] - center.view(1, 3), dim=-1)
    return (torch.einsum('nj,njc->nc', sh_basis(dirs, sh_deg), sh32) + 0.5).clamp_min(0.0)
