"""TEST INFRASTRUCTURE ONLY — torch restatement of the reference's inference packing (render.py:168-235:
morton_order, pack_foam, bake_colors), the checker of the device packing (vg_infer_pack /
vg_bake_colors). Pinned to the layouts the reference's own render.py produced (tests/golden/
foam_small.npz, tests/test_pack_host.py). Runs on CPU or GPU tensors; `conic` is the conic function to
use (the product's ext.conic on the GPU, ext.conic_reference on the CPU). The product never imports it.
"""

from __future__ import annotations

import math

import torch


def morton_order(points, bits=10):
    """Z-order permutation of the points' bounding box (render.py:168-176), stable for equal codes."""
    lo, hi = points.amin(0), points.amax(0)
    q = ((points - lo) / (hi - lo).clamp_min(1e-12) * (2 ** bits - 1)).long()
    code = torch.zeros(len(points), dtype=torch.long, device=points.device)
    for b in range(bits):
        for a in range(3):
            code |= ((q[:, a] >> b) & 1) << (3 * b + a)
    return torch.argsort(code, stable=True)


@torch.no_grad()
def pack_foam(model, conic, scale_floor=0.0, eps_density=0.0, sh_half=False, reorder=False):
    """render.py:179-225 restated with torch gathers (same outputs as the device packing)."""
    g = model.graph
    n = len(g.points)
    dev = g.points.device
    raw = model.raw.clamp(max=30.0)
    if eps_density > 0:
        s_max2 = (torch.exp(2 * model.d_log_scale.clamp(-20, 20)) + scale_floor ** 2).amax(-1)
        r2 = 2 * s_max2 * (raw - math.log(eps_density)).clamp_min(0) * (1 + 2 ** -9)
    else:
        r2 = torch.full_like(raw, float('inf'))
    lam = 1.0 / (torch.exp(2 * model.c_log_scale.clamp(-20, 20)) + scale_floor ** 2).amax(-1)
    lam = (lam * (1 - 2 ** -9)).clamp(max=65000.0)
    cut = torch.stack([r2, lam], -1).half().view(torch.float32)[:, 0]
    off = g.offsets.long()
    deg = off[1:] - off[:-1]
    offsets = off + torch.arange(n + 1, device=dev)
    row = torch.repeat_interleave(torch.arange(n, device=dev), deg)
    nbr = torch.empty(len(g.adj) + n, dtype=torch.long, device=dev)
    nbr[offsets[:-1]] = torch.arange(n, device=dev)
    nbr[torch.arange(len(g.adj), device=dev) + row + 1] = g.adj.long()
    edge = torch.cat([g.points[nbr], cut[nbr, None]], 1).contiguous()
    points = torch.cat([g.points, torch.zeros_like(raw)[:, None]], 1).contiguous()
    dA = conic(model.d_log_scale, model.d_quat, scale_floor)
    cA = conic(model.c_log_scale, model.c_quat, scale_floor)
    z = torch.zeros_like(raw)[:, None]
    attr = torch.cat([dA, raw[:, None], z, cA, z, z, z, z, z, z], 1).contiguous()
    sh = model.sh().contiguous()
    perm = inv = None
    if reorder:
        perm = morton_order(g.points)
        inv = torch.empty_like(perm)
        inv[perm] = torch.arange(n, device=dev)
        size = (deg + 1)[perm]
        new_off = torch.cat([torch.zeros_like(size[:1]), torch.cumsum(size, 0)])
        cell = torch.repeat_interleave(torch.arange(n, device=dev), size)
        old = offsets[perm][cell] + torch.arange(len(nbr), device=dev) - new_off[cell]
        offsets, nbr, edge = new_off, inv[nbr[old]], edge[old].contiguous()
        points, attr, sh = points[perm].contiguous(), attr[perm].contiguous(), sh[perm].contiguous()
    return {'points': points, 'offsets': offsets.int().contiguous(), 'nbr': nbr.int().contiguous(), 'edge': edge,
            'attr': attr, 'sh': sh.half() if sh_half else sh, 'sh32': sh, 'perm': perm, 'inv': inv,
            'orig': (perm if reorder else torch.empty(0, device=dev)).int().contiguous()}


def sh_basis(d, deg):
    """(B, 16) real SH basis, the reference's constants (render.py:143-165)."""
    x, y, z = d.unbind(-1)
    b = torch.zeros(len(d), 16, device=d.device, dtype=d.dtype)
    b[:, 0] = 0.28209479177387814
    if deg >= 1:
        b[:, 1], b[:, 2], b[:, 3] = -0.4886025119029199 * y, 0.4886025119029199 * z, -0.4886025119029199 * x
    if deg >= 2:
        xx, yy, zz = x * x, y * y, z * z
        b[:, 4], b[:, 5] = 1.0925484305920792 * x * y, -1.0925484305920792 * y * z
        b[:, 6], b[:, 7] = 0.31539156525252005 * (2 * zz - xx - yy), -1.0925484305920792 * x * z
        b[:, 8] = 0.5462742152960396 * (xx - yy)
    if deg >= 3:
        b[:, 9], b[:, 10] = -0.5900435899266435 * y * (3 * xx - yy), 2.890611442640554 * x * y * z
        b[:, 11] = -0.4570457994644658 * y * (4 * zz - xx - yy)
        b[:, 12] = 0.3731763325901154 * z * (2 * zz - 3 * xx - 3 * yy)
        b[:, 13] = -0.4570457994644658 * x * (4 * zz - xx - yy)
        b[:, 14], b[:, 15] = 1.445305721320277 * z * (xx - yy), -0.5900435899266435 * x * (xx - 3 * yy)
    return b


@torch.no_grad()
def baked_colors(points4, sh32, sh_deg, center):
    """render.py:228-235: max(SH_k(d_k) + 1/2, 0), d_k the unit direction from `center` to site k."""
    dirs = torch.nn.functional.normalize(points4[:, :3] - center.view(1, 3), dim=-1)
    return torch.einsum('nj,njc->nc', sh_basis(dirs, sh_deg), sh32).add_(0.5).clamp_min_(0.0)
