"""Trained-scene checkpoints in the reference's format, so scenes trained by voronoi-gauss load here.

The reference's train.py (train.py:168-170) saves one ``torch.save`` dict:
``state`` (the model's state_dict: raw, d_log_scale, d_quat, c_log_scale, c_quat, sh_dc, sh_rest,
bg_logit), ``points`` (N, 3), ``offsets`` (N + 1) and ``adj`` (M) (the fixed sites and their Delaunay
CSR), ``sh_deg`` (the active SH degree), ``normalization`` (the scene transform) and ``args``.
``load_model`` rebuilds a ``VoronoiGaussField`` from it the way bench_fps.load_model does
(bench_fps.py:19-28); ``save_model`` writes the same dict.
"""

from __future__ import annotations

import torch

from .model import VoronoiGaussField


def load_model(path, device='cuda', requires_grad=False):
    """(model, checkpoint dict) from a reference checkpoint; parameters on `device`."""
    ck = torch.load(path, map_location=device, weights_only=False)
    pts = ck['points'].to(device)
    n = len(pts)
    model = VoronoiGaussField(pts, ck['offsets'].to(device), ck['adj'].to(device), torch.zeros(n, 3, device=device),
                              torch.ones(n, device=device))
    model.load_state_dict(ck['state'])
    model.sh_deg = int(ck['sh_deg'])
    model.requires_grad_(requires_grad)
    return model, ck


def save_model(model, path, normalization=None, args=None):
    """Writes `model` in the reference's checkpoint format (train.py:168-170)."""
    g = model.graph
    record = dict(state=model.state_dict(), points=g.points, offsets=g.offsets, adj=g.adj, sh_deg=model.sh_deg,
                  normalization=normalization, args=dict(args or {}))
    torch.save(record, path)
