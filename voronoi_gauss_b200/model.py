"""Per-site parameters of the field, with the reference's parameterisation (voronoi-gauss model.py:19-59).

Every site carries a density Gaussian (raw = log rho, log-scale (N, 3), quaternion (N, 4)), a colour
Gaussian (log-scale, quaternion) and SH colour coefficients (sh_dc (N, 1, 3) + sh_rest (N, 15, 3)); one
learned background colour (bg_logit (3,)) sits behind the scene. The sites and their adjacency are fixed.
The parameter names, shapes and registration order are those of the reference's checkpoints
(train.py:168-170), so its state dicts load here unchanged.
"""

from __future__ import annotations

import math

import torch
import torch.nn as nn

from .ext import Graph

C0 = 0.28209479177387814  # band-0 SH constant: a site's base colour is C0 sh_dc + 1/2

# per-site parameters in registration order, with their shapes after the site axis
LAYOUT = (('raw', ()), ('d_log_scale', (3,)), ('d_quat', (4,)), ('c_log_scale', (3,)), ('c_quat', (4,)),
          ('sh_dc', (1, 3)), ('sh_rest', (15, 3)))

# learning-rate groups (the keys of the `lr` dict of param_groups) and their parameters
GROUPS = (('raw', ('raw',)), ('scale', ('d_log_scale', 'c_log_scale')), ('quat', ('d_quat', 'c_quat')),
          ('sh_dc', ('sh_dc',)), ('sh_rest', ('sh_rest',)), ('bg', ('bg_logit',)))


def initial_state(colors, spacing, init_alpha=0.1, device=None):
    """Initial per-site tensors (model.py:23-39): isotropic Gaussians of scale s = max(spacing, 1e-4) for
    density and colour, with rho chosen so that a ray through the centre of a lone site absorbs init_alpha
    (rho s sqrt(2 pi) = -ln(1 - init_alpha)); identity rotations; base colour `colors` (clamped to
    [0, 1]) in the DC band, higher bands zero. New tensors go to `device` (default: spacing's)."""
    s = spacing.clamp_min(1e-4)
    n = len(s)
    device = s.device if device is None else device
    log_s = s.log().unsqueeze(1).repeat(1, 3)
    unit = torch.zeros(n, 4, device=device)
    unit[:, 0] = 1.0
    absorb = -math.log(1.0 - init_alpha)
    return {'raw': (absorb / (s * math.sqrt(2.0 * math.pi))).log(), 'd_log_scale': log_s, 'd_quat': unit,
            'c_log_scale': log_s.clone(), 'c_quat': unit.clone(),
            'sh_dc': ((colors.clamp(0, 1) - 0.5) / C0).unsqueeze(1),
            'sh_rest': torch.zeros(n, 15, 3, device=device)}


class VoronoiGaussField(nn.Module):
    """points (N, 3) fixed sites; offsets / adj their Delaunay adjacency; colors (N, 3) in [0, 1]; spacing (N,)
    mean distance to the nearest sites, the initial isotropic scale of both Gaussians. The active SH degree
    `sh_deg` starts at 0 and is raised by the caller, up to `max_sh_deg`."""

    def __init__(self, points, offsets, adj, colors, spacing, init_alpha=0.1, sh_deg=3):
        super().__init__()
        self._attach(Graph(points, offsets, adj), initial_state(colors, spacing, init_alpha, points.device),
                     max_sh_deg=sh_deg, sh_deg=0)

    def _attach(self, graph, state, max_sh_deg, sh_deg):
        self.graph = graph
        self.max_sh_deg, self.sh_deg = max_sh_deg, sh_deg
        for name, _ in LAYOUT:
            setattr(self, name, nn.Parameter(state[name]))
        self.bg_logit = nn.Parameter(torch.zeros(3, device=graph.points.device))

    @classmethod
    def from_params(cls, points, offsets, adj, params):
        """Model holding copies of the tensors of scenes.make_params (already on the target device)."""
        m = cls.__new__(cls)
        nn.Module.__init__(m)
        state = {name: params[name].clone() for name, _ in LAYOUT[:5]}
        state['sh_dc'], state['sh_rest'] = params['sh'][:, :1].clone(), params['sh'][:, 1:].clone()
        m._attach(Graph(points, offsets, adj), state, max_sh_deg=3, sh_deg=int(params['sh_deg']))
        return m

    @property
    def n_sites(self):
        return len(self.raw)

    def sh(self):
        """All SH coefficients (N, 16, 3): the DC band followed by the higher ones."""
        return torch.cat([self.sh_dc, self.sh_rest], 1)

    def walk(self, o, d, z, start):
        """Nearest sites of the sorted samples o + z d (model.py:48-49)."""
        return self.graph.walk(o, d, z, start)

    def param_groups(self, lr):
        """Optimizer groups keyed by the names of `lr` (raw, scale, quat, sh_dc, sh_rest, bg)."""
        return [{'params': [getattr(self, p) for p in names], 'lr': lr[group], 'name': group}
                for group, names in GROUPS]
