"""Per-site parameters of the field, with the reference's parameterisation (voronoi-gauss model.py:19-59):
density Gaussian (raw = log rho, log-scale (N, 3), quaternion (N, 4)), colour Gaussian (log-scale,
quaternion) and SH colour (sh_dc (N, 1, 3) + sh_rest (N, 15, 3)); the sites and their adjacency are fixed."""

from __future__ import annotations

import math

import torch
import torch.nn as nn

from .ext import Graph

C0 = 0.28209479177387814


def identity_quat(n, device):
    q = torch.zeros(n, 4, device=device)
    q[:, 0] = 1.0
    return q


class VoronoiGaussField(nn.Module):
    """points (N, 3) fixed sites; offsets / adj their Delaunay adjacency; colors (N, 3) in [0, 1]; spacing (N,)
    mean distance to the nearest sites, the initial isotropic scale of both Gaussians (model.py:23-39)."""

    def __init__(self, points, offsets, adj, colors, spacing, init_alpha=0.1, sh_deg=3):
        super().__init__()
        device = points.device
        n = len(points)
        self.graph = Graph(points, offsets, adj)
        self.max_sh_deg, self.sh_deg = sh_deg, 0
        s = spacing.clamp_min(1e-4)
        # a ray through the centre of a lone Gaussian has opacity init_alpha: rho s sqrt(2 pi) = -ln(1 - a)
        rho = -math.log(1.0 - init_alpha) / (s * math.sqrt(2.0 * math.pi))
        self.raw = nn.Parameter(rho.log())
        self.d_log_scale = nn.Parameter(s.log()[:, None].repeat(1, 3))
        self.d_quat = nn.Parameter(identity_quat(n, device))
        self.c_log_scale = nn.Parameter(s.log()[:, None].repeat(1, 3))
        self.c_quat = nn.Parameter(identity_quat(n, device))
        self.sh_dc = nn.Parameter(((colors.clamp(0, 1) - 0.5) / C0)[:, None])
        self.sh_rest = nn.Parameter(torch.zeros(n, 15, 3, device=device))
        self.bg_logit = nn.Parameter(torch.zeros(3, device=device))

    @classmethod
    def from_params(cls, points, offsets, adj, params):
        """Model holding the tensors of scenes.make_params (already on the target device)."""
        m = cls.__new__(cls)
        nn.Module.__init__(m)
        m.graph = Graph(points, offsets, adj)
        m.max_sh_deg = 3
        m.sh_deg = int(params['sh_deg'])
        m.raw = nn.Parameter(params['raw'].clone())
        m.d_log_scale = nn.Parameter(params['d_log_scale'].clone())
        m.d_quat = nn.Parameter(params['d_quat'].clone())
        m.c_log_scale = nn.Parameter(params['c_log_scale'].clone())
        m.c_quat = nn.Parameter(params['c_quat'].clone())
        m.sh_dc = nn.Parameter(params['sh'][:, :1].clone())
        m.sh_rest = nn.Parameter(params['sh'][:, 1:].clone())
        m.bg_logit = nn.Parameter(torch.zeros(3, device=params['raw'].device))
        return m

    @property
    def n_sites(self):
        return len(self.raw)

    def sh(self):
        return torch.cat([self.sh_dc, self.sh_rest], 1)

    def walk(self, o, d, z, start):
        """Nearest sites of the sorted samples o + z d (model.py:48-49)."""
        return self.graph.walk(o, d, z, start)

    def param_groups(self, lr):
        return [
            {'params': [self.raw], 'lr': lr['raw'], 'name': 'raw'},
            {'params': [self.d_log_scale, self.c_log_scale], 'lr': lr['scale'], 'name': 'scale'},
            {'params': [self.d_quat, self.c_quat], 'lr': lr['quat'], 'name': 'quat'},
            {'params': [self.sh_dc], 'lr': lr['sh_dc'], 'name': 'sh_dc'},
            {'params': [self.sh_rest], 'lr': lr['sh_rest'], 'name': 'sh_rest'},
            {'params': [self.bg_logit], 'lr': lr['bg'], 'name': 'bg'},
        ]
