"""Checkpoints in the reference's format (train.py:168-170) load into VoronoiGaussField and round-trip:
tests/golden/ckpt_small.pth was written by the reference's own model class (tests/golden/make_golden.py)."""

import os

import torch

from conftest import GOLDEN


def test_reference_checkpoint_loads_and_round_trips(tmp_path):
    from voronoi_gauss_b200.checkpoint import load_model, save_model
    path = os.path.join(GOLDEN, 'ckpt_small.pth')
    model, ck = load_model(path, device='cpu')
    assert model.sh_deg == 2 and model.n_sites == len(ck['points'])
    for k, v in ck['state'].items():
        assert torch.equal(getattr(model, k).detach(), v), k
    assert not any(p.requires_grad for p in model.parameters())
    assert torch.equal(model.graph.adj, ck['adj'].int())
    out = tmp_path / 'model.pth'
    save_model(model, out, normalization=ck['normalization'], args=ck['args'])
    again, ck2 = load_model(out, device='cpu')
    assert set(ck2) == set(ck) and ck2['sh_deg'] == 2
    for k, v in ck['state'].items():
        assert torch.equal(getattr(again, k).detach(), v), k


def test_initial_parameters_match_the_reference_constructor():
    """VoronoiGaussField's initial state against the reference's constructor (tests/golden/model_init.npz):
    same parameter names in the same order, bit-identical values."""
    import numpy as np
    import torch
    from conftest import golden
    from voronoi_gauss_b200.model import VoronoiGaussField
    z = golden('model_init.npz')
    n = len(z['points'])
    m = VoronoiGaussField(torch.tensor(z['points']), torch.zeros(n + 1, dtype=torch.int32),
                          torch.zeros(0, dtype=torch.int32), torch.tensor(z['colors']), torch.tensor(z['spacing']),
                          init_alpha=0.2, sh_deg=2)
    sd = m.state_dict()
    assert list(sd) == list(z['keys'])
    for k, v in sd.items():
        assert np.array_equal(v.numpy(), z[f'state_{k}']), k
    assert (m.max_sh_deg, m.sh_deg) == (2, 0)
