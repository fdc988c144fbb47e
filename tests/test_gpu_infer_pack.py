"""The device inference packing (render.pack_foam / bake_colors on vg_infer_pack / vg_bake_colors)
against its torch checker (oracle/pack_ref.py, pinned to the reference's render.py layouts by
test_pack_host.py) run on the same GPU tensors: integer arrays, positions and fp16 cut bits identical,
conics within 1e-6, and the layouts against the reference's own golden layouts."""

from types import SimpleNamespace

import numpy as np
import pytest
import torch

from conftest import cuda

pytestmark = pytest.mark.gpu

OPTS = [('plain', {}), ('morton', dict(reorder=True)), ('eps', dict(eps_density=1e-3, sh_half=True)),
        ('eps_morton', dict(eps_density=1e-3, sh_half=True, reorder=True, scale_floor=0.01))]


@pytest.fixture()
def model(foam_small):
    from voronoi_gauss_b200 import ext
    z = foam_small
    graph = ext.Graph(cuda(z['points']), cuda(z['offsets'], torch.int32), cuda(z['adj'], torch.int32))
    t = {k: cuda(z[k], torch.float32) for k in ('raw', 'ls', 'quat', 'cls', 'cquat', 'sh')}
    return SimpleNamespace(graph=graph, raw=t['raw'], d_log_scale=t['ls'], d_quat=t['quat'], c_log_scale=t['cls'],
                           c_quat=t['cquat'], sh=lambda: t['sh'], sh_deg=3)


@pytest.mark.parametrize('tag,kw', OPTS)
def test_device_pack_matches_torch_checker_and_reference(foam_small, model, tag, kw):
    from oracle import pack_ref
    from voronoi_gauss_b200 import ext, render
    pk = render.pack_foam(model, **kw)
    ref = pack_ref.pack_foam(model, ext.conic, **kw)
    for key in ('offsets', 'nbr', 'orig', 'points'):
        assert torch.equal(pk[key], ref[key]), key
    assert torch.equal(pk['edge'].view(torch.int32), ref['edge'].view(torch.int32))
    assert torch.equal(pk['sh'], ref['sh']) and torch.equal(pk['sh32'], ref['sh32'])
    torch.testing.assert_close(pk['attr'], ref['attr'], rtol=1e-6, atol=1e-7)
    if kw.get('reorder'):
        assert torch.equal(pk['perm'], ref['perm']) and torch.equal(pk['inv'], ref['inv'])
    z = foam_small
    for key in ('offsets', 'nbr', 'orig', 'points'):
        assert np.array_equal(pk[key].cpu().numpy(), z[f'pack_{tag}_{key}']), key
    e, ze = pk['edge'].cpu().numpy(), z[f'pack_{tag}_edge']
    assert np.array_equal(e[:, :3], ze[:, :3])
    h = np.ascontiguousarray(e[:, 3]).view(np.uint16).astype(np.int32)
    zh = np.ascontiguousarray(ze[:, 3]).view(np.uint16).astype(np.int32)
    assert np.abs(h - zh).max() <= 1  # fp16 cuts: libm vs CUDA expf may differ by one unit before rounding


def test_bake_colors_matches_torch_checker(model):
    from oracle import pack_ref
    from voronoi_gauss_b200 import render
    pk = render.pack_foam(model, reorder=True)
    center = torch.tensor([0.3, -2.5, 1.2], device='cuda')
    render.bake_colors(model, pk, center)
    ref = pack_ref.baked_colors(pk['points'], pk['sh32'], 3, center)
    torch.testing.assert_close(pk['attr'][:, 16:19], ref, rtol=1e-5, atol=1e-6)
    assert (pk['attr'][:, 19] == 0).all() and (pk['attr'][:, 14:16] == 0).all()
