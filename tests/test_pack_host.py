"""The checker of the device inference packing (oracle/pack_ref.py: pack_foam / morton_order / sh_basis
restated in torch) against the layouts the reference's own render.py produced for the same scene
(tests/golden/make_golden.py), and render.sh_basis. The conics are computed with the torch twin on both
sides, so the comparison runs on the CPU."""

from types import SimpleNamespace

import numpy as np
import pytest
import torch

from conftest import golden


@pytest.fixture()
def model_and_ext(foam_small):
    z = foam_small
    graph = SimpleNamespace(points=torch.tensor(z['points']), offsets=torch.tensor(z['offsets']),
                            adj=torch.tensor(z['adj']))
    t = {k: torch.tensor(z[k]) for k in ('raw', 'ls', 'quat', 'cls', 'cquat', 'sh')}
    model = SimpleNamespace(graph=graph, raw=t['raw'], d_log_scale=t['ls'], d_quat=t['quat'], c_log_scale=t['cls'],
                            c_quat=t['cquat'], sh=lambda: t['sh'], sh_deg=3)
    return model


@pytest.mark.parametrize('tag,kw', [('plain', {}), ('morton', dict(reorder=True)),
                                    ('eps', dict(eps_density=1e-3, sh_half=True)),
                                    ('eps_morton', dict(eps_density=1e-3, sh_half=True, reorder=True,
                                                        scale_floor=0.01))])
def test_pack_foam_matches_reference_layout(foam_small, model_and_ext, tag, kw):
    from oracle import pack_ref
    from voronoi_gauss_b200 import ext
    model = model_and_ext
    z = foam_small
    pk = pack_ref.pack_foam(model, ext.conic_reference, **kw)
    for key in ('offsets', 'nbr', 'orig'):
        assert np.array_equal(pk[key].numpy(), z[f'pack_{tag}_{key}']), key
    assert np.array_equal(pk['points'].numpy(), z[f'pack_{tag}_points'])
    assert np.array_equal(pk['edge'].numpy().view(np.int32), z[f'pack_{tag}_edge'].view(np.int32))
    np.testing.assert_allclose(pk['attr'].numpy(), z[f'pack_{tag}_attr'], rtol=1e-6, atol=1e-7)
    assert np.array_equal(pk['sh'].numpy(), z[f'pack_{tag}_sh'])


def test_morton_order_matches_reference(foam_small):
    from oracle import pack_ref
    from voronoi_gauss_b200 import render
    perm = render.morton_order(torch.tensor(foam_small['points']))
    assert np.array_equal(perm.numpy(), foam_small['morton_perm'])
    assert np.array_equal(pack_ref.morton_order(torch.tensor(foam_small['points'])).numpy(), foam_small['morton_perm'])


def test_sh_basis_matches_reference():
    from voronoi_gauss_b200 import render
    z = golden('sh_basis.npz')
    from oracle import pack_ref
    for deg in range(4):
        np.testing.assert_allclose(render.sh_basis(torch.tensor(z['dirs']), deg).numpy(), z[f'b{deg}'], rtol=0,
                                   atol=1e-15)
        np.testing.assert_allclose(pack_ref.sh_basis(torch.tensor(z['dirs']), deg).numpy(), z[f'b{deg}'], rtol=0,
                                   atol=1e-15)
