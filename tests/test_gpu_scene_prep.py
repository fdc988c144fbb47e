"""Scene preparation on the device: camera rays (vg_camera_rays) against the torch pinhole rays of
scenes.camera_rays (colmap.py:129-134) in the same pixel-tile order, and nearest sites (vg_nearest_sites)
against the k-d tree of sites.nearest_sites (sites.py:38-39)."""

import numpy as np
import pytest
import torch

from conftest import cuda

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize('W,H,tile', [(64, 64, (4, 8)), (37, 23, (4, 8)), (30, 18, None), (800, 800, (4, 8))])
def test_camera_rays_match_torch_rays_in_tile_order(W, H, tile):
    from voronoi_gauss_b200 import scenes
    centre, c2w = scenes.orbit_camera(3, 10)
    order = scenes.tile_order(H, W, *tile) if tile else None
    o_ref, d_ref = scenes.camera_rays(centre, c2w, W, H, 50.0, order=order)
    o, d = scenes.camera_rays_device(centre, c2w, W, H, 50.0, tile=tile)
    torch.testing.assert_close(o.cpu(), o_ref, rtol=0, atol=1e-6)
    torch.testing.assert_close(d.cpu(), d_ref, rtol=0, atol=2e-6)


def test_nearest_sites_match_kd_tree(foam_small):
    from scipy.spatial import cKDTree

    from voronoi_gauss_b200 import ext
    z = foam_small
    g = ext.Graph(cuda(z['points']), cuda(z['offsets'], torch.int32), cuda(z['adj'], torch.int32))
    rng = np.random.default_rng(5)
    q = np.concatenate([rng.uniform(-1, 1, (4000, 3)), rng.uniform(-4, 4, (1000, 3))]).astype(np.float32)
    got = ext.nearest_sites(g, cuda(q)).cpu().numpy()
    dist, idx = cKDTree(z['points'].astype(np.float64)).query(q.astype(np.float64), k=2)
    tie = dist[:, 1] - dist[:, 0] <= 1e-6 * np.maximum(dist[:, 0], 1e-12)
    assert (got[~tie] == idx[~tie, 0]).all()
    d_got = np.linalg.norm(q - z['points'][got], axis=1)
    assert np.all(d_got <= dist[:, 0] * (1 + 1e-6) + 1e-7)
    assert ext.nearest_sites(g, torch.zeros(0, 3, device='cuda')).numel() == 0
