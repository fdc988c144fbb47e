"""Host scene preparation against the reference's own code: pinhole rays (colmap.py:129-134) and the
4x8 pixel-tile order of the inference benchmark (bench_infer.py:37-41), from `tests/golden/camera_rays.npz`
(made by make_golden.py from the reference's ColmapScene.rays and tile_order on a 37x23 image whose edge
tiles are partial)."""

import os

import numpy as np
import torch

from voronoi_gauss_b200 import scenes

GOLD = np.load(os.path.join(os.path.dirname(__file__), 'golden', 'camera_rays.npz'))
W, H, FOV = int(GOLD['W']), int(GOLD['H']), float(GOLD['fov'])


def test_tile_order_matches_reference():
    assert np.array_equal(scenes.tile_order(H, W), GOLD['order'])


def test_camera_rays_match_reference():
    o, d = scenes.camera_rays(GOLD['centre'], GOLD['rot'], W, H, FOV)
    # the same float32 operations up to the order of the matrix products' sums
    assert torch.allclose(o, torch.from_numpy(GOLD['o']), atol=0, rtol=0)
    assert (d - torch.from_numpy(GOLD['d'])).abs().max().item() < 1e-6
    assert torch.allclose(d.norm(dim=-1), torch.ones(H * W), atol=1e-6)


def test_camera_rays_in_tile_order():
    order = scenes.tile_order(H, W)
    _, d = scenes.camera_rays(GOLD['centre'], GOLD['rot'], W, H, FOV, order=order)
    assert (d - torch.from_numpy(GOLD['d'][order])).abs().max().item() < 1e-6
