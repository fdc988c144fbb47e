"""Host arithmetic behind bench.py's JSON line: the algorithmic-byte model of the roofline and the count
of library kernel launches per training step (checked against the ncu launch list of a config-3 step:
44 kernels in vg_foam_forward, 51 in vg_foam_backward, 2 conic forwards and 2 conic backwards)."""

import os
import sys

import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
import bench  # noqa: E402


def _records(cells_per_ray, K):
    rec = torch.zeros(len(cells_per_ray), K, 8)
    for r, cells in enumerate(cells_per_ray):
        for s, c in enumerate(cells[:K]):
            rec[r, s, 1] = torch.tensor([c], dtype=torch.int32).view(torch.float32)[0]
    return rec


def test_algorithmic_bytes_by_hand():
    # three cells of degree 2, 3 and 4 (neighbourhoods of 3, 4 and 5 sites)
    offsets = torch.tensor([0, 2, 5, 9], dtype=torch.int32)
    K = 4
    # ray 0 visits cells 0, 1 (2 samples); ray 1 visits 2, 2, 1 (3 samples); ray 2 has 6 samples > K and is
    # left out of the neighbourhood mean (its records stop at K)
    rec = _records([[0, 1], [2, 2, 1], [0, 0, 0, 0]], K)
    stats = torch.tensor([[2, 1, 3], [3, 0, 1], [6, 2, 0]], dtype=torch.int32)  # samples, coloured, walk
    nb = 16
    fwd, bwd, n_bar = bench.algorithmic_bytes(stats, rec, offsets, nb)
    n = (3 + 4 + 5 + 5 + 4) / 5
    assert abs(n_bar - n) < 1e-12
    S, C, W, B = 2 + 3 + 6, (1 + 1) + 0 + (2 + 1), 3 + 1 + 0, 3
    assert abs(fwd - (44 * n * S + (24 + 12 * nb) * n * C + 16 * n * W + 68 * B)) < 1e-6
    assert abs(bwd - (100 * n * S + (24 + 12 * nb + 8 * (6 + 3 * nb)) * n * C + 16 * n * W + 84 * B)) < 1e-6


def test_launches_per_step_matches_the_launch_list():
    # 1080p with record_cap 256: 8 passes of 2^26 record slots
    assert bench.launches_per_step(1920 * 1080, 256) == 2 + 44 + 51 + 2
    # one pass
    assert bench.launches_per_step(4096, 256) == 2 + (3 + 5 + 1) + (2 + 6 + 1) + 2


def test_scene_build_failure_reaches_the_waiting_ranks(tmp_path, monkeypatch):
    """A rank-0 failure while building the scene cache makes the other ranks raise at their next poll
    instead of waiting for a cache that will never come; a marker from another launch is ignored."""
    import time
    import pytest
    from voronoi_gauss_b200 import scenes
    monkeypatch.setenv('VG_SCENE_CACHE', str(tmp_path))
    monkeypatch.setenv('TORCHELASTIC_RUN_ID', 'launch-a')

    def broken(cfg, n=None, **kw):
        raise MemoryError('no room for the triangulation')
    monkeypatch.setattr(scenes, 'build_graph', broken)
    with pytest.raises(MemoryError):
        bench.load_scene(1, 500, rank=0)
    t0 = time.time()
    with pytest.raises(RuntimeError, match='no room for the triangulation'):
        bench.load_scene(1, 500, rank=1, poll_s=0.05, wait_s=30)
    assert time.time() - t0 < 5
    # a later launch does not read launch-a's marker: it waits (and here times out quickly)
    monkeypatch.setenv('TORCHELASTIC_RUN_ID', 'launch-b')
    with pytest.raises(TimeoutError):
        bench.load_scene(1, 500, rank=1, poll_s=0.05, wait_s=0.2)
