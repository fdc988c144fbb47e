"""Host arithmetic behind bench.py's JSON line: the work units and algorithmic bytes of the roofline, the
choice of the dominant kernel, the march bounds, and the count of library kernel launches per training
step (checked against the ncu launch list of a config-3 step: 44 kernels in vg_foam_forward, 51 in
vg_foam_backward, 2 conic forwards and 2 conic backwards)."""

import os
import sys

import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
import bench  # noqa: E402


def _records(cells_per_ray, K, coloured=()):
    """(B, K, 8) records: field 1 the cell id bits, field 7 > 0 for the (ray, sample) pairs in coloured."""
    rec = torch.zeros(len(cells_per_ray), K, 8)
    for r, cells in enumerate(cells_per_ray):
        for s, c in enumerate(cells[:K]):
            rec[r, s, 1] = torch.tensor([c], dtype=torch.int32).view(torch.float32)[0]
    for r, s in coloured:
        rec[r, s, 7] = 0.5
    return rec


def test_training_units_and_bytes_by_hand(monkeypatch):
    # three cells of degree 2, 3 and 4 (neighbourhoods of 3, 4 and 5 sites); chunks of 2 samples, passes of
    # 2 rays x K slots
    monkeypatch.setattr(bench, 'CM_CHUNK', 2)
    K = 4
    monkeypatch.setattr(bench, 'CM_SLOTS', 2 * K)
    offsets = torch.tensor([0, 2, 5, 9], dtype=torch.int32)
    # pass 0: ray 0 visits cells 0, 1; ray 1 visits 2, 2, 2, 1. pass 1: ray 2 has 6 samples > K (re-traced,
    # left out of the cell-major passes)
    rec = _records([[0, 1], [2, 2, 2, 1], [0, 0, 0, 0]], K, coloured=[(0, 0), (1, 0), (1, 1), (1, 2)])
    stats = torch.tensor([[2, 1, 3], [4, 2, 1], [6, 2, 0]], dtype=torch.int32)  # samples, coloured, walk
    u = bench.training_units(stats, rec, offsets, K)
    # scatter, pass 0: cell 0: 1 sample (1 chunk, n 3), cell 1: 2 (1 chunk, n 4), cell 2: 3 (2 chunks, n 5)
    assert (u['sc_chunks'], u['sc_nbr'], u['sc_samples']) == (4, 3 + 4 + 2 * 5, 6)
    # colour pass: cell 0: 1 sample, cell 2: 3 samples
    assert (u['col_chunks'], u['col_nbr'], u['col_samples']) == (3, 3 + 2 * 5, 4)
    n = (3 + 4 + 5 + 5 + 5 + 4) / 6
    assert abs(u['cell_n'] - n) < 1e-12
    nb = 16
    b = bench.algorithmic_bytes_training(stats, u, nb, K)
    S, W, B, rec_s = 2 + 4 + 6, 3 + 1 + 0, 3, 2 + 4 + 4
    assert abs(b['traversal'] - (44 * n * S + 16 * n * W + 68 * B + 32 * rec_s)) < 1e-6
    assert b['color'] == (40 + 12 * nb) * 13 + 88 * 4
    assert b['replay'] == 96 * 6 + 44 * B
    assert b['scatter'] == (68 + 12 * nb + 8 * (13 + 3 * nb)) * 17 + 64 * 6


def test_roofline_takes_the_dominant_kernel():
    times = {'traversal': (30.0, 5), 'scatter': (100.0, 40), 'color': (20.0, 40)}
    nbytes = {'traversal': 1e9, 'scatter': 8e9, 'color': 1e9}
    r = bench.roofline(times, nbytes, steps=5, peak=8000.0, peak_kind='measured')
    assert r['kernel'] == 'scatter'
    # 8 launches per step: 1e9 bytes per launch in 2.5 ms
    assert abs(r['algorithmic_bytes_per_launch'] - 1e9) < 1
    assert abs(r['achieved'] - 400.0) < 1e-6 and abs(r['frac'] - 0.05) < 1e-9


def test_march_bounds_enter_and_leave_the_unit_ball():
    o = torch.tensor([[3.0, 0.0, 0.0], [3.0, 0.0, 0.0]])
    d = torch.tensor([[-1.0, 0.0, 0.0], [0.0, 1.0, 0.0]])
    from voronoi_gauss_b200 import scenes
    near, mid, far = scenes.march_bounds(o, d)
    assert torch.allclose(near, torch.tensor([2.0, 0.02])) and torch.allclose(mid, torch.tensor([4.0, 0.02]))
    assert torch.allclose(far - mid, torch.full((2,), 1e-3), atol=1e-6)


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
