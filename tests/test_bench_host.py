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
