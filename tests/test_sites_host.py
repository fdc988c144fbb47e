"""Host scene graph construction against the reference's own outputs: the Delaunay CSR of the
test_foam.py scene (300 sites drawn from default_rng(2), sites.py:24-35) stored in
tests/golden/foam_small.npz by make_golden.py, rebuilt here from the same draw."""

import numpy as np

from voronoi_gauss_b200 import sites


def test_delaunay_graph_matches_reference(foam_small):
    pts0 = np.random.default_rng(2).uniform(-0.9, 0.9, (300, 3))
    pts, kept, offsets, adj = sites.delaunay_graph(pts0)
    assert np.array_equal(pts.astype(np.float32), foam_small['points'])
    assert np.array_equal(offsets, foam_small['offsets']) and np.array_equal(adj, foam_small['adj'])
    assert offsets.dtype == np.int32 and adj.dtype == np.int32
    assert np.array_equal(pts, pts0[kept])


def test_delaunay_graph_drops_coincident_points():
    rng = np.random.default_rng(5)
    p = rng.uniform(-1, 1, (400, 3))
    p = np.concatenate([p, p[:3], np.zeros((2, 3))])  # exact duplicates are left out by Qhull
    pts, kept, offsets, adj = sites.delaunay_graph(p)
    assert len(pts) < len(p) and (np.diff(offsets) > 0).all()
    assert len(np.unique(np.round(pts, 12), axis=0)) == len(pts)
    # symmetric adjacency
    rows = np.repeat(np.arange(len(pts)), np.diff(offsets))
    pairs = set(zip(rows.tolist(), adj.tolist()))
    assert all((b, a) in pairs for a, b in pairs)


def test_nearest_sites_and_spacing():
    rng = np.random.default_rng(6)
    p = rng.uniform(-1, 1, (500, 3))
    q = rng.uniform(-1, 1, (50, 3))
    brute = np.argmin(((q[:, None] - p[None]) ** 2).sum(-1), 1)
    got = sites.nearest_sites(p, q)
    assert got.dtype == np.int32 and np.array_equal(got, brute)
    d = np.sqrt(((p[:, None] - p[None]) ** 2).sum(-1))
    np.fill_diagonal(d, np.inf)
    want = np.sort(d, 1)[:, :3].mean(1)
    assert np.allclose(sites.neighbor_spacing(p, 3), want, rtol=1e-12)
