"""Sites of the field and their Delaunay (Voronoi-neighbour) adjacency, built on the host.

Same contract as the reference's scene preprocessing (sites.py:24-45 of voronoi-gauss):

* ``delaunay_graph(points)`` -> (points kept, index of the kept points, CSR offsets (N + 1) int32,
  adjacency (M) int32). Points that Qhull leaves out of the triangulation are dropped and the
  triangulation is rebuilt (sites.py:24-35).
* ``nearest_sites(points, queries)`` -> int32 site index of every query (k-d tree, sites.py:38-39).
* ``neighbor_spacing(points, k=3)`` -> mean distance to the k nearest other sites (sites.py:42-45).

The triangulation is one global Qhull run (as the reference): a slab-parallel build cannot resolve the
tetrahedra next to the convex hull of a cube-shaped point set locally (their circumspheres span the
whole domain), so large scenes are built once and cached by ``scenes.build_graph``.
"""

from __future__ import annotations

import numpy as np
from scipy.spatial import Delaunay, cKDTree


def delaunay_graph(points):
    """-> (points kept, kept index, offsets (N + 1) int32, adj (M) int32). sites.py:24-35."""
    points = np.asarray(points, dtype=np.float64)
    idx = np.arange(len(points))
    for _ in range(3):
        tri = Delaunay(points[idx])
        offsets, adj = tri.vertex_neighbor_vertices
        alone = np.diff(offsets) == 0
        if not alone.any():
            return points[idx], idx, offsets.astype(np.int32), adj.astype(np.int32)
        idx = idx[~alone]
    raise RuntimeError('Delaunay triangulation keeps dropping points')


def nearest_sites(points, queries):
    """Nearest site of every query point (sites.py:38-39)."""
    return cKDTree(np.asarray(points)).query(np.asarray(queries))[1].astype(np.int32)


def neighbor_spacing(points, k=3):
    """Mean distance to the k nearest other sites (sites.py:42-45)."""
    d, _ = cKDTree(np.asarray(points)).query(np.asarray(points), k + 1)
    return d[:, 1:].mean(1)
