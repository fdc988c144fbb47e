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


def _neighbour_csr(points):
    """CSR Delaunay adjacency (offsets (N + 1), neighbours) of one Qhull triangulation of `points`."""
    return Delaunay(points).vertex_neighbor_vertices


def delaunay_graph(points, attempts=3):
    """-> (points kept, kept index, offsets (N + 1) int32, adj (M) int32) (sites.py:24-35). Qhull leaves
    nearly coincident or degenerate points out of the triangulation (they come back with no neighbours);
    those are removed and the rest triangulated again, at most `attempts` times."""
    pts = np.asarray(points, dtype=np.float64)
    kept = np.arange(len(pts))
    for _ in range(attempts):
        offsets, adj = _neighbour_csr(pts[kept])
        lonely = np.flatnonzero(np.diff(offsets) == 0)
        if lonely.size == 0:
            return pts[kept], kept, offsets.astype(np.int32), adj.astype(np.int32)
        kept = np.delete(kept, lonely)
    raise RuntimeError(f'Qhull still leaves {lonely.size} sites out of the triangulation after {attempts} attempts')


def nearest_sites(points, queries):
    """Index (int32) of the site nearest to each query point (sites.py:38-39)."""
    _, index = cKDTree(np.asarray(points)).query(np.asarray(queries))
    return np.asarray(index, dtype=np.int32)


def neighbor_spacing(points, k=3):
    """Mean distance from each site to its k nearest other sites (sites.py:42-45): the k + 1 nearest
    points of a site include the site itself at distance 0, which is left out."""
    pts = np.asarray(points)
    dist, _ = cKDTree(pts).query(pts, k + 1)
    return dist[:, 1:].mean(axis=1)
