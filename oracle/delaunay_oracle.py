"""CPU Delaunay adjacency oracle -- TEST INFRASTRUCTURE ONLY (tests/ may use
it; the product never does).

The reference builds its Delaunay tetrahedralisation on the GPU
(src/delaunay/*.cu) and cannot be compiled here; for points in general
position the Delaunay tetrahedralisation is unique, so scipy.spatial.Delaunay
(Qhull) gives the same tet set.  The CSR is then written exactly as the
reference's find_adjacency does (src/delaunay/delaunay.cu:146-229): the six
edges of every tet, sorted by (min, max) and made unique; each edge emitted
as (a -> b) and (b -> a) and sorted by source (rows therefore list
neighbours in ascending order); offsets filled with UINT32_MAX, offsets[0] = 0,
offsets[N] = 2 * edges, and offsets[key + 1] = i wherever the source key
changes at position i.  Parity with the reference is unpinned (no reference
output exists here); tests compare the GPU kernels with this restatement.
"""
from __future__ import annotations

import numpy as np

U32_NONE = 0xFFFFFFFF


def delaunay_tets(points: np.ndarray) -> np.ndarray:
    from scipy.spatial import Delaunay
    p = np.ascontiguousarray(points, np.float64)
    return Delaunay(p).simplices.astype(np.int64)


def csr_from_tets(tets: np.ndarray, num_points: int):
    t = np.sort(np.asarray(tets, np.int64), axis=1)
    pairs = np.concatenate([t[:, [0, 1]], t[:, [0, 2]], t[:, [0, 3]], t[:, [1, 2]], t[:, [1, 3]], t[:, [2, 3]]])
    key = pairs[:, 0] * num_points + pairs[:, 1]
    key = np.unique(key)
    a, b = key // num_points, key % num_points
    src = np.empty(2 * a.size, np.int64)
    dst = np.empty(2 * a.size, np.int64)
    src[0::2], dst[0::2] = a, b
    src[1::2], dst[1::2] = b, a
    order = np.argsort(src, kind="stable")
    src, dst = src[order], dst[order]
    offsets = np.full(num_points + 1, U32_NONE, np.uint32)
    offsets[0] = 0
    offsets[num_points] = src.size
    change = np.nonzero(src[1:] != src[:-1])[0] + 1
    offsets[src[change - 1] + 1] = change
    return dst.astype(np.uint32), offsets


def delaunay_adjacency(points: np.ndarray):
    """(point_adjacency uint32 [E], offsets uint32 [N+1]) of the Delaunay
    tetrahedralisation of points, in the given order."""
    p = np.asarray(points, np.float32)
    return csr_from_tets(delaunay_tets(p), p.shape[0])
