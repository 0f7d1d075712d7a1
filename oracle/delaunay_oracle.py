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

Qhull is floating point: for near-degenerate sites it can return tets whose
circumsphere strictly contains another site.  empty_sphere_violations()
checks the property exactly (float filter, rational arithmetic where the
filter cannot decide); the test sets the GPU comparison uses pass it.
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


def tet_structure(points: np.ndarray, tets: np.ndarray):
    """The reference's tet arrays for a tet set, as Triangulation.tets(),
    tet_adjacency() and vert_to_tet() return them (find_adjacency,
    src/delaunay/delaunay.cu:32-144):
      * tets sorted by their sorted vertex sets (the SortedMap<IndexedTet>
        order, set_less, src/utils/geometry.h:217-232), each with ascending
        vertices and the last two swapped where needed so that
        IndexedTet::volume > 0 (geometry.h:488-494), i.e. the determinant of
        (v1 - v0, v2 - v0, v3 - v0), expanded along its first row in double,
        is not positive;
      * tet_adjacency[4 t + j] = 4 t' + j' of the tet sharing the face
        opposite vertex j (IndexedTet::face, geometry.h:474-485), UINT32_MAX
        on the hull;
      * vert_to_tet[v] = the smallest tet containing v, UINT32_MAX for none.
    Returns (tets uint32 [T, 4], tet_adjacency uint32 [T, 4], vert_to_tet
    uint32 [N])."""
    p = np.asarray(points, np.float64)
    n = p.shape[0]
    t = np.sort(np.asarray(tets, np.int64), axis=1)
    t = t[np.lexsort((t[:, 3], t[:, 2], t[:, 1], t[:, 0]))]
    q = [p[t[:, k]] - p[t[:, 0]] for k in (1, 2, 3)]
    det = (q[0][:, 0] * (q[1][:, 1] * q[2][:, 2] - q[1][:, 2] * q[2][:, 1])
           - q[0][:, 1] * (q[1][:, 0] * q[2][:, 2] - q[1][:, 2] * q[2][:, 0])
           + q[0][:, 2] * (q[1][:, 0] * q[2][:, 1] - q[1][:, 1] * q[2][:, 0]))
    swap = det > 0.0
    t[swap, 2], t[swap, 3] = t[swap, 3].copy(), t[swap, 2].copy()
    num = t.shape[0]
    # faces: the sorted triple opposite each vertex, keyed as one integer
    f = np.stack([np.delete(t, j, axis=1) for j in range(4)], 1)  # [T, 4, 3]
    f = np.sort(f, axis=2).reshape(-1, 3)
    key = (f[:, 0] * n + f[:, 1]) * n + f[:, 2]
    order = np.argsort(key, kind="stable")
    ks = key[order]
    adj = np.full(4 * num, U32_NONE, np.uint32)
    same = np.nonzero(ks[1:] == ks[:-1])[0]
    if same.size and np.any(np.diff(same) == 1):
        raise ValueError("a face is shared by more than two tets")
    a, b = order[same], order[same + 1]
    adj[a] = b
    adj[b] = a
    v2t = np.full(n, U32_NONE, np.int64)
    np.minimum.at(v2t, t.reshape(-1), np.repeat(np.arange(num), 4))
    return t.astype(np.uint32), adj.reshape(num, 4), v2t.astype(np.uint32)


def _lifted_det_sign(rows):
    """Exact sign of det [[x, y, z, x^2 + y^2 + z^2]] over 4 rows of
    Fractions (the insphere determinant relative to the fifth point)."""
    m = [[r[0], r[1], r[2], r[0] * r[0] + r[1] * r[1] + r[2] * r[2]] for r in rows]
    return _sign(_det(m))


def _det(m):
    n = len(m)
    if n == 1:
        return m[0][0]
    if n == 2:
        return m[0][0] * m[1][1] - m[0][1] * m[1][0]
    total = 0
    for j in range(n):
        if m[0][j] == 0:
            continue
        minor = [row[:j] + row[j + 1:] for row in m[1:]]
        total += (-1) ** j * m[0][j] * _det(minor)
    return total


def _sign(x):
    return (x > 0) - (x < 0)


def empty_sphere_violations(points: np.ndarray, tets: np.ndarray, max_report: int = 10):
    """Tets whose circumsphere strictly contains another site, decided
    exactly: a float64 filter with a conservative error bound, and exact
    rational arithmetic on the float32 coordinates where the filter cannot
    decide (sites exactly on a sphere are not violations).  Returns up to
    max_report (tet index, site) pairs; empty for a Delaunay tetrahedralisation."""
    from fractions import Fraction
    from scipy.spatial import cKDTree
    p32 = np.asarray(points, np.float32)
    p = p32.astype(np.float64)
    t = np.asarray(tets, np.int64)
    a, b, c, d = (p[t[:, k]] for k in range(4))
    # circumcentres and radii (float64) to collect candidates
    ba, ca, da = b - a, c - a, d - a
    rhs = 0.5 * np.stack([(ba * ba).sum(1), (ca * ca).sum(1), (da * da).sum(1)], 1)
    mat = np.stack([ba, ca, da], 1)
    ok = np.abs(np.linalg.det(mat)) > 0
    centre = np.zeros_like(a)
    centre[ok] = a[ok] + np.linalg.solve(mat[ok], rhs[ok][..., None])[..., 0]
    radius = np.linalg.norm(centre - a, axis=1)
    tree = cKDTree(p)
    # orientation sign of the reference inside case, to read the determinant
    ref = [[Fraction(v) for v in row] for row in ([-0.25, -0.25, -0.25], [0.75, -0.25, -0.25],
                                                   [-0.25, 0.75, -0.25], [-0.25, -0.25, 0.75])]
    ref_orient = _sign(_det([[ref[i][k] - ref[0][k] for k in range(3)] for i in (1, 2, 3)]))
    inside_sign = _lifted_det_sign(ref) * ref_orient
    found = []
    for ti in range(t.shape[0]):
        if not ok[ti]:
            continue
        cand = tree.query_ball_point(centre[ti], radius[ti] * (1 + 1e-7) + 1e-12)
        verts = set(t[ti].tolist())
        for e in cand:
            if e in verts:
                continue
            rows = p[t[ti]] - p[e]
            lifted = np.concatenate([rows, (rows * rows).sum(1, keepdims=True)], 1)
            det = np.linalg.det(lifted)
            perm = np.abs(lifted).prod(1).sum() * 24.0
            o = np.linalg.det(p[t[ti][1:]] - p[t[ti][0]])
            operm = np.abs(p[t[ti][1:]] - p[t[ti][0]]).prod(1).sum() * 6.0
            if abs(det) > 1e-10 * perm and abs(o) > 1e-10 * operm:
                s = (1 if det > 0 else -1) * (1 if o > 0 else -1)
            else:
                fe = [Fraction(float(v)) for v in p32[e]]
                fr = [[Fraction(float(v)) - fe[k] for k, v in enumerate(p32[i])] for i in t[ti]]
                fa = [Fraction(float(v)) for v in p32[t[ti][0]]]
                orient = _sign(_det([[Fraction(float(v)) - fa[k] for k, v in enumerate(p32[i])]
                                     for i in t[ti][1:]]))
                s = _lifted_det_sign(fr) * orient
            if s == inside_sign:
                found.append((ti, e))
                if len(found) >= max_report:
                    return found
    return found


def delaunay_adjacency(points: np.ndarray):
    """(point_adjacency uint32 [E], offsets uint32 [N+1]) of the Delaunay
    tetrahedralisation of points, in the given order."""
    p = np.asarray(points, np.float32)
    return csr_from_tets(delaunay_tets(p), p.shape[0])
