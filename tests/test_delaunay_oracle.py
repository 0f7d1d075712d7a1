"""The Delaunay oracle (Qhull written as the reference's CSR) checked for
the empty-circumsphere property with exact arithmetic where floating point
cannot decide: random sites pass; on a near-degenerate grid Qhull's own
floating point shows and the check reports it (confirmed independently);
a planted non-Delaunay tet is reported."""
from fractions import Fraction

import numpy as np

from oracle.delaunay_oracle import delaunay_tets, empty_sphere_violations


def test_random_sites_are_delaunay():
    pts = np.random.default_rng(0).uniform(-1, 1, (1500, 3)).astype(np.float32)
    tets = delaunay_tets(pts)
    assert tets.shape[0] > 8000
    assert empty_sphere_violations(pts, tets) == []


def _exact_inside(tet_pts, q):
    """Circumsphere of four float32 sites and a fifth, in rationals."""
    a = [Fraction(float(x)) for x in tet_pts[0]]
    rows, rhs = [], []
    for t in tet_pts[1:]:
        v = [Fraction(float(x)) - a[k] for k, x in enumerate(t)]
        rows.append(v)
        rhs.append(sum(x * x for x in v) / 2)

    def det3(m):
        return (m[0][0] * (m[1][1] * m[2][2] - m[1][2] * m[2][1]) - m[0][1] * (m[1][0] * m[2][2] - m[1][2] * m[2][0])
                + m[0][2] * (m[1][0] * m[2][1] - m[1][1] * m[2][0]))

    D = det3(rows)
    x = []
    for j in range(3):
        m = [r[:] for r in rows]
        for i in range(3):
            m[i][j] = rhs[i]
        x.append(det3(m) / D)
    c = [a[k] + x[k] for k in range(3)]
    r2 = sum((a[k] - c[k]) ** 2 for k in range(3))
    e = [Fraction(float(v)) for v in q]
    return sum((e[k] - c[k]) ** 2 for k in range(3)) < r2


def test_qhull_is_inexact_on_near_degenerate_sites_and_the_check_says_so():
    """A grid perturbed by 1e-7: Qhull (floating point) returns tets whose
    circumspheres strictly contain other sites by ~1e-13 relative; the
    exact check reports them, and an independent rational computation of
    the circumsphere confirms each one."""
    g = np.arange(5, dtype=np.float32) * 0.25
    pts = np.stack(np.meshgrid(g, g, g, indexing="ij"), -1).reshape(-1, 3)
    pts = pts + np.float32(1e-7) * np.random.default_rng(1).integers(0, 2, pts.shape).astype(np.float32)
    tets = delaunay_tets(pts)
    found = empty_sphere_violations(pts, tets, max_report=6)
    assert found
    for t, e in found:
        assert _exact_inside(pts[tets[t]], pts[e])


def test_planted_violation_is_reported():
    inner = np.random.default_rng(2).uniform(-0.5, 0.5, (200, 3)).astype(np.float32)
    corners = np.array([[-1, -1, -1], [1, -1, -1], [-1, 1, -1], [-1, -1, 1]], np.float32)
    pts = np.concatenate([corners, inner])
    found = empty_sphere_violations(pts, np.array([[0, 1, 2, 3]]), max_report=5)
    assert len(found) == 5 and all(t == 0 and e >= 4 for t, e in found)
