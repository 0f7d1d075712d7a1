"""CPU checks of the parity oracle (oracle/sdfoam_oracle.c).

The reference ships no golden vectors and cannot be built here, so the
oracle is pinned by (a) the accuracy of its scalar building blocks against
exact references and (b) finite-difference self-consistency: its backward
(restating pipeline.cu:267-550 / 553-791) must be the derivative of its
forward (pipeline.cu:36-264) for the attribute and sharpness gradients.
"""
import numpy as np
import pytest

from oracle import oracle as orc
from sdfoam_b200 import synthetic as syn


def test_expf_within_two_ulp():
    rng = np.random.default_rng(0)
    x = np.concatenate([
        rng.uniform(-104.0, 88.7, 2_000_000),
        rng.uniform(-1.0, 1.0, 500_000),
        np.array([0.0, -0.0, 1e-30, -1e-30, 88.7, -87.3, -100.0, -103.9, 0.5, -0.5]),
    ]).astype(np.float32)
    y = orc.expf_array(x).astype(np.float64)
    ref = np.exp(x.astype(np.float64))
    normal = ref >= np.finfo(np.float32).tiny
    ulp = np.spacing(ref[normal].astype(np.float32)).astype(np.float64)
    err_ulp = np.abs(y[normal] - ref[normal]) / ulp
    assert err_ulp.max() <= 2.0, err_ulp.max()
    # subnormal / underflowing results: absolute error within one subnormal step
    sub = ~normal
    assert np.all(np.abs(y[sub] - ref[sub]) <= 2 * 1.401298464324817e-45)
    assert np.isinf(orc.expf(89.0)) and orc.expf(-110.0) == 0.0
    assert np.isnan(orc.expf(float("nan")))


def test_half_conversion_matches_ieee():
    rng = np.random.default_rng(1)
    bits = rng.integers(0, 2**32, 3_000_000, dtype=np.uint64).astype(np.uint32)
    x = bits.view(np.float32)
    x = x[np.isfinite(x)]
    special = np.array([65504.0, 65519.99, 65520.0, 6.1e-5, 5.96e-8, 2.98e-8, 2.99e-8,
                        1.0 + 2**-11, 1.0 + 3 * 2**-11, -0.0, 0.0, 1e-8, -1e-8], np.float32)
    small = rng.uniform(-2.0, 2.0, 1_000_000).astype(np.float32)
    x = np.concatenate([x, special, small])
    h = orc.f2h_array(x)
    ref = x.astype(np.float16).view(np.uint16)
    assert np.array_equal(h, ref)
    allh = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    f = orc.h2f_array(allh)
    ref_f = allh.view(np.float16).astype(np.float32)
    both_nan = np.isnan(f) & np.isnan(ref_f)
    assert np.array_equal(f.view(np.uint32)[~both_nan], ref_f.view(np.uint32)[~both_nan])


def test_csr_contract():
    tets = np.array([[0, 1, 2, 3], [1, 2, 3, 4]])
    adj, off = syn.csr_from_tets(5, tets)
    assert off.tolist() == [0, 3, 7, 11, 15, 18]
    rows = [adj[off[i]:off[i + 1]].tolist() for i in range(5)]
    assert rows == [[1, 2, 3], [0, 2, 3, 4], [0, 1, 3, 4], [0, 1, 2, 4], [1, 2, 3]]


def test_sort_points_permutation_structure():
    rng = np.random.default_rng(4)
    p = rng.uniform(-1, 1, (5000, 3)).astype(np.float32)
    perm = syn.sort_points_permutation(p)
    assert np.array_equal(np.sort(perm), np.arange(5000))
    # with 8192 = pow2(5000) the last round sorts 1024-site blocks by axis
    # (13 - 1) % 3 = 0 ... rounds: seg 8192..2 = 13 rounds, last dim = 12 % 3 = 0
    q = p[perm]
    for b in range(0, 5000, 1024):
        blk = q[b:b + 1024, 0]
        assert np.all(np.diff(blk) >= 0)


def _scene(foam):
    return orc.OracleScene(foam.points, foam.attributes, foam.adjacency, foam.offsets, foam.sh_degree)


def test_forward_walk_is_adjacent_and_bounded(mini_foam):
    foam, rays, start = mini_foam
    sc = _scene(foam)
    st = orc.settings(neus=True, sharpness=50.0)
    out = orc.trace_forward(sc, st, rays, start, record_sequences=True)
    n = out["num_intersections"]
    assert n.min() >= 1 and n.max() <= 1025
    a = out["rgba"][:, 3]
    assert np.all((a >= 0) & (a <= 1))
    off, cells, cnt = out["seq_offsets"], out["seq_cells"], out["seq_count"]
    assert np.all(cnt <= n)
    adj_sets = [set(foam.adjacency[foam.offsets[i]:foam.offsets[i + 1]].tolist()) for i in range(len(foam.points))]
    for r in range(0, rays.shape[0], 7):
        seq = cells[off[r]:off[r] + cnt[r]]
        assert seq[0] == start[r] or cnt[r] == 0
        for u, v in zip(seq[:-1], seq[1:]):
            assert v in adj_sets[u]


def _loss(sc, st, rays, start, g, attrs=None):
    if attrs is not None:
        sc.attributes[...] = attrs
    out = orc.trace_forward(sc, st, rays, start, return_contribution=False, threads=1)
    return float((out["rgba"].astype(np.float64) * g).sum()), out


@pytest.mark.parametrize("neus", [True, False])
def test_backward_matches_finite_differences(mini_foam, neus):
    foam, rays, start = mini_foam
    rng = np.random.default_rng(11)
    attrs0 = foam.attributes.copy()
    if not neus:
        attrs0[:, -1] = np.log1p(np.exp(rng.normal(0, 1, attrs0.shape[0]))).astype(np.float32) * 4.0
    sc = orc.OracleScene(foam.points, attrs0, foam.adjacency, foam.offsets, 3)
    st = orc.settings(neus=neus, sharpness=20.0)
    # a handful of rays that hit something, one at a time (keeps L ~ O(1))
    full = orc.trace_forward(sc, st, rays, start, threads=1)
    hit = np.nonzero(full["rgba"][:, 3] > 0.2)[0][:4]
    assert hit.size >= 2
    checked = 0
    for r in hit:
        ray, st0 = rays[r:r + 1], start[r:r + 1]
        g = rng.normal(0, 1, (1, 4)).astype(np.float64)
        _, fw = _loss(sc, st, ray, st0, g, attrs0)
        b = orc.trace_backward(sc, st, ray, st0, fw["rgba"], g.astype(np.float32), threads=1)
        seq = orc.trace_forward(sc, st, ray, st0, threads=1, record_sequences=True)
        sites = np.unique(seq["seq_cells"][: seq["seq_count"][0]])
        # attribute entries of visited sites with a non-negligible gradient
        cand = [(s, c) for s in sites for c in (0, 1, 2, 5, 20, 48)]
        grads = np.array([b["attr_grad"][s, c] for s, c in cand])
        order = np.argsort(-np.abs(grads))[:12]
        for k in order:
            s, c = cand[k]
            if abs(grads[k]) < 1e-3:
                continue
            h = 2e-2 if c < 48 else (2e-4 if neus else 2e-3)
            a = attrs0.copy()
            a[s, c] += h
            lp, _ = _loss(sc, st, ray, st0, g, a)
            a[s, c] -= 2 * h
            lm, _ = _loss(sc, st, ray, st0, g, a)
            fd = (lp - lm) / (2 * h)
            assert abs(fd - grads[k]) <= 2e-2 * abs(grads[k]) + 2e-3, (r, s, c, fd, grads[k])
            checked += 1
        if neus:
            h = 1e-2
            st_p = orc.settings(neus=True, sharpness=20.0 + h)
            st_m = orc.settings(neus=True, sharpness=20.0 - h)
            lp, _ = _loss(sc, st_p, ray, st0, g, attrs0)
            lm, _ = _loss(sc, st_m, ray, st0, g, attrs0)
            fd = (lp - lm) / (2 * h)
            an = float(b["sharpness_grad"][0])
            assert abs(fd - an) <= 3e-2 * abs(an) + 2e-3, (fd, an)
    sc.attributes[...] = attrs0
    assert checked >= 8


def test_walk_exits_through_the_nearest_face(mini_foam):
    """Geometry, independent of any implementation: at every shaded step
    the face the walk leaves through is, in float64 geometry with the true
    bisector planes, the first face the ray meets after entering (the
    smallest t > t0 among faces with d . (q - p) > 0).  The reference's walk
    uses binary16 plane offsets, so a ray passing within their rounding of a
    Voronoi edge may leave through the other face of the edge: every such
    swap must be the binary16 planes' own order (checked in float64), and
    the walk's later cells are then not compared."""
    foam, rays, start = mini_foam
    sc = _scene(foam)
    st = orc.settings(neus=True, sharpness=50.0)
    out = orc.trace_forward(sc, st, rays, start, record_sequences=True)
    off, cells, cnt, nint = out["seq_offsets"], out["seq_cells"], out["seq_count"], out["num_intersections"]
    P = foam.points.astype(np.float64)
    steps = swapped = 0
    worst = 0.0
    for r in range(rays.shape[0]):
        seq = cells[off[r]:off[r] + cnt[r]].astype(np.int64)
        if seq.size < 2 or nint[r] != cnt[r] + 1:
            continue  # only walks whose every step was shaded
        o = rays[r, :3].astype(np.float64)
        d = rays[r, 3:].astype(np.float64)
        d /= np.linalg.norm(d)
        t0 = 0.0
        for k in range(seq.size - 1):
            c, nxt = seq[k], seq[k + 1]
            nb = foam.adjacency[foam.offsets[c]:foam.offsets[c + 1]].astype(np.int64)
            n = P[nb] - P[c]
            dp = n @ d
            t = ((0.5 * (P[nb] + P[c]) - o) * n).sum(1) / np.where(dp > 0, dp, 1.0)
            t_exit = t[nb == nxt][0]
            cand = (dp > 0) & (t > t0 - 1e-4)
            steps += 1
            t_min = t[cand].min()
            if t_exit != t_min:
                # a swap near a Voronoi edge: with the binary16 plane offsets
                # the walk uses (evaluated in float64) its face must come
                # first, up to float32 rounding
                swapped += 1
                f16 = (foam.points[nb] - foam.points[c]).astype(np.float16).astype(np.float64)
                t16 = ((P[c] + 0.5 * f16 - o) * f16).sum(1) / (f16 @ d)
                j_min = np.nonzero(cand & (t == t_min))[0][0]
                worst = max(worst, (t16[nb == nxt][0] - t16[j_min]) / abs(t16[j_min]))
                break  # the rest of this walk follows the cells on the other side
            t0 = max(t0, t_exit)
    assert steps > 5000
    # rare, and each one explained by the binary16 planes
    assert swapped < 0.002 * steps and worst < 1e-6, (worst, swapped, steps)


def test_sh_basis_is_orthonormal_real_sh():
    """The SH constants and polynomials of the restated basis (the
    reference's sh_utils.cuh:8-70, bit-identical on the GPU through the walk
    tests) form an orthonormal basis of real spherical harmonics up to
    degree 3: a Fibonacci-sphere quadrature of Y_i Y_j gives delta_ij."""
    n = 400_000
    k = np.arange(n) + 0.5
    z = 1.0 - 2.0 * k / n
    phi = np.pi * (3.0 - np.sqrt(5.0)) * k
    r = np.sqrt(1.0 - z * z)
    dirs = np.stack([r * np.cos(phi), r * np.sin(phi), z], 1).astype(np.float32)
    Y = orc.sh_basis(dirs).astype(np.float64)
    gram = 4.0 * np.pi * (Y.T @ Y) / n
    np.testing.assert_allclose(gram, np.eye(16), atol=2e-5)
    # and the degree-1 signs of the reference: Y1 = -C1 y, Y2 = C1 z, Y3 = -C1 x
    e = orc.sh_basis(np.array([[1, 0, 0], [0, 1, 0], [0, 0, 1]], np.float32))
    assert e[0, 3] < 0 and e[1, 1] < 0 and e[2, 2] > 0
