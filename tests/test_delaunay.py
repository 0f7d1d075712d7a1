"""Delaunay adjacency (sdfoam_b200.Triangulation, the reference's
Triangulation / find_adjacency): the GPU Voronoi-cell kernels through the C
ABI against Qhull's tetrahedralisation written as the reference's CSR
(oracle/delaunay_oracle.py).  Bit-exact CSR is the bar."""
import numpy as np
import pytest

from oracle import delaunay_oracle as dor
from oracle import spatial_oracle as so
from sdfoam_b200 import synthetic as syn


def _check_csr(adj, off, n):
    assert off[0] == 0 and off[n] == adj.size
    for i in range(n):
        row = adj[off[i]:off[i + 1]]
        assert np.all(np.diff(row.astype(np.int64)) > 0)
        assert np.all(row != i)


def test_oracle_csr_conventions():
    rng = np.random.default_rng(0)
    p = rng.uniform(-1, 1, (300, 3)).astype(np.float32)
    adj, off = dor.delaunay_adjacency(p)
    _check_csr(adj, off, 300)
    # symmetric: j in row i <=> i in row j
    pairs = {(i, int(j)) for i in range(300) for j in adj[off[i]:off[i + 1]]}
    assert all((j, i) in pairs for i, j in pairs)
    # the scene generator's CSR (an independent writer of the same contract)
    adj2, off2 = syn.delaunay_adjacency(p)
    assert np.array_equal(adj, adj2) and np.array_equal(off, off2)


def test_oracle_csr_empty_rows():
    # rows with no edges keep UINT32_MAX the way find_adjacency leaves them:
    # the entry after an empty row, and the one after the last non-empty row
    tets = np.array([[0, 1, 2, 3], [1, 2, 3, 5]])
    adj, off = dor.csr_from_tets(tets, 7)
    assert off.tolist() == [0, 3, 7, 11, 15, 0xFFFFFFFF, 0xFFFFFFFF, 18]
    assert adj[15:].tolist() == [1, 2, 3]


def _gpu_triangulate(p):
    import torch
    import sdfoam_b200 as sdfoam
    tri = sdfoam.Triangulation(torch.from_numpy(p).cuda())
    return tri


CASES = ["tiny", "uniform", "band", "small", "high_degree", "clustered"]


def _case_points(case):
    rng = np.random.default_rng(7)
    if case == "tiny":
        p, _ = syn.make_sites("tiny", None, 0)
    elif case == "uniform":
        p = rng.uniform(-1, 1, (20000, 3)).astype(np.float32)
    elif case == "band":  # sites on a thin spherical shell: many near-cospherical sets
        d = rng.normal(size=(20000, 3))
        d /= np.linalg.norm(d, axis=1, keepdims=True)
        p = (d * (0.5 + rng.uniform(-0.01, 0.01, (20000, 1)))).astype(np.float32)
    elif case == "small":  # 40 sites: almost every cell reaches the convex hull
        p = rng.normal(size=(40, 3)).astype(np.float32)
    elif case == "clustered":  # the densify loop's growth: three rounds of 10 % jittered copies of the same sites
        p = rng.uniform(-1, 1, (16000, 3))
        for _ in range(3):
            parents = np.argsort(np.abs(p[:, 0] + 0.5 * p[:, 1]), kind="stable")[:p.shape[0] // 10]
            p = np.concatenate([p, p[parents] + rng.normal(0.0, 0.004, (parents.shape[0], 3))])
        p = p.astype(np.float32)
    else:  # a site inside a jittered shell of 200: degree ~200, past the first pass's cell
        d = rng.normal(size=(200, 3))
        d /= np.linalg.norm(d, axis=1, keepdims=True)
        shell = d * (1.0 + rng.uniform(-0.01, 0.01, (200, 1)))
        far = rng.uniform(-3, 3, (2000, 3))
        far = far[np.linalg.norm(far, axis=1) > 1.6]
        p = np.concatenate([[[0.0, 0.0, 0.0]], shell, far]).astype(np.float32)
    return p


@pytest.mark.parametrize("case", CASES)
def test_oracle_is_delaunay_on_the_gpu_test_sets(case):
    """Qhull is floating point and can return non-Delaunay tets for
    near-degenerate sites; on the sets the GPU comparison below uses, the
    oracle's tets pass the exact empty-circumsphere check."""
    p = _case_points(case)
    assert dor.empty_sphere_violations(p, dor.delaunay_tets(p)) == []


@pytest.mark.gpu
@pytest.mark.parametrize("case", CASES)
def test_adjacency_matches_qhull(case):
    p = _case_points(case)
    tri = _gpu_triangulate(p)
    perm = tri.permutation().cpu().numpy().astype(np.int64)
    assert np.array_equal(perm, so.sort_permutation(p))
    ps = p[perm]
    adj = tri.point_adjacency().cpu().numpy()
    off = tri.point_adjacency_offsets().cpu().numpy()
    ref_adj, ref_off = dor.delaunay_adjacency(ps)
    st = tri.last_status
    assert st["failed_cells"] == 0 and st["duplicates"] == 0
    if case == "high_degree":
        assert np.diff(ref_off.astype(np.int64)).max() > 150
    assert np.array_equal(off, ref_off), (st, int(np.sum(off != ref_off)))
    assert np.array_equal(adj, ref_adj), st


@pytest.mark.gpu
def test_incremental_rebuild_keeps_order():
    import torch
    rng = np.random.default_rng(9)
    p = rng.uniform(-1, 1, (5000, 3)).astype(np.float32)
    tri = _gpu_triangulate(p)
    perm = tri.permutation().clone()
    ps = torch.from_numpy(p).cuda()[perm.long()]
    moved = ps + 1e-3 * torch.randn_like(ps)
    assert tri.rebuild(moved, incremental=True) is False
    assert torch.equal(tri.permutation(), perm)
    ref_adj, ref_off = dor.delaunay_adjacency(moved.cpu().numpy())
    assert np.array_equal(tri.point_adjacency_offsets().cpu().numpy(), ref_off)
    assert np.array_equal(tri.point_adjacency().cpu().numpy(), ref_adj)
    # a full rebuild re-sorts
    assert tri.rebuild(moved, incremental=False) is True


@pytest.mark.gpu
def test_triangulation_errors():
    import torch
    import sdfoam_b200 as sdfoam
    from sdfoam_b200.triangulation import TriangulationFailedError
    with pytest.raises(RuntimeError, match="does not support less than 32 points"):
        sdfoam.Triangulation(torch.rand(31, 3, device="cuda"))
    with pytest.raises(RuntimeError, match="points must have float32 dtype"):
        sdfoam.Triangulation(torch.rand(64, 3, device="cuda", dtype=torch.float64))
    p = torch.rand(64, 3, device="cuda")
    p[10] = p[3]
    with pytest.raises(TriangulationFailedError, match="duplicate points found"):
        sdfoam.Triangulation(p)


def test_oracle_tet_structure_conventions():
    """The restated tet arrays: volume > 0, symmetric face links between
    tets that share the linked faces, vert_to_tet the smallest tet."""
    rng = np.random.default_rng(3)
    p = rng.uniform(-1, 1, (400, 3)).astype(np.float32)
    t, a, v = dor.tet_structure(p, dor.delaunay_tets(p))
    key = [tuple(sorted(r)) for r in t.tolist()]
    assert key == sorted(key)
    q = p.astype(np.float64)
    vol = np.einsum("ij,ij->i", np.cross(q[t[:, 2]] - q[t[:, 0]], q[t[:, 1]] - q[t[:, 0]]), q[t[:, 3]] - q[t[:, 0]])
    assert (vol > 0).all()
    hull = 0
    for i in range(t.shape[0]):
        for j in range(4):
            x = int(a[i, j])
            if x == dor.U32_NONE:
                hull += 1
                continue
            i2, j2 = divmod(x, 4)
            assert int(a[i2, j2]) == 4 * i + j
            assert set(np.delete(t[i], j)) == set(np.delete(t[i2], j2))
    assert hull > 0
    for k in range(p.shape[0]):
        assert v[k] == min(np.nonzero((t == k).any(axis=1))[0])


@pytest.mark.gpu
@pytest.mark.parametrize("case", CASES)
def test_tets_match_qhull(case):
    """Triangulation.tets(), tet_adjacency() and vert_to_tet() against the
    same arrays built from Qhull's tets (tet order, vertex order and
    orientation, face links, smallest tet per site: all exact)."""
    p = _case_points(case)
    tri = _gpu_triangulate(p)
    ps = p[tri.permutation().cpu().numpy().astype(np.int64)]
    ref_t, ref_a, ref_v = dor.tet_structure(ps, dor.delaunay_tets(ps))
    t = tri.tets().cpu().numpy()
    assert t.shape == ref_t.shape, (t.shape, ref_t.shape)
    assert np.array_equal(t, ref_t)
    assert np.array_equal(tri.tet_adjacency().cpu().numpy(), ref_a)
    assert np.array_equal(tri.vert_to_tet().cpu().numpy(), ref_v)


@pytest.mark.gpu
def test_large_mixture_matches_qhull():
    """150k sites: a uniform background, a thin band around three spheres (the
    headline's mixture, 80 % in the band) and two rounds of densify-style
    jittered copies -- CSR, tets, face links and vert_to_tet against Qhull.
    (Qhull is not exact; on random sites in general position its tets are
    the Delaunay tets.)"""
    rng = np.random.default_rng(12)
    n = 120_000
    d = rng.normal(size=(n, 3))
    d /= np.linalg.norm(d, axis=1, keepdims=True)
    centres = np.array([[0.0, 0.0, 0.0], [0.6, 0.2, -0.1], [-0.5, -0.3, 0.3]])
    radii = np.array([0.45, 0.25, 0.3])
    k = rng.integers(0, 3, n)
    band = centres[k] + d * (radii[k] + rng.uniform(-0.02, 0.02, n))[:, None]
    p = np.concatenate([rng.uniform(-1, 1, (n // 4, 3)), band])
    for _ in range(2):
        parents = rng.choice(p.shape[0], p.shape[0] // 20, replace=False)
        p = np.concatenate([p, p[parents] + rng.normal(0.0, 0.003, (parents.shape[0], 3))])
    p = p.astype(np.float32)
    _, first = np.unique(p, axis=0, return_index=True)
    p = p[np.sort(first)]
    tri = _gpu_triangulate(p)
    ps = p[tri.permutation().cpu().numpy().astype(np.int64)]
    ref_tets = dor.delaunay_tets(ps)
    ref_adj, ref_off = dor.csr_from_tets(ref_tets, ps.shape[0])
    assert np.array_equal(tri.point_adjacency_offsets().cpu().numpy(), ref_off)
    assert np.array_equal(tri.point_adjacency().cpu().numpy(), ref_adj)
    ref_t, ref_a, ref_v = dor.tet_structure(ps, ref_tets)
    assert np.array_equal(tri.tets().cpu().numpy(), ref_t)
    assert np.array_equal(tri.tet_adjacency().cpu().numpy(), ref_a)
    assert np.array_equal(tri.vert_to_tet().cpu().numpy(), ref_v)
