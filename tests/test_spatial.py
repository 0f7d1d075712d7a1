"""AABB tree (build_aabb_tree) and nearest-site seeding (nn): GPU kernels
through the C ABI against the CPU restatement in oracle/spatial_oracle.py.
Trees must match bit for bit (boxes are min / max); nn indices must match
exactly (squared float32 distances, ties to the lowest index)."""
import numpy as np
import pytest
import torch

from oracle import spatial_oracle as so
from sdfoam_b200 import synthetic as syn


def test_tree_oracle_structure():
    rng = np.random.default_rng(0)
    p = rng.uniform(-1, 1, (1000, 3)).astype(np.float32)
    t = so.build_aabb_tree(p)
    assert t.shape == (1024, 2, 3)
    # root (last used node, index 1022) is the bounding box of all sites
    assert np.array_equal(t[1022, 0], p.min(0)) and np.array_equal(t[1022, 1], p.max(0))
    # the padded leaves repeat the last site
    assert np.array_equal(t[511, 0], p[999]) and np.array_equal(t[511, 1], p[999])


def test_nn_oracle_ties_lowest_index():
    p = np.array([[0, 0, 0], [1, 0, 0], [1, 0, 0], [-1, 0, 0]], np.float32)
    q = np.array([[0.5, 0, 0], [1, 0, 0], [0.9, 0, 0]], np.float32)
    assert so.nn(p, q).tolist() == [0, 1, 1]


@pytest.mark.gpu
@pytest.mark.parametrize("n", [1, 2, 3, 5, 1000, 4096, 40000])
def test_aabb_tree_bit_exact(n):
    import sdfoam_b200 as sdfoam
    rng = np.random.default_rng(n)
    p = rng.normal(0, 1, (n, 3)).astype(np.float32)
    tree = sdfoam.build_aabb_tree(torch.from_numpy(p).cuda()).cpu().numpy()
    ref = so.build_aabb_tree(p)
    assert tree.shape == ref.shape
    if n > 1:
        assert np.array_equal(tree[:-1], ref[:-1])  # the last slot of pow2 nodes is unused
    else:
        assert np.array_equal(tree, ref)


@pytest.mark.gpu
def test_nn_matches_brute_force(tiny_foam):
    import sdfoam_b200 as sdfoam
    foam, _, _ = tiny_foam
    rng = np.random.default_rng(1)
    q = np.concatenate([rng.uniform(-1.5, 1.5, (3000, 3)), rng.normal(0, 3, (500, 3)),
                        foam.points[:200], foam.points[:100] + 1e-7,
                        np.array([c.position for c in syn.views("surface")])]).astype(np.float32)
    pts = torch.from_numpy(foam.points).cuda()
    tree = sdfoam.build_aabb_tree(pts)
    got = sdfoam.nn(pts, tree, torch.from_numpy(q).cuda().reshape(-1, 1, 3)).cpu().numpy()
    assert got.shape == (q.shape[0], 1)
    assert np.array_equal(got.reshape(-1), so.nn(foam.points, q))
    # a site queried at its own position is its own nearest site
    assert np.array_equal(got.reshape(-1)[3500:3700], np.arange(200))


@pytest.mark.gpu
def test_nn_small_foams_and_errors():
    import sdfoam_b200 as sdfoam
    for n in (1, 2, 7):
        p = np.random.default_rng(n).uniform(-1, 1, (n, 3)).astype(np.float32)
        q = np.random.default_rng(n + 1).uniform(-1, 1, (50, 3)).astype(np.float32)
        pts = torch.from_numpy(p).cuda()
        got = sdfoam.nn(pts, sdfoam.build_aabb_tree(pts), torch.from_numpy(q).cuda()).cpu().numpy()
        assert np.array_equal(got, so.nn(p, q))
    with pytest.raises(RuntimeError, match="points and queries must have the same dtype"):
        sdfoam.nn(pts, sdfoam.build_aabb_tree(pts), torch.zeros(3, 3, dtype=torch.float64, device="cuda"))
    with pytest.raises(RuntimeError, match="points must have 3 as the last dimension"):
        sdfoam.build_aabb_tree(torch.zeros(4, 2, device="cuda"))


def test_farthest_neighbor_oracle_basics():
    from oracle import oracle as orc
    p = np.array([[0, 0, 0], [1, 0, 0], [0, 2, 0], [0, 0, 2]], np.float32)
    adj = np.array([1, 2, 3, 0, 0, 0], np.uint32)
    off = np.array([0, 3, 4, 5, 6], np.uint32)
    idx, rad = orc.farthest_neighbor(p, adj, off)
    assert idx.tolist() == [2, 0, 0, 0]          # first of the two farthest (2 and 3)
    assert np.isclose(rad[0], (0.5 + 1 + 1) / 3) and np.isclose(rad[2], 1.0)


@pytest.mark.gpu
def test_farthest_neighbor_bit_exact(tiny_foam):
    import sdfoam_b200 as sdfoam
    from oracle import oracle as orc
    foam, _, _ = tiny_foam
    idx, rad = sdfoam.farthest_neighbor(torch.from_numpy(foam.points).cuda(), torch.from_numpy(foam.adjacency).cuda(),
                                        torch.from_numpy(foam.offsets).cuda())
    ridx, rrad = orc.farthest_neighbor(foam.points, foam.adjacency, foam.offsets)
    assert np.array_equal(idx.cpu().numpy(), ridx)
    assert np.array_equal(rad.cpu().numpy().view(np.uint32), rrad.view(np.uint32))


def _order_keys(p):
    u = np.ascontiguousarray(p, np.float32).view(np.uint32)
    return np.where((u & 0x80000000) != 0, ~u, u ^ 0x80000000).astype(np.uint32)


def test_sort_oracle_small_is_lexicographic():
    # up to 1024 sites every round sorts the whole block, so r stable rounds
    # by axes 0, 1, 2, 0, ... are one lexicographic sort, last axis first
    rng = np.random.default_rng(3)
    p = np.round(rng.normal(0, 1, (700, 3)), 1).astype(np.float32)  # many ties
    p[:5] = [[0.0, 0, 0], [-0.0, 0, 0], [0.0, -0.0, 1], [-1, 2, 3], [-1, 2, 3]]
    k = _order_keys(p)
    rounds = 10  # pow2(700) = 1024
    expect = np.lexsort(tuple(k[:, r % 3] for r in range(rounds)))
    assert np.array_equal(so.sort_permutation(p), expect)
    assert np.array_equal(syn.sort_points_permutation(p), expect)


def test_sort_oracle_global_rounds_forget_segments():
    # above 1024 sites the first rounds sort all sites at once (the reference's
    # global CUB sort): with 2048 sites, round 0 (x, one segment) is global and
    # the ten block rounds then sort each 1024 block by axes 1, 2, 0, ...
    rng = np.random.default_rng(4)
    p = rng.normal(0, 1, (2048, 3)).astype(np.float32)
    k = _order_keys(p)
    first = np.argsort(k[:, 0], kind="stable")
    out = []
    for b in range(2):
        idx = first[b * 1024:(b + 1) * 1024]
        kk = k[idx]
        out.append(idx[np.lexsort(tuple(kk[:, (1 + r) % 3] for r in range(10)))])
    assert np.array_equal(so.sort_permutation(p), np.concatenate(out))


@pytest.mark.gpu
@pytest.mark.parametrize("n", [1, 2, 3, 1000, 1024, 1025, 4096, 5000, 100000, 2_200_000, 4_500_000])
def test_sort_points_matches_oracle(n):
    """Permutation bit-exact against the CPU restatement; sorted sites are the
    gathered originals bit for bit.  2.2M sites reach the per-segment round
    (2048-site segments, more than 1024 of them), 4.5M two of them (4096- and
    2048-site segments, a partial last segment)."""
    import sdfoam_b200 as sdfoam
    rng = np.random.default_rng(n)
    p = rng.normal(0, 1, (n, 3)).astype(np.float32)
    if n >= 1000:  # ties, signed zeros
        p[: n // 4] = np.round(p[: n // 4], 1)
        p[:4] = [[0.0, -0.0, 0.0], [-0.0, 0.0, -0.0], [0.0, 0.0, 0.0], [-0.0, -0.0, -0.0]]
    sorted_p, perm = sdfoam.sort_points(torch.from_numpy(p).cuda())
    perm = perm.cpu().numpy().astype(np.int64)
    ref = so.sort_permutation(p)
    assert np.array_equal(perm, ref)
    assert np.array_equal(sorted_p.cpu().numpy().view(np.uint32), p[ref].view(np.uint32))


@pytest.mark.gpu
def test_sort_points_errors():
    import sdfoam_b200 as sdfoam
    with pytest.raises(RuntimeError, match="points must have 3 as the last dimension"):
        sdfoam.sort_points(torch.zeros((4, 2), device="cuda"))
    with pytest.raises(RuntimeError, match="unsupported scalar type"):
        sdfoam.sort_points(torch.zeros((4, 3), dtype=torch.float64, device="cuda"))
    s, perm = sdfoam.sort_points(torch.zeros((0, 3), device="cuda"))
    assert s.shape == (0, 3) and perm.shape == (0,)
