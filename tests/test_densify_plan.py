"""prune_and_densify_plan (the site selection of the reference's
SDFoamScene.prune_and_densify, scene.py:546-623) on a small foam, with the
CPU restatement's farthest_neighbor standing in for the library's: the
pruning rule checked site by site, the sampling's count, uniqueness,
weights and geometry."""
import numpy as np
import torch

from oracle import oracle as orc
from oracle.delaunay_oracle import delaunay_adjacency
from sdfoam_b200.densify import prune_and_densify_plan


def _foam(seed=0):
    rng = np.random.default_rng(seed)
    # a sparse background and a tight cluster whose cells are below 1e-3
    pts = np.concatenate([rng.uniform(-1, 1, (1500, 3)), 0.3 + rng.uniform(0, 0.004, (400, 3))]).astype(np.float32)
    adj, off = delaunay_adjacency(pts)
    return pts, adj, off, rng


def _fn(points, adjacency, offsets):
    return orc.farthest_neighbor(points.numpy(), adjacency.numpy(), offsets.numpy())


def test_prune_rule_and_sampling():
    pts, adj, off, rng = _foam()
    n = pts.shape[0]
    contrib = rng.uniform(0, 0.02, (n, 1)).astype(np.float32)
    contrib[rng.uniform(size=n) < 0.5] = 0.0
    error = rng.normal(0, 1, (n, 1)).astype(np.float32)  # negative errors count as zero
    P, A, O = torch.from_numpy(pts), torch.from_numpy(adj.astype(np.int32)), torch.from_numpy(off.astype(np.int32))
    g = torch.Generator().manual_seed(5)
    new_pts, parents, prune = prune_and_densify_plan(P, A, O, torch.from_numpy(error), torch.from_numpy(contrib),
                                                     upsample_factor=1.2, generator=g, farthest_neighbor_fn=_fn)
    m = int((1.2 - 1) * n)  # the reference's float arithmetic: 379 for n = 1900
    assert new_pts.shape == (m, 3) and parents.shape == (m,) and prune.shape == (n + m,)
    assert not prune[n:].any()
    # pruning, site by site.  The reference counts contributing neighbours
    # with an inclusive prefix sum, nsum[off[i+1]] - nsum[off[i]], i.e. over
    # CSR entries off[i] + 1 .. off[i+1]: its row shifted by one entry (the
    # first neighbour left out, the next row's first neighbour counted, a
    # zero appended past the end).  The plan keeps that window.
    far, radius = orc.farthest_neighbor(pts, adj, off)
    window_src = np.concatenate([adj, [0]])
    shifted_diff = 0
    for i in range(n):
        window = window_src[off[i] + 1:off[i + 1] + 1]
        valid = np.arange(off[i] + 1, off[i + 1] + 1) < adj.shape[0]
        expect = (contrib[i, 0] <= 1e-2 and (contrib[window[valid], 0] <= 1e-2).all() and radius[i] < 1e-3)
        assert bool(prune[i]) == bool(expect), i
        row = adj[off[i]:off[i + 1]]
        shifted_diff += bool(expect) != bool(contrib[i, 0] <= 1e-2 and (contrib[row, 0] <= 1e-2).all()
                                             and radius[i] < 1e-3)
    assert shifted_diff > 0  # the window matters on this foam
    assert prune[:n].any() and not prune[:n].all()
    # sampling: distinct parents with positive weight, each new site within
    # 0.275 of the way to its parent's farthest neighbour
    par = parents.numpy()
    assert len(set(par.tolist())) == m
    assert (np.maximum(error[par, 0], 0) * radius[par] > 0).all()
    d = np.linalg.norm(pts[far[par]] - pts[par], axis=1)
    moved = np.linalg.norm(new_pts.numpy() - pts[par], axis=1)
    assert (moved <= 0.275 * d * (1 + 1e-5) + 1e-7).all() and (moved >= 0.225 * d * (1 - 1e-5) - 1e-7).all()
    # the same generator state gives the same plan
    g2 = torch.Generator().manual_seed(5)
    new2, par2, prune2 = prune_and_densify_plan(P, A, O, torch.from_numpy(error), torch.from_numpy(contrib),
                                                upsample_factor=1.2, generator=g2, farthest_neighbor_fn=_fn)
    assert torch.equal(new2, new_pts) and torch.equal(par2, parents) and torch.equal(prune2, prune)


def test_collect_error_map_accumulates_per_image():
    """Error = sum over images of |d L1 / d position| per site, contribution
    = per-site maximum, on a differentiable stand-in for the tracer."""
    from sdfoam_b200.densify import collect_error_map
    torch.manual_seed(0)
    n, H, W = 40, 6, 8
    points = torch.randn(n, 3, requires_grad=True)
    rays = [torch.randn(1, H, W, 6) for _ in range(3)]
    rgbs = [torch.rand(1, H, W, 3) for _ in range(3)]
    contribs = [torch.rand(n, 1) for _ in range(3)]
    mix = torch.randn(6, n)

    def forward_fn(r, k):
        w = torch.softmax(r @ mix, -1)                       # [1, h, w, n]
        c = w @ torch.sigmoid(points)                        # [1, h, w, 3]
        rgba = torch.cat([c, w[..., :1]], -1)
        return rgba, contribs[k]

    g = torch.Generator().manual_seed(3)
    err, con = collect_error_map(forward_fn, points, rays, rgbs, [0, 1, 2], white_bkg=True, downsample=2,
                                 generator=g)
    # the same draws, done by hand
    g = torch.Generator().manual_seed(3)
    ref = torch.zeros(n, 1)
    for i in range(3):
        d = torch.randint(0, 2, (2,), generator=g)
        r = rays[i][:, d[0]::2, d[1]::2]
        t = rgbs[i][:, d[0]::2, d[1]::2]
        p = points.detach().clone().requires_grad_(True)
        w = torch.softmax(r @ mix, -1)
        rgba = torch.cat([w @ torch.sigmoid(p), w[..., :1]], -1)
        rgb = rgba[..., :3] + (1 - rgba[..., 3:])
        (t - rgb).abs().mean(-1).sum().backward()
        ref += p.grad.norm(dim=-1, keepdim=True)
    assert torch.allclose(err, ref, rtol=1e-5, atol=1e-7)
    assert torch.equal(con, torch.maximum(torch.maximum(contribs[0], contribs[1]), contribs[2]))
    assert points.grad is None
