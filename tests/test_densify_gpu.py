"""The densify helpers on the GPU path: collect_error_map through TraceRays
(the real forward and backward kernels) on the mini foam against the same
maps built from the CPU restatement, and prune_and_densify_plan with the
library's farthest_neighbor against the restatement's.

collect_error_map follows the reference's SDFoamScene.collect_error_map
(sdfoam_model/scene.py:625-677): per image a 1/4 subset of the rays (random
row and column offsets), one start point broadcast to the image's rays as
scene.forward does (scene.py:301-304), the L1 error against the image
composited over white, and |d error / d position| summed per site; the
contribution keeps the per-site maximum.  The restatement's side applies the
chain rule by hand: d error / d rgb = -sign(t - rgb')/3 and
d error / d alpha = sum_c sign(t_c - rgb'_c)/3, with rgb' = rgb + 1 - alpha."""
import numpy as np
import pytest
import torch

from oracle import oracle as orc

pytestmark = pytest.mark.gpu

H = W = 24
IMAGES = 3
# few enough new sites that every draw has a site with positive weight
UPSAMPLE = 1.02


def _targets():
    rng = np.random.default_rng(21)
    return [rng.uniform(0, 1, (1, H, W, 3)).astype(np.float32) for _ in range(IMAGES)]


def _oracle_maps(foam, rays, start, targets, seed):
    sc = orc.OracleScene(foam.points, foam.attributes, foam.adjacency, foam.offsets, 3)
    st = orc.settings(neus=True, sharpness=50.0)
    n = foam.points.shape[0]
    error = np.zeros((n,), np.float64)
    contribution = np.zeros((n,), np.float32)
    image = rays.reshape(1, H, W, 6)
    g = torch.Generator().manual_seed(seed)
    for i in range(IMAGES):
        d = torch.randint(0, 2, (2,), generator=g)
        r = np.ascontiguousarray(image[:, d[0]::2, d[1]::2, :].reshape(-1, 6))
        t = targets[i][:, d[0]::2, d[1]::2, :].reshape(-1, 3)
        s = np.full((r.shape[0],), start[0], np.uint32)
        rf = orc.trace_forward(sc, st, r, s)
        rgba = rf["rgba"]
        sgn = np.sign(t - (rgba[:, :3] + 1.0 - rgba[:, 3:4]))
        grad = np.concatenate([-sgn / 3.0, sgn.sum(1, keepdims=True) / 3.0], 1).astype(np.float32)
        rb = orc.trace_backward(sc, st, r, s, rgba, grad)
        error += np.linalg.norm(rb["points_grad"].astype(np.float64), axis=1)
        contribution = np.maximum(contribution, rf["contribution"])
    return error, contribution


def test_collect_error_map_and_plan_on_the_gpu(mini_foam):
    import sdfoam_b200 as sdfoam
    from sdfoam_b200.densify import collect_error_map, prune_and_densify_plan
    from sdfoam_b200.render import TraceRays
    from sdfoam_b200.spatial import farthest_neighbor

    foam, rays, start = mini_foam
    assert np.all(start == start[0])  # one camera: one start point, as collect_error_map takes it
    dev = torch.device("cuda:0")
    pipe = sdfoam.create_pipeline(3)
    points = torch.from_numpy(foam.points).to(dev).requires_grad_(True)
    attributes = torch.from_numpy(foam.attributes).to(dev)
    adj = torch.from_numpy(foam.adjacency).to(dev)
    off = torch.from_numpy(foam.offsets).to(dev)
    inv_s = torch.tensor([50.0], device=dev)
    image = torch.from_numpy(rays.reshape(1, H, W, 6)).to(dev)
    targets = _targets()
    starts = [torch.from_numpy(start[:1].copy()).to(dev) for _ in range(IMAGES)]

    def forward_fn(r, s):
        r = r.contiguous()
        s = torch.broadcast_to(s, r.shape[:-1]).contiguous()
        rgba, _depth, contrib, *_ = TraceRays.apply(pipe, points, attributes, adj, off, r, s, None, True, True,
                                                   inv_s, 1e-6, attributes.shape[-1] - 1)
        return rgba, contrib

    seed = 9
    err, con = collect_error_map(forward_fn, points, [image] * IMAGES, [torch.from_numpy(t).to(dev) for t in targets],
                                 starts, white_bkg=True, downsample=2, generator=torch.Generator().manual_seed(seed))
    torch.cuda.synchronize()
    ref_err, ref_con = _oracle_maps(foam, rays, start, targets, seed)
    e = err.reshape(-1).cpu().numpy().astype(np.float64)
    assert (ref_err > 0).sum() > 100  # the images reach many sites
    assert np.all(np.abs(e - ref_err) <= 1e-3 * ref_err + 1e-5 * ref_err.max()), np.abs(e - ref_err).max()
    c = con.reshape(-1).cpu().numpy()
    assert np.all(np.abs(c - ref_con) <= 1e-4 * np.abs(ref_con) + 1e-6)

    # the plan: pruning is deterministic given the maps, the draws are not
    # comparable across devices (CUDA against CPU generators)
    gen = torch.Generator(device=dev).manual_seed(3)
    new_pts, parents, prune = prune_and_densify_plan(points.detach(), adj, off, err, con, upsample_factor=UPSAMPLE,
                                                     generator=gen, farthest_neighbor_fn=farthest_neighbor)

    def oracle_fn(p, a, o):
        return orc.farthest_neighbor(p.numpy(), a.numpy(), o.numpy())

    _, _, prune_ref = prune_and_densify_plan(torch.from_numpy(foam.points), torch.from_numpy(foam.adjacency),
                                             torch.from_numpy(foam.offsets), err.cpu(), con.cpu(),
                                             upsample_factor=UPSAMPLE, generator=torch.Generator().manual_seed(3),
                                             farthest_neighbor_fn=oracle_fn)
    assert torch.equal(prune.cpu(), prune_ref)
    n = foam.points.shape[0]
    m = int((UPSAMPLE - 1) * n)
    assert new_pts.shape == (m, 3) and parents.shape == (m,)
    par = parents.cpu().numpy()
    assert len(set(par.tolist())) == m
    far, radius = orc.farthest_neighbor(foam.points, foam.adjacency, foam.offsets)
    weight = np.maximum(e, 0) * radius
    assert (weight[par] > 0).all()
    d = np.linalg.norm(foam.points[far[par]] - foam.points[par], axis=1)
    moved = np.linalg.norm(new_pts.cpu().numpy() - foam.points[par], axis=1)
    assert (moved <= 0.275 * d * (1 + 1e-5) + 1e-7).all() and (moved >= 0.225 * d * (1 - 1e-5) - 1e-7).all()
