"""The rebuild step around the tracer when sites move or multiply: the
reference's SDFoamScene.update_triangulation (sdfoam_model/scene.py:204-244)
and the site growth of prune_and_densify (scene.py:546-623), for one GPU or
several.

With several ranks (one process per GPU) the Delaunay rebuild runs on rank 0
only and its result -- the site permutation, the CSR offsets and the
adjacency -- is broadcast to the other ranks; every rank then permutes its
copy of the per-site tensors, rebuilds its own AABB tree and seeds its own
rays (cheap, deterministic, no exchange).  The broadcast is the only
collective of the rebuild.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from .distributed import broadcast_triangulation


def rebuild(points: torch.Tensor, triangulate, world: int = 1, group=None):
    """Rebuilds the adjacency of `points` on rank 0 with
    triangulate(points) -> (perm, adjacency, offsets) and shares it.  Returns
    (perm, adjacency, offsets) on every rank; the adjacency refers to
    points[perm]."""
    rank = dist.get_rank(group) if world > 1 else 0
    perm = adjacency = offsets = None
    if rank == 0:
        perm, adjacency, offsets = triangulate(points)
    if world > 1:
        perm, adjacency, offsets = broadcast_triangulation(perm, adjacency, offsets, points.shape[0],
                                                           points.device, 0, group)
    return perm, adjacency, offsets


def gpu_triangulate(triangulation=None, on_failure=None, seed: int = 0):
    """triangulate() for rebuild(): a full sdfoam_b200.Triangulation rebuild
    (sort_points order), keeping the Triangulation between calls as the
    reference's scene keeps self.triangulation.  On TriangulationFailedError
    it follows the reference's update_triangulation (scene.py:204-244): jitter
    the sites by 1e-6 N(0, 1), doubling the jitter after every failure, and
    give up after 25 failures.  The adjacency then belongs to the jittered
    sites, which (as in the reference, for up to 5 failures) stand in for
    the caller's.  on_failure(points, error) sees every failing site set;
    triangulate.failures counts the failures of the last call."""
    from .triangulation import TriangulationFailedError
    state = {"tri": triangulation}
    gen = torch.Generator(device="cpu").manual_seed(seed)

    def attempt(points):
        from .triangulation import Triangulation
        if state["tri"] is None:
            state["tri"] = Triangulation(points)
        else:
            state["tri"].rebuild(points, incremental=False)
        tri = state["tri"]
        return tri.permutation(), tri.point_adjacency(), tri.point_adjacency_offsets()

    def triangulate(points):
        triangulate.failures = 0
        perturbation = 1e-6
        current = points
        while True:
            try:
                return attempt(current)
            except TriangulationFailedError as e:
                if on_failure is not None:
                    on_failure(current, e)
                triangulate.failures += 1
                if triangulate.failures > 25:
                    raise RuntimeError("aborted triangulation after 25 attempts") from e
                perturbation *= 2
                noise = torch.randn(points.shape, generator=gen).to(points.device, points.dtype)
                current = points + perturbation * noise

    triangulate.failures = 0
    return triangulate


def prune_and_densify_plan(points: torch.Tensor, point_adjacency: torch.Tensor,
                           point_adjacency_offsets: torch.Tensor, point_error: torch.Tensor,
                           point_contribution: torch.Tensor, upsample_factor: float = 1.2,
                           generator: torch.Generator | None = None, farthest_neighbor_fn=None):
    """The site selection of the reference's SDFoamScene.prune_and_densify
    (sdfoam_model/scene.py:546-623), without the optimizer-state surgery
    around it: returns (new_points [M, 3], parent indices [M] (int64),
    prune_mask [N + M] (bool)) for the caller's densification_postfix /
    prune_points.

      * M = int((upsample_factor - 1) * N) new sites, parents drawn without
        replacement with weights max(point_error, 0) * cell_radius
        (torch.multinomial); each new site is its parent moved a quarter of
        the way to its farthest Delaunay neighbour plus 0.1 x that length in a
        random direction;
      * a site is pruned when its contribution and its neighbours' are at
        most 1e-2 and its cell radius is below 1e-3 (new sites are kept).
        The neighbours are counted as the reference counts them, with an
        inclusive prefix sum over the CSR entries: nsum[off[i+1]] -
        nsum[off[i]] covers entries off[i] + 1 .. off[i+1], the row shifted
        by one entry; kept as is so that the same sites are pruned.

    farthest_neighbor_fn(points, adjacency, offsets) -> (index, radius)
    defaults to the library's farthest_neighbor; random draws come from
    `generator` (the global generator when None), in the reference's order."""
    if farthest_neighbor_fn is None:
        from .spatial import farthest_neighbor as farthest_neighbor_fn
    with torch.no_grad():
        n = points.shape[0]
        num_new = int((upsample_factor - 1) * n)
        error = point_error.clip(min=0).reshape(-1)
        far, cell_radius = farthest_neighbor_fn(points, point_adjacency, point_adjacency_offsets)
        far = torch.as_tensor(far, device=points.device).to(torch.int64)
        cell_radius = torch.as_tensor(cell_radius, device=points.device).reshape(-1)
        # pruning: no contribution here or at any Delaunay neighbour, small cell
        self_mask = point_contribution.reshape(-1) > 1e-2
        adj = point_adjacency.to(torch.int64)
        neighbor_mask = torch.cat([self_mask.to(torch.int64)[adj], adj.new_zeros(1)])
        nsum = torch.cumsum(neighbor_mask, 0)
        off = point_adjacency_offsets.to(torch.int64)
        n_masked = nsum[off[1:]] - nsum[off[:-1]]
        prune_mask = (n_masked == 0) & ~self_mask & (cell_radius < 1e-3)
        # sampling: a quarter of the way to the farthest neighbour, jittered
        perturbation = 0.25 * (points[far] - points)
        delta = torch.randn(perturbation.shape, generator=generator, device=points.device, dtype=points.dtype)
        delta = delta / delta.norm(dim=-1, keepdim=True)
        perturbation = perturbation + 0.1 * perturbation.norm(dim=-1, keepdim=True) * delta
        parents = torch.multinomial(error * cell_radius, num_new, replacement=False, generator=generator)
        new_points = (points + perturbation)[parents]
        prune_mask = torch.cat([prune_mask, torch.zeros(num_new, dtype=torch.bool, device=points.device)])
        return new_points, parents, prune_mask


def collect_error_map(forward_fn, points: torch.Tensor, ray_batches, rgb_batches, start_points,
                      white_bkg: bool = True, downsample: int = 2, generator: torch.Generator | None = None):
    """The per-site error and contribution maps that drive
    prune_and_densify_plan (SDFoamScene.collect_error_map, scene.py:625-677).
    For every image: a 1/downsample^2 subset of its rays (row and column
    offsets drawn at random) is traced, the per-ray L1 colour error against
    the image (composited over white when white_bkg) is summed and
    back-propagated, and |d error / d site position| is added per site; the
    contribution map keeps each site's maximum over the images.

    forward_fn(rays, start) -> (rgba, contribution) traces one ray batch
    ([1, H, W, 6]) through the scene with `points` (a leaf tensor that
    requires grad) among its inputs, e.g. TraceRays with
    return_contribution=True.  Returns (point_error [N, 1], point_contribution
    [N, 1])."""
    n = points.shape[0]
    error = torch.zeros((n, 1), dtype=points.dtype, device=points.device)
    contribution = torch.zeros((n, 1), dtype=points.dtype, device=points.device)
    for i in range(len(ray_batches)):
        rays, rgbs = ray_batches[i], rgb_batches[i]
        d = torch.randint(0, downsample, (2,), generator=generator)
        rays = rays[:, d[0]::downsample, d[1]::downsample, :]
        rgbs = rgbs[:, d[0]::downsample, d[1]::downsample, :]
        points.grad = None
        rgba, contrib = forward_fn(rays, start_points[i])
        opacity = rgba[..., -1:]
        rgb = rgba[..., :3] + (1 - opacity) if white_bkg else rgba[..., :3]
        (rgbs - rgb).abs().mean(dim=-1).sum().backward()
        error += points.grad.norm(dim=-1, keepdim=True).detach()
        contribution = torch.maximum(contribution, contrib.detach().reshape(n, 1).to(contribution.dtype))
        points.grad = None
    return error, contribution


def densify(points: torch.Tensor, attributes: torch.Tensor, score: torch.Tensor, fraction: float, sigma: float,
            generator: torch.Generator):
    """Appends round(fraction * N) new sites: copies of the sites with the
    largest score (ties to the lower index), jittered by N(0, sigma^2) per
    coordinate, inheriting their parents' attributes.  Deterministic for a
    given generator state, so every rank grows the same foam."""
    n = points.shape[0]
    k = int(round(fraction * n))
    if k == 0:
        return points, attributes
    # stable descending order by score, ties to the lower index
    order = torch.sort(score.reshape(-1), descending=True, stable=True).indices[:k]
    jitter = torch.randn((k, 3), generator=generator, device=points.device, dtype=points.dtype) * sigma
    new_points = torch.cat([points, points[order] + jitter])
    new_attributes = torch.cat([attributes, attributes[order]])
    return new_points, new_attributes
