"""TraceRays autograd op: drop-in for sdfoam_model/render.py (reference
sdfoam_model/render.py:10-189), same arguments and outputs.

The forward builds the cell records once and hands them to the backward
through ctx, where the reference recomputes its neighbour diffs in both
passes (pipeline.cu:1271, 1329).  In NeuS mode it also records each ray's
exit face per walk step (one byte for each of the first EXIT_RECORD_STEPS
steps) so that the backward, whose walk takes the same steps, replays them
instead of searching every cell's faces again.

With pipeline.sort_rays set, the op walks the batch in a coherent order --
rays of one start site (camera) together, then by direction along a Morton
curve -- and hands every per-ray output back in the caller's order.  Each
ray's walk is independent, so per-ray results are the same bits; only the
order of the per-site atomic sums changes (as between any two launches).
Training draws rays in random order, which leaves the lanes of a warp in
unrelated cells.
"""
from __future__ import annotations

import torch

# Walk steps per ray kept in the exit record (steps past it are searched);
# 512 bytes per ray, 4.3 GB for an 8M-ray batch.
EXIT_RECORD_STEPS = 512
# Walk steps per ray the forward records for the backward -- the site
# entered, the exit distance and the colour (steps past it are replayed from
# the exit record or searched, their SH rows gathered and evaluated again);
# 5 KB per ray, 43 GB for an 8M-ray batch.
COLOR_RECORD_STEPS = 256


def _spread_bits16(x: torch.Tensor) -> torch.Tensor:
    x = (x | (x << 8)) & 0x00FF00FF
    x = (x | (x << 4)) & 0x0F0F0F0F
    x = (x | (x << 2)) & 0x33333333
    return (x | (x << 1)) & 0x55555555


def coherent_order(rays: torch.Tensor, start_point: torch.Tensor) -> torch.Tensor:
    """Permutation (int64) that sorts the rays by (start site, Morton code of
    their direction on the octahedral map, 16 bits per axis)."""
    r = rays.reshape(-1, 6).float()
    d = r[:, 3:6]
    d = d / d.abs().sum(dim=1, keepdim=True).clamp_min(1e-30)
    u, v = d[:, 0], d[:, 1]
    lower = d[:, 2] < 0
    # fold the lower hemisphere onto the outer triangles of the square
    u, v = (torch.where(lower, (1 - v.abs()) * torch.where(u >= 0, 1.0, -1.0), u),
            torch.where(lower, (1 - u.abs()) * torch.where(v >= 0, 1.0, -1.0), v))
    qu = ((u * 0.5 + 0.5) * 65535.0).round().clamp(0, 65535).to(torch.int64)
    qv = ((v * 0.5 + 0.5) * 65535.0).round().clamp(0, 65535).to(torch.int64)
    key = (start_point.reshape(-1).to(torch.int64) << 32) | _spread_bits16(qu) | (_spread_bits16(qv) << 1)
    return torch.argsort(key)


def _unsort(x: torch.Tensor, perm: torch.Tensor, shape) -> torch.Tensor:
    """out[perm] = x (rows), for uint32 outputs through an int32 view (torch
    has no index_put for uint32)."""
    u32 = x.dtype == torch.uint32
    src = x.view(torch.int32) if u32 else x
    out = torch.empty_like(src)
    out[perm] = src
    if u32:
        out = out.view(torch.uint32)
    return out.reshape(shape)


class ErrorBox:
    def __init__(self):
        self.ray_error = None
        self.point_error = None


class TraceRays(torch.autograd.Function):
    @staticmethod
    def forward(ctx, pipeline, _points, _attributes, _point_adjacency, _point_adjacency_offsets, rays,
                start_point, depth_quantiles, return_contribution, use_sdfoam: bool = False,
                inv_s=50.0, eps: float = 1e-6, sdf_channel=None):
        ctx.rays = rays
        ctx.start_point = start_point
        ctx.pipeline = pipeline
        ctx.points = _points
        ctx.attributes = _attributes
        ctx.point_adjacency = _point_adjacency
        ctx.point_adjacency_offsets = _point_adjacency_offsets
        ctx.depth_quantiles = depth_quantiles
        ctx.use_sdfoam = bool(use_sdfoam)
        ctx.inv_s = inv_s
        ctx.eps = float(eps)
        ctx.sdf_channel = (int(sdf_channel) if sdf_channel is not None
                           else (_attributes.shape[-1] - 1 if use_sdfoam else -1))
        cells = pipeline.build_cells(_points, _attributes, _point_adjacency, _point_adjacency_offsets)
        ctx.cells = cells
        num_rays = rays.numel() // 6
        ctx.perm = None
        if getattr(pipeline, "sort_rays", False) and num_rays > 1:
            perm = coherent_order(rays, start_point)
            ctx.perm = perm
            ctx.batch_shape = tuple(rays.shape[:-1])
            rays = rays.reshape(-1, 6)[perm]
            # uint32 has no CUDA gather: permute its int32 bit pattern
            start_point = start_point.reshape(-1).view(torch.int32)[perm].view(torch.uint32)
            if depth_quantiles is not None:
                depth_quantiles = depth_quantiles.reshape(num_rays, -1)[perm]
            ctx.rays, ctx.start_point, ctx.depth_quantiles = rays, start_point, depth_quantiles
        # NeuS mode: the backward replays the forward's exit faces
        exits = (pipeline.exit_record(num_rays, EXIT_RECORD_STEPS, rays.device)
                 if ctx.use_sdfoam and num_rays > 0 else None)
        record = ctx.use_sdfoam and num_rays > 0 and hasattr(pipeline, "color_record")
        colors = pipeline.color_record(num_rays, COLOR_RECORD_STEPS, rays.device) if record else None
        sites = pipeline.site_record(num_rays, COLOR_RECORD_STEPS, rays.device) if record else None
        ctx.exits = exits
        ctx.colors = colors
        ctx.sites = sites
        results = pipeline.trace_forward(
            _points, _attributes, _point_adjacency, _point_adjacency_offsets, rays, start_point,
            depth_quantiles=depth_quantiles, return_contribution=return_contribution,
            alpha_mode="sdfoam" if ctx.use_sdfoam else "standard", inv_s=ctx.inv_s, eps=ctx.eps,
            sdf_channel=ctx.sdf_channel, cells=cells, exits=exits,
            **({"colors": colors, "sites": sites} if colors is not None else {}))
        ctx.rgba = results["rgba"]
        ctx.depth_indices = results.get("depth_indices", None)
        errbox = ErrorBox()
        ctx.errbox = errbox
        rgba, depth, nint = results["rgba"], results.get("depth", None), results["num_intersections"]
        if ctx.perm is not None:
            bs = ctx.batch_shape
            rgba = _unsort(rgba, ctx.perm, bs + (4,))
            nint = _unsort(nint, ctx.perm, bs + (1,))
            if depth is not None:
                depth = _unsort(depth, ctx.perm, bs + (depth.shape[-1],))
        return (rgba, depth, results.get("contribution", None), nint, errbox, results["alpha"])

    @staticmethod
    def backward(ctx, grad_rgba, grad_depth, grad_contribution, grad_num_intersections, errbox_grad, grad_alpha):
        del grad_contribution, grad_num_intersections, errbox_grad, grad_alpha
        ray_error = ctx.errbox.ray_error
        if ctx.perm is not None:
            # per-ray inputs in the order the forward walked
            R = ctx.perm.numel()
            grad_rgba = grad_rgba.reshape(R, 4)[ctx.perm]
            if grad_depth is not None:
                grad_depth = grad_depth.reshape(R, -1)[ctx.perm]
            if ray_error is not None:
                ray_error = ray_error.reshape(R, -1)[ctx.perm]
        results = ctx.pipeline.trace_backward(
            ctx.points, ctx.attributes, ctx.point_adjacency, ctx.point_adjacency_offsets, ctx.rays,
            ctx.start_point, ctx.rgba, grad_rgba, ctx.depth_quantiles, ctx.depth_indices, grad_depth,
            ray_error, alpha_mode="sdfoam" if ctx.use_sdfoam else "standard", inv_s=ctx.inv_s,
            eps=ctx.eps, sdf_channel=ctx.sdf_channel, cells=ctx.cells, exits=ctx.exits,
            **({"colors": ctx.colors, "sites": ctx.sites} if ctx.colors is not None else {}))
        points_grad = results["points_grad"].contiguous()
        attr_grad = results["attr_grad"].contiguous()
        sharpness_grad = results["sharpness_grad"].contiguous()
        if sharpness_grad is not None and isinstance(ctx.inv_s, torch.Tensor):
            sharpness_grad = sharpness_grad.to(ctx.inv_s.dtype).view_as(ctx.inv_s)
        ctx.errbox.point_error = results.get("point_error", None)
        # render.py:154-157: non-finite gradients are zeroed
        torch.nan_to_num_(points_grad, nan=0.0, posinf=0.0, neginf=0.0)
        torch.nan_to_num_(attr_grad, nan=0.0, posinf=0.0, neginf=0.0)
        if sharpness_grad is not None:
            torch.nan_to_num_(sharpness_grad, nan=0.0, posinf=0.0, neginf=0.0)
        use_sdfoam = ctx.use_sdfoam
        del (ctx.rays, ctx.start_point, ctx.pipeline, ctx.rgba, ctx.points, ctx.attributes, ctx.point_adjacency,
             ctx.point_adjacency_offsets, ctx.depth_quantiles, ctx.cells, ctx.exits, ctx.colors, ctx.sites)
        inv_s_grad = sharpness_grad if (use_sdfoam and isinstance(ctx.inv_s, torch.Tensor)) else None
        return (None, points_grad, attr_grad, None, None, None, None, None, None, None, inv_s_grad, None, None)
