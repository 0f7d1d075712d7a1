"""TraceRays autograd op: drop-in for sdfoam_model/render.py (reference
sdfoam_model/render.py:10-189), same arguments and outputs.

The forward builds the cell records once and hands them to the backward
through ctx, where the reference recomputes its neighbour diffs in both
passes (pipeline.cu:1271, 1329).  In NeuS mode it also records each ray's
exit face per walk step (one byte for each of the first EXIT_RECORD_STEPS
steps) so that the backward, whose walk takes the same steps, replays them
instead of searching every cell's faces again.
"""
from __future__ import annotations

import torch

# Walk steps per ray kept in the exit record (steps past it are searched);
# 512 bytes per ray, 4.3 GB for an 8M-ray batch.
EXIT_RECORD_STEPS = 512


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
        # NeuS mode: the backward replays the forward's exit faces
        num_rays = rays.numel() // 6
        exits = (pipeline.exit_record(num_rays, EXIT_RECORD_STEPS, rays.device)
                 if ctx.use_sdfoam and num_rays > 0 else None)
        ctx.exits = exits
        results = pipeline.trace_forward(
            _points, _attributes, _point_adjacency, _point_adjacency_offsets, rays, start_point,
            depth_quantiles=depth_quantiles, return_contribution=return_contribution,
            alpha_mode="sdfoam" if ctx.use_sdfoam else "standard", inv_s=ctx.inv_s, eps=ctx.eps,
            sdf_channel=ctx.sdf_channel, cells=cells, exits=exits)
        ctx.rgba = results["rgba"]
        ctx.depth_indices = results.get("depth_indices", None)
        errbox = ErrorBox()
        ctx.errbox = errbox
        return (results["rgba"], results.get("depth", None), results.get("contribution", None),
                results["num_intersections"], errbox, results["alpha"])

    @staticmethod
    def backward(ctx, grad_rgba, grad_depth, grad_contribution, grad_num_intersections, errbox_grad, grad_alpha):
        del grad_contribution, grad_num_intersections, errbox_grad, grad_alpha
        results = ctx.pipeline.trace_backward(
            ctx.points, ctx.attributes, ctx.point_adjacency, ctx.point_adjacency_offsets, ctx.rays,
            ctx.start_point, ctx.rgba, grad_rgba, ctx.depth_quantiles, ctx.depth_indices, grad_depth,
            ctx.errbox.ray_error, alpha_mode="sdfoam" if ctx.use_sdfoam else "standard", inv_s=ctx.inv_s,
            eps=ctx.eps, sdf_channel=ctx.sdf_channel, cells=ctx.cells, exits=ctx.exits)
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
             ctx.point_adjacency_offsets, ctx.depth_quantiles, ctx.cells)
        inv_s_grad = sharpness_grad if (use_sdfoam and isinstance(ctx.inv_s, torch.Tensor)) else None
        return (None, points_grad, attr_grad, None, None, None, None, None, None, None, inv_s_grad, None, None)
