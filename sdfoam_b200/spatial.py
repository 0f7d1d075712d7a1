"""AABB tree and nearest-site query: build_aabb_tree / nn of the reference's
triangulation bindings (torch_bindings/triangulation_bindings.cpp:117-181),
same arguments, outputs and error messages, computed by libsdfoam_b200.so;
sort_points, the site order the reference's Triangulation establishes before
it triangulates (src/aabb_tree/aabb_tree.cu:62-190).

Differences: nn accepts foams of any size (the reference's warp-cooperative
query needs at least 32 sites), and exact distance ties go to the lowest
site index.
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib


def _stream(device):
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def sort_points(points: torch.Tensor):
    """(sorted_points, permutation): sorted_points[i] = points[permutation[i]],
    permutation uint32, in the reference's sort_points order (what
    Triangulation.permutation() returns after a rebuild)."""
    if points.size(-1) != 3:
        raise RuntimeError("points must have 3 as the last dimension")
    if points.dim() != 2:
        raise RuntimeError("points must have 2 dimensions")
    if points.device.type != "cuda":
        raise RuntimeError("points must be on CUDA device")
    if points.dtype != torch.float32:
        raise RuntimeError("unsupported scalar type")
    p = points.contiguous()
    n = p.size(0)
    lib = _lib.load()
    sorted_points = torch.empty_like(p)
    perm = torch.empty((n,), dtype=torch.uint32, device=p.device)
    if n == 0:
        return sorted_points, perm
    ws_bytes = lib.sdfoam_sort_points_workspace_bytes(n)
    ws = torch.empty((ws_bytes,), dtype=torch.uint8, device=p.device)
    with torch.cuda.device(p.device):
        _lib.check(lib.sdfoam_sort_points(ctypes.c_void_p(p.data_ptr()), n, ctypes.c_void_p(sorted_points.data_ptr()),
                                          ctypes.c_void_p(perm.data_ptr()), ctypes.c_void_p(ws.data_ptr()), ws_bytes,
                                          _stream(p.device)))
    return sorted_points, perm


def build_aabb_tree(points: torch.Tensor) -> torch.Tensor:
    """[pow2(N), 2, 3] tree over (already sorted) sites, leaves first."""
    if points.size(-1) != 3:
        raise RuntimeError("points must have 3 as the last dimension")
    if points.dim() != 2:
        raise RuntimeError("points must have 2 dimensions")
    if points.device.type != "cuda":
        raise RuntimeError("points must be on CUDA device")
    if points.dtype != torch.float32:
        raise RuntimeError("unsupported scalar type")
    p = points.contiguous()
    lib = _lib.load()
    n = p.size(0)
    tree = torch.empty((lib.sdfoam_aabb_tree_nodes(n), 2, 3), dtype=p.dtype, device=p.device)
    with torch.cuda.device(p.device):
        _lib.check(lib.sdfoam_build_aabb_tree(ctypes.c_void_p(p.data_ptr()), n, ctypes.c_void_p(tree.data_ptr()),
                                              _stream(p.device)))
    return tree


def nn(points: torch.Tensor, tree: torch.Tensor, queries: torch.Tensor) -> torch.Tensor:
    """uint32 index of the nearest site to each query, shape queries[..., :-1]."""
    if points.dtype != queries.dtype:
        raise RuntimeError("points and queries must have the same dtype")
    if points.dtype != tree.dtype:
        raise RuntimeError("points and tree must have the same dtype")
    if points.device.type != "cuda":
        raise RuntimeError("points must be on CUDA device")
    if tree.device.type != "cuda":
        raise RuntimeError("tree must be on CUDA device")
    if queries.device.type != "cuda":
        raise RuntimeError("queries must be on CUDA device")
    if points.dtype != torch.float32:
        raise RuntimeError("unsupported scalar type")
    p = points.contiguous()
    t = tree.contiguous()
    q = queries.contiguous()
    n = p.numel() // 3
    nq = q.numel() // 3
    out = torch.zeros(tuple(q.shape[:-1]), dtype=torch.uint32, device=q.device)
    lib = _lib.load()
    with torch.cuda.device(q.device):
        _lib.check(lib.sdfoam_nn(ctypes.c_void_p(p.data_ptr()), n, ctypes.c_void_p(t.data_ptr()),
                                 ctypes.c_void_p(q.data_ptr()), nq, ctypes.c_void_p(out.data_ptr()),
                                 _stream(q.device)))
    return out


def farthest_neighbor(points: torch.Tensor, point_adjacency: torch.Tensor, point_adjacency_offsets: torch.Tensor):
    """(uint32 farthest Delaunay neighbour, float32 mean half-edge length) per
    site (triangulation_bindings.cpp:183-217); used by the densify step."""
    p = points.contiguous()
    adj = point_adjacency.contiguous()
    off = point_adjacency_offsets.contiguous()
    if p.device.type != "cuda":
        raise RuntimeError("points must be on CUDA device")
    if p.dtype != torch.float32:
        raise RuntimeError("unsupported scalar type")
    n = p.size(0)
    shape = tuple(p.shape[:-1])
    indices = torch.zeros(shape, dtype=torch.uint32, device=p.device)
    radius = torch.zeros(shape, dtype=torch.float32, device=p.device)
    lib = _lib.load()
    with torch.cuda.device(p.device):
        _lib.check(lib.sdfoam_farthest_neighbor(ctypes.c_void_p(p.data_ptr()), ctypes.c_void_p(adj.data_ptr()),
                                                ctypes.c_void_p(off.data_ptr()), n, adj.numel(),
                                                ctypes.c_void_p(indices.data_ptr()),
                                                ctypes.c_void_p(radius.data_ptr()), _stream(p.device)))
    return indices, radius
