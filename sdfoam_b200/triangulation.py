"""sdfoam.Triangulation on the GPU (torch_bindings/triangulation_bindings.cpp:
219-237, src/delaunay/delaunay.cu:233-395): the Delaunay adjacency of the
sites after the reference's sort_points order, computed by libsdfoam_b200.so.

    tri = Triangulation(points)          # rebuild(points, incremental=False)
    sorted_ = tri.rebuild(points, incremental=False)   # True: sites were re-sorted
    perm = tri.permutation()             # uint32 [N]: sorted site i = points[perm[i]]
    adj, off = tri.point_adjacency(), tri.point_adjacency_offsets()

As in the reference, the adjacency refers to the sorted order: the caller
permutes its per-site tensors by permutation() when rebuild returns True
(sdfoam_model/scene.py:216-237), and an incremental rebuild of the same
number of sites keeps the caller's order and the previous permutation.
Failures raise TriangulationFailedError (a RuntimeError), which the reference's
scene.py answers by jittering the sites and retrying.

    tets = tri.tets()                    # uint32 [T, 4], sorted by vertex set, volume > 0
    tadj = tri.tet_adjacency()           # uint32 [T, 4]: 4 t' + j' across face j, UINT32_MAX on the hull
    v2t = tri.vert_to_tet()              # uint32 [N]: smallest tet containing each site

The tet-level getters are computed from the adjacency on first use after a
rebuild (the reference computes them inside rebuild; nothing on the tracing
path reads them).
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib
from .spatial import build_aabb_tree, sort_points


class TriangulationFailedError(RuntimeError):
    """Raised when the adjacency cannot be built (duplicate sites, a cell
    that does not close); the reference registers the same name."""


def _check_points(points: torch.Tensor):
    if points.size(-1) != 3:
        raise RuntimeError("points must have 3 as the last dimension")
    if points.device.type != "cuda":
        raise RuntimeError("points must be on CUDA device")
    if points.dtype != torch.float32:
        raise RuntimeError("points must have float32 dtype")


class Triangulation:
    def __init__(self, points: torch.Tensor):
        _check_points(points)
        self._num_points = 0
        self._perm = None
        self._adjacency = None
        self._offsets = None
        self.last_status = None
        self.rebuild(points, False)

    def rebuild(self, points: torch.Tensor, incremental: bool = False) -> bool:
        _check_points(points)
        p = points.reshape(-1, 3).contiguous()
        n = p.size(0)
        if n < 32:
            raise RuntimeError("Delaunay triangulation does not support less than 32 points")
        if incremental and n == self._num_points:
            sorted_points, resorted = p, False
        else:
            sorted_points, perm = sort_points(p)
            self._perm = perm
            self._num_points = n
            resorted = True
        self._adjacency, self._offsets, self.last_status = _adjacency(sorted_points)
        self._sorted_points = sorted_points
        self._tets = None
        return resorted

    def permutation(self) -> torch.Tensor:
        return self._perm

    def num_points(self) -> int:
        return self._num_points

    def point_adjacency(self) -> torch.Tensor:
        return self._adjacency

    def point_adjacency_offsets(self) -> torch.Tensor:
        return self._offsets

    def tets(self) -> torch.Tensor:
        return self._tet_data()[0]

    def tet_adjacency(self) -> torch.Tensor:
        return self._tet_data()[1]

    def vert_to_tet(self) -> torch.Tensor:
        return self._tet_data()[2]

    def _tet_data(self):
        if self._tets is None:
            self._tets = _tets(self._sorted_points, self._adjacency, self._offsets)
        return self._tets


def _adjacency(points: torch.Tensor):
    p = points.contiguous()
    n = p.size(0)
    lib = _lib.load()
    dev = p.device
    stream = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
    tree = build_aabb_tree(p)
    ws_bytes = lib.sdfoam_delaunay_workspace_bytes(n)
    ws = torch.empty((ws_bytes,), dtype=torch.uint8, device=dev)
    offsets = torch.empty((n + 1,), dtype=torch.uint32, device=dev)
    status = (ctypes.c_uint32 * 6)()
    with torch.cuda.device(dev):
        _lib.check(lib.sdfoam_delaunay_neighbors(ctypes.c_void_p(p.data_ptr()), n, ctypes.c_void_p(tree.data_ptr()),
                                                 ctypes.c_void_p(ws.data_ptr()), ws_bytes,
                                                 ctypes.c_void_p(offsets.data_ptr()), stream))
        _lib.check(lib.sdfoam_delaunay_status(ctypes.c_void_p(ws.data_ptr()), n, status, stream))
    failed, duplicates, asymmetric, open_cells, guard, guard_index = (int(x) for x in status)
    info = {"failed_cells": failed, "duplicates": duplicates, "asymmetric_pairs": asymmetric,
            "open_cells": open_cells, "self_check": guard, "self_check_index": guard_index}
    if duplicates:
        raise TriangulationFailedError("duplicate points found")
    if guard:
        raise TriangulationFailedError(f"index self-check {guard} failed at {guard_index}")
    if failed or asymmetric > n:
        raise TriangulationFailedError(f"{failed} Voronoi cells did not close")
    size = int(offsets[n].item())
    adjacency = torch.empty((size,), dtype=torch.uint32, device=dev)
    with torch.cuda.device(dev):
        _lib.check(lib.sdfoam_delaunay_adjacency(ctypes.c_void_p(ws.data_ptr()), n,
                                                 ctypes.c_void_p(adjacency.data_ptr()), size, stream))
    return adjacency, offsets, info


def _tets(points: torch.Tensor, adjacency: torch.Tensor, offsets: torch.Tensor):
    """(tets [T, 4], tet_adjacency [T, 4], vert_to_tet [N]) of the sorted sites
    and their CSR adjacency (find_adjacency, src/delaunay/delaunay.cu:32-144)."""
    lib = _lib.load()
    p = points.contiguous()
    n = p.size(0)
    dev = p.device
    stream = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
    adj = adjacency.contiguous()
    off = offsets.contiguous()
    status = (ctypes.c_uint32 * 4)()
    count = ctypes.c_uint32(0)
    ws_bytes = lib.sdfoam_delaunay_tets_workspace_bytes(n, 0)
    ws = torch.empty((ws_bytes,), dtype=torch.uint8, device=dev)
    with torch.cuda.device(dev):
        _lib.check(lib.sdfoam_delaunay_tets_count(ctypes.c_void_p(p.data_ptr()), n, ctypes.c_void_p(adj.data_ptr()),
                                                  adj.numel(), ctypes.c_void_p(off.data_ptr()),
                                                  ctypes.c_void_p(ws.data_ptr()), ws_bytes, ctypes.byref(count),
                                                  status, stream))
    t = int(count.value)
    ws_bytes = lib.sdfoam_delaunay_tets_workspace_bytes(n, t)
    ws = torch.empty((ws_bytes,), dtype=torch.uint8, device=dev)
    tets = torch.empty((t, 4), dtype=torch.uint32, device=dev)
    tet_adjacency = torch.empty((t, 4), dtype=torch.uint32, device=dev)
    vert_to_tet = torch.empty((n,), dtype=torch.uint32, device=dev)
    with torch.cuda.device(dev):
        _lib.check(lib.sdfoam_delaunay_tets(ctypes.c_void_p(p.data_ptr()), n, ctypes.c_void_p(adj.data_ptr()),
                                            adj.numel(), ctypes.c_void_p(off.data_ptr()),
                                            ctypes.c_void_p(ws.data_ptr()), ws_bytes, t,
                                            ctypes.c_void_p(tets.data_ptr()), ctypes.c_void_p(tet_adjacency.data_ptr()),
                                            ctypes.c_void_p(vert_to_tet.data_ptr()), status, stream))
    failed, ambiguous, too_long, _ = (int(x) for x in status)
    if ambiguous:
        raise TriangulationFailedError("ambiguous triangulation")
    if failed or too_long:
        raise TriangulationFailedError(f"{failed + too_long} Voronoi cells could not be rebuilt for their tets")
    return tets, tet_adjacency, vert_to_tet


def delaunay_adjacency(points: torch.Tensor):
    """(point_adjacency, point_adjacency_offsets) of the sites in the order
    given (no sort_points; best with sites already in that order, which keeps
    the AABB tree tight) -- what an incremental Triangulation.rebuild
    computes."""
    _check_points(points)
    p = points.reshape(-1, 3)
    if p.size(0) < 32:
        raise RuntimeError("Delaunay triangulation does not support less than 32 points")
    adjacency, offsets, _ = _adjacency(p)
    return adjacency, offsets
