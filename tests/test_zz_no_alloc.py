"""The allocation-free forward entry point, sdfoam_trace_forward_noalloc.

It serves callers that cannot allocate device memory (C-ABI hosts without a
device allocator, frame loops that must not call cudaMalloc).  It keeps the
cell records in a fixed 64 MiB device array instead of a caller-owned
workspace; its outputs must match the regular sdfoam_trace_forward path, call
after call, even though the array keeps the previous call's records.

This file is collected last on purpose: it runs the entry point's one-time
per-device set-up, and must pass both alone in a fresh process and after the
rest of the suite.
"""
import ctypes

import numpy as np
import pytest
import torch

from sdfoam_b200 import _lib, synthetic as syn

INV_S = 50.0


def _c_call(lib, pipe, pts, att, adj, off, rays, start, sharp):
    """Runs the no-alloc entry point through the C ABI; returns its outputs."""
    dev = rays.device
    R = rays.shape[0]
    N = pts.shape[0]
    rgba = torch.empty((R, 4), dtype=torch.float32, device=dev)
    nint = torch.empty((R,), dtype=torch.uint32, device=dev)
    contrib = torch.zeros((N,), dtype=torch.float32, device=dev)
    alpha = torch.zeros((N,), dtype=torch.float32, device=dev)
    foam = _lib.Foam(N, adj.numel(), 3, _lib.SDFOAM_F32, pts.data_ptr(), att.data_ptr(), adj.data_ptr(),
                     off.data_ptr())
    st = _lib.TraceSettings(1e-7, 1024, _lib.SDFOAM_ALPHA_NEUS, 48, 1e-6)
    io = _lib.ForwardIO(R, rays.data_ptr(), start.data_ptr(), 0, None, sharp.data_ptr(), rgba.data_ptr(), None,
                        None, nint.data_ptr(), contrib.data_ptr(), alpha.data_ptr(), None, None, None, None)
    stream = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
    _lib.check(lib.sdfoam_trace_forward_noalloc(ctypes.byref(foam), ctypes.byref(st), ctypes.byref(io), stream))
    torch.cuda.synchronize()
    return rgba.cpu().numpy(), nint.cpu().numpy(), contrib.cpu().numpy(), alpha.cpu().numpy()


@pytest.mark.gpu
def test_noalloc_forward_matches_regular_entry_point_twice():
    import sdfoam_b200 as sdfoam
    lib = _lib.load()
    dev = torch.device("cuda:0")
    pipe = sdfoam.create_pipeline(3)
    # two different foams in a row, so stale records from call 1 would show in call 2
    cases = []
    for seed, n, w in ((3, 4096, 24), (5, 6000, 32)):
        foam = syn.make_foam("tiny", num_points=n, seed=seed)
        cam = syn.look_at((2.2, -1.1, 0.7), fov_deg=40.0, width=w, height=w)
        rays, start = syn.camera_rays(foam, [cam], tile=(8, 4))
        cases.append((foam, rays, start))
    for foam, rays, start in cases:
        pts = torch.from_numpy(foam.points).to(dev)
        att = torch.from_numpy(foam.attributes).to(dev)
        adj = torch.from_numpy(foam.adjacency).to(dev)
        off = torch.from_numpy(foam.offsets).to(dev)
        rr = torch.from_numpy(rays).to(dev)
        ss = torch.from_numpy(start).to(dev)
        sharp = torch.tensor([INV_S], device=dev)
        rgba, nint, contrib, alpha = _c_call(lib, pipe, pts, att, adj, off, rr, ss, sharp)
        ref = pipe.trace_forward(pts, att, adj, off, rr, ss, return_contribution=True, alpha_mode="sdfoam",
                                 inv_s=sharp)
        torch.cuda.synchronize()
        assert np.array_equal(nint, ref["num_intersections"].cpu().numpy().reshape(-1))
        r_rgba = ref["rgba"].cpu().numpy()
        assert np.all(np.abs(rgba - r_rgba) <= 1e-4 * np.abs(r_rgba) + 1e-6)
        r_con = ref["contribution"].cpu().numpy().reshape(-1)
        assert np.all(np.abs(contrib - r_con) <= 1e-4 * np.abs(r_con) + 1e-6)
        # alpha is a last-writer-wins store, so only sites that exactly one
        # walk step visited have a deterministic value; unvisited sites stay 0
        n64 = ref["num_intersections"].reshape(-1).to(torch.int64)
        offs = torch.zeros(n64.numel() + 1, dtype=torch.int64, device=dev)
        offs[1:] = torch.cumsum(n64, 0)
        seq = {"offsets": offs.to(torch.uint64),
               "cells": torch.zeros(int(offs[-1].item()), dtype=torch.uint32, device=dev),
               "count": torch.zeros(n64.numel(), dtype=torch.uint32, device=dev)}
        ref2 = pipe.trace_forward(pts, att, adj, off, rr, ss, alpha_mode="sdfoam", inv_s=sharp, _sequences=seq)
        torch.cuda.synchronize()
        o, c, k = (seq["offsets"].cpu().numpy(), seq["cells"].cpu().numpy(), seq["count"].cpu().numpy())
        visited = np.concatenate([c[o[i]:o[i] + k[i]] for i in range(k.shape[0])])
        visits = np.bincount(visited, minlength=pts.shape[0])
        r_alpha = ref2["alpha"].cpu().numpy().reshape(-1)
        once = visits == 1
        assert once.sum() > 0
        assert np.array_equal(alpha[once], r_alpha[once])
        assert np.all(alpha[visits == 0] == 0) and np.all(r_alpha[visits == 0] == 0)


def test_noalloc_rejects_foams_beyond_the_static_scratch():
    lib = _lib.load()
    big = _lib.Foam(4_000_000, 60_000_000, 3, _lib.SDFOAM_F32, 256, 256, 256, 256)
    st = _lib.TraceSettings(1e-7, 1024, _lib.SDFOAM_ALPHA_NEUS, 48, 1e-6)
    io = _lib.ForwardIO()
    rc = lib.sdfoam_trace_forward_noalloc(ctypes.byref(big), ctypes.byref(st), ctypes.byref(io), None)
    assert rc == 1
    assert b"static scratch holds 67108864 bytes" in lib.sdfoam_last_error()
    # an SH degree no entry point takes: sdfoam_build_cells' code and message
    deg4 = _lib.Foam(1000, 15000, 4, _lib.SDFOAM_F32, 256, 256, 256, 256)
    rc = lib.sdfoam_trace_forward_noalloc(ctypes.byref(deg4), ctypes.byref(st), ctypes.byref(io), None)
    assert rc == 2  # SDFOAM_ERR_UNSUPPORTED
    assert b"Unsupported SH degree" in lib.sdfoam_last_error()
