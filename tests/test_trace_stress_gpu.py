"""GPU parity on a foam built to reach the walk's rare paths.

The tiny and mini foams never exercise three paths that the benchmarked 4M-site
foam does:
  * cell rows longer than 254 faces: the exit record stores a face position in
    one byte, so an exit through face 254 or later is recorded as "unknown"
    and the NeuS backward searches that step instead of replaying it;
  * rays of more than 512 walk steps: past the record's 512 bytes per ray the
    backward searches every step;
  * max_intersections 4096 (the unbounded configuration's cap).

The foam here is the surface mixture (80 % within +-0.02 of three spheres,
20 % uniform) at 100k sites, plus
  * a hub: one site in an emptied ball whose shell of 300 nearly cospherical
    sites gives it a 300-face cell, seen by a camera aimed at it;
  * a tube: 40k sites packed along a thin box 2 units long, traced by rays
    along its axis (~600 cells each) through sites whose SDF keeps them
    transparent.
GPU (C ABI) against the CPU oracle, with the tolerances of test_trace_gpu.py.
"""
import numpy as np
import pytest
import torch

from oracle import oracle as orc
from sdfoam_b200 import synthetic as syn

pytestmark = pytest.mark.gpu

HUB = np.array([0.0, -0.7, -0.3])
HUB_SHELL = 300
TUBE_Y, TUBE_Z, TUBE_HALF = -0.85, 0.85, 0.015
MAX_STEPS = 4096


def _unit(rng, n):
    v = rng.normal(size=(n, 3))
    return v / np.linalg.norm(v, axis=1, keepdims=True)


def stress_foam(seed=5):
    rng = np.random.default_rng(seed)
    p, _ = syn.make_sites("surface", num_points=100_000, seed=seed)
    p = p.astype(np.float64)
    # the hub's emptied ball and the tube's box
    p = p[np.linalg.norm(p - HUB, axis=1) > 0.1]
    in_tube = (np.abs(p[:, 1] - TUBE_Y) < 2 * TUBE_HALF) & (np.abs(p[:, 2] - TUBE_Z) < 2 * TUBE_HALF)
    p = p[~in_tube]
    shell = HUB + _unit(rng, HUB_SHELL) * (0.05 * (1.0 + rng.uniform(-0.005, 0.005, (HUB_SHELL, 1))))
    tube = np.stack([rng.uniform(-1.0, 1.0, 40_000),
                     TUBE_Y + rng.uniform(-TUBE_HALF, TUBE_HALF, 40_000),
                     TUBE_Z + rng.uniform(-TUBE_HALF, TUBE_HALF, 40_000)], 1)
    p = np.concatenate([p, HUB[None], shell, tube]).astype(np.float32)
    _, first = np.unique(p, axis=0, return_index=True)
    p = p[np.sort(first)]
    p = np.ascontiguousarray(p[syn.sort_points_permutation(p)])
    sdf = (syn.spheres_sdf(p.astype(np.float64)) + rng.normal(0, 0.01, p.shape[0])).astype(np.float32)
    attrs = syn.make_attributes(p, sdf, 3, "neus", seed=seed + 1)
    adj, off = syn.delaunay_adjacency(p)
    foam = syn.Foam(p, attrs, adj, off, sdf, 3)
    hub_dir = np.array([1.0, 0.6, 0.3]) / np.linalg.norm([1.0, 0.6, 0.3])
    cams = [syn.look_at((0.8, -2.2, 0.9), fov_deg=45.0, width=64, height=48),
            syn.look_at(HUB + 0.4 * hub_dir, target=HUB, fov_deg=12.0, width=32, height=32),
            syn.look_at((-1.4, TUBE_Y, TUBE_Z), target=(1.0, TUBE_Y, TUBE_Z), up=(0.0, 1.0, 0.0), fov_deg=0.4,
                        width=8, height=8)]
    rays, start = syn.camera_rays(foam, cams, tile=(8, 4))
    return foam, rays, start


@pytest.fixture(scope="module")
def stress():
    return stress_foam()


def _assert_grads(gpu, ref, ref_abs, what):
    a = np.asarray(gpu, np.float64)
    b = np.asarray(ref, np.float64)
    floor = 3e-5 * np.asarray(ref_abs, np.float64) + 1e-7
    bad = np.abs(a - b) > 1e-3 * np.abs(b) + floor
    assert not bad.any(), f"{what}: {bad.sum()} of {bad.size} differ; worst abs {np.abs(a - b)[bad].max()}"


def test_stress_foam_reaches_the_rare_paths(stress):
    foam, rays, start = stress
    deg = np.diff(foam.offsets.astype(np.int64))
    assert deg.max() >= 280, deg.max()
    assert rays.shape[0] == 64 * 48 + 32 * 32 + 64


def test_stress_parity(stress):
    import sdfoam_b200 as sdfoam
    foam, rays, start = stress
    dev = torch.device("cuda:0")
    pipe = sdfoam.create_pipeline(3, "float32")
    pts = torch.from_numpy(foam.points).to(dev)
    att = torch.from_numpy(foam.attributes).to(dev)
    adj = torch.from_numpy(foam.adjacency).to(dev)
    off = torch.from_numpy(foam.offsets).to(dev)
    rr = torch.from_numpy(rays).to(dev)
    ss = torch.from_numpy(start).to(dev)
    inv = torch.tensor([50.0], device=dev)
    R = rays.shape[0]

    # forward with the exit record (zeroed, so unwritten bytes read as 0)
    ex = pipe.exit_record(R, 512, dev)
    ex.zero_()
    n = torch.zeros(R + 1, dtype=torch.int64, device=dev)
    fw0 = pipe.trace_forward(pts, att, adj, off, rr, ss, alpha_mode="sdfoam", inv_s=inv,
                             max_intersections=MAX_STEPS)
    n[1:] = torch.cumsum(fw0["num_intersections"].reshape(-1).to(torch.int64), 0)
    seq = {"offsets": n.to(torch.uint64),
           "cells": torch.full((int(n[-1].item()),), 0xFFFFFFFF, dtype=torch.uint32, device=dev),
           "count": torch.zeros(R, dtype=torch.uint32, device=dev)}
    # the step record covers 256 steps: rays past it replay the exit record,
    # then search, and evaluate their later colours again
    col = pipe.color_record(R, 256, dev)
    sit = pipe.site_record(R, 256, dev)
    fw = pipe.trace_forward(pts, att, adj, off, rr, ss, return_contribution=True, alpha_mode="sdfoam", inv_s=inv,
                            max_intersections=MAX_STEPS, exits=ex, colors=col, sites=sit, _sequences=seq)
    g = np.random.default_rng(11).normal(0, 1, (R, 4)).astype(np.float32)
    gd = torch.from_numpy(g).to(dev)
    bw = pipe.trace_backward(pts, att, adj, off, rr, ss, fw["rgba"], gd, alpha_mode="sdfoam", inv_s=inv,
                             max_intersections=MAX_STEPS, exits=ex, colors=col, sites=sit)
    torch.cuda.synchronize()

    sc = orc.OracleScene(foam.points, foam.attributes, foam.adjacency, foam.offsets, 3)
    st = orc.settings(neus=True, sharpness=50.0, max_intersections=MAX_STEPS)
    rf = orc.trace_forward(sc, st, rays, start, record_sequences=True, ambiguity=True)
    nint = fw["num_intersections"].cpu().numpy().reshape(-1)

    # the walk reached the paths this foam was built for
    assert nint.max() > 600, nint.max()
    codes = ex.cpu().numpy()
    steps = np.minimum(nint.astype(np.int64), 512)
    recorded = np.arange(512)[None, :] < steps[:, None]
    assert (codes[recorded] == 255).sum() > 0, "no exit through face position >= 254 was recorded"

    # bit-exact walk
    assert np.array_equal(nint, rf["num_intersections"])
    gseq = seq["cells"].cpu().numpy()
    gcnt = seq["count"].cpu().numpy()
    assert np.array_equal(gcnt, rf["seq_count"])
    for r in range(R):
        o = int(rf["seq_offsets"][r])
        assert np.array_equal(gseq[o:o + gcnt[r]], rf["seq_cells"][o:o + gcnt[r]]), f"ray {r}: cells differ"
    rgba = fw["rgba"].cpu().numpy()
    assert np.all(np.abs(rgba - rf["rgba"]) <= 1e-4 * np.abs(rf["rgba"]) + 1e-6)
    assert np.all(rf["ambiguous"] == 0)

    # backward replaying the record where it can, searching past 512 steps
    # and after the unknown codes
    rb = orc.trace_backward(sc, st, rays, start, rf["rgba"], g, with_abs=True)
    _assert_grads(bw["attr_grad"].cpu().numpy(), rb["attr_grad"], rb["attr_grad_abs"], "attr_grad")
    _assert_grads(bw["points_grad"].cpu().numpy(), rb["points_grad"], rb["points_grad_abs"], "points_grad")
    sg = float(bw["sharpness_grad"].reshape(-1)[0])
    ref = float(rb["sharpness_grad"][0])
    assert abs(sg - ref) <= 1e-3 * abs(ref) + 1e-4, (sg, ref)
