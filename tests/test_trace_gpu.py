"""GPU parity: libsdfoam_b200.so (through its C ABI) against the CPU oracle.

Contract (cell walk of src/tracing/tracing_utils.cuh:17-109 with the functors
of src/tracing/pipeline.cu:36-791):
  * bit-exact: per-ray cell sequences, num_intersections, depth_indices;
  * rgba / depth within 1e-4 relative (absolute floor 1e-6);
  * gradients within 1e-3 relative, with an absolute floor proportional to
    the sum of |terms| accumulated into that entry (float atomics sum in an
    unspecified order on both sides);
  * alpha[N]: the reference's store is last-writer-wins, so each site's value
    must be the alpha of one of that site's visits.
"""
import numpy as np
import pytest
import torch

from oracle import oracle as orc
from sdfoam_b200 import synthetic as syn

pytestmark = pytest.mark.gpu

RTOL_FWD = 1e-4
RTOL_GRAD = 1e-3


@pytest.fixture(scope="module")
def sdfoam():
    import sdfoam_b200
    return sdfoam_b200


def dev_tensors(foam, rays, start, attrs=None):
    d = torch.device("cuda:0")
    return (torch.from_numpy(foam.points).to(d),
            torch.from_numpy(foam.attributes if attrs is None else attrs).to(d),
            torch.from_numpy(foam.adjacency).to(d),
            torch.from_numpy(foam.offsets).to(d),
            torch.from_numpy(rays).to(d),
            torch.from_numpy(start).to(d))


def gpu_forward(pipe, T, with_seq=False, **kw):
    pts, att, adj, off, rays, start = T
    seq = None
    if with_seq:
        first = pipe.trace_forward(pts, att, adj, off, rays, start, **kw)
        n = first["num_intersections"].reshape(-1).to(torch.int64)
        offs = torch.zeros(n.numel() + 1, dtype=torch.int64, device=n.device)
        offs[1:] = torch.cumsum(n, 0)
        seq = {"offsets": offs.to(torch.uint64),
               "cells": torch.full((int(offs[-1].item()),), 0xFFFFFFFF, dtype=torch.uint32, device=n.device),
               "count": torch.zeros(n.numel(), dtype=torch.uint32, device=n.device)}
    out = pipe.trace_forward(pts, att, adj, off, rays, start, _sequences=seq, **kw)
    torch.cuda.synchronize()
    res = {k: v.cpu().numpy() for k, v in out.items()}
    if seq is not None:
        res["seq_offsets"] = seq["offsets"].cpu().numpy()
        res["seq_cells"] = seq["cells"].cpu().numpy()
        res["seq_count"] = seq["count"].cpu().numpy()
    return res


def assert_close(a, b, rtol, atol, what):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    bad = np.abs(a - b) > rtol * np.abs(b) + atol
    assert not bad.any(), f"{what}: {bad.sum()} of {bad.size} differ; worst {np.abs(a - b)[bad].max()}"


def assert_grads(gpu, ref, ref_abs, what):
    a = np.asarray(gpu, np.float64)
    b = np.asarray(ref, np.float64)
    floor = 3e-5 * np.asarray(ref_abs, np.float64) + 1e-7
    bad = np.abs(a - b) > RTOL_GRAD * np.abs(b) + floor
    assert not bad.any(), f"{what}: {bad.sum()} of {bad.size} differ; worst abs {np.abs(a - b)[bad].max()}"


def check_alpha_sets(gpu_alpha, ref):
    """Each site's GPU alpha equals the alpha of one of the site's visits."""
    cells = np.concatenate([ref["seq_cells"][ref["seq_offsets"][r]:ref["seq_offsets"][r] + ref["seq_count"][r]]
                            for r in range(ref["seq_count"].shape[0])])
    alphas = np.concatenate([ref["seq_alpha"][ref["seq_offsets"][r]:ref["seq_offsets"][r] + ref["seq_count"][r]]
                             for r in range(ref["seq_count"].shape[0])])
    ga = gpu_alpha.reshape(-1)
    visited = np.zeros(ga.shape[0], bool)
    visited[cells] = True
    assert np.all(ga[~visited] == 0.0)
    key = cells.astype(np.uint64) << np.uint64(32) | alphas.view(np.uint32).astype(np.uint64)
    want = np.unique(key)
    got = np.nonzero(visited)[0].astype(np.uint64) << np.uint64(32) | ga[visited].view(np.uint32).astype(np.uint64)
    assert np.isin(got, want).all()


def seq_equal(g, r):
    assert np.array_equal(g["seq_count"], r["seq_count"])
    for k in range(g["seq_count"].shape[0]):
        a = g["seq_cells"][g["seq_offsets"][k]:g["seq_offsets"][k] + g["seq_count"][k]]
        b = r["seq_cells"][r["seq_offsets"][k]:r["seq_offsets"][k] + r["seq_count"][k]]
        if not np.array_equal(a, b):
            raise AssertionError(f"ray {k}: cell sequences differ")


def _oracle(foam, attrs=None):
    return orc.OracleScene(foam.points, foam.attributes if attrs is None else attrs, foam.adjacency, foam.offsets,
                           foam.sh_degree)


@pytest.mark.parametrize("neus", [True, False])
def test_forward_parity_tiny(sdfoam, tiny_foam, neus):
    foam, rays, start = tiny_foam
    attrs = foam.attributes
    if not neus:
        attrs = syn.make_attributes(foam.points, foam.sdf, 3, "standard", seed=7)
    pipe = sdfoam.create_pipeline(3, "float32")
    T = dev_tensors(foam, rays, start, attrs)
    inv_s = torch.tensor([50.0], device="cuda:0")
    mode = "sdfoam" if neus else "standard"
    g = gpu_forward(pipe, T, with_seq=True, return_contribution=True, alpha_mode=mode, inv_s=inv_s)
    sc = _oracle(foam, attrs)
    st = orc.settings(neus=neus, sharpness=50.0 if neus else 1.0)
    r = orc.trace_forward(sc, st, rays, start, record_sequences=True)
    assert np.array_equal(g["num_intersections"].reshape(-1), r["num_intersections"])
    seq_equal(g, r)
    assert_close(g["rgba"], r["rgba"], RTOL_FWD, 1e-6, "rgba")
    exact = np.mean(g["rgba"].view(np.uint32) == r["rgba"].view(np.uint32))
    assert exact > 0.99, f"bit-identical rgba fraction {exact}"
    assert_close(g["contribution"].reshape(-1), r["contribution"], 1e-4, 1e-6, "contribution")
    check_alpha_sets(g["alpha"], r)


@pytest.mark.parametrize("neus", [True, False])
def test_backward_parity_tiny(sdfoam, tiny_foam, neus):
    foam, rays, start = tiny_foam
    attrs = foam.attributes
    if not neus:
        attrs = syn.make_attributes(foam.points, foam.sdf, 3, "standard", seed=7)
    pipe = sdfoam.create_pipeline(3, "float32")
    T = dev_tensors(foam, rays, start, attrs)
    pts, att, adj, off, rr, ss = T
    inv_s = torch.full((pts.shape[0], 1), 50.0, device="cuda:0")  # training passes [N,1]
    mode = "sdfoam" if neus else "standard"
    fw = pipe.trace_forward(pts, att, adj, off, rr, ss, alpha_mode=mode, inv_s=inv_s)
    grad = np.random.default_rng(3).normal(0, 1, (rays.shape[0], 4)).astype(np.float32)
    bw = pipe.trace_backward(pts, att, adj, off, rr, ss, fw["rgba"], torch.from_numpy(grad).cuda(),
                             alpha_mode=mode, inv_s=inv_s)
    torch.cuda.synchronize()
    sc = _oracle(foam, attrs)
    st = orc.settings(neus=neus, sharpness=50.0 if neus else 1.0)
    rf = orc.trace_forward(sc, st, rays, start)
    assert np.array_equal(fw["num_intersections"].cpu().numpy().reshape(-1), rf["num_intersections"])
    rb = orc.trace_backward(sc, st, rays, start, rf["rgba"], grad, with_abs=True)
    assert_grads(bw["attr_grad"].cpu().numpy(), rb["attr_grad"], rb["attr_grad_abs"], "attr_grad")
    assert_grads(bw["points_grad"].cpu().numpy(), rb["points_grad"], rb["points_grad_abs"], "points_grad")
    assert bw["sharpness_grad"].shape == inv_s.shape
    if neus:
        sg = float(bw["sharpness_grad"].reshape(-1)[0])
        ref = float(rb["sharpness_grad"][0])
        assert abs(sg - ref) <= RTOL_GRAD * abs(ref) + 1e-4, (sg, ref)
        assert torch.all(bw["sharpness_grad"].reshape(-1)[1:] == 0)


@pytest.mark.parametrize("deg", [0, 1, 2])
def test_lower_sh_degrees(sdfoam, mini_foam, deg):
    foam, rays, start = mini_foam
    attrs = syn.make_attributes(foam.points, foam.sdf, deg, "neus", seed=5)
    sub = syn.Foam(foam.points, attrs, foam.adjacency, foam.offsets, foam.sdf, deg)
    pipe = sdfoam.create_pipeline(deg)
    T = dev_tensors(sub, rays, start)
    inv_s = torch.tensor([30.0], device="cuda:0")
    g = gpu_forward(pipe, T, return_contribution=True, alpha_mode="sdfoam", inv_s=inv_s)
    sc = _oracle(sub)
    st = orc.settings(neus=True, sharpness=30.0, attr_dim=attrs.shape[1])
    r = orc.trace_forward(sc, st, rays, start)
    assert np.array_equal(g["num_intersections"].reshape(-1), r["num_intersections"])
    assert_close(g["rgba"], r["rgba"], RTOL_FWD, 1e-6, "rgba")
    grad = np.random.default_rng(deg).normal(0, 1, (rays.shape[0], 4)).astype(np.float32)
    pts, att, adj, off, rr, ss = T
    fw = pipe.trace_forward(pts, att, adj, off, rr, ss, alpha_mode="sdfoam", inv_s=inv_s)
    bw = pipe.trace_backward(pts, att, adj, off, rr, ss, fw["rgba"], torch.from_numpy(grad).cuda(),
                             alpha_mode="sdfoam", inv_s=inv_s)
    rb = orc.trace_backward(sc, st, rays, start, r["rgba"], grad, with_abs=True)
    assert_grads(bw["attr_grad"].cpu().numpy(), rb["attr_grad"], rb["attr_grad_abs"], "attr_grad")
    assert_grads(bw["points_grad"].cpu().numpy(), rb["points_grad"], rb["points_grad_abs"], "points_grad")


@pytest.mark.parametrize("neus", [True, False])
def test_depth_quantiles(sdfoam, tiny_foam, neus):
    foam, rays, start = tiny_foam
    attrs = foam.attributes if neus else syn.make_attributes(foam.points, foam.sdf, 3, "standard", seed=7)
    rng = np.random.default_rng(9)
    # train.py:259-261 draws two random quantiles per ray, sorted descending
    q = np.sort(rng.uniform(0, 1, (rays.shape[0], 2)).astype(np.float32), axis=1)[:, ::-1].copy()
    pipe = sdfoam.create_pipeline(3)
    T = dev_tensors(foam, rays, start, attrs)
    pts, att, adj, off, rr, ss = T
    mode = "sdfoam" if neus else "standard"
    inv_s = torch.tensor([50.0], device="cuda:0")
    dq = torch.from_numpy(q).cuda()
    fw = pipe.trace_forward(pts, att, adj, off, rr, ss, depth_quantiles=dq, alpha_mode=mode, inv_s=inv_s)
    sc = _oracle(foam, attrs)
    st = orc.settings(neus=neus, sharpness=50.0 if neus else 1.0)
    rf = orc.trace_forward(sc, st, rays, start, quantiles=q)
    assert np.array_equal(fw["depth_indices"].cpu().numpy(), rf["depth_indices"])
    assert_close(fw["depth"].cpu().numpy(), rf["depth"], RTOL_FWD, 1e-6, "depth")
    grad = rng.normal(0, 1, (rays.shape[0], 4)).astype(np.float32)
    dgrad = rng.normal(0, 1, (rays.shape[0], 2)).astype(np.float32)
    bw = pipe.trace_backward(pts, att, adj, off, rr, ss, fw["rgba"], torch.from_numpy(grad).cuda(),
                             depth_quantiles=dq, depth_indices=fw["depth_indices"],
                             depth_grad_in=torch.from_numpy(dgrad).cuda(), alpha_mode=mode, inv_s=inv_s)
    rb = orc.trace_backward(sc, st, rays, start, rf["rgba"], grad, quantiles=q, depth_indices=rf["depth_indices"],
                            depth_grad=dgrad, with_abs=True)
    assert_grads(bw["attr_grad"].cpu().numpy(), rb["attr_grad"], rb["attr_grad_abs"], "attr_grad")
    assert_grads(bw["points_grad"].cpu().numpy(), rb["points_grad"], rb["points_grad_abs"], "points_grad")


def test_ray_error_point_error(sdfoam, mini_foam):
    foam, rays, start = mini_foam
    pipe = sdfoam.create_pipeline(3)
    T = dev_tensors(foam, rays, start)
    pts, att, adj, off, rr, ss = T
    inv_s = torch.tensor([50.0], device="cuda:0")
    fw = pipe.trace_forward(pts, att, adj, off, rr, ss, alpha_mode="sdfoam", inv_s=inv_s)
    err = np.random.default_rng(2).uniform(0, 1, rays.shape[0]).astype(np.float32)
    grad = np.zeros((rays.shape[0], 4), np.float32)
    bw = pipe.trace_backward(pts, att, adj, off, rr, ss, fw["rgba"], torch.from_numpy(grad).cuda(),
                             ray_error=torch.from_numpy(err).cuda(), alpha_mode="sdfoam", inv_s=inv_s)
    sc = _oracle(foam)
    st = orc.settings(neus=True, sharpness=50.0)
    rf = orc.trace_forward(sc, st, rays, start)
    rb = orc.trace_backward(sc, st, rays, start, rf["rgba"], grad, ray_error=err)
    assert bw["point_error"].shape == (foam.points.shape[0], 1)
    assert_close(bw["point_error"].cpu().numpy().reshape(-1), rb["point_error"], 1e-4, 1e-6, "point_error")


def test_edge_cases(sdfoam, mini_foam):
    foam, rays, start = mini_foam
    pipe = sdfoam.create_pipeline(3)
    pts, att, adj, off, rr, ss = dev_tensors(foam, rays, start)
    inv_s = torch.tensor([50.0], device="cuda:0")
    # no rays
    out = pipe.trace_forward(pts, att, adj, off, rr[:0], ss[:0], alpha_mode="sdfoam", inv_s=inv_s)
    assert out["rgba"].shape == (0, 4) and out["num_intersections"].shape == (0, 1)
    # start site out of range: no walk (n = 0, transparent)
    bad = ss.clone()
    bad[:5] = foam.points.shape[0] + 7
    out = pipe.trace_forward(pts, att, adj, off, rr, bad, alpha_mode="sdfoam", inv_s=inv_s)
    torch.cuda.synchronize()
    assert torch.all(out["num_intersections"][:5] == 0)
    assert torch.all(out["rgba"][:5] == 0)
    # max_intersections cap: n = cap + 1 for rays that reach it
    out = pipe.trace_forward(pts, att, adj, off, rr, ss, max_intersections=3, alpha_mode="sdfoam", inv_s=inv_s)
    sc = _oracle(foam)
    st = orc.settings(neus=True, sharpness=50.0, max_intersections=3)
    r = orc.trace_forward(sc, st, rays, start)
    assert np.array_equal(out["num_intersections"].cpu().numpy().reshape(-1), r["num_intersections"])
    assert r["num_intersections"].max() == 4
    # batched ray shapes keep their leading dims
    out = pipe.trace_forward(pts, att, adj, off, rr.reshape(24, 24, 6), ss.reshape(24, 24), alpha_mode="sdfoam",
                             inv_s=inv_s)
    assert out["rgba"].shape == (24, 24, 4) and out["num_intersections"].shape == (24, 24, 1)


def test_reference_error_messages(sdfoam, mini_foam):
    foam, rays, start = mini_foam
    pipe = sdfoam.create_pipeline(3)
    pts, att, adj, off, rr, ss = dev_tensors(foam, rays, start)
    with pytest.raises(RuntimeError, match="rays must have 6 as the last dimension"):
        pipe.trace_forward(pts, att, adj, off, rr[:, :5], ss)
    with pytest.raises(RuntimeError, match="start_point must have uint32 dtype"):
        pipe.trace_forward(pts, att, adj, off, rr, ss.to(torch.int64))
    with pytest.raises(RuntimeError, match="attributes had dimension 48 along axis -1, expected 49"):
        pipe.trace_forward(pts, att[:, :48], adj, off, rr, ss)
    with pytest.raises(RuntimeError, match="point_adjacency_offsets must have num_points"):
        pipe.trace_forward(pts, att, adj, off[:-1], rr, ss)
    fw = pipe.trace_forward(pts, att, adj, off, rr, ss, depth_quantiles=torch.full((rr.shape[0], 1), 0.5,
                                                                                 device="cuda:0"))
    with pytest.raises(RuntimeError, match="depth_grad must be provided if depth_quantiles is provided"):
        pipe.trace_backward(pts, att, adj, off, rr, ss, fw["rgba"], torch.zeros_like(fw["rgba"]),
                            depth_quantiles=torch.full((rr.shape[0], 1), 0.5, device="cuda:0"),
                            depth_indices=fw["depth_indices"])
    with pytest.raises(RuntimeError, match="Unsupported SH degree"):
        sdfoam.create_pipeline(4)
    with pytest.raises(RuntimeError, match="Unsupported attribute type"):
        sdfoam.create_pipeline(3, "float64")


def test_trace_rays_autograd(sdfoam, mini_foam):
    from sdfoam_b200.render import TraceRays
    foam, rays, start = mini_foam
    pipe = sdfoam.create_pipeline(3)
    pts, att, adj, off, rr, ss = dev_tensors(foam, rays, start)
    pts = pts.clone().requires_grad_(True)
    att = att.clone().requires_grad_(True)
    inv_s = torch.full((pts.shape[0], 1), 50.0, device="cuda:0", requires_grad=True)
    rgba, depth, contrib, nint, errbox, alpha = TraceRays.apply(pipe, pts, att, adj, off, rr, ss, None, True, True,
                                                               inv_s, 1e-6, att.shape[-1] - 1)
    g = torch.randn_like(rgba)
    (rgba * g).sum().backward()
    direct = pipe.trace_backward(pts.detach(), att.detach(), adj, off, rr, ss, rgba.detach(), g,
                                 alpha_mode="sdfoam", inv_s=inv_s.detach(), sdf_channel=48)
    torch.cuda.synchronize()
    assert torch.allclose(att.grad, direct["attr_grad"], rtol=1e-3, atol=1e-5)
    assert torch.allclose(pts.grad, direct["points_grad"], rtol=1e-3, atol=1e-4)
    assert inv_s.grad.shape == inv_s.shape
    assert contrib.shape == (pts.shape[0], 1) and alpha.shape == (pts.shape[0], 1)


def test_float16_pipeline(sdfoam, mini_foam):
    """float16 attributes (create_pipeline(deg, "float16"), used by the
    reference's benchmark.py and extract_mesh.py).  As in the reference, the
    NeuS sharpness is the first two bytes of the float32 inv_s buffer read as
    binary16: 0x42485640 (= 50.08 as float32) is read as 0x5640 = 100.0."""
    foam, rays, start = mini_foam
    att16 = foam.attributes.astype(np.float16)
    inv_bits = np.array([0x42485640], np.uint32)
    inv = torch.from_numpy(inv_bits.view(np.float32)).cuda()
    pipe = sdfoam.create_pipeline(3, "float16")
    pts, _, adj, off, rr, ss = dev_tensors(foam, rays, start)
    att = torch.from_numpy(att16).cuda()
    fw = pipe.trace_forward(pts, att, adj, off, rr, ss, return_contribution=True, alpha_mode="sdfoam", inv_s=inv)
    assert fw["rgba"].dtype == torch.float16 and fw["contribution"].dtype == torch.float16
    sc = _oracle(foam, att16.astype(np.float32))
    st = orc.settings(neus=True, sharpness=100.0)
    rf = orc.trace_forward(sc, st, rays, start)
    assert np.array_equal(fw["num_intersections"].cpu().numpy().reshape(-1), rf["num_intersections"])
    assert np.array_equal(fw["rgba"].cpu().numpy(), rf["rgba"].astype(np.float16))
    con = fw["contribution"].cpu().numpy().reshape(-1).astype(np.float32)
    assert np.all(np.abs(con - rf["contribution"]) <= 1e-2 * np.abs(rf["contribution"]) + 1e-3)
    grad = np.random.default_rng(4).normal(0, 1, (rays.shape[0], 4)).astype(np.float16)
    bw = pipe.trace_backward(pts, att, adj, off, rr, ss, fw["rgba"], torch.from_numpy(grad).cuda(),
                             alpha_mode="sdfoam", inv_s=inv)
    assert bw["attr_grad"].dtype == torch.float16 and bw["points_grad"].dtype == torch.float32
    rb = orc.trace_backward(sc, st, rays, start, fw["rgba"].cpu().numpy().astype(np.float32),
                            grad.astype(np.float32), with_abs=True)
    ga = bw["attr_grad"].cpu().numpy().astype(np.float64)
    floor = 3e-5 * rb["attr_grad_abs"] + 1e-6
    assert np.all(np.abs(ga - rb["attr_grad"]) <= 1e-3 * np.abs(rb["attr_grad"]) + floor + 1e-3 * np.abs(ga))
    assert_grads(bw["points_grad"].cpu().numpy(), rb["points_grad"], rb["points_grad_abs"], "points_grad")
    # inv_s = 50.0 (0x42480000) has zero low bits: the reference's float16
    # kernels see a sharpness of 0, so nothing is opaque
    fz = pipe.trace_forward(pts, att, adj, off, rr, ss, alpha_mode="sdfoam",
                            inv_s=torch.tensor([50.0], device="cuda:0"))
    assert torch.all(fz["rgba"][:, 3] == 0)


@pytest.mark.gpu
@pytest.mark.parametrize("steps", [8, 64, 1024])
def test_backward_replaying_exit_record_matches_search(tiny_foam, steps):
    """The NeuS backward that replays the forward's exit record takes the same
    steps as the one that searches: same gradients (up to the order of the
    atomic sums), whether the record covers all steps or only the first few."""
    import torch
    import sdfoam_b200 as sdfoam
    foam, rays, start = tiny_foam
    dev = torch.device("cuda:0")
    pipe = sdfoam.create_pipeline(3)
    pts = torch.from_numpy(foam.points).to(dev)
    att = torch.from_numpy(foam.attributes).to(dev)
    adj = torch.from_numpy(foam.adjacency).to(dev)
    off = torch.from_numpy(foam.offsets).to(dev)
    rr = torch.from_numpy(rays).to(dev)
    ss = torch.from_numpy(start).to(dev)
    inv = torch.tensor([50.0], device=dev)
    g = torch.from_numpy(np.random.default_rng(1).normal(0, 1, (rr.shape[0], 4)).astype(np.float32)).to(dev)
    ex = pipe.exit_record(rr.shape[0], steps, dev)
    fw = pipe.trace_forward(pts, att, adj, off, rr, ss, alpha_mode="sdfoam", inv_s=inv, exits=ex)
    fw0 = pipe.trace_forward(pts, att, adj, off, rr, ss, alpha_mode="sdfoam", inv_s=inv)
    assert torch.equal(fw["rgba"], fw0["rgba"]) and torch.equal(fw["num_intersections"], fw0["num_intersections"])
    a = pipe.trace_backward(pts, att, adj, off, rr, ss, fw["rgba"], g, alpha_mode="sdfoam", inv_s=inv, exits=ex)
    b = pipe.trace_backward(pts, att, adj, off, rr, ss, fw["rgba"], g, alpha_mode="sdfoam", inv_s=inv)
    for k in ("attr_grad", "points_grad", "sharpness_grad"):
        x, y = a[k].double(), b[k].double()
        assert torch.allclose(x, y, rtol=1e-4, atol=1e-6 * y.abs().max().item()), k


@pytest.mark.gpu
@pytest.mark.parametrize("steps", [16, 256])
@pytest.mark.parametrize("with_sites", [False, True])
def test_backward_reading_the_step_record_matches(tiny_foam, steps, with_sites):
    """The NeuS backward that reads the forward's step record (step-major:
    each step's colour and exit distance, and with the site record the site
    it entered) instead of testing exit faces and gathering and evaluating
    each site's SH row: the same gradients up to the order of the atomic
    sums, whether the record covers every step or only the first ones; the
    forward's outputs do not change when it writes the record."""
    import sdfoam_b200 as sdfoam
    foam, rays, start = tiny_foam
    dev = torch.device("cuda:0")
    pipe = sdfoam.create_pipeline(3)
    pts = torch.from_numpy(foam.points).to(dev)
    att = torch.from_numpy(foam.attributes).to(dev)
    adj = torch.from_numpy(foam.adjacency).to(dev)
    off = torch.from_numpy(foam.offsets).to(dev)
    rr = torch.from_numpy(rays).to(dev)
    ss = torch.from_numpy(start).to(dev)
    inv = torch.tensor([50.0], device=dev)
    g = torch.from_numpy(np.random.default_rng(2).normal(0, 1, (rr.shape[0], 4)).astype(np.float32)).to(dev)
    ex = pipe.exit_record(rr.shape[0], 512, dev)
    col = pipe.color_record(rr.shape[0], steps, dev)
    sit = pipe.site_record(rr.shape[0], steps, dev) if with_sites else None
    fw = pipe.trace_forward(pts, att, adj, off, rr, ss, alpha_mode="sdfoam", inv_s=inv, exits=ex, colors=col,
                            sites=sit)
    fw0 = pipe.trace_forward(pts, att, adj, off, rr, ss, alpha_mode="sdfoam", inv_s=inv)
    assert torch.equal(fw["rgba"], fw0["rgba"]) and torch.equal(fw["num_intersections"], fw0["num_intersections"])
    a = pipe.trace_backward(pts, att, adj, off, rr, ss, fw["rgba"], g, alpha_mode="sdfoam", inv_s=inv, exits=ex,
                            colors=col, sites=sit)
    b = pipe.trace_backward(pts, att, adj, off, rr, ss, fw["rgba"], g, alpha_mode="sdfoam", inv_s=inv, exits=ex)
    for k in ("attr_grad", "points_grad", "sharpness_grad"):
        x, y = a[k].double(), b[k].double()
        assert torch.allclose(x, y, rtol=1e-4, atol=1e-6 * y.abs().max().item()), k
    with pytest.raises(RuntimeError, match="colors must be"):
        pipe.trace_forward(pts, att, adj, off, rr, ss, alpha_mode="sdfoam", inv_s=inv, colors=col[:, :5])
    with pytest.raises(RuntimeError, match="sites must be"):
        pipe.trace_forward(pts, att, adj, off, rr, ss, alpha_mode="sdfoam", inv_s=inv, colors=col,
                           sites=pipe.site_record(rr.shape[0], steps + 1, dev))
