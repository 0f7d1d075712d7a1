"""Headless render (Pipeline.trace_benchmark, the reference's benchmark kernel
pipeline.cu:1067-1199): the GPU frame through the C ABI against the CPU
restatement (oracle.render), pixel for pixel."""
import math

import numpy as np
import pytest

from oracle import oracle as orc
from sdfoam_b200 import synthetic as syn


def _camera(cam, model="pinhole", width=None, height=None, fov=None):
    return {"position": cam.position, "forward": cam.forward, "right": cam.right, "up": cam.up,
            "fov": float(cam.fov if fov is None else fov), "width": int(width or cam.width),
            "height": int(height or cam.height), "model": model}


def _unpack(img):
    img = np.asarray(img, np.uint32)
    return np.stack([(img >> s) & 255 for s in (0, 8, 16, 24)], -1).astype(np.int32)


def test_oracle_render_matches_forward(mini_foam):
    """The render driver (ray per pixel, bottom-up rows, background, RGBA8
    packing) agrees with the forward walk of the same pinhole rays."""
    foam, _, _ = mini_foam
    cam = syn.look_at((2.2, 1.1, 0.7), fov_deg=40.0, width=24, height=20)
    sc = orc.OracleScene(foam.points, foam.attributes, foam.adjacency, foam.offsets, 3)
    st = orc.settings(neus=True, sharpness=50.0, weight_threshold=0.05)
    start = int(syn.nearest_site(foam.points, cam.position[None, :])[0])
    img = orc.render(sc, st, _camera(cam), start)
    rays = syn.pinhole_rays(cam, tile=None)  # row-major: ray j * W + i
    fwd = orc.trace_forward(sc, st, rays, np.full(rays.shape[0], start, np.uint32), return_contribution=False)
    rgba = fwd["rgba"]
    T = 1.0 - rgba[:, 3]
    col = np.clip(rgba[:, :3] + T[:, None], 0.0, 1.0)
    expect = (col * 255.0).astype(np.int32)
    W, H = cam.width, cam.height
    got = _unpack(img).reshape(H, W, 4)[::-1].reshape(-1, 4)  # back to top-down rows
    assert np.all(got[:, 3] == 255)
    close = np.abs(got[:, :3] - expect).max(axis=1) <= 1
    assert close.mean() > 0.98
    # the walks are not all empty: some pixels are darker than the white background
    assert (got[:, :3] < 250).any()


def _density(attributes):
    """Standard (RadFoam) mode reads the last channel as a density."""
    a = attributes.copy()
    a[:, -1] = np.abs(a[:, -1]) * 5.0
    return a


def _gpu_scene(foam, pipe_dtype="float32", attributes=None):
    import torch
    import sdfoam_b200 as sdfoam
    dev = torch.device("cuda:0")
    pipe = sdfoam.create_pipeline(3, pipe_dtype)
    dt = torch.float16 if pipe_dtype == "float16" else torch.float32
    pts = torch.from_numpy(foam.points).to(dev)
    att = torch.from_numpy(foam.attributes if attributes is None else attributes).to(dev, dt)
    adj = torch.from_numpy(foam.adjacency.astype(np.uint32)).to(dev)
    off = torch.from_numpy(foam.offsets.astype(np.uint32)).to(dev)
    return pipe, pts, att, adj, off


def _diffs_like_benchmark_py(pts, adj, off):
    """adjacent_offsets as the reference's benchmark.py:41-51 builds them."""
    import torch
    self_idx = torch.zeros_like(adj.long())
    scatter = off[1:-1].long()
    self_idx.scatter_add_(0, scatter, torch.ones_like(scatter))
    self_idx = torch.cumsum(self_idx, dim=0)
    d = pts[adj.long()] - pts[self_idx]
    return torch.cat([d, torch.zeros_like(d[:, :1])], dim=1).to(torch.half)


@pytest.mark.gpu
@pytest.mark.parametrize("mode", ["sdfoam", "standard"])
def test_render_pinhole_bit_exact(tiny_foam, mode):
    import torch
    foam, _, _ = tiny_foam
    neus = mode == "sdfoam"
    attrs = foam.attributes if neus else _density(foam.attributes)
    pipe, pts, att, adj, off = _gpu_scene(foam, attributes=attrs)
    cam = syn.views("tiny")[0]
    start_i = int(syn.nearest_site(foam.points, cam.position[None, :])[0])
    sc = orc.OracleScene(foam.points, attrs, foam.adjacency, foam.offsets, 3)
    diffs = torch.from_numpy(sc.diffs.view(np.float16)).cuda()
    start = torch.tensor([start_i], dtype=torch.uint32, device="cuda")
    out = torch.zeros((cam.height, cam.width), dtype=torch.uint32, device="cuda")
    kw = {"weight_threshold": 0.05}
    if neus:
        kw.update(alpha_mode="sdfoam", inv_s=torch.tensor(50.0))
    pipe.trace_benchmark(pts, att, adj, off, diffs, _camera(cam), start, out, **kw)
    st = orc.settings(neus=neus, sharpness=50.0, weight_threshold=0.05)
    ref = orc.render(sc, st, _camera(cam), start_i)
    got = out.cpu().numpy().reshape(-1)
    assert np.array_equal(got, ref), f"{(got != ref).sum()} of {got.size} pixels differ"
    assert len(np.unique(got)) > 50  # a real image, not a flat background


@pytest.mark.gpu
def test_render_background_options_and_fisheye(tiny_foam):
    import torch
    foam, _, _ = tiny_foam
    pipe, pts, att, adj, off = _gpu_scene(foam)
    cam = syn.views("tiny")[0]
    start_i = int(syn.nearest_site(foam.points, cam.position[None, :])[0])
    sc = orc.OracleScene(foam.points, foam.attributes, foam.adjacency, foam.offsets, 3)
    diffs = torch.from_numpy(sc.diffs.view(np.float16)).cuda()
    start = torch.tensor([start_i], dtype=torch.uint32, device="cuda")
    st = orc.settings(neus=True, sharpness=50.0, weight_threshold=0.05)
    kw = {"weight_threshold": 0.05, "alpha_mode": "sdfoam", "inv_s": torch.tensor(50.0)}
    # checkerboard and a coloured background, non-square frame
    c = _camera(cam, width=100, height=60)
    out = torch.zeros(60 * 100, dtype=torch.uint32, device="cuda")
    pipe.trace_benchmark(pts, att, adj, off, diffs, c, start, out, checker_bg=True, **kw)
    assert np.array_equal(out.cpu().numpy(), orc.render(sc, st, c, start_i, checker_bg=True))
    pipe.trace_benchmark(pts, att, adj, off, diffs, c, start, out, bg_color=(0.2, 0.4, 0.9), **kw)
    assert np.array_equal(out.cpu().numpy(), orc.render(sc, st, c, start_i, bg_color=(0.2, 0.4, 0.9)))
    # fisheye: atan2 / sin / cos are the platform's on each side, so a few
    # pixels may take a different walk; pixels outside the lens are background
    c = _camera(cam, model="fisheye", width=64, height=64, fov=1.4)
    out = torch.zeros(64 * 64, dtype=torch.uint32, device="cuda")
    pipe.trace_benchmark(pts, att, adj, off, diffs, c, start, out, **kw)
    got, ref = _unpack(out.cpu().numpy()), _unpack(orc.render(sc, st, c, start_i))
    diff = np.abs(got - ref).max(axis=1)
    assert (diff <= 1).mean() > 0.97
    u = (2.0 * np.arange(64) / 64 - 1.0)
    outside = np.hypot(u[None, :], (1.0 - 2.0 * np.arange(64) / 64)[::-1, None]) * 1.4 >= math.pi + 1e-3
    assert np.all(got.reshape(64, 64, 4)[outside][:, :3] == 255)


@pytest.mark.gpu
def test_render_float16_pipeline_and_cache(tiny_foam):
    import torch
    foam, _, _ = tiny_foam
    attrs = _density(foam.attributes)
    pipe, pts, att, adj, off = _gpu_scene(foam, "float16", attributes=attrs)
    cam = syn.views("tiny")[0]
    start_i = int(syn.nearest_site(foam.points, cam.position[None, :])[0])
    att16 = attrs.astype(np.float16).astype(np.float32)
    sc = orc.OracleScene(foam.points, att16, foam.adjacency, foam.offsets, 3)
    diffs = _diffs_like_benchmark_py(pts, adj, off)
    # benchmark.py's torch diffs are the reference prefetch's bits
    assert np.array_equal(diffs.view(torch.int16).cpu().numpy().view(np.uint16), sc.diffs)
    start = torch.tensor([start_i], dtype=torch.uint32, device="cuda")
    out = torch.zeros(cam.height * cam.width, dtype=torch.uint32, device="cuda")
    st = orc.settings(neus=False, weight_threshold=0.05)
    pipe.trace_benchmark(pts, att, adj, off, diffs, _camera(cam), start, out, weight_threshold=0.05)
    assert np.array_equal(out.cpu().numpy(), orc.render(sc, st, _camera(cam), start_i))
    # an in-place update of the attributes rebuilds the cached cell records
    att.mul_(0.5)
    pipe.trace_benchmark(pts, att, adj, off, diffs, _camera(cam), start, out, weight_threshold=0.05)
    sc2 = orc.OracleScene(foam.points, (att16 * np.float32(0.5)).astype(np.float16).astype(np.float32),
                          foam.adjacency, foam.offsets, 3)
    assert np.array_equal(out.cpu().numpy(), orc.render(sc2, st, _camera(cam), start_i))


@pytest.mark.gpu
def test_render_errors(mini_foam):
    import torch
    foam, _, _ = mini_foam
    pipe, pts, att, adj, off = _gpu_scene(foam)
    cam = syn.look_at((2.2, 1.1, 0.7), width=8, height=8)
    diffs = torch.zeros((adj.numel(), 4), dtype=torch.half, device="cuda")
    start = torch.zeros(1, dtype=torch.uint32, device="cuda")
    out = torch.zeros(64, dtype=torch.uint32, device="cuda")
    with pytest.raises(RuntimeError, match="Invalid camera model"):
        pipe.trace_benchmark(pts, att, adj, off, diffs, _camera(cam, model="ortho"), start, out)
    with pytest.raises(RuntimeError, match="start_point must have a single element"):
        pipe.trace_benchmark(pts, att, adj, off, diffs, _camera(cam), start.repeat(2), out)
    with pytest.raises(RuntimeError, match="output_rgba must have width \\* height elements"):
        pipe.trace_benchmark(pts, att, adj, off, diffs, _camera(cam), start, out[:10])
    with pytest.raises(RuntimeError, match="output_rgba must have uint32 dtype"):
        pipe.trace_benchmark(pts, att, adj, off, diffs, _camera(cam), start, out.float())
