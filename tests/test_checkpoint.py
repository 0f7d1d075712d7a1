"""model.pt / scene.ply in the reference's formats (SDFoamScene.save_pt /
load_pt / save_ply, sdfoam_model/scene.py:679-823): round trips, the
'module.' prefix of wrapped state dicts, the SH-width check, the trace
attributes of a loaded scene, and the PLY layout."""
import numpy as np
import pytest
import torch

from sdfoam_b200 import checkpoint as ck
from sdfoam_b200.sdfnet import SDFNetwork, SingleVarianceNetwork


def _scene(n=300, sh_degree=3, seed=0):
    rng = np.random.default_rng(seed)
    pts = torch.from_numpy(rng.uniform(-1, 1, (n, 3)).astype(np.float32))
    deg = rng.integers(3, 9, n)
    off = np.concatenate([[0], np.cumsum(deg)]).astype(np.int64)
    adj = rng.integers(0, n, off[-1]).astype(np.int64)
    k = 3 * ((sh_degree + 1) ** 2 - 1)
    net = SDFNetwork(point_cloud=pts, generator=torch.Generator().manual_seed(1))
    var = SingleVarianceNetwork(0.3)
    return ck.SceneCheckpoint(
        points=pts, color_dc=torch.from_numpy(rng.normal(0, 1, (n, 3)).astype(np.float32)),
        color_sh=torch.from_numpy(rng.normal(0, 0.1, (n, k)).astype(np.float32)),
        adjacency=torch.from_numpy(adj).to(torch.uint32), adjacency_offsets=torch.from_numpy(off).to(torch.uint32),
        alpha=torch.from_numpy(rng.uniform(0, 1, (n, 1)).astype(np.float32)),
        sdf=net.state_dict(), variance=var.state_dict()), net


def test_pt_round_trip_and_trace_attributes(tmp_path):
    sc, net = _scene()
    path = tmp_path / "model.pt"
    ck.save_pt(path, sc)
    raw = torch.load(path, weights_only=False)
    assert set(raw) == {"xyz", "color_dc", "color_sh", "adjacency", "adjacency_offsets", "alpha", "sdf", "variance"}
    assert raw["adjacency"].dtype == torch.int64 and raw["adjacency_offsets"].dtype == torch.int64
    got = ck.load_pt(path)
    for name in ("points", "color_dc", "color_sh", "alpha"):
        assert torch.equal(getattr(got, name), getattr(sc, name)), name
    assert got.adjacency.dtype == torch.uint32 and torch.equal(got.adjacency, sc.adjacency)
    assert torch.equal(got.adjacency_offsets, sc.adjacency_offsets)
    att = ck.trace_attributes(got)
    assert att.shape == (300, 49)
    assert torch.equal(att[:, :3], sc.color_dc) and torch.equal(att[:, 3:48], sc.color_sh)
    np.testing.assert_allclose(att[:, 48].detach().numpy(), net(sc.points)[:, 0].detach().numpy(), rtol=1e-6)
    inv_s = ck.variance_network(got)(torch.zeros(1, 3)).detach()
    assert abs(float(inv_s[0, 0]) - float(np.exp(0.3))) < 1e-6


def test_wrapped_state_dicts_and_sh_width(tmp_path):
    sc, _ = _scene()
    raw = {"xyz": sc.points, "color_dc": sc.color_dc, "color_sh": sc.color_sh,
           "adjacency": sc.adjacency.to(torch.int64), "adjacency_offsets": sc.adjacency_offsets.to(torch.int64),
           "alpha": sc.alpha, "sdf": {"module." + k: v for k, v in sc.sdf.items()},
           "variance": {"module." + k: v for k, v in sc.variance.items()}}
    torch.save(raw, tmp_path / "wrapped.pt")
    got = ck.load_pt(tmp_path / "wrapped.pt")
    ck.sdf_network(got)  # strict load succeeds after the prefix is stripped
    with pytest.raises(AssertionError, match="Expected 24 SH coeffs per-point, got 45"):
        ck.load_pt(tmp_path / "wrapped.pt", sh_degree=2)


def test_radfoam_density_scene(tmp_path):
    sc, _ = _scene()
    rad = ck.SceneCheckpoint(points=sc.points, color_dc=sc.color_dc, color_sh=sc.color_sh, adjacency=sc.adjacency,
                             adjacency_offsets=sc.adjacency_offsets, alpha=sc.alpha,
                             density=torch.randn(300, 1))
    ck.save_pt(tmp_path / "rad.pt", rad)
    got = ck.load_pt(tmp_path / "rad.pt")
    assert not got.use_sdfoam
    att = ck.trace_attributes(got, activation_scale=2.0)
    ref = 2.0 * torch.nn.functional.softplus(rad.density, beta=10)
    assert torch.allclose(att[:, 48:], ref)


def test_ply_layout_and_round_trip(tmp_path):
    sc, net = _scene(n=50)
    att = torch.cat([sc.color_dc, sc.color_sh], 1)
    sdf = net(sc.points)[:, :1].detach()
    path = tmp_path / "scene.ply"
    ck.save_ply(path, sc.points, att, sc.adjacency, sc.adjacency_offsets, sdf)
    header = open(path, "rb").read().split(b"end_header\n")[0].decode().splitlines()
    assert header[:3] == ["ply", "format binary_little_endian 1.0", "element vertex 50"]
    assert header[3:11] == ["property float x", "property float y", "property float z", "property uchar red",
                            "property uchar green", "property uchar blue", "property float density",
                            "property uint adjacency_offset"]
    assert header[11] == "property float color_sh_0" and header[11 + 44] == "property float color_sh_44"
    assert header[-2:] == [f"element adjacency {sc.adjacency.numel()}", "property uint adjacency"]
    pts, col, last, adj, off = ck.load_ply(path)
    assert np.array_equal(pts, sc.points.numpy()) and np.array_equal(adj, sc.adjacency.numpy())
    assert np.array_equal(off, sc.adjacency_offsets.numpy()) and np.array_equal(col[:, 3:], sc.color_sh.numpy())
    np.testing.assert_allclose(last, sdf[:, 0].numpy())
    # the DC colour goes through 8 bits, clipped to [0, 255]
    rgb8 = np.clip(255 * (0.5 + ck.SH_C0 * sc.color_dc.numpy()), 0, 255).astype(np.uint8)
    np.testing.assert_allclose(col[:, :3], (rgb8 / 255.0 - 0.5) / ck.SH_C0, rtol=1e-6, atol=1e-6)
