"""The multi-GPU host path on world-size-2 gloo process groups (CPU): the
bucketed gradient all-reduce and max-over-ranks timing, the broadcast of a
rank-0 Delaunay rebuild, ray sharding whose all-reduced gradients equal the
unsharded backward, and the deterministic densify step."""
import socket

import numpy as np
import torch
import torch.multiprocessing as mp

import dist_workers


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _spawn(fn, tmp_path):
    mp.spawn(fn, args=(2, _port(), str(tmp_path)), nprocs=2, join=True)


def test_shard_batches():
    from sdfoam_b200.distributed import shard_batches
    assert shard_batches(5, 2, 0) == [0, 2, 4] and shard_batches(5, 2, 1) == [1, 3]
    assert shard_batches(1, 4, 3) == [0]  # every rank steps
    seen = sorted(b for r in range(3) for b in shard_batches(10, 3, r))
    assert seen == list(range(10))


def test_allreduce_and_max_gloo(tmp_path):
    _spawn(dist_workers.allreduce_worker, tmp_path)
    a, b = np.load(tmp_path / "in0.npy"), np.load(tmp_path / "in1.npy")
    o0, o1 = np.load(tmp_path / "out0.npy"), np.load(tmp_path / "out1.npy")
    assert np.array_equal(o0, o1)
    # fp32 parts exact; the bf16 part (elements 15..21) is summed in bf16
    np.testing.assert_allclose(o0[:15], a[:15] + b[:15], rtol=1e-6)
    np.testing.assert_allclose(o0[22:], a[22:] + b[22:], rtol=1e-6)
    np.testing.assert_allclose(o0[15:22], a[15:22] + b[15:22], rtol=1e-2, atol=1e-2)
    assert np.load(tmp_path / "max0.npy")[0] == np.load(tmp_path / "max1.npy")[0] == 4.5


def test_rebuild_broadcast_gloo(tmp_path):
    _spawn(dist_workers.broadcast_worker, tmp_path)
    t0, t1 = np.load(tmp_path / "tri0.npz"), np.load(tmp_path / "tri1.npz")
    for k in ("perm", "adj", "off"):
        assert np.array_equal(t0[k], t1[k]), k
    assert t0["calls"].tolist() == [0] and t1["calls"].tolist() == []  # only rank 0 rebuilds
    assert t0["off"][-1] == t0["adj"].size and t0["perm"][0] == 299


def test_sharded_gradients_equal_unsharded_gloo(tmp_path):
    from oracle import oracle as orc
    from sdfoam_b200 import synthetic as syn
    _spawn(dist_workers.sharded_gradient_worker, tmp_path)
    g0, g1 = np.load(tmp_path / "grad0.npz"), np.load(tmp_path / "grad1.npz")
    assert np.array_equal(g0["attr"], g1["attr"]) and np.array_equal(g0["pts"], g1["pts"])
    foam = syn.make_foam("tiny", num_points=4096, seed=3)
    cam = syn.look_at((2.2, 1.1, 0.7), fov_deg=40.0, width=32, height=32)
    rays, start = syn.camera_rays(foam, [cam], tile=None)
    sc = orc.OracleScene(foam.points, foam.attributes, foam.adjacency, foam.offsets, 3)
    st = orc.settings(neus=True, sharpness=50.0)
    g = np.random.default_rng(9).normal(0, 1, (rays.shape[0], 4)).astype(np.float32)
    fw = orc.trace_forward(sc, st, rays, start, threads=1)
    bw = orc.trace_backward(sc, st, rays, start, fw["rgba"], g, threads=1)
    scale = np.abs(bw["attr_grad"]).max()
    np.testing.assert_allclose(g0["attr"], bw["attr_grad"], rtol=1e-4, atol=1e-5 * scale)
    np.testing.assert_allclose(g0["pts"], bw["points_grad"], rtol=1e-4, atol=1e-5 * np.abs(bw["points_grad"]).max())


def test_densify_is_deterministic():
    from sdfoam_b200.densify import densify
    pts = torch.rand(100, 3)
    att = torch.rand(100, 49)
    score = torch.rand(100)
    score[7] = score[3] = 10.0  # a tie: the lower index first
    a = densify(pts, att, score, 0.1, 0.005, torch.Generator().manual_seed(4))
    b = densify(pts, att, score, 0.1, 0.005, torch.Generator().manual_seed(4))
    assert torch.equal(a[0], b[0]) and torch.equal(a[1], b[1])
    assert a[0].shape == (110, 3) and torch.equal(a[1][100], att[3]) and torch.equal(a[1][101], att[7])
    assert (a[0][100] - pts[3]).abs().max() < 0.05


def test_sharded_sdfnet_gradients_equal_unsharded_gloo(tmp_path):
    """The per-site MLP split over the ranks (each site evaluated by one
    rank, gathered everywhere) gives the single-process SDF and, after the
    gradient all-reduce, its gradients."""
    _spawn(dist_workers.sharded_mlp_worker, tmp_path)
    for r in range(2):
        z = np.load(tmp_path / f"mlp{r}.npz")
        np.testing.assert_allclose(z["sdf"], z["ref_sdf"], rtol=1e-6, atol=1e-7)
        np.testing.assert_allclose(z["pts"], z["ref_pts"], rtol=1e-4, atol=1e-6)
        np.testing.assert_allclose(z["w"], z["ref_w"], rtol=1e-4, atol=1e-6 * np.abs(z["ref_w"]).max())


def test_overlapped_allreduce_gloo(tmp_path):
    _spawn(dist_workers.overlapped_worker, tmp_path)
    a, b = np.load(tmp_path / "ov0.npz"), np.load(tmp_path / "ov1.npz")
    for k in ("big", "small", "other"):
        assert np.array_equal(a[k], b[k]), k
        np.testing.assert_allclose(a[k], a["r" + k], rtol=1e-6, atol=1e-6)
    np.testing.assert_allclose(a["big0"] * 2, a["big"], rtol=1e-6)
