"""Rank bodies of the world-size-2 gloo tests (tests/test_distributed.py);
a separate module so that spawned processes can import them."""
import os

import numpy as np
import torch
import torch.distributed as dist


def _init(rank, world, port):
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)


def allreduce_worker(rank, world, port, out_dir):
    from sdfoam_b200.distributed import allreduce_grads, max_over_ranks
    _init(rank, world, port)
    g = torch.Generator().manual_seed(100 + rank)
    grads = [torch.randn(5, 3, generator=g), torch.randn(7, generator=g).to(torch.bfloat16),
             torch.randn(2, 2, generator=g), None]
    np.save(os.path.join(out_dir, f"in{rank}.npy"),
            np.concatenate([t.float().reshape(-1).numpy() for t in grads if t is not None]))
    allreduce_grads(grads)
    np.save(os.path.join(out_dir, f"out{rank}.npy"),
            np.concatenate([t.float().reshape(-1).numpy() for t in grads if t is not None]))
    m = max_over_ranks(float(rank) * 3.5 + 1.0, torch.device("cpu"))
    np.save(os.path.join(out_dir, f"max{rank}.npy"), np.array([m]))
    dist.barrier()
    dist.destroy_process_group()


def broadcast_worker(rank, world, port, out_dir):
    from oracle import delaunay_oracle as dor
    from sdfoam_b200.densify import rebuild

    _init(rank, world, port)
    rng = np.random.default_rng(5)
    pts = torch.from_numpy(rng.uniform(-1, 1, (300, 3)).astype(np.float32))
    calls = []

    def triangulate(points):  # the CPU oracle stands in for the GPU rebuild
        calls.append(rank)
        perm = np.arange(points.shape[0])[::-1].copy()
        adj, off = dor.delaunay_adjacency(points.numpy()[perm])
        return (torch.from_numpy(perm.astype(np.uint32)), torch.from_numpy(adj), torch.from_numpy(off))

    perm, adj, off = rebuild(pts, triangulate, world=world)
    np.savez(os.path.join(out_dir, f"tri{rank}.npz"), perm=perm.numpy(), adj=adj.numpy(), off=off.numpy(),
             calls=np.array(calls, np.int64))
    dist.barrier()
    dist.destroy_process_group()


def sharded_gradient_worker(rank, world, port, out_dir):
    """Each rank runs the CPU restatement's backward on its shard of the rays;
    the all-reduced gradients must equal the backward over all rays."""
    from oracle import oracle as orc
    from sdfoam_b200 import synthetic as syn
    from sdfoam_b200.distributed import allreduce_grads, shard_batches

    _init(rank, world, port)
    foam = syn.make_foam("tiny", num_points=4096, seed=3)
    cam = syn.look_at((2.2, 1.1, 0.7), fov_deg=40.0, width=32, height=32)
    rays, start = syn.camera_rays(foam, [cam], tile=None)
    sc = orc.OracleScene(foam.points, foam.attributes, foam.adjacency, foam.offsets, 3)
    st = orc.settings(neus=True, sharpness=50.0)
    g = np.random.default_rng(9).normal(0, 1, (rays.shape[0], 4)).astype(np.float32)
    batch = 128
    nb = rays.shape[0] // batch
    attr = torch.zeros(foam.points.shape[0], 49, dtype=torch.float64)
    pts = torch.zeros(foam.points.shape[0], 3, dtype=torch.float64)
    for b in shard_batches(nb, world, rank):
        sl = slice(b * batch, (b + 1) * batch)
        fw = orc.trace_forward(sc, st, rays[sl], start[sl], threads=1)
        bw = orc.trace_backward(sc, st, rays[sl], start[sl], fw["rgba"], g[sl], threads=1)
        attr += torch.from_numpy(bw["attr_grad"].astype(np.float64))
        pts += torch.from_numpy(bw["points_grad"].astype(np.float64))
    allreduce_grads([attr, pts])
    np.savez(os.path.join(out_dir, f"grad{rank}.npz"), attr=attr.numpy(), pts=pts.numpy())
    dist.barrier()
    dist.destroy_process_group()


def sharded_mlp_worker(rank, world, port, out_dir):
    """sdfnet over 101 sites split across the ranks (sharded_rows) with
    per-rank losses; the all-reduced gradients against one process
    evaluating every site."""
    from sdfoam_b200.distributed import allreduce_grads, sharded_rows
    from sdfoam_b200.sdfnet import SDFNetwork
    _init(rank, world, port)
    g = torch.Generator().manual_seed(7)
    pts0 = torch.rand(101, 3, generator=g) * 2 - 1
    w = [torch.randn(101, 1, generator=g) for _ in range(world)]
    net = SDFNetwork(d_hidden=64, init="xavier", point_cloud=pts0, generator=torch.Generator().manual_seed(2))
    pts = pts0.clone().requires_grad_(True)
    sdf = sharded_rows(net, pts)
    (w[rank] * sdf).sum().backward()
    params = [p for p in net.parameters()]
    allreduce_grads([pts.grad] + [p.grad for p in params])
    ref_net = SDFNetwork(d_hidden=64, init="xavier", point_cloud=pts0, generator=torch.Generator().manual_seed(2))
    ref_pts = pts0.clone().requires_grad_(True)
    ref_sdf = ref_net(ref_pts)
    (sum(w) * ref_sdf).sum().backward()
    np.savez(os.path.join(out_dir, f"mlp{rank}.npz"), sdf=sdf.detach().numpy(), ref_sdf=ref_sdf.detach().numpy(),
             pts=pts.grad.numpy(), ref_pts=ref_pts.grad.numpy(),
             w=np.concatenate([p.grad.reshape(-1).numpy() for p in params]),
             ref_w=np.concatenate([p.grad.reshape(-1).numpy() for p in ref_net.parameters()]))
    dist.barrier()
    dist.destroy_process_group()


def overlapped_worker(rank, world, port, out_dir):
    """A backward whose leaf gradients are all-reduced by the hooks of
    OverlappedAllReduce (large ones as soon as they are ready, small ones at
    finish()), twice in a row, against the plain bucketed all-reduce."""
    from sdfoam_b200.distributed import OverlappedAllReduce, allreduce_grads
    _init(rank, world, port)
    g = torch.Generator().manual_seed(7)  # the same leaves on every rank
    big = torch.randn(300000, generator=g).requires_grad_(True)
    small = torch.randn(17, generator=g).requires_grad_(True)
    other = torch.randn(5, 3, generator=g).requires_grad_(True)
    x = torch.randn(300000, generator=torch.Generator().manual_seed(50 + rank))
    red = OverlappedAllReduce([big, small, other], small_bytes=4096)
    outs = []
    for step in range(2):
        loss = (big * x).sum() * (step + 1) + (small ** 2).sum() * rank + (other * 3.0).sum()
        loss.backward()
        red.finish()
        outs.append([big.grad.clone(), small.grad.clone(), other.grad.clone()])
        for p in (big, small, other):
            p.grad = None
    red.remove()
    # the same sums with the plain all-reduce
    ref = [(x * 2).clone(), (2 * small.detach() * rank).clone(), torch.full((5, 3), 3.0)]
    allreduce_grads(ref)
    np.savez(os.path.join(out_dir, f"ov{rank}.npz"), big=outs[1][0].numpy(), small=outs[1][1].numpy(),
             other=outs[1][2].numpy(), big0=outs[0][0].numpy(), rbig=ref[0].numpy(), rsmall=ref[1].numpy(),
             rother=ref[2].numpy())
    dist.barrier()
    dist.destroy_process_group()
