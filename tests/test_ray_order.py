"""TraceRays with pipeline.sort_rays: the batch is walked in coherent order
and every per-ray output comes back in the caller's order.  Checked on the
host with a stand-in pipeline whose per-ray results are functions of the
ray alone (integer-valued, so per-site sums are order-free) and whose
backward checks that it sees the forward's rays, outputs and gradients in
one consistent order."""
import pytest
import torch

from sdfoam_b200.render import TraceRays, coherent_order

N, A = 50, 49


class StandIn:
    def __init__(self, sort_rays):
        self.sort_rays = sort_rays

    def build_cells(self, *args):
        return None

    @staticmethod
    def exit_record(n, steps, device):
        return torch.zeros((n, 8), dtype=torch.uint8)

    @staticmethod
    def _rgba(rays, start):
        r = rays.reshape(-1, 6)
        s = start.reshape(-1).to(r.dtype)
        return torch.stack([r[:, 3] + s, 2 * r[:, 4], r[:, 5] - r[:, 0], r[:, 1] * r[:, 2]], -1)

    def trace_forward(self, points, attributes, adj, off, rays, start, depth_quantiles=None,
                      return_contribution=False, alpha_mode=None, inv_s=None, eps=None, sdf_channel=None,
                      cells=None, exits=None):
        rgba = self._rgba(rays, start)
        s = start.reshape(-1).long()
        out = {"rgba": rgba.reshape(rays.shape[:-1] + (4,)),
               "num_intersections": (s % 7).to(torch.uint32).reshape(rays.shape[:-1] + (1,)),
               "alpha": torch.zeros(N, 1)}
        if return_contribution:
            out["contribution"] = torch.zeros(N, 1).index_add_(0, s, rgba[:, 3:4])
        if depth_quantiles is not None:
            q = depth_quantiles.reshape(s.numel(), -1)
            out["depth"] = (q * rgba[:, :1]).reshape(rays.shape[:-1] + (q.shape[1],))
            out["depth_indices"] = s[:, None].expand(-1, q.shape[1]).to(torch.uint32).reshape(out["depth"].shape)
        return out

    def trace_backward(self, points, attributes, adj, off, rays, start, rgb_out, grad_in, depth_quantiles,
                       depth_indices, depth_grad, ray_error, alpha_mode=None, inv_s=None, eps=None,
                       sdf_channel=None, cells=None, exits=None):
        # the backward sees the forward's order: rgb_out must be the forward's
        # rgba of these very rays
        assert torch.equal(rgb_out.reshape(-1, 4), self._rgba(rays, start))
        r = rays.reshape(-1, 6)
        s = start.reshape(-1).long()
        g = grad_in.reshape(-1, 4)
        if depth_grad is not None:
            g = g + depth_grad.reshape(s.numel(), -1).sum(1, keepdim=True)
        if ray_error is not None:
            g = g * ray_error.reshape(-1, 1)
        out = {"points_grad": torch.zeros(N, 3).index_add_(0, s, g[:, :3] * r[:, 3:6]),
               "attr_grad": torch.zeros(N, A).index_add_(0, s, g.sum(1, keepdim=True).expand(-1, A).contiguous()),
               "sharpness_grad": (g * rgb_out.reshape(-1, 4)).sum().reshape(1)}
        if ray_error is not None:
            out["point_error"] = torch.zeros(N, 1).index_add_(0, s, ray_error.reshape(-1, 1))
        return out


def _run(sort_rays, quantiles):
    g = torch.Generator().manual_seed(0)
    rays = torch.randint(-5, 6, (4, 9, 6), generator=g).float()
    start = torch.randint(0, N, (4, 9), generator=g).to(torch.uint32)  # the pipeline's dtypes
    dq = torch.randint(0, 3, (4, 9, 2), generator=g).float() if quantiles else None
    pts = torch.zeros(N, 3, requires_grad=True)
    att = torch.zeros(N, A, requires_grad=True)
    inv_s = torch.tensor([2.0], requires_grad=True)
    out = TraceRays.apply(StandIn(sort_rays), pts, att, None, None, rays, start, dq, True, True, inv_s, 1e-6, 48)
    rgba, depth, contrib, nint, errbox, alpha = out
    errbox.ray_error = torch.randint(1, 4, (4, 9, 1), generator=g).float()
    grad = torch.randint(-3, 4, (4, 9, 4), generator=g).float()
    loss = (rgba * grad).sum() + (depth.sum() if depth is not None else 0.0)
    loss.backward()
    return rgba, depth, contrib, nint, pts.grad, att.grad, inv_s.grad, errbox.point_error


def test_sorted_walk_returns_the_callers_order():
    for quantiles in (False, True):
        a = _run(False, quantiles)
        b = _run(True, quantiles)
        for x, y in zip(a, b):
            if x is None:
                assert y is None
            else:
                assert torch.equal(x, y)


def test_coherent_order_groups_start_sites_and_directions():
    g = torch.Generator().manual_seed(1)
    d = torch.randn(2000, 3, generator=g)
    rays = torch.cat([torch.zeros(2000, 3), d / d.norm(dim=1, keepdim=True)], 1)
    start = torch.randint(0, 5, (2000,), generator=g)
    perm = coherent_order(rays, start)
    assert torch.equal(torch.sort(perm).values, torch.arange(2000))
    s = start[perm]
    assert (s[1:] >= s[:-1]).all()
    # consecutive rays of one start site point in similar directions
    dd = rays[perm, 3:]
    same = s[1:] == s[:-1]
    cos = (dd[1:] * dd[:-1]).sum(1)[same]
    assert cos.median() > 0.9


@pytest.mark.gpu
def test_sorted_walk_matches_caller_order_on_the_gpu(tiny_foam):
    """The real kernels with pipeline.sort_rays on and off, rays shuffled as
    training draws them: the same per-ray outputs bit for bit (each ray's
    walk is independent) and the same gradients up to the order of the
    per-site atomic sums, through the exit-record replay in sorted order."""
    import numpy as np
    import sdfoam_b200 as sdfoam

    foam, rays, start = tiny_foam
    dev = torch.device("cuda:0")
    perm = np.random.default_rng(17).permutation(rays.shape[0])
    rr = torch.from_numpy(rays[perm]).to(dev)
    ss = torch.from_numpy(start[perm]).to(dev)
    g = torch.from_numpy(np.random.default_rng(5).normal(0, 1, (rays.shape[0], 4)).astype(np.float32)).to(dev)
    out = {}
    for sort in (False, True):
        pipe = sdfoam.create_pipeline(3)
        pipe.sort_rays = sort
        pts = torch.from_numpy(foam.points).to(dev).requires_grad_(True)
        att = torch.from_numpy(foam.attributes).to(dev).requires_grad_(True)
        inv = torch.full((pts.shape[0], 1), 50.0, device=dev, requires_grad=True)
        adj = torch.from_numpy(foam.adjacency).to(dev)
        off = torch.from_numpy(foam.offsets).to(dev)
        rgba, _, contrib, nint, _, _ = TraceRays.apply(pipe, pts, att, adj, off, rr, ss, None, True, True, inv,
                                                       1e-6, 48)
        (rgba * g).sum().backward()
        torch.cuda.synchronize()
        out[sort] = (rgba.detach(), nint, contrib.detach(), att.grad, pts.grad, inv.grad)
    a, b = out[False], out[True]
    assert torch.equal(a[0], b[0]) and torch.equal(a[1], b[1])
    for x, y in zip(a[2:], b[2:]):
        x, y = x.double(), y.double()
        assert torch.allclose(x, y, rtol=1e-4, atol=1e-6 * y.abs().max().item())
