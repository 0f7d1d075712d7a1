"""Host side of the multi-GPU path (one process per GPU, torch.distributed):
rays shard across ranks with the foam replicated, so the data path has one
exchange -- the sum of the per-site gradients -- plus, when sites move, the
broadcast of the Delaunay rebuild that rank 0 computes.

Everything here also runs on the gloo backend with CPU tensors, which is how
the tests exercise it without GPUs.
"""
from __future__ import annotations

from typing import List, Sequence

import torch
import torch.distributed as dist
from torch._utils import _flatten_dense_tensors, _unflatten_dense_tensors


def shard_batches(num_batches: int, world: int, rank: int) -> List[int]:
    """Batches of this rank: round robin, at least one per rank (a rank with
    no batch of its own repeats one, so that every rank steps)."""
    mine = [b for b in range(num_batches) if b % world == rank]
    return mine or [rank % max(1, num_batches)]


def allreduce_grads(tensors: Sequence[torch.Tensor], group=None) -> None:
    """Sums the tensors over the group in place, one collective per dtype
    (the gradients are flattened into a bucket, reduced and copied back)."""
    by_dtype = {}
    for t in tensors:
        if t is not None:
            by_dtype.setdefault(t.dtype, []).append(t)
    for ts in by_dtype.values():
        flat = _flatten_dense_tensors(ts)
        dist.all_reduce(flat, group=group)
        for t, r in zip(ts, _unflatten_dense_tensors(flat, ts)):
            t.copy_(r)


class OverlappedAllReduce:
    """Sums the gradients of `leaves` over the group while the backward is
    still running.

    A post-accumulate-grad hook on every leaf starts an asynchronous
    all-reduce of that leaf's gradient as soon as autograd has written it
    (NCCL orders it after the work already queued on the current stream), so
    the reduction of the per-site gradients, which the walk's backward
    produces first, overlaps the rest of the backward (the sdfnet's).  Leaves
    smaller than `small_bytes` wait and are reduced together in finish(),
    one bucket per dtype.  finish() waits for everything; every rank must
    run the same backward, so the collectives line up in the same order."""

    def __init__(self, leaves: Sequence[torch.Tensor], group=None, small_bytes: int = 1 << 20):
        self.leaves = list(leaves)
        self.group = group
        self.small_bytes = small_bytes
        self.works = []
        self.small = []
        self.enabled = True  # False: the hooks do nothing (a backward that is not reduced)
        self.handles = [p.register_post_accumulate_grad_hook(self._ready) for p in self.leaves]

    def _ready(self, p: torch.Tensor) -> None:
        if not self.enabled:
            return
        g = p.grad
        if g.numel() * g.element_size() < self.small_bytes:
            self.small.append(g)
        else:
            self.works.append(dist.all_reduce(g, group=self.group, async_op=True))

    def finish(self) -> None:
        """Reduces the small gradients and waits for every reduction of this
        backward (the results are then ordered before later work on the
        current stream)."""
        small = sorted(self.small, key=lambda t: next(i for i, p in enumerate(self.leaves) if p.grad is t))
        allreduce_grads(small, group=self.group)
        for w in self.works:
            w.wait()
        self.works, self.small = [], []

    def remove(self) -> None:
        for h in self.handles:
            h.remove()
        self.handles = []


class _GatherRows(torch.autograd.Function):
    """Every rank's [n, C] block stacked in rank order; the backward sums the
    gradient over the ranks and returns this rank's block of it."""

    @staticmethod
    def forward(ctx, local, group):
        ctx.group = group
        ctx.rank = dist.get_rank(group)
        ctx.n = local.shape[0]
        local = local.contiguous()
        parts = [torch.empty_like(local) for _ in range(dist.get_world_size(group))]
        dist.all_gather(parts, local, group=group)
        return torch.cat(parts, 0)

    @staticmethod
    def backward(ctx, grad):
        g = grad.contiguous().clone()
        dist.all_reduce(g, group=ctx.group)
        return g[ctx.rank * ctx.n:(ctx.rank + 1) * ctx.n], None


def sharded_rows(fn, inputs: torch.Tensor, group=None) -> torch.Tensor:
    """fn applied to all rows of `inputs` with the rows split over the ranks:
    this rank evaluates fn on its 1/world of them (the last shard padded to
    equal size with copies of row 0, whose outputs are dropped), the results
    are gathered to every rank, and the backward sends each rank the summed
    gradient of its own rows -- so the per-site sdfnet runs once per site in
    the whole job instead of once per rank.  Parameter and input gradients
    then hold this rank's shard's part and are summed with the other
    gradients (allreduce_grads)."""
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    n = inputs.shape[0]
    per = (n + world - 1) // world
    lo, hi = min(n, rank * per), min(n, (rank + 1) * per)
    local = inputs[lo:hi]
    if hi - lo < per:
        local = torch.cat([local, inputs[:1].expand(per - (hi - lo), *inputs.shape[1:])], 0)
    return _GatherRows.apply(fn(local), group)[:n]


def max_over_ranks(value: float, device, group=None) -> float:
    """The largest of the ranks' values (per-rank device times)."""
    t = torch.tensor([value], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t.item())


def _as_i32(t: torch.Tensor) -> torch.Tensor:
    # uint32 payloads travel as int32 bit patterns
    return t.view(torch.int32) if t.dtype == torch.uint32 else t


def broadcast_triangulation(perm, adjacency, offsets, num_points: int, device, src: int = 0, group=None):
    """(perm, adjacency, offsets) of rank src on every rank of the group.

    On src the three uint32 tensors are given; elsewhere pass None and they
    are allocated here.  The adjacency size travels first (one int64), then
    the payloads."""
    rank = dist.get_rank(group)
    size = torch.zeros(1, dtype=torch.int64, device=device)
    if rank == src:
        size[0] = adjacency.numel()
    dist.broadcast(size, src, group=group)
    e = int(size.item())
    if rank != src:
        perm = torch.empty(num_points, dtype=torch.uint32, device=device)
        adjacency = torch.empty(e, dtype=torch.uint32, device=device)
        offsets = torch.empty(num_points + 1, dtype=torch.uint32, device=device)
    for t in (perm, offsets, adjacency):
        dist.broadcast(_as_i32(t), src, group=group)
    return perm, adjacency, offsets
