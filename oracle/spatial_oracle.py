"""CPU restatement of the AABB tree, the nearest-site query and the site sort.

Test infrastructure only (checker for sdfoam_b200's GPU kernels).

  build_aabb_tree  src/aabb_tree/aabb_tree.cu:192-341: level-major complete
                   binary tree, leaves (site pairs 2j, 2j+1, clamped to the
                   last site) first, [pow2(N), 2, 3] (min, max)
  nn               src/aabb_tree/aabb_tree.cu:343-415 / nn_cpu 417-478: the
                   nearest site; distance (dx*dx + dy*dy) + dz*dz in float32,
                   ties to the lowest index (the reference leaves ties to its
                   warp sort; this restatement fixes the rule)
  sort_points      src/aabb_tree/aabb_tree.cu:62-190 (see sort_permutation)
"""
from __future__ import annotations

import math

import numpy as np


def pow2_round_up(x: int) -> int:
    p = 1
    while p < x:
        p <<= 1
    return p


def build_aabb_tree(points: np.ndarray) -> np.ndarray:
    p = np.ascontiguousarray(points, np.float32).reshape(-1, 3)
    n = p.shape[0]
    nodes = pow2_round_up(n)
    tree = np.zeros((nodes, 2, 3), np.float32)
    leaves = nodes // 2
    if leaves == 0:
        tree[0, 0] = p[0]
        tree[0, 1] = p[0]
        return tree
    a = np.minimum(np.arange(leaves) * 2, n - 1)
    b = np.arange(leaves) * 2 + 1
    b = np.where(b >= n, a, b)
    lo = np.minimum(p[a], p[b])
    hi = np.maximum(p[a], p[b])
    tree[:leaves, 0] = lo
    tree[:leaves, 1] = hi
    off, width = 0, leaves
    while width > 1:
        up = width // 2
        c = tree[off:off + width]
        tree[off + width:off + width + up, 0] = np.minimum(c[0::2, 0], c[1::2, 0])
        tree[off + width:off + width + up, 1] = np.maximum(c[0::2, 1], c[1::2, 1])
        off += width
        width = up
    return tree


def nn(points: np.ndarray, queries: np.ndarray, chunk: int = 2048) -> np.ndarray:
    p = np.ascontiguousarray(points, np.float32).reshape(-1, 3)
    q = np.ascontiguousarray(queries, np.float32).reshape(-1, 3)
    out = np.empty(q.shape[0], np.uint32)
    for s in range(0, q.shape[0], chunk):
        d = q[s:s + chunk, None, :] - p[None, :, :]          # float32 differences
        d2 = (d[..., 0] * d[..., 0] + d[..., 1] * d[..., 1]) + d[..., 2] * d[..., 2]
        out[s:s + chunk] = np.argmin(d2, axis=1)              # first index of the minimum
    return out


def sort_permutation(points: np.ndarray) -> np.ndarray:
    """perm[i] = original index of the i-th site after sort_points: rounds of
    stable sorts by the order-preserving u32 key of one axis (x, y, z, x, ...),
    segment size pow2(N) halving each round; segments above 1024 sites sort
    globally while there are at most 1024 of them (aabb_tree.cu:135-152) and
    per segment otherwise; smaller segments sort whole 1024-site blocks
    (aabb_tree.cu:154-163)."""
    p = np.ascontiguousarray(points, np.float32)
    n = p.shape[0]
    u = p.view(np.uint32).copy()
    keys = np.where((u & 0x80000000) != 0, ~u, u ^ 0x80000000).astype(np.uint32)
    perm = np.arange(n, dtype=np.int64)
    seg = pow2_round_up(n)
    dim = 0
    while seg > 1:
        nseg = (n + seg - 1) // seg
        k = keys[perm, dim]
        if seg > 1024 and nseg <= 1024:
            order = np.argsort(k, kind="stable")
        else:
            unit = seg if seg > 1024 else 1024
            order = np.lexsort((k, np.arange(n) // unit))
        perm = perm[order]
        seg >>= 1
        dim = (dim + 1) % 3
    return perm


def log2_levels(n: int) -> int:
    return int(math.log2(pow2_round_up(n)))
