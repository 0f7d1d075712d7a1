"""Seeded synthetic foams and camera rays.

The reference trains on DTU / Mip-NeRF 360 / Deep Blending captures, none of
which are available here; these seeded scenes stand in for them with the
shapes, sizes and value distributions of the benchmark configurations:

  tiny     32,768 sites: 50% U[-1,1]^3, 50% within +-0.05 of the r=0.5 sphere;
           one 128x128 pinhole view at radius 3, fov 40 deg.
  medium   1M sites, same mixture around a torus (R=0.6, r=0.2); 8 views of
           800x800 on a ring at radius 3.
  surface  4M sites, 80% within +-0.02 of a union of three spheres, 20%
           U[-1,1]^3; 49 views of 1600x1200 on a hemisphere at radius 2.5,
           traced in 8M-ray batches.
  unbounded 6M sites, log-radial out to r=50 plus a dense core, 1/4 of the SH
           coefficients non-zero; 16 views of 1236x820, jittered cameras.

Rays follow the data loaders' layout ([..., 6] = origin, unit direction) and
the pinhole model of cast_ray (src/tracing/camera.h:56-85).  Sites are put in
the order of the reference's sort_points permutation
(src/aabb_tree/aabb_tree.cu:62-190), which is the order a trained scene holds
them in (sdfoam_model/scene.py:80-81, 235-237).
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np

SH_SIGMA = 0.1


# --------------------------------------------------------------------------
# sites
# --------------------------------------------------------------------------

def _unit_vectors(rng, n):
    v = rng.normal(size=(n, 3))
    v /= np.linalg.norm(v, axis=1, keepdims=True)
    return v


def sphere_sdf(p, r=0.5):
    return np.linalg.norm(p, axis=-1) - r


def torus_sdf(p, R=0.6, r=0.2):
    q = np.sqrt(p[..., 0] ** 2 + p[..., 1] ** 2) - R
    return np.sqrt(q ** 2 + p[..., 2] ** 2) - r


SPHERES = np.array([[-0.40, 0.00, 0.00, 0.35],
                    [0.40, 0.00, 0.00, 0.35],
                    [0.00, 0.30, 0.35, 0.30]], dtype=np.float64)


def spheres_sdf(p):
    d = [np.linalg.norm(p - s[:3], axis=-1) - s[3] for s in SPHERES]
    return np.min(np.stack(d, 0), axis=0)


def _band_samples(rng, n, band, kind):
    """n points with |sdf| <= band around the chosen surface."""
    out = []
    have = 0
    while have < n:
        m = int((n - have) * 1.3) + 1024
        if kind == "sphere":
            p = _unit_vectors(rng, m) * (0.5 + rng.uniform(-band, band, (m, 1)))
            f = sphere_sdf(p)
        elif kind == "torus":
            u = rng.uniform(0, 2 * np.pi, m)
            v = rng.uniform(0, 2 * np.pi, m)
            rr = 0.2 + rng.uniform(-band, band, m)
            p = np.stack([(0.6 + rr * np.cos(v)) * np.cos(u),
                          (0.6 + rr * np.cos(v)) * np.sin(u),
                          rr * np.sin(v)], 1)
            f = torus_sdf(p)
        elif kind == "spheres":
            area = SPHERES[:, 3] ** 2
            which = rng.choice(3, size=m, p=area / area.sum())
            s = SPHERES[which]
            p = s[:, :3] + _unit_vectors(rng, m) * (s[:, 3:4] + rng.uniform(-band, band, (m, 1)))
            f = spheres_sdf(p)
        else:
            raise ValueError(kind)
        keep = np.abs(f) <= band
        p = p[keep]
        out.append(p)
        have += p.shape[0]
    return np.concatenate(out, 0)[:n]


def make_sites(config: str, num_points: int | None = None, seed: int = 0):
    """Returns (points float32 [N,3], sdf float32 [N]) in generation order."""
    rng = np.random.default_rng(seed)
    if config == "tiny":
        n = num_points or 32768
        nb = n // 2
        p = np.concatenate([rng.uniform(-1, 1, (n - nb, 3)), _band_samples(rng, nb, 0.05, "sphere")])
        base = sphere_sdf
    elif config == "medium":
        n = num_points or 1 << 20
        nb = n // 2
        p = np.concatenate([rng.uniform(-1, 1, (n - nb, 3)), _band_samples(rng, nb, 0.05, "torus")])
        base = torus_sdf
    elif config == "surface":
        n = num_points or 4 << 20
        nb = int(round(n * 0.8))
        p = np.concatenate([rng.uniform(-1, 1, (n - nb, 3)), _band_samples(rng, nb, 0.02, "spheres")])
        base = spheres_sdf
    elif config == "unbounded":
        n = num_points or 6 << 20
        nc = n // 2
        r = np.exp(rng.uniform(0.0, math.log(50.0), n - nc))[:, None]
        p = np.concatenate([rng.uniform(-1, 1, (nc, 3)), _unit_vectors(rng, n - nc) * r])
        base = spheres_sdf
    else:
        raise ValueError(f"unknown config {config!r}")
    p = p.astype(np.float32)
    # drop exact duplicates (a Delaunay adjacency needs distinct sites)
    _, first = np.unique(p, axis=0, return_index=True)
    if first.shape[0] != p.shape[0]:
        p = p[np.sort(first)]
    sdf = (base(p.astype(np.float64)) + rng.normal(0, 0.01, p.shape[0])).astype(np.float32)
    return p, sdf


def sort_points_permutation(points: np.ndarray) -> np.ndarray:
    """Site permutation of the reference's sort_points
    (src/aabb_tree/aabb_tree.cu:62-190): order-preserving u32 keys of the
    float bits, segment size pow2(N) halving every round with the axis cycling
    x, y, z; rounds whose segments exceed 1024 sites sort globally while there
    are at most 1024 segments (aabb_tree.cu:135-152) and per segment otherwise;
    smaller segments sort whole 1024-site blocks (aabb_tree.cu:154-163).  All
    sorts are stable.  perm[i] = original index of the i-th sorted site."""
    p = np.ascontiguousarray(points, np.float32)
    n = p.shape[0]
    u = p.view(np.uint32).copy()
    neg = (u & 0x80000000) != 0
    keys = np.where(neg, ~u, u ^ 0x80000000).astype(np.uint32)
    perm = np.arange(n, dtype=np.int64)
    seg = 1 << max(0, int(math.ceil(math.log2(n))) if n > 1 else 0)
    dim = 0
    while seg > 1:
        nseg = (n + seg - 1) // seg
        k = keys[perm, dim]
        if seg > 1024 and nseg <= 1024:
            order = np.argsort(k, kind="stable")
        else:
            unit = seg if seg > 1024 else 1024
            blk = np.arange(n, dtype=np.int64) // unit
            order = np.lexsort((k, blk))  # stable: by block, then key
        perm = perm[order]
        seg >>= 1
        dim = (dim + 1) % 3
    return perm


def make_attributes(points, sdf, sh_degree=3, mode="neus", sh_fraction=1.0, seed=1):
    """[N, 1 + 3*(deg+1)^2] float32: SH coefficients (3k+c layout) ~ N(0, 0.1)
    and, in the last channel, the SDF (NeuS mode) or a softplus(N(0,1))
    density (standard mode)."""
    rng = np.random.default_rng(seed)
    n = points.shape[0]
    nsh = 3 * (sh_degree + 1) ** 2
    sh = rng.normal(0.0, SH_SIGMA, (n, nsh)).astype(np.float32)
    if sh_fraction < 1.0:
        keep = max(3, int(round(nsh * sh_fraction)) // 3 * 3)
        sh[:, keep:] = 0.0
    if mode == "neus":
        last = sdf.astype(np.float32)
    else:
        z = rng.normal(0.0, 1.0, n)
        last = np.log1p(np.exp(z)).astype(np.float32)
    return np.concatenate([sh, last[:, None]], 1).astype(np.float32)


# --------------------------------------------------------------------------
# adjacency
# --------------------------------------------------------------------------

def csr_from_tets(num_points: int, tets: np.ndarray):
    """Site adjacency in the reference's CSR contract (find_adjacency,
    src/delaunay/delaunay.cu:150-229): unique undirected edges of the tets,
    both directions, rows in ascending site order and each row's neighbours in
    ascending index order; offsets[N] = 2 * #edges."""
    t = np.asarray(tets, dtype=np.int64)
    pairs = np.concatenate([t[:, [a, b]] for a, b in ((0, 1), (0, 2), (0, 3), (1, 2), (1, 3), (2, 3))])
    lo = np.minimum(pairs[:, 0], pairs[:, 1])
    hi = np.maximum(pairs[:, 0], pairs[:, 1])
    key = np.unique(lo * num_points + hi)
    a = key // num_points
    b = key % num_points
    src = np.concatenate([a, b])
    dst = np.concatenate([b, a])
    order = np.lexsort((dst, src))
    src = src[order]
    dst = dst[order]
    counts = np.bincount(src, minlength=num_points)
    offsets = np.zeros(num_points + 1, np.int64)
    np.cumsum(counts, out=offsets[1:])
    return dst.astype(np.uint32), offsets.astype(np.uint32)


def delaunay_adjacency(points: np.ndarray):
    """Delaunay site adjacency via scipy's Qhull on the float32 sites (exact in
    float64).  Used to build synthetic test scenes."""
    from scipy.spatial import Delaunay

    tri = Delaunay(np.asarray(points, np.float64))
    return csr_from_tets(points.shape[0], tri.simplices)


# --------------------------------------------------------------------------
# cameras and rays
# --------------------------------------------------------------------------

@dataclass
class Camera:
    position: np.ndarray
    forward: np.ndarray
    right: np.ndarray
    up: np.ndarray
    fov: float
    width: int
    height: int


def look_at(position, target=(0.0, 0.0, 0.0), up=(0.0, 0.0, 1.0), fov_deg=40.0, width=128, height=128):
    """look_at (src/tracing/camera.h:36-53)."""
    pos = np.asarray(position, np.float32)
    fwd = np.asarray(target, np.float32) - pos
    fwd /= np.linalg.norm(fwd)
    right = np.cross(fwd, np.asarray(up, np.float32))
    right /= np.linalg.norm(right)
    upv = np.cross(right, fwd)
    upv /= np.linalg.norm(upv)
    return Camera(pos, fwd.astype(np.float32), right.astype(np.float32), upv.astype(np.float32),
                  math.radians(fov_deg), int(width), int(height))


def pinhole_rays(cam: Camera, tile=None):
    """[H*W, 6] float32 rays of cast_ray's pinhole model (camera.h:56-85):
    u = (2 i/W - 1) W/H, v = 1 - 2 j/H, dir = normalize(w fwd + u right + v up).
    tile=(tw, th) orders pixels in tw x th tiles (one warp per tile)."""
    W, H = cam.width, cam.height
    i = np.arange(W, dtype=np.float32)
    j = np.arange(H, dtype=np.float32)
    x = i / np.float32(W)
    y = j / np.float32(H)
    u = (2.0 * x - 1.0) * (np.float32(W) / np.float32(H))
    v = 1.0 - 2.0 * y
    w = np.float32(1.0 / math.tan(cam.fov * 0.5))
    uu, vv = np.meshgrid(u, v)  # [H, W]
    d = w * cam.forward[None, None, :] + uu[..., None] * cam.right + vv[..., None] * cam.up
    d = d / np.linalg.norm(d, axis=-1, keepdims=True)
    o = np.broadcast_to(cam.position, d.shape)
    rays = np.concatenate([o, d], -1).astype(np.float32)  # [H, W, 6]
    if tile is not None:
        tw, th = tile
        if W % tw == 0 and H % th == 0:
            rays = rays.reshape(H // th, th, W // tw, tw, 6).transpose(0, 2, 1, 3, 4)
        else:
            # partial tiles at the right and bottom edges: pixels ordered by
            # (tile row, tile column, row in tile, column in tile)
            jj, ii = np.meshgrid(np.arange(H), np.arange(W), indexing="ij")
            order = np.lexsort(((ii % tw).ravel(), (jj % th).ravel(), (ii // tw).ravel(), (jj // th).ravel()))
            rays = rays.reshape(-1, 6)[order]
    return np.ascontiguousarray(rays.reshape(-1, 6))


def fibonacci_hemisphere(n):
    k = np.arange(n) + 0.5
    z = 1.0 - k / n  # (0, 1]
    phi = k * math.pi * (3.0 - math.sqrt(5.0))
    r = np.sqrt(1.0 - z * z)
    return np.stack([r * np.cos(phi), r * np.sin(phi), z], 1)


def views(config: str, seed: int = 2):
    rng = np.random.default_rng(seed)
    if config == "tiny":
        d = np.array([1.0, 0.45, 0.3])
        d /= np.linalg.norm(d)
        return [look_at(3.0 * d, fov_deg=40.0, width=128, height=128)]
    if config == "medium":
        out = []
        for k in range(8):
            a = 2 * math.pi * k / 8 + 0.1
            out.append(look_at((3.0 * math.cos(a), 3.0 * math.sin(a), 0.6), fov_deg=40.0, width=800, height=800))
        return out
    if config == "surface":
        dirs = fibonacci_hemisphere(49)
        # keep cameras off the exact pole so that up = +z stays well defined
        dirs[:, 2] = np.minimum(dirs[:, 2], 0.95)
        dirs /= np.linalg.norm(dirs, axis=1, keepdims=True)
        return [look_at(2.5 * d, fov_deg=45.0, width=1600, height=1200) for d in dirs]
    if config == "unbounded":
        out = []
        for k in range(16):
            a = 2 * math.pi * k / 16
            pos = np.array([2.0 * math.cos(a), 2.0 * math.sin(a), 0.3]) + rng.normal(0, 0.2, 3)
            out.append(look_at(pos, fov_deg=60.0, width=1236, height=820))
        return out
    raise ValueError(config)


def nearest_site(points: np.ndarray, queries: np.ndarray, chunk: int = 4096) -> np.ndarray:
    """Brute-force nearest site (ties -> lowest index), float64 distances."""
    p = np.asarray(points, np.float64)
    q = np.asarray(queries, np.float64).reshape(-1, 3)
    out = np.empty(q.shape[0], np.uint32)
    pn = (p * p).sum(1)
    for s in range(0, q.shape[0], chunk):
        qq = q[s:s + chunk]
        d = pn[None, :] - 2.0 * qq @ p.T + (qq * qq).sum(1)[:, None]
        out[s:s + chunk] = np.argmin(d, axis=1)
    return out


# --------------------------------------------------------------------------
# whole scenes
# --------------------------------------------------------------------------

@dataclass
class Foam:
    points: np.ndarray       # [N,3] f32, in sort_points order
    attributes: np.ndarray   # [N,A] f32
    adjacency: np.ndarray    # [E] u32
    offsets: np.ndarray      # [N+1] u32
    sdf: np.ndarray          # [N] f32
    sh_degree: int


def make_foam(config="tiny", num_points=None, sh_degree=3, mode="neus", seed=0, sort=True,
              adjacency_fn=delaunay_adjacency, sh_fraction=None):
    p, sdf = make_sites(config, num_points, seed)
    if sort:
        perm = sort_points_permutation(p)
        p = np.ascontiguousarray(p[perm])
        sdf = np.ascontiguousarray(sdf[perm])
    if sh_fraction is None:
        sh_fraction = 0.25 if config == "unbounded" else 1.0
    attrs = make_attributes(p, sdf, sh_degree, mode, sh_fraction=sh_fraction, seed=seed + 1)
    adj, off = adjacency_fn(p)
    return Foam(p, attrs, adj, off, sdf, sh_degree)


def camera_rays(foam: Foam, cams, tile=(8, 4)):
    """Concatenated rays of the given views plus each ray's start site (the
    site nearest the camera position, as SDFoamScene.get_starting_point does
    with the AABB-tree NN query)."""
    rays, starts = [], []
    for cam in cams:
        r = pinhole_rays(cam, tile)
        s = nearest_site(foam.points, cam.position[None, :])[0]
        rays.append(r)
        starts.append(np.full(r.shape[0], s, np.uint32))
    return np.concatenate(rays), np.concatenate(starts)
