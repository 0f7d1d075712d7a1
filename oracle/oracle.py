"""ctypes front end of the CPU restatement in sdfoam_oracle.c.

Test infrastructure only: tests/, __graft_entry__.smoke() and bench.py's
cpu_baseline / --impl reference legs use it as the checker.  The product
(sdfoam_b200) never imports it.

Parity status: unpinned against the reference binary (mmlab-cv/SDFoam cannot
be built here and ships no golden vectors); see the header of
sdfoam_oracle.c for what each function follows.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")
_lib = None

U32_NONE = 0xFFFFFFFF


def build(force: bool = False) -> str:
    """Compile liboracle.so with the committed Makefile."""
    src = os.path.join(_HERE, "sdfoam_oracle.c")
    if force or not os.path.exists(_LIB_PATH) or os.path.getmtime(_LIB_PATH) < os.path.getmtime(src):
        subprocess.run(["make", "-s", "-C", _HERE, "liboracle.so"], check=True)
    return _LIB_PATH


class Scene(ctypes.Structure):
    _fields_ = [
        ("num_points", ctypes.c_uint32),
        ("adjacency_size", ctypes.c_uint32),
        ("attr_dim", ctypes.c_uint32),
        ("sh_degree", ctypes.c_int),
        ("points", ctypes.c_void_p),
        ("attributes", ctypes.c_void_p),
        ("adjacency", ctypes.c_void_p),
        ("offsets", ctypes.c_void_p),
        ("diffs", ctypes.c_void_p),
    ]


class Settings(ctypes.Structure):
    _fields_ = [
        ("weight_threshold", ctypes.c_float),
        ("max_intersections", ctypes.c_uint32),
        ("neus", ctypes.c_int),
        ("sdf_channel", ctypes.c_int),
        ("sharpness", ctypes.c_float),
    ]


class FwdIO(ctypes.Structure):
    _fields_ = [
        ("num_rays", ctypes.c_uint32),
        ("rays", ctypes.c_void_p),
        ("start", ctypes.c_void_p),
        ("num_quantiles", ctypes.c_uint32),
        ("quantiles", ctypes.c_void_p),
        ("rgba", ctypes.c_void_p),
        ("depth", ctypes.c_void_p),
        ("depth_indices", ctypes.c_void_p),
        ("num_intersections", ctypes.c_void_p),
        ("contribution", ctypes.c_void_p),
        ("alpha_out", ctypes.c_void_p),
        ("seq_offsets", ctypes.c_void_p),
        ("seq_cells", ctypes.c_void_p),
        ("seq_alpha", ctypes.c_void_p),
        ("seq_count", ctypes.c_void_p),
        ("ambiguous", ctypes.c_void_p),
    ]


class Camera(ctypes.Structure):
    _fields_ = [
        ("position", ctypes.c_float * 3),
        ("forward", ctypes.c_float * 3),
        ("right", ctypes.c_float * 3),
        ("up", ctypes.c_float * 3),
        ("fov", ctypes.c_float),
        ("width", ctypes.c_uint32),
        ("height", ctypes.c_uint32),
        ("model", ctypes.c_uint32),
        ("bg", ctypes.c_float * 3),
        ("checker", ctypes.c_int),
    ]


class BwdIO(ctypes.Structure):
    _fields_ = [
        ("num_rays", ctypes.c_uint32),
        ("rays", ctypes.c_void_p),
        ("start", ctypes.c_void_p),
        ("num_quantiles", ctypes.c_uint32),
        ("quantiles", ctypes.c_void_p),
        ("depth_indices", ctypes.c_void_p),
        ("rgba", ctypes.c_void_p),
        ("rgba_grad", ctypes.c_void_p),
        ("depth_grad", ctypes.c_void_p),
        ("ray_error", ctypes.c_void_p),
        ("points_grad", ctypes.c_void_p),
        ("attr_grad", ctypes.c_void_p),
        ("point_error", ctypes.c_void_p),
        ("sharpness_grad", ctypes.c_void_p),
        ("points_grad_abs", ctypes.c_void_p),
        ("attr_grad_abs", ctypes.c_void_p),
    ]


def lib():
    global _lib
    if _lib is None:
        build()
        _lib = ctypes.CDLL(_LIB_PATH)
        _lib.oracle_f2h.restype = ctypes.c_uint16
        _lib.oracle_f2h.argtypes = [ctypes.c_float]
        _lib.oracle_h2f.restype = ctypes.c_float
        _lib.oracle_h2f.argtypes = [ctypes.c_uint16]
        _lib.oracle_expf.restype = ctypes.c_float
        _lib.oracle_expf.argtypes = [ctypes.c_float]
        _lib.oracle_build_diffs.restype = None
        _lib.oracle_build_diffs.argtypes = [ctypes.c_uint32, ctypes.c_void_p, ctypes.c_void_p,
                                            ctypes.c_void_p, ctypes.c_uint32, ctypes.c_void_p]
        _lib.oracle_trace_forward.restype = None
        _lib.oracle_trace_forward.argtypes = [ctypes.POINTER(Scene), ctypes.POINTER(Settings),
                                              ctypes.POINTER(FwdIO), ctypes.c_int]
        for name, a, b in (("oracle_expf_array", ctypes.c_void_p, ctypes.c_void_p),
                           ("oracle_f2h_array", ctypes.c_void_p, ctypes.c_void_p),
                           ("oracle_h2f_array", ctypes.c_void_p, ctypes.c_void_p)):
            fn = getattr(_lib, name)
            fn.restype = None
            fn.argtypes = [a, b, ctypes.c_size_t]
        _lib.oracle_farthest_neighbor.restype = None
        _lib.oracle_sh_basis_array.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t]
        _lib.oracle_sh_basis_array.restype = None
        _lib.oracle_farthest_neighbor.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                                  ctypes.c_uint32, ctypes.c_uint32, ctypes.c_void_p,
                                                  ctypes.c_void_p]
        _lib.oracle_render.restype = None
        _lib.oracle_render.argtypes = [ctypes.POINTER(Scene), ctypes.POINTER(Settings), ctypes.POINTER(Camera),
                                       ctypes.c_uint32, ctypes.c_void_p, ctypes.c_int]
        _lib.oracle_trace_backward.restype = None
        _lib.oracle_trace_backward.argtypes = [ctypes.POINTER(Scene), ctypes.POINTER(Settings),
                                               ctypes.POINTER(BwdIO), ctypes.c_int]
    return _lib


def _ptr(a):
    return None if a is None else a.ctypes.data


def _c(a, dtype):
    return None if a is None else np.ascontiguousarray(a, dtype=dtype)


def expf(x: float) -> float:
    return lib().oracle_expf(float(x))


def expf_array(x):
    x = np.ascontiguousarray(x, np.float32)
    y = np.empty_like(x)
    lib().oracle_expf_array(_ptr(x), _ptr(y), x.size)
    return y


def f2h_array(x):
    x = np.ascontiguousarray(x, np.float32)
    y = np.empty(x.shape, np.uint16)
    lib().oracle_f2h_array(_ptr(x), _ptr(y), x.size)
    return y


def h2f_array(h):
    h = np.ascontiguousarray(h, np.uint16)
    y = np.empty(h.shape, np.float32)
    lib().oracle_h2f_array(_ptr(h), _ptr(y), h.size)
    return y


def sh_basis(dirs):
    """[n, 16] SH basis (degree 3) of unit directions [n, 3], float32."""
    d = _c(dirs, np.float32).reshape(-1, 3)
    y = np.zeros((d.shape[0], 16), np.float32)
    lib().oracle_sh_basis_array(_ptr(d), _ptr(y), d.shape[0])
    return y


def farthest_neighbor(points, adjacency, offsets):
    p = _c(points, np.float32).reshape(-1, 3)
    adj = _c(adjacency, np.uint32).reshape(-1)
    off = _c(offsets, np.uint32).reshape(-1)
    idx = np.zeros(p.shape[0], np.uint32)
    rad = np.zeros(p.shape[0], np.float32)
    lib().oracle_farthest_neighbor(_ptr(p), _ptr(adj), _ptr(off), p.shape[0], adj.shape[0], _ptr(idx), _ptr(rad))
    return idx, rad


def f2h(x: float) -> int:
    return lib().oracle_f2h(float(x))


def h2f(h: int) -> float:
    return lib().oracle_h2f(int(h))


class OracleScene:
    """Holds contiguous numpy copies of a foam plus its fp16 neighbour diffs."""

    def __init__(self, points, attributes, adjacency, offsets, sh_degree: int):
        self.points = _c(points, np.float32).reshape(-1, 3)
        self.attributes = _c(attributes, np.float32)
        self.attributes = self.attributes.reshape(self.points.shape[0], -1)
        self.adjacency = _c(adjacency, np.uint32).reshape(-1)
        self.offsets = _c(offsets, np.uint32).reshape(-1)
        self.sh_degree = int(sh_degree)
        self.attr_dim = self.attributes.shape[1]
        assert self.attr_dim == 1 + 3 * (self.sh_degree + 1) ** 2
        self.diffs = np.zeros((self.adjacency.shape[0], 4), np.uint16)
        lib().oracle_build_diffs(self.points.shape[0], _ptr(self.points), _ptr(self.adjacency),
                                 _ptr(self.offsets), self.adjacency.shape[0], _ptr(self.diffs))
        self._c = Scene(self.points.shape[0], self.adjacency.shape[0], self.attr_dim,
                        self.sh_degree, _ptr(self.points), _ptr(self.attributes),
                        _ptr(self.adjacency), _ptr(self.offsets), _ptr(self.diffs))

    @property
    def num_points(self):
        return self.points.shape[0]


def settings(neus=True, sharpness=50.0, sdf_channel=None, attr_dim=49,
             weight_threshold=1e-7, max_intersections=1024):
    if sdf_channel is None:
        sdf_channel = attr_dim - 1 if neus else -1
    return Settings(float(weight_threshold), int(max_intersections), int(bool(neus)),
                    int(sdf_channel), float(sharpness))


def trace_forward(scene: OracleScene, st: Settings, rays, start, quantiles=None,
                  return_contribution=True, threads=0, record_sequences=False,
                  seq_capacity=None, ambiguity=False):
    """Returns a dict like Pipeline.trace_forward (numpy arrays).  With
    record_sequences, also the per-ray cell sequences (CSR) and alphas.  With
    ambiguity, also "ambiguous" (uint8 [R]): 1 for rays whose termination or
    quantile crossings could fall on another walk step under the reference's
    __expf, whose documented error bound is wider than this oracle's exp
    (exp_interval in sdfoam_oracle.c)."""
    rays = _c(rays, np.float32).reshape(-1, 6)
    start = _c(start, np.uint32).reshape(-1)
    R = rays.shape[0]
    Q = 0
    if quantiles is not None:
        quantiles = _c(quantiles, np.float32).reshape(R, -1)
        Q = quantiles.shape[1]
    N = scene.num_points
    out = {
        "rgba": np.zeros((R, 4), np.float32),
        "num_intersections": np.zeros((R,), np.uint32),
        "alpha": np.zeros((N,), np.float32),
    }
    if return_contribution:
        out["contribution"] = np.zeros((N,), np.float32)
    if quantiles is not None:
        out["depth"] = np.zeros((R, Q), np.float32)
        out["depth_indices"] = np.zeros((R, Q), np.uint32)
    if ambiguity:
        out["ambiguous"] = np.zeros((R,), np.uint8)
    seq_off = seq_cells = seq_alpha = seq_count = None
    if record_sequences:
        if seq_capacity is None:
            # first pass for the lengths
            first = trace_forward(scene, st, rays, start, quantiles, False, threads)
            seq_capacity = first["num_intersections"].astype(np.uint64)
        cap = np.asarray(seq_capacity, np.uint64).reshape(-1)
        seq_off = np.zeros(R + 1, np.uint64)
        np.cumsum(cap, out=seq_off[1:])
        seq_cells = np.full(int(seq_off[-1]), U32_NONE, np.uint32)
        seq_alpha = np.zeros(int(seq_off[-1]), np.float32)
        seq_count = np.zeros(R, np.uint32)
    io = FwdIO(R, _ptr(rays), _ptr(start), Q, _ptr(quantiles), _ptr(out["rgba"]),
               _ptr(out.get("depth")), _ptr(out.get("depth_indices")),
               _ptr(out["num_intersections"]), _ptr(out.get("contribution")),
               _ptr(out["alpha"]), _ptr(seq_off), _ptr(seq_cells), _ptr(seq_alpha),
               _ptr(seq_count), _ptr(out.get("ambiguous")))
    lib().oracle_trace_forward(ctypes.byref(scene._c), ctypes.byref(st), ctypes.byref(io),
                               int(threads))
    if record_sequences:
        out["seq_offsets"] = seq_off
        out["seq_cells"] = seq_cells
        out["seq_alpha"] = seq_alpha
        out["seq_count"] = seq_count
    return out


def trace_backward(scene: OracleScene, st: Settings, rays, start, rgba, rgba_grad,
                   quantiles=None, depth_indices=None, depth_grad=None, ray_error=None,
                   threads=0, with_abs=False):
    rays = _c(rays, np.float32).reshape(-1, 6)
    start = _c(start, np.uint32).reshape(-1)
    R = rays.shape[0]
    rgba = _c(rgba, np.float32).reshape(R, 4)
    rgba_grad = _c(rgba_grad, np.float32).reshape(R, 4)
    Q = 0
    if quantiles is not None:
        quantiles = _c(quantiles, np.float32).reshape(R, -1)
        Q = quantiles.shape[1]
        depth_grad = _c(depth_grad, np.float32).reshape(R, Q)
        depth_indices = _c(depth_indices, np.uint32).reshape(R, Q)
    if ray_error is not None:
        ray_error = _c(ray_error, np.float32).reshape(R)
    N, D = scene.num_points, scene.attr_dim
    out = {
        "points_grad": np.zeros((N, 3), np.float32),
        "attr_grad": np.zeros((N, D), np.float32),
        "sharpness_grad": np.zeros((1,), np.float32),
    }
    if ray_error is not None:
        out["point_error"] = np.zeros((N,), np.float32)
    if with_abs:
        out["points_grad_abs"] = np.zeros((N, 3), np.float32)
        out["attr_grad_abs"] = np.zeros((N, D), np.float32)
    io = BwdIO(R, _ptr(rays), _ptr(start), Q, _ptr(quantiles), _ptr(depth_indices),
               _ptr(rgba), _ptr(rgba_grad), _ptr(depth_grad), _ptr(ray_error),
               _ptr(out["points_grad"]), _ptr(out["attr_grad"]), _ptr(out.get("point_error")),
               _ptr(out["sharpness_grad"]), _ptr(out.get("points_grad_abs")),
               _ptr(out.get("attr_grad_abs")))
    lib().oracle_trace_backward(ctypes.byref(scene._c), ctypes.byref(st), ctypes.byref(io),
                                int(threads))
    return out


def render(scene: OracleScene, st: Settings, camera: dict, start: int, bg_color=(1.0, 1.0, 1.0),
           checker_bg=False, threads=0, diffs=None):
    """trace_benchmark's frame (pipeline.cu:1067-1199): uint32 [height * width]
    RGBA8, rows bottom-up.  diffs (binary16 [E, 4] bits) replaces the scene's
    own neighbour offsets, as the reference's adjacent_diff argument does."""
    c = Camera()
    for k in ("position", "forward", "right", "up"):
        getattr(c, k)[:] = [float(x) for x in np.asarray(camera[k], np.float32).reshape(-1)[:3]]
    c.fov = float(camera["fov"])
    c.width = int(camera["width"])
    c.height = int(camera["height"])
    c.model = {"pinhole": 0, "fisheye": 1}[camera["model"]]
    c.bg[:] = [float(x) for x in bg_color]
    c.checker = 1 if checker_bg else 0
    out = np.zeros(c.width * c.height, np.uint32)
    sc = scene._c
    if diffs is not None:
        d = _c(diffs, np.uint16).reshape(-1, 4)
        sc = Scene(sc.num_points, sc.adjacency_size, sc.attr_dim, sc.sh_degree, sc.points, sc.attributes,
                   sc.adjacency, sc.offsets, _ptr(d))
    lib().oracle_render(ctypes.byref(sc), ctypes.byref(st), ctypes.byref(c), int(start), _ptr(out), int(threads))
    return out
