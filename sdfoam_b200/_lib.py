"""ctypes binding of libsdfoam_b200.so (declarations: include/sdfoam_b200.h).

The library is required: importing the tracer without it raises, there is no
CPU fallback.
"""
from __future__ import annotations

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
# SDFOAM_B200_LIB selects another build of the same library (same ABI).
LIB_PATH = os.environ.get("SDFOAM_B200_LIB") or os.path.join(HERE, "libsdfoam_b200.so")

SDFOAM_OK = 0
SDFOAM_F32 = 0
SDFOAM_F16 = 1
SDFOAM_ALPHA_STANDARD = 0
SDFOAM_ALPHA_NEUS = 1
SDFOAM_PINHOLE = 0
SDFOAM_FISHEYE = 1

EXPORTED = (
    "sdfoam_cells_bytes",
    "sdfoam_build_cells",
    "sdfoam_trace_forward",
    "sdfoam_backward_workspace_bytes",
    "sdfoam_trace_backward",
    "sdfoam_last_error",
    "sdfoam_abi_version",
    "sdfoam_trace_forward_noalloc",
    "sdfoam_aabb_tree_nodes",
    "sdfoam_build_aabb_tree",
    "sdfoam_nn",
    "sdfoam_farthest_neighbor",
    "sdfoam_sort_points_workspace_bytes",
    "sdfoam_sort_points",
    "sdfoam_build_cells_from_diffs",
    "sdfoam_trace_benchmark",
    "sdfoam_delaunay_workspace_bytes",
    "sdfoam_delaunay_neighbors",
    "sdfoam_delaunay_status",
    "sdfoam_delaunay_adjacency",
    "sdfoam_delaunay_tets_workspace_bytes",
    "sdfoam_delaunay_tets_count",
    "sdfoam_delaunay_tets",
    "sdfoam_mlp_layer",
    "sdfoam_mlp_layer_backward",
    "sdfoam_mlp_layer_dot",
    "sdfoam_mlp_wgrad",
    "sdfoam_mlp_input_grad",
    "sdfoam_mlp_layer_tangent",
    "sdfoam_mlp_layer_second",
    "sdfoam_mlp_encode_jvp",
    "sdfoam_mlp_decode_hessian",
    "sdfoam_mlp_encode",
    "sdfoam_mlp_activate",
    "sdfoam_mlp_deactivate",
    "sdfoam_mlp_decode",
)


class Foam(ctypes.Structure):
    _fields_ = [
        ("num_points", ctypes.c_uint32),
        ("adjacency_size", ctypes.c_uint32),
        ("sh_degree", ctypes.c_uint32),
        ("attr_dtype", ctypes.c_uint32),
        ("points", ctypes.c_void_p),
        ("attributes", ctypes.c_void_p),
        ("point_adjacency", ctypes.c_void_p),
        ("point_adjacency_offsets", ctypes.c_void_p),
    ]


class TraceSettings(ctypes.Structure):
    _fields_ = [
        ("weight_threshold", ctypes.c_float),
        ("max_intersections", ctypes.c_uint32),
        ("alpha_mode", ctypes.c_uint32),
        ("sdf_channel", ctypes.c_int32),
        ("eps", ctypes.c_float),
    ]


class ForwardIO(ctypes.Structure):
    _fields_ = [
        ("num_rays", ctypes.c_uint32),
        ("rays", ctypes.c_void_p),
        ("start_point", ctypes.c_void_p),
        ("num_depth_quantiles", ctypes.c_uint32),
        ("depth_quantiles", ctypes.c_void_p),
        ("sharpness", ctypes.c_void_p),
        ("ray_rgba", ctypes.c_void_p),
        ("depth", ctypes.c_void_p),
        ("depth_indices", ctypes.c_void_p),
        ("num_intersections", ctypes.c_void_p),
        ("point_contribution", ctypes.c_void_p),
        ("alpha", ctypes.c_void_p),
        ("seq_offsets", ctypes.c_void_p),
        ("seq_cells", ctypes.c_void_p),
        ("seq_count", ctypes.c_void_p),
        ("face_tests", ctypes.c_void_p),
        ("exits", ctypes.c_void_p),
        ("exits_stride", ctypes.c_uint32),
        ("step_colors", ctypes.c_void_p),
        ("step_colors_steps", ctypes.c_uint32),
        ("step_sites", ctypes.c_void_p),
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
    ]


class BackwardIO(ctypes.Structure):
    _fields_ = [
        ("num_rays", ctypes.c_uint32),
        ("rays", ctypes.c_void_p),
        ("start_point", ctypes.c_void_p),
        ("num_depth_quantiles", ctypes.c_uint32),
        ("depth_quantiles", ctypes.c_void_p),
        ("depth_indices", ctypes.c_void_p),
        ("ray_rgba", ctypes.c_void_p),
        ("ray_rgba_grad", ctypes.c_void_p),
        ("depth_grad", ctypes.c_void_p),
        ("ray_error", ctypes.c_void_p),
        ("sharpness", ctypes.c_void_p),
        ("points_grad", ctypes.c_void_p),
        ("attr_grad", ctypes.c_void_p),
        ("point_error", ctypes.c_void_p),
        ("sharpness_grad", ctypes.c_void_p),
        ("workspace", ctypes.c_void_p),
        ("workspace_bytes", ctypes.c_size_t),
        ("exits", ctypes.c_void_p),
        ("exits_stride", ctypes.c_uint32),
        ("step_colors", ctypes.c_void_p),
        ("step_colors_steps", ctypes.c_uint32),
        ("step_sites", ctypes.c_void_p),
    ]


_lib = None


def load():
    """Loads the library (building it first if the sources are newer)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise RuntimeError(
            f"{LIB_PATH} is missing: build it with `python -m sdfoam_b200.build` "
            "(the tracer has no CPU fallback)")
    lib = ctypes.CDLL(LIB_PATH)
    lib.sdfoam_cells_bytes.restype = ctypes.c_size_t
    lib.sdfoam_cells_bytes.argtypes = [ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint32]
    lib.sdfoam_build_cells.restype = ctypes.c_int
    lib.sdfoam_build_cells.argtypes = [ctypes.POINTER(Foam), ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p]
    lib.sdfoam_trace_forward.restype = ctypes.c_int
    lib.sdfoam_trace_forward.argtypes = [ctypes.POINTER(Foam), ctypes.c_void_p, ctypes.POINTER(TraceSettings),
                                         ctypes.POINTER(ForwardIO), ctypes.c_void_p]
    lib.sdfoam_backward_workspace_bytes.restype = ctypes.c_size_t
    lib.sdfoam_backward_workspace_bytes.argtypes = [ctypes.c_uint32, ctypes.c_uint32]
    lib.sdfoam_trace_backward.restype = ctypes.c_int
    lib.sdfoam_trace_backward.argtypes = [ctypes.POINTER(Foam), ctypes.c_void_p, ctypes.POINTER(TraceSettings),
                                          ctypes.POINTER(BackwardIO), ctypes.c_void_p]
    lib.sdfoam_last_error.restype = ctypes.c_char_p
    lib.sdfoam_last_error.argtypes = []
    lib.sdfoam_abi_version.restype = ctypes.c_int
    lib.sdfoam_abi_version.argtypes = []
    lib.sdfoam_trace_forward_noalloc.restype = ctypes.c_int
    lib.sdfoam_trace_forward_noalloc.argtypes = [ctypes.POINTER(Foam), ctypes.POINTER(TraceSettings),
                                                 ctypes.POINTER(ForwardIO), ctypes.c_void_p]
    lib.sdfoam_aabb_tree_nodes.restype = ctypes.c_uint32
    lib.sdfoam_aabb_tree_nodes.argtypes = [ctypes.c_uint32]
    lib.sdfoam_build_aabb_tree.restype = ctypes.c_int
    lib.sdfoam_build_aabb_tree.argtypes = [ctypes.c_void_p, ctypes.c_uint32, ctypes.c_void_p, ctypes.c_void_p]
    lib.sdfoam_nn.restype = ctypes.c_int
    lib.sdfoam_nn.argtypes = [ctypes.c_void_p, ctypes.c_uint32, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_uint32,
                              ctypes.c_void_p, ctypes.c_void_p]
    lib.sdfoam_farthest_neighbor.restype = ctypes.c_int
    lib.sdfoam_farthest_neighbor.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_uint32,
                                             ctypes.c_uint32, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
    vp, u32, i32, f32 = ctypes.c_void_p, ctypes.c_uint32, ctypes.c_int, ctypes.c_float
    lib.sdfoam_sort_points_workspace_bytes.restype = ctypes.c_size_t
    lib.sdfoam_sort_points_workspace_bytes.argtypes = [u32]
    lib.sdfoam_sort_points.restype = ctypes.c_int
    lib.sdfoam_sort_points.argtypes = [vp, u32, vp, vp, vp, ctypes.c_size_t, vp]
    lib.sdfoam_delaunay_workspace_bytes.restype = ctypes.c_size_t
    lib.sdfoam_delaunay_workspace_bytes.argtypes = [u32]
    lib.sdfoam_delaunay_neighbors.restype = ctypes.c_int
    lib.sdfoam_delaunay_neighbors.argtypes = [vp, u32, vp, vp, ctypes.c_size_t, vp, vp]
    lib.sdfoam_delaunay_status.restype = ctypes.c_int
    lib.sdfoam_delaunay_status.argtypes = [vp, u32, ctypes.POINTER(ctypes.c_uint32), vp]
    lib.sdfoam_delaunay_adjacency.restype = ctypes.c_int
    lib.sdfoam_delaunay_adjacency.argtypes = [vp, u32, vp, u32, vp]
    lib.sdfoam_delaunay_tets_workspace_bytes.restype = ctypes.c_size_t
    lib.sdfoam_delaunay_tets_workspace_bytes.argtypes = [u32, u32]
    u32p = ctypes.POINTER(ctypes.c_uint32)
    lib.sdfoam_delaunay_tets_count.restype = ctypes.c_int
    lib.sdfoam_delaunay_tets_count.argtypes = [vp, u32, vp, u32, vp, vp, ctypes.c_size_t, u32p, u32p, vp]
    lib.sdfoam_delaunay_tets.restype = ctypes.c_int
    lib.sdfoam_delaunay_tets.argtypes = [vp, u32, vp, u32, vp, vp, ctypes.c_size_t, u32, vp, vp, vp, u32p, vp]
    lib.sdfoam_build_cells_from_diffs.restype = ctypes.c_int
    lib.sdfoam_build_cells_from_diffs.argtypes = [ctypes.POINTER(Foam), vp, vp, ctypes.c_size_t, vp]
    lib.sdfoam_trace_benchmark.restype = ctypes.c_int
    lib.sdfoam_trace_benchmark.argtypes = [ctypes.POINTER(Foam), vp, ctypes.POINTER(TraceSettings),
                                           ctypes.POINTER(Camera), vp, vp, ctypes.POINTER(ctypes.c_float), i32, vp,
                                           vp]
    for name, args in (("sdfoam_mlp_layer", [vp, i32, i32, u32, vp, i32, i32, vp, i32, i32, i32, f32, vp, i32, vp, vp]),
                       ("sdfoam_mlp_layer_backward",
                        [vp, i32, i32, u32, vp, i32, i32, vp, i32, i32, f32, vp, i32, vp, i32, vp, vp]),
                       ("sdfoam_mlp_layer_dot",
                        [vp, i32, i32, u32, vp, i32, i32, vp, i32, i32, i32, f32, vp, i32, vp, vp, f32, vp, vp]),
                       ("sdfoam_mlp_wgrad", [vp, i32, i32, u32, vp, i32, i32, vp, i32, i32, vp, vp]),
                       ("sdfoam_mlp_input_grad", [vp, i32, i32, u32, vp, i32, i32, vp, i32, i32, vp, i32, vp, vp]),
                       ("sdfoam_mlp_layer_tangent",
                        [vp, i32, i32, u32, vp, i32, i32, vp, i32, i32, f32, vp, i32, i32, vp, i32, vp, i32, vp, vp]),
                       ("sdfoam_mlp_layer_second",
                        [vp, i32, i32, u32, vp, i32, i32, vp, i32, i32, f32, vp, i32, vp, i32, vp, i32, vp, i32, vp,
                         vp]),
                       ("sdfoam_mlp_encode_jvp", [vp, vp, u32, i32, vp, i32, vp, vp]),
                       ("sdfoam_mlp_decode_hessian", [vp, vp, u32, i32, vp, vp, i32, vp, vp, vp]),
                       ("sdfoam_mlp_encode", [vp, vp, u32, i32, i32, vp, vp]),
                       ("sdfoam_mlp_activate", [vp, i32, i32, u32, vp, i32, i32, f32, i32, vp, vp]),
                       ("sdfoam_mlp_deactivate", [vp, i32, vp, i32, f32, u32, i32, vp, i32, vp]),
                       ("sdfoam_mlp_decode", [vp, vp, u32, i32, vp, i32, vp, vp])):
        fn = getattr(lib, name)
        fn.restype = ctypes.c_int
        fn.argtypes = args
    _lib = lib
    return lib


def check(rc: int) -> None:
    if rc != SDFOAM_OK:
        msg = load().sdfoam_last_error().decode("utf-8", "replace")
        raise RuntimeError(msg)
