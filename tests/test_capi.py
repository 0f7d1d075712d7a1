"""CPU checks of the C-ABI boundary: the library loads, exports every entry
point include/sdfoam_b200.h declares, sizes its workspaces, and rejects bad
arguments with the reference's messages -- all without touching a GPU."""
import ctypes
import os
import re

import pytest
import torch

from sdfoam_b200 import _lib, build

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "sdfoam_b200.h")


@pytest.fixture(scope="module")
def lib():
    build.build()
    return _lib.load()


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(sdfoam_\w+)\s*\(", text)))


def test_header_declares_python_bound_symbols():
    assert declared_functions() == sorted(_lib.EXPORTED)


def test_library_exports_every_declared_symbol(lib):
    for name in declared_functions():
        assert hasattr(lib, name), name
    assert lib.sdfoam_abi_version() == 5


def test_workspace_sizes(lib):
    def align(x):
        return (x + 255) // 256 * 256
    n, e = 1000, 15000
    # site records: 32-byte head + SH row rounded to 128-byte lines; then
    # 16-byte face records; then 8-byte plane records, E + 3N + 8 slots
    # rounded to 4
    planes = (e + 3 * n + 8 + 3) // 4 * 4
    for deg, site_bytes in ((3, 256), (2, 256), (1, 128), (0, 128)):
        assert lib.sdfoam_cells_bytes(n, e, deg) == align(align(align(n * site_bytes) + e * 16) + planes * 8)
    assert lib.sdfoam_cells_bytes(n, e, 4) == 0
    # plane rows are addressed in 32 bits
    assert lib.sdfoam_cells_bytes(1 << 30, (1 << 32) - 1 - 3 * (1 << 30) - 8, 0) > 0
    assert lib.sdfoam_cells_bytes(1 << 30, (1 << 32) - 3 * (1 << 30) - 8, 0) == 0
    assert lib.sdfoam_backward_workspace_bytes(n, 3) == align(align(n * 13 * 16) + n * 16)


def test_invalid_arguments_are_reported_without_a_gpu(lib):
    rc = lib.sdfoam_build_cells(None, None, 0, None)
    assert rc == 1 and lib.sdfoam_last_error() == b"foam is NULL"
    foam = _lib.Foam(10, 20, 4, _lib.SDFOAM_F32, 8, 8, 8, 8)
    rc = lib.sdfoam_build_cells(ctypes.byref(foam), ctypes.c_void_p(256), 1 << 20, None)
    assert rc == 2 and lib.sdfoam_last_error() == b"Unsupported SH degree"
    foam.sh_degree = 3
    foam.attr_dtype = 7
    rc = lib.sdfoam_build_cells(ctypes.byref(foam), ctypes.c_void_p(256), 1 << 20, None)
    assert rc == 2 and lib.sdfoam_last_error() == b"Unsupported attribute type"
    foam.attr_dtype = _lib.SDFOAM_F32
    rc = lib.sdfoam_build_cells(ctypes.byref(foam), ctypes.c_void_p(256), 16, None)
    assert rc == 1 and b"workspace too small" in lib.sdfoam_last_error()
    # the walk reads cell records with 256-bit loads
    rc = lib.sdfoam_build_cells(ctypes.byref(foam), ctypes.c_void_p(272), 1 << 20, None)
    assert rc == 1 and lib.sdfoam_last_error() == b"cells must be 32-byte aligned"
    # plane rows are addressed in 32 bits
    big = _lib.Foam(1 << 30, (1 << 32) - 3 * (1 << 30) - 8, 3, _lib.SDFOAM_F32, 8, 8, 8, 8)
    rc = lib.sdfoam_build_cells(ctypes.byref(big), ctypes.c_void_p(256), 1 << 20, None)
    assert rc == 1 and b"foam too large" in lib.sdfoam_last_error()
    st = _lib.TraceSettings(1e-7, 1024, 1, 49, 1e-6)
    rc = lib.sdfoam_trace_forward(ctypes.byref(foam), ctypes.c_void_p(256), ctypes.byref(st), None, None)
    assert rc == 1 and b"sdf_channel" in lib.sdfoam_last_error()
    with pytest.raises(RuntimeError, match="sdf_channel"):
        _lib.check(1)


def test_mlp_stage_arguments_are_checked_without_a_gpu(lib):
    p = ctypes.c_void_p(256)
    # activate: 256 softplus columns + 1 bias column do not fit a 256-wide row
    rc = lib.sdfoam_mlp_activate(p, 256, 256, 10, None, 0, 0, 1.0, 256, p, None)
    assert rc == 1 and lib.sdfoam_last_error() == b"inconsistent row widths"
    # rows must be whole 16-byte vectors
    rc = lib.sdfoam_mlp_activate(p, 252, 217, 10, None, 0, 0, 1.0, 264, p, None)
    assert rc == 1 and b"multiples of 8" in lib.sdfoam_last_error()
    rc = lib.sdfoam_mlp_activate(ctypes.c_void_p(258), 256, 256, 10, None, 0, 0, 1.0, 264, p, None)
    assert rc == 1 and b"16-byte aligned" in lib.sdfoam_last_error()
    rc = lib.sdfoam_mlp_activate(p, 256, 217, 10, None, 48, 39, 1.0, 264, p, None)
    assert rc == 1 and b"enc" in lib.sdfoam_last_error()
    # tcgen05 layers: at most 320 input columns forward, 256 backward
    rc = lib.sdfoam_mlp_layer(p, 328, 328, 10, p, 328, 256, None, 0, 0, 256, 1.0, p, 264, p, None)
    assert rc == 1 and lib.sdfoam_last_error() == b"inconsistent layer shapes"
    rc = lib.sdfoam_mlp_layer_backward(p, 264, 264, 10, p, 264, 256, p, 264, 256, 1.0, p, 256, None, 0, p, None)
    assert rc == 1 and lib.sdfoam_last_error() == b"inconsistent layer shapes"
    # deactivate: dz wider than the activation rows, a non-positive scale
    rc = lib.sdfoam_mlp_deactivate(p, 264, p, 224, 1.0, 10, 217, p, 256, None)
    assert rc == 1 and lib.sdfoam_last_error() == b"inconsistent row widths"
    rc = lib.sdfoam_mlp_deactivate(p, 264, p, 264, 0.0, 10, 217, p, 224, None)
    assert rc == 1 and lib.sdfoam_last_error() == b"inconsistent row widths"
    rc = lib.sdfoam_mlp_encode(p, None, 10, 6, 32, p, None)
    assert rc == 1 and lib.sdfoam_last_error() == b"encoding row too short"
    # the output dot needs the plain 256-column hidden layer
    rc = lib.sdfoam_mlp_layer_dot(p, 264, 264, 10, p, 264, 224, p, 48, 39, 217, 1.0, p, 264, p, p, 1.0, p, None)
    assert rc == 1 and b"output dot" in lib.sdfoam_last_error()
    # weight gradients: k a multiple of 4 that fits dw, a bias column past k
    rc = lib.sdfoam_mlp_wgrad(p, 256, 256, 10, p, 264, 258, p, 264, -1, p, None)
    assert rc == 1 and lib.sdfoam_last_error() == b"inconsistent weight-gradient shapes"
    rc = lib.sdfoam_mlp_wgrad(p, 256, 256, 10, p, 264, 256, p, 264, 100, p, None)
    assert rc == 1 and lib.sdfoam_last_error() == b"inconsistent weight-gradient shapes"
    rc = lib.sdfoam_mlp_wgrad(p, 256, 257, 10, p, 264, 256, p, 264, 256, p, None)
    assert rc == 1 and lib.sdfoam_last_error() == b"inconsistent weight-gradient shapes"
    # input gradient: the addend wider than the output
    rc = lib.sdfoam_mlp_input_grad(p, 256, 256, 10, p, 256, 48, p, 64, 56, p, 48, p, None)
    assert rc == 1 and lib.sdfoam_last_error() == b"inconsistent input-gradient shapes"
    # eikonal sweeps: the tangent's output at most 256 wide, its derivative
    # columns within the weight rows; the second sweep's dz narrower than cols
    rc = lib.sdfoam_mlp_layer_tangent(p, 256, 256, 10, p, 264, 224, p, 264, 256, 1.0, None, 48, 0, p, 256, p, 256,
                                      p, None)
    assert rc == 1 and lib.sdfoam_last_error() == b"inconsistent tangent-layer shapes"
    rc = lib.sdfoam_mlp_layer_second(p, 256, 256, 10, p, 256, 256, p, 264, 256, 1.0, p, 224, p, 256, p, 256, None,
                                     0, p, None)
    assert rc == 1 and lib.sdfoam_last_error() == b"inconsistent second-sweep shapes"
    rc = lib.sdfoam_mlp_encode_jvp(p, None, 10, 6, p, 32, p, None)
    assert rc == 1 and b"ld too small" in lib.sdfoam_last_error()


def test_python_surface_validates_on_host(lib):
    import sdfoam_b200 as sdfoam
    with pytest.raises(RuntimeError, match="Unsupported SH degree"):
        sdfoam.create_pipeline(5)
    with pytest.raises(RuntimeError, match="Unsupported attribute type"):
        sdfoam.create_pipeline(3, "float64")
    with pytest.raises(RuntimeError, match="unsupported dtype 'int8'"):
        sdfoam.create_pipeline(3, "int8")
    pipe = sdfoam.create_pipeline(3, "torch.float32")
    assert pipe.attribute_dim() == 49 and pipe.attribute_type() == torch.float32
    assert pipe in sdfoam.pipeline_registry
    pts = torch.zeros(40, 3)
    att = torch.zeros(40, 49)
    adj = torch.zeros(10, dtype=torch.uint32)
    off = torch.zeros(41, dtype=torch.uint32)
    rays = torch.zeros(5, 6)
    start = torch.zeros(5, dtype=torch.uint32)
    with pytest.raises(RuntimeError, match="points must be on CUDA device"):
        pipe.trace_forward(pts, att, adj, off, rays, start)


def test_sort_points_workspace_and_errors(lib):
    def align(x):
        return (x + 255) // 256 * 256
    assert lib.sdfoam_sort_points_workspace_bytes(0) == 0
    # no radix rounds up to 1024 sites: four key / permutation arrays only
    assert lib.sdfoam_sort_points_workspace_bytes(1000) == 4 * align(4000)
    # 5000 sites: three global rounds over ceil(5000 / 2048) = 3 tiles: digit
    # counts per tile, then one unit's 256 digit totals
    assert lib.sdfoam_sort_points_workspace_bytes(5000) == 4 * align(20000) + align(256 * 3 * 4) + align(256 * 4)
    p = ctypes.c_void_p(4096)
    rc = lib.sdfoam_sort_points(p, 100, ctypes.c_void_p(4096 + 600), p, p, 1 << 20, None)
    assert rc == 1 and lib.sdfoam_last_error() == b"sorted_points must not overlap points"
    rc = lib.sdfoam_sort_points(p, 100, ctypes.c_void_p(1 << 20), p, p, 16, None)
    assert rc == 1 and b"sort workspace" in lib.sdfoam_last_error()
    assert lib.sdfoam_sort_points(None, 0, None, None, None, 0, None) == 0


def test_tets_arguments_are_checked_without_a_gpu(lib):
    assert lib.sdfoam_delaunay_tets_workspace_bytes(31, 0) == 0
    small = lib.sdfoam_delaunay_tets_workspace_bytes(1000, 0)
    # 16-byte face records: four per tet
    assert lib.sdfoam_delaunay_tets_workspace_bytes(1000, 100) == small + 100 * 4 * 16
    status = (ctypes.c_uint32 * 4)()
    count = ctypes.c_uint32(0)
    p = ctypes.c_void_p(4096)
    rc = lib.sdfoam_delaunay_tets_count(p, 20, p, 10, p, p, 1 << 30, ctypes.byref(count), status, None)
    assert rc == 1 and b"32 to 2^27 points" in lib.sdfoam_last_error()
    rc = lib.sdfoam_delaunay_tets_count(p, 1000, p, 10, p, p, 16, ctypes.byref(count), status, None)
    assert rc == 1 and b"workspace too small" in lib.sdfoam_last_error()
    rc = lib.sdfoam_delaunay_tets_count(p, 1000, p, 10, None, p, small, ctypes.byref(count), status, None)
    assert rc == 1 and b"non-NULL" in lib.sdfoam_last_error()
    rc = lib.sdfoam_delaunay_tets(p, 1000, p, 10, p, p, small + 6400, 100, ctypes.c_void_p(4104), p, p, status,
                                  None)
    assert rc == 1 and lib.sdfoam_last_error() == b"tets must be 16-byte aligned"
