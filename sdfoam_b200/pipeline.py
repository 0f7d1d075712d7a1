"""Host-side mirror of the reference's tracing-pipeline operator surface.

Same names, arguments, defaults, output dictionaries and error messages as the
reference's pybind module (torch_bindings/pipeline_bindings.cpp:138-334,
336-607, 734-751, 799-860); the work is done by libsdfoam_b200.so through its
C ABI on the current CUDA stream.  Differences that callers can observe:

* ``attr_grad`` / ``points_grad`` are written completely by the library, so
  they are allocated empty rather than zeroed.
* ``inv_s`` is never read back to the host (the reference calls ``.item()`` on
  it, pipeline_bindings.cpp:231, which synchronises the device; its kernels
  never use that value).
* ``cells=`` (keyword only) accepts the records of :meth:`Pipeline.build_cells`
  so a forward and its backward share one build.
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib

_ATTR_TYPES = {
    "float32": torch.float32, "torch.float32": torch.float32,
    "float16": torch.float16, "torch.float16": torch.float16,
    "float64": torch.float64, "torch.float64": torch.float64,
}

_NEUS_NAMES = ("sdfoam", "sdf", "alpha_neus")

# Pipelines stay alive for the life of the module, like the reference's
# pipeline_registry (pipeline_bindings.cpp:10, 747-751).
pipeline_registry: list = []


def _ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream(device):
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _dtype_name(dt):
    return str(dt).replace("torch.", "")


def inv_s_to_tensor(inv_s, like: torch.Tensor) -> torch.Tensor:
    """pipeline_bindings.cpp:124-136: None -> ones(1) float32; otherwise a
    contiguous float32 tensor on the device of ``like``."""
    if inv_s is None:
        return torch.ones((1,), dtype=torch.float32, device=like.device)
    if not isinstance(inv_s, torch.Tensor):
        inv_s = torch.tensor([float(inv_s)], dtype=torch.float32)
    s = inv_s.contiguous()
    if s.device != like.device or s.dtype != torch.float32:
        s = s.to(like.device, torch.float32).contiguous()
    return s


class Pipeline:
    """One (sh_degree, attribute dtype) entry of create_pipeline's dispatch
    table (src/tracing/pipeline.cu:1477-1506)."""

    def __init__(self, sh_degree: int, attr_type: torch.dtype):
        if sh_degree not in (0, 1, 2, 3):
            raise RuntimeError("Unsupported SH degree")
        if attr_type not in (torch.float32, torch.float16):
            raise RuntimeError("Unsupported attribute type")
        self.sh_degree = int(sh_degree)
        self._attr_type = attr_type
        self._lib = _lib.load()
        # TraceRays: walk the rays of a batch in coherent order (by start site
        # and direction) and return the results in the caller's order; off by
        # default (render.coherent_order)
        self.sort_rays = False
        # The step cap used when a call passes max_intersections=None (the
        # reference's default 1024 while this is None).  TraceRays passes
        # None, so this is how a training step reaches another cap.
        self.max_intersections = None

    # -- reference accessors ------------------------------------------------
    def attribute_dim(self) -> int:
        return 1 + 3 * (1 + self.sh_degree) * (1 + self.sh_degree)

    def attribute_type(self) -> torch.dtype:
        return self._attr_type

    # -- validation (pipeline_bindings.cpp:12-75) -----------------------------
    def _validate_scene(self, points, attributes, point_adjacency, point_adjacency_offsets):
        if points.size(-1) != 3:
            raise RuntimeError(f"points had dimension {points.size(-1)} along axis -1, expected 3")
        if points.dtype != torch.float32:
            raise RuntimeError(f"points had dtype {_dtype_name(points.dtype)}, expected float32")
        if points.device.type != "cuda":
            raise RuntimeError("points must be on CUDA device")
        num_points = points.numel() // 3
        A = self.attribute_dim()
        if attributes.size(-1) != A:
            raise RuntimeError(f"attributes had dimension {attributes.size(-1)} along axis -1, expected {A}")
        if attributes.numel() // A != num_points:
            raise RuntimeError("attributes must have the same number of rows as points")
        if attributes.dtype != self._attr_type:
            raise RuntimeError(f"attributes had dtype {_dtype_name(attributes.dtype)}, "
                               f"expected {_dtype_name(self._attr_type)}")
        if attributes.device.type != "cuda":
            raise RuntimeError("attributes must be on CUDA device")
        if point_adjacency_offsets.dtype != torch.uint32:
            raise RuntimeError("point_adjacency_offsets must have uint32 dtype")
        if point_adjacency_offsets.device.type != "cuda":
            raise RuntimeError("point_adjacency_offsets must be on CUDA device")
        if point_adjacency_offsets.numel() != num_points + 1:
            raise RuntimeError("point_adjacency_offsets must have num_points + 1 elements")
        if point_adjacency.dtype != torch.uint32:
            raise RuntimeError("point_adjacency must have uint32 dtype")
        if point_adjacency.device.type != "cuda":
            raise RuntimeError("point_adjacency must be on CUDA device")

    def _check_rays(self, rays, start_point, num_rays):
        if rays.size(-1) != 6:
            raise RuntimeError("rays must have 6 as the last dimension")
        if rays.dtype != torch.float32:
            raise RuntimeError("rays must have float32 dtype")
        if rays.device.type != "cuda":
            raise RuntimeError("rays must be on CUDA device")
        if start_point.numel() != num_rays:
            raise RuntimeError("start_point must have the same batch size as rays")
        if start_point.dtype != torch.uint32:
            raise RuntimeError("start_point must have uint32 dtype")
        if start_point.device.type != "cuda":
            raise RuntimeError("start_point must be on CUDA device")

    def _settings(self, weight_threshold, max_intersections, alpha_mode, eps, sdf_channel):
        s = _lib.TraceSettings(1e-7, 1024, _lib.SDFOAM_ALPHA_STANDARD, -1, 1e-6)
        if weight_threshold is not None:
            s.weight_threshold = float(weight_threshold)
        if max_intersections is not None:
            s.max_intersections = int(max_intersections)
        elif self.max_intersections is not None:
            s.max_intersections = int(self.max_intersections)
        if alpha_mode is not None:
            s.alpha_mode = (_lib.SDFOAM_ALPHA_NEUS if str(alpha_mode).lower() in _NEUS_NAMES
                            else _lib.SDFOAM_ALPHA_STANDARD)
        if eps is not None:
            s.eps = float(eps)
        if sdf_channel is not None:
            s.sdf_channel = int(sdf_channel)
        elif s.alpha_mode == _lib.SDFOAM_ALPHA_NEUS:
            s.sdf_channel = self.attribute_dim() - 1
        return s

    @staticmethod
    def _check_colors(colors, num_rays, sites=None):
        if colors is not None and (colors.dtype != torch.float32 or colors.dim() != 3 or colors.shape[1] != num_rays
                                   or colors.shape[2] != 4 or not colors.is_contiguous()
                                   or colors.device.type != "cuda"):
            raise RuntimeError("colors must be a contiguous CUDA float32 [steps, num_rays, 4] buffer "
                               "(Pipeline.color_record)")
        if sites is not None and (colors is None or sites.dtype != torch.uint32 or sites.dim() != 2
                                  or tuple(sites.shape) != tuple(colors.shape[:2]) or not sites.is_contiguous()
                                  or sites.device.type != "cuda"):
            raise RuntimeError("sites must be a contiguous CUDA uint32 [steps, num_rays] buffer matching colors "
                               "(Pipeline.site_record)")

    def _foam(self, points, attributes, point_adjacency, point_adjacency_offsets):
        dtype = _lib.SDFOAM_F16 if self._attr_type == torch.float16 else _lib.SDFOAM_F32
        return _lib.Foam(points.numel() // 3, point_adjacency.numel(), self.sh_degree, dtype,
                         points.data_ptr(), attributes.data_ptr(), point_adjacency.data_ptr(),
                         point_adjacency_offsets.data_ptr())

    # -- exit record (forward -> NeuS backward) --------------------------------
    @staticmethod
    def exit_record(num_rays: int, steps: int, device) -> torch.Tensor:
        """A buffer for trace_forward(..., exits=e) / trace_backward(...,
        exits=e): one byte per walk step for the first `steps` steps of each
        ray (rounded up to 8).  With it the NeuS backward replays the
        forward's exit faces instead of searching again; results are equal."""
        stride = (max(8, steps) + 7) // 8 * 8
        return torch.empty((num_rays, stride), dtype=torch.uint8, device=device)

    @staticmethod
    def color_record(num_rays: int, steps: int, device) -> torch.Tensor:
        """A buffer for trace_forward(..., colors=c) / trace_backward(...,
        colors=c): the SH colour and the exit distance of each of the first
        `steps` walk steps of every ray, step-major [steps, num_rays, 4]
        float32.  With it the NeuS backward reads each step's colour
        (coalesced) instead of gathering and evaluating the site's SH row;
        results are equal."""
        return torch.empty((max(1, steps), num_rays, 4), dtype=torch.float32, device=device)

    @staticmethod
    def site_record(num_rays: int, steps: int, device) -> torch.Tensor:
        """A buffer for trace_forward(..., colors=c, sites=s) /
        trace_backward(..., colors=c, sites=s): the site each of the first
        `steps` walk steps of every ray entered, step-major [steps, num_rays]
        uint32.  With it (and the colour record) the NeuS backward replays
        those steps without testing their exit faces again; results are
        equal."""
        return torch.empty((max(1, steps), num_rays), dtype=torch.uint32, device=device)

    # -- cell records (replaces prefetch_adjacent_diff) -----------------------
    def build_cells(self, points, attributes, point_adjacency, point_adjacency_offsets) -> torch.Tensor:
        points = points.contiguous()
        attributes = attributes.contiguous()
        point_adjacency = point_adjacency.contiguous()
        point_adjacency_offsets = point_adjacency_offsets.contiguous()
        self._validate_scene(points, attributes, point_adjacency, point_adjacency_offsets)
        foam = self._foam(points, attributes, point_adjacency, point_adjacency_offsets)
        nbytes = self._lib.sdfoam_cells_bytes(foam.num_points, foam.adjacency_size, self.sh_degree)
        cells = torch.empty((nbytes,), dtype=torch.uint8, device=points.device)
        with torch.cuda.device(points.device):
            _lib.check(self._lib.sdfoam_build_cells(ctypes.byref(foam), _ptr(cells), nbytes,
                                                    _stream(points.device)))
        return cells

    # -- forward (pipeline_bindings.cpp:138-334) ------------------------------
    def trace_forward(self, points, attributes, point_adjacency, point_adjacency_offsets, rays, start_point,
                      depth_quantiles=None, weight_threshold=None, max_intersections=None,
                      return_contribution=False, alpha_mode=None, inv_s=None, eps=None, sdf_channel=None,
                      *, cells=None, exits=None, colors=None, sites=None, _sequences=None, _face_tests=None):
        points_c = points.contiguous()
        attributes_c = attributes.contiguous()
        adj = point_adjacency.contiguous()
        off = point_adjacency_offsets.contiguous()
        rays_c = rays.contiguous()
        start = start_point.contiguous()
        sharpness = inv_s_to_tensor(inv_s, rays_c)
        self._validate_scene(points, attributes, point_adjacency, point_adjacency_offsets)
        num_points = points_c.size(0)
        num_rays = rays_c.numel() // 6
        self._check_rays(rays_c, start, num_rays)
        self._check_colors(colors, num_rays, sites)
        Q = 0
        dq = None
        if depth_quantiles is not None:
            dq = depth_quantiles.contiguous()
            Q = dq.size(-1)
            if dq.dtype != torch.float32:
                raise RuntimeError("depth_quantiles must have float32 dtype")
            if dq.device.type != "cuda":
                raise RuntimeError("depth_quantiles must be on CUDA device")
            if Q == 0 or dq.numel() // Q != num_rays:
                raise RuntimeError("depth_quantiles must have the same batch size as rays")
        settings = self._settings(weight_threshold, max_intersections, alpha_mode, eps, sdf_channel)
        dev = rays_c.device
        lead = list(rays_c.shape[:-1])
        rgba = torch.empty(lead + [4], dtype=self._attr_type, device=dev)
        nint = torch.empty(lead + [1], dtype=torch.uint32, device=dev)
        contrib = torch.zeros((num_points, 1), dtype=self._attr_type, device=dev) if return_contribution else None
        depth = depth_idx = None
        if dq is not None:
            depth = torch.zeros(lead + [Q], dtype=torch.float32, device=dev)
            depth_idx = torch.zeros(lead + [Q], dtype=torch.uint32, device=dev)
        alpha = torch.zeros((num_points, 1), dtype=torch.float32, device=dev)
        if cells is None:
            cells = self.build_cells(points_c, attributes_c, adj, off)
        foam = self._foam(points_c, attributes_c, adj, off)
        seq = _sequences or {}
        io = _lib.ForwardIO(num_rays, rays_c.data_ptr(), start.data_ptr(), Q, _ptr(dq), _ptr(sharpness),
                            rgba.data_ptr(), _ptr(depth), _ptr(depth_idx), nint.data_ptr(), _ptr(contrib),
                            alpha.data_ptr(), _ptr(seq.get("offsets")), _ptr(seq.get("cells")),
                            _ptr(seq.get("count")), _ptr(_face_tests), _ptr(exits),
                            exits.shape[-1] if exits is not None else 0, _ptr(colors),
                            colors.shape[0] if colors is not None else 0, _ptr(sites))
        with torch.cuda.device(dev):
            _lib.check(self._lib.sdfoam_trace_forward(ctypes.byref(foam), _ptr(cells), ctypes.byref(settings),
                                                      ctypes.byref(io), _stream(dev)))
        out = {"rgba": rgba}
        if dq is not None:
            out["depth"] = depth
            out["depth_indices"] = depth_idx
        if return_contribution:
            out["contribution"] = contrib
        out["num_intersections"] = nint
        out["alpha"] = alpha
        return out

    # -- backward (pipeline_bindings.cpp:336-607) -----------------------------
    def trace_backward(self, points, attributes, point_adjacency, point_adjacency_offsets, rays, start_point,
                       rgb_out, grad_in, depth_quantiles=None, depth_indices=None, depth_grad_in=None,
                       ray_error=None, weight_threshold=None, max_intersections=None, alpha_mode=None,
                       inv_s=None, eps=None, sdf_channel=None, *, cells=None, exits=None, colors=None,
                       sites=None):
        points_c = points.contiguous()
        attributes_c = attributes.contiguous()
        adj = point_adjacency.contiguous()
        off = point_adjacency_offsets.contiguous()
        rays_c = rays.contiguous()
        start = start_point.contiguous()
        sharpness = inv_s_to_tensor(inv_s, rays_c)
        self._validate_scene(points, attributes, point_adjacency, point_adjacency_offsets)
        num_points = points_c.size(0)
        num_rays = rays_c.numel() // 6
        self._check_rays(rays_c, start, num_rays)
        self._check_colors(colors, num_rays, sites)
        g = grad_in.contiguous()
        if g.size(-1) != 4:
            raise RuntimeError("rgb_grad_in must have 4 as the last dimension")
        if g.dtype != self._attr_type:
            raise RuntimeError(f"rgb_grad_in had dtype {_dtype_name(g.dtype)}, expected {_dtype_name(self._attr_type)}")
        if g.device.type != "cuda":
            raise RuntimeError("rgb_grad_in must be on CUDA device")
        if g.numel() // 4 != num_rays:
            raise RuntimeError("rgb_grad_in must have the same batch size as rays")
        rgba = rgb_out.contiguous()
        if rgba.dtype != self._attr_type or rgba.numel() != 4 * num_rays:
            raise RuntimeError("rgb_out must be the forward's rgba output")
        Q = 0
        dq = di = dg = None
        if depth_quantiles is not None:
            dq = depth_quantiles.contiguous()
            Q = dq.size(-1)
            if dq.dtype != torch.float32:
                raise RuntimeError("depth_quantiles must have float32 dtype")
            if dq.device.type != "cuda":
                raise RuntimeError("depth_quantiles must be on CUDA device")
            if dq.numel() != num_rays * Q:
                raise RuntimeError("depth_quantiles must have the same batch size as rays")
            if depth_grad_in is None:
                raise RuntimeError("depth_grad must be provided if depth_quantiles is provided")
            di = depth_indices.contiguous()
            if di.dtype != torch.uint32:
                raise RuntimeError("depth_indices must have uint32 dtype")
            if di.device.type != "cuda":
                raise RuntimeError("depth_indices must be on CUDA device")
            if di.numel() != num_rays * Q:
                raise RuntimeError("depth_indices must have the same batch size as rays")
            dg = depth_grad_in.contiguous()
            if dg.size(-1) != Q:
                raise RuntimeError("depth_grad must have the same number of depth quantiles as depth_quantiles")
            if dg.dtype != torch.float32:
                raise RuntimeError(f"depth_grad had dtype {_dtype_name(dg.dtype)}, expected float32")
            if dg.device.type != "cuda":
                raise RuntimeError("depth_grad must be on CUDA device")
            if dg.numel() != num_rays * Q:
                raise RuntimeError("depth_grad must have the same batch size as rays")
        err = perr = None
        dev = rays_c.device
        if ray_error is not None:
            err = ray_error.contiguous()
            if err.dtype != self._attr_type:
                raise RuntimeError(f"ray_error had dtype {_dtype_name(err.dtype)}, "
                                   f"expected {_dtype_name(self._attr_type)}")
            if err.device.type != "cuda":
                raise RuntimeError("ray_error must be on CUDA device")
            if err.numel() != num_rays:
                raise RuntimeError("ray_error must have the same batch size as rays")
            perr = torch.zeros((num_points, 1), dtype=self._attr_type, device=dev)
        settings = self._settings(weight_threshold, max_intersections, alpha_mode, eps, sdf_channel)
        A = self.attribute_dim()
        attr_grad = torch.empty((attributes_c.size(0), A), dtype=self._attr_type, device=dev)
        points_grad = torch.empty((num_points, 3), dtype=rays_c.dtype, device=dev)
        ray_grad = torch.empty_like(rays_c)
        sharpness_grad = torch.zeros_like(sharpness, dtype=torch.float32)
        if cells is None:
            cells = self.build_cells(points_c, attributes_c, adj, off)
        foam = self._foam(points_c, attributes_c, adj, off)
        wbytes = self._lib.sdfoam_backward_workspace_bytes(num_points, self.sh_degree)
        ws = torch.empty((max(wbytes, 16),), dtype=torch.uint8, device=dev)
        io = _lib.BackwardIO(num_rays, rays_c.data_ptr(), start.data_ptr(), Q, _ptr(dq), _ptr(di),
                             rgba.data_ptr(), g.data_ptr(), _ptr(dg), _ptr(err), _ptr(sharpness),
                             points_grad.data_ptr(), attr_grad.data_ptr(), _ptr(perr), sharpness_grad.data_ptr(),
                             ws.data_ptr(), ws.numel(), _ptr(exits), exits.shape[-1] if exits is not None else 0,
                             _ptr(colors), colors.shape[0] if colors is not None else 0, _ptr(sites))
        with torch.cuda.device(dev):
            _lib.check(self._lib.sdfoam_trace_backward(ctypes.byref(foam), _ptr(cells), ctypes.byref(settings),
                                                       ctypes.byref(io), _stream(dev)))
        out = {"points_grad": points_grad, "attr_grad": attr_grad, "ray_grad": ray_grad,
               "sharpness_grad": sharpness_grad}
        if ray_error is not None:
            out["point_error"] = perr
        return out


    # -- headless render (pipeline_bindings.cpp:609-732) ----------------------
    def trace_benchmark(self, points, attributes, point_adjacency, point_adjacency_offsets, adjacent_diff, camera,
                        start_point, output_rgba, weight_threshold=None, max_intersections=None, alpha_mode=None,
                        inv_s=None, eps=None, sdf_channel=None, *, bg_color=None, checker_bg=False):
        """Renders one frame into output_rgba (uint32 [height * width], RGBA8,
        rows bottom-up) from the single start site.  adjacent_diff ([E, 4]
        binary16 q - p per CSR entry) is used as given.  The cell records are
        cached on the pipeline and rebuilt when any scene tensor changes
        (another tensor, or an in-place update).  bg_color / checker_bg expose
        the visualisation settings the reference fixes to white."""
        points_c = points.contiguous()
        attributes_c = attributes.contiguous()
        adj = point_adjacency.contiguous()
        off = point_adjacency_offsets.contiguous()
        diff = adjacent_diff.contiguous()
        sharpness = inv_s_to_tensor(inv_s, output_rgba)
        self._validate_scene(points, attributes, point_adjacency, point_adjacency_offsets)
        cam = camera_from_dict(camera)
        if start_point.numel() != 1:
            raise RuntimeError("start_point must have a single element")
        if start_point.dtype != torch.uint32:
            raise RuntimeError("start_point must have uint32 dtype")
        if start_point.device.type != "cuda":
            raise RuntimeError("start_point must be on CUDA device")
        if output_rgba.numel() != cam.width * cam.height:
            raise RuntimeError("output_rgba must have width * height elements")
        if output_rgba.dtype != torch.uint32:
            raise RuntimeError("output_rgba must have uint32 dtype")
        if output_rgba.device.type != "cuda":
            raise RuntimeError("output_rgba must be on CUDA device")
        if diff.dtype != torch.float16 or diff.numel() != 4 * adj.numel():
            raise RuntimeError("adjacent_diff must be float16 with 4 values per adjacency entry")
        if diff.device.type != "cuda":
            raise RuntimeError("adjacent_diff must be on CUDA device")
        settings = self._settings(weight_threshold, max_intersections, alpha_mode, eps, sdf_channel)
        key = tuple((t.data_ptr(), t._version, t.numel()) for t in (points_c, attributes_c, adj, off, diff))
        cached = getattr(self, "_render_cells", None)
        foam = self._foam(points_c, attributes_c, adj, off)
        dev = output_rgba.device
        if cached is None or cached[0] != key:
            nbytes = self._lib.sdfoam_cells_bytes(foam.num_points, foam.adjacency_size, self.sh_degree)
            cells = torch.empty((nbytes,), dtype=torch.uint8, device=dev)
            with torch.cuda.device(dev):
                _lib.check(self._lib.sdfoam_build_cells_from_diffs(ctypes.byref(foam), _ptr(diff), _ptr(cells),
                                                                   nbytes, _stream(dev)))
            self._render_cells = cached = (key, cells)
        out = output_rgba if output_rgba.is_contiguous() else output_rgba.contiguous()
        bg = None
        if bg_color is not None:
            bg = (ctypes.c_float * 3)(*[float(x) for x in bg_color])
        start = start_point.contiguous()
        with torch.cuda.device(dev):
            _lib.check(self._lib.sdfoam_trace_benchmark(ctypes.byref(foam), _ptr(cached[1]), ctypes.byref(settings),
                                                        ctypes.byref(cam), _ptr(start), _ptr(sharpness), bg,
                                                        1 if checker_bg else 0, _ptr(out), _stream(dev)))
        if out is not output_rgba:
            output_rgba.copy_(out.view_as(output_rgba))

def _camera_vec(camera, key):
    v = camera[key]
    if isinstance(v, torch.Tensor):
        v = v.detach().to("cpu", torch.float32).reshape(-1).tolist()
    v = [float(x) for x in v]
    if len(v) < 3:
        raise RuntimeError(f"camera {key} must have 3 elements")
    return v[:3]


def camera_from_dict(camera: dict) -> "_lib.Camera":
    """The camera dict of trace_benchmark (pipeline_bindings.cpp:636-654):
    position / forward / up / right (3-vectors), fov (radians), width,
    height, model ("pinhole" or "fisheye")."""
    model = str(camera["model"])
    if model == "pinhole":
        m = _lib.SDFOAM_PINHOLE
    elif model == "fisheye":
        m = _lib.SDFOAM_FISHEYE
    else:
        raise RuntimeError("Invalid camera model")
    c = _lib.Camera()
    c.position[:] = _camera_vec(camera, "position")
    c.forward[:] = _camera_vec(camera, "forward")
    c.right[:] = _camera_vec(camera, "right")
    c.up[:] = _camera_vec(camera, "up")
    c.fov = float(camera["fov"])
    c.width = int(camera["width"])
    c.height = int(camera["height"])
    c.model = m
    return c


def dtype_string_to_scalar_type(dtype: str) -> torch.dtype:
    if dtype in _ATTR_TYPES:
        return _ATTR_TYPES[dtype]
    raise RuntimeError(f"unsupported dtype '{dtype}'")


def create_pipeline(sh_degree: int, attr_dtype: str = "float32") -> Pipeline:
    """create_pipeline (pipeline_bindings.cpp:747-751, 856-860)."""
    if isinstance(attr_dtype, torch.dtype):
        attr_dtype = str(attr_dtype)
    t = dtype_string_to_scalar_type(attr_dtype)
    if t == torch.float64:
        raise RuntimeError("Unsupported attribute type")
    p = Pipeline(sh_degree, t)
    pipeline_registry.append(p)
    return p
