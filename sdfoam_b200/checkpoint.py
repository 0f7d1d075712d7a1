"""Trained-foam checkpoints in the reference's formats, so that a scene
trained with SDFoam loads into this library and back.

  model.pt   torch.save of {"xyz", "color_dc", "color_sh", "adjacency"
             (int64), "adjacency_offsets" (int64), "alpha", and "sdf" +
             "variance" state dicts (SDFoam) or "density" (RadFoam)}
             (SDFoamScene.save_pt / load_pt, sdfoam_model/scene.py:744-823)
  scene.ply  binary little-endian PLY with a "vertex" element (x, y, z,
             red, green, blue, density, adjacency_offset = the row's end,
             color_sh_0 ...) and an "adjacency" element
             (SDFoamScene.save_ply, scene.py:679-742)

The trace attributes of a loaded scene are [color_dc, color_sh, last], the
last channel being the SDF network's output at the sites (SDFoam) or the
activated density (RadFoam) (SDFoamScene.get_trace_data, scene.py:256-265).
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np
import torch

from .sdfnet import SDFNetwork, SingleVarianceNetwork

SH_C0 = 0.28209479177387814


@dataclass
class SceneCheckpoint:
    points: torch.Tensor              # [N, 3] float32
    color_dc: torch.Tensor            # [N, 3]
    color_sh: torch.Tensor            # [N, 3 ((d+1)^2 - 1)]
    adjacency: torch.Tensor           # [E] uint32
    adjacency_offsets: torch.Tensor   # [N+1] uint32
    alpha: torch.Tensor               # [N, 1]
    sdf: dict | None = None           # SDFNetwork state dict (SDFoam)
    variance: dict | None = None      # SingleVarianceNetwork state dict (SDFoam)
    density: torch.Tensor | None = None  # [N, 1] pre-activation density (RadFoam)
    extra: dict = field(default_factory=dict)

    @property
    def use_sdfoam(self) -> bool:
        return self.sdf is not None


def _strip_module_prefix(sd):
    """State dicts saved through a wrapper (DataParallel, DDP) carry a
    'module.' prefix on every key (scene.py:777-784)."""
    if isinstance(sd, dict) and any(k.startswith("module.") for k in sd.keys()):
        return {k[len("module."):]: v for k, v in sd.items()}
    return sd


def load_pt(path, sh_degree: int = 3, attr_dtype=torch.float32, device=None) -> SceneCheckpoint:
    """Reads a model.pt written by the reference (or by save_pt) and checks
    the SH width against sh_degree with the reference's message."""
    data = torch.load(path, map_location="cpu", weights_only=False)
    dev = torch.device(device) if device is not None else torch.device("cpu")
    exp_sh = 3 * ((1 + sh_degree) * (1 + sh_degree) - 1)
    got_sh = data["color_sh"].shape[-1]
    assert exp_sh == got_sh, f"Expected {exp_sh} SH coeffs per-point, got {got_sh}"
    known = {"xyz", "color_dc", "color_sh", "adjacency", "adjacency_offsets", "alpha", "sdf", "variance", "density"}
    return SceneCheckpoint(
        points=data["xyz"].float().to(dev),
        color_dc=data["color_dc"].to(attr_dtype).to(dev),
        color_sh=data["color_sh"].to(attr_dtype).to(dev),
        adjacency=data["adjacency"].to(dev).to(torch.uint32),
        adjacency_offsets=data["adjacency_offsets"].to(dev).to(torch.uint32),
        alpha=data["alpha"].to(dev).to(attr_dtype),
        sdf=_strip_module_prefix(data.get("sdf")),
        variance=_strip_module_prefix(data.get("variance")),
        density=data["density"].to(dev) if "density" in data else None,
        extra={k: v for k, v in data.items() if k not in known},
    )


def save_pt(path, ckpt: SceneCheckpoint) -> None:
    """Writes the reference's model.pt dictionary (adjacency as int64)."""
    out = {
        "xyz": ckpt.points.detach().float().cpu(),
        "color_dc": ckpt.color_dc.detach().float().cpu(),
        "color_sh": ckpt.color_sh.detach().float().cpu(),
        "adjacency": ckpt.adjacency.cpu().to(torch.int64),
        "adjacency_offsets": ckpt.adjacency_offsets.cpu().to(torch.int64),
        "alpha": ckpt.alpha.detach().float().cpu(),
    }
    if ckpt.use_sdfoam:
        out["sdf"] = ckpt.sdf
        out["variance"] = ckpt.variance
    else:
        out["density"] = ckpt.density.detach().float().cpu()
    torch.save(out, path)


def sdf_network(ckpt: SceneCheckpoint, dtype=torch.float32, device=None) -> SDFNetwork:
    """The scene's SDF network with the reference's construction
    (scene.py:795-802: 8 x 256, skip at 4, multires 6, centred on the sites)
    and its trained weights (strict load)."""
    net = SDFNetwork(d_in=3, d_out=1, d_hidden=256, n_layers=8, skip_in=(4,), multires=6, bias=0.5, scale=1.0,
                     geometric_init=True, weight_norm=True, point_cloud=ckpt.points.detach().cpu(), dtype=dtype)
    net.load_state_dict(ckpt.sdf, strict=True)
    return net.to(device if device is not None else ckpt.points.device)


def variance_network(ckpt: SceneCheckpoint, device=None) -> SingleVarianceNetwork:
    net = SingleVarianceNetwork(init_val=0.3, device=device if device is not None else ckpt.points.device)
    net.load_state_dict(ckpt.variance, strict=True)
    return net


def trace_attributes(ckpt: SceneCheckpoint, sdf_net: SDFNetwork | None = None, activation_scale: float = 1.0,
                     attr_dtype=torch.float32) -> torch.Tensor:
    """[color_dc, color_sh, last] as the tracer reads it: last = the SDF
    network at the sites (SDFoam) or activation_scale * softplus(density,
    beta=10) (RadFoam) (scene.py:246-265)."""
    if ckpt.use_sdfoam:
        net = sdf_net if sdf_net is not None else sdf_network(ckpt)
        last = net(ckpt.points)[:, :1].float()
    else:
        last = activation_scale * torch.nn.functional.softplus(ckpt.density.float(), beta=10)
    return torch.cat([ckpt.color_dc.float(), ckpt.color_sh.float(), last], dim=-1).to(attr_dtype).contiguous()


# ---------------------------------------------------------------------------
# PLY
# ---------------------------------------------------------------------------

_PLY_TYPES = {np.dtype(np.float32): "float", np.dtype(np.uint8): "uchar", np.dtype(np.uint32): "uint"}
_PLY_NUMPY = {"float": "<f4", "float32": "<f4", "uchar": "u1", "uint8": "u1", "uint": "<u4", "uint32": "<u4",
              "int": "<i4", "int32": "<i4", "double": "<f8", "float64": "<f8", "char": "i1", "int8": "i1",
              "ushort": "<u2", "uint16": "<u2", "short": "<i2", "int16": "<i2"}


def _vertex_dtype(num_sh: int):
    fields = [("x", "<f4"), ("y", "<f4"), ("z", "<f4"), ("red", "u1"), ("green", "u1"), ("blue", "u1"),
              ("density", "<f4"), ("adjacency_offset", "<u4")]
    fields += [(f"color_sh_{i}", "<f4") for i in range(num_sh)]
    return np.dtype(fields)


def save_ply(path, points, color_attributes, adjacency, adjacency_offsets, last=None) -> None:
    """scene.ply as the reference writes it: per vertex the position, the DC
    colour as 8-bit RGB (clip(255 (0.5 + C0 dc))), the last channel ("density":
    the SDF for SDFoam, 1 when absent), the end of its adjacency row and the
    remaining colour coefficients; then the adjacency list."""
    pts = np.asarray(torch.as_tensor(points).detach().float().cpu(), np.float32).reshape(-1, 3)
    att = np.asarray(torch.as_tensor(color_attributes).detach().float().cpu(), np.float32)
    adj = np.asarray(torch.as_tensor(adjacency).cpu().to(torch.int64), np.int64).astype(np.uint32).reshape(-1)
    off = np.asarray(torch.as_tensor(adjacency_offsets).cpu().to(torch.int64), np.int64).astype(np.uint32)
    n = pts.shape[0]
    v = np.zeros(n, dtype=_vertex_dtype(att.shape[1] - 3))
    v["x"], v["y"], v["z"] = pts[:, 0], pts[:, 1], pts[:, 2]
    for k, name in enumerate(("red", "green", "blue")):
        v[name] = np.clip(255 * (0.5 + SH_C0 * att[:, k]), 0, 255).astype(np.uint8)
    if last is None:
        v["density"] = 1.0
    else:
        v["density"] = np.asarray(torch.as_tensor(last).detach().float().cpu(), np.float32).reshape(-1)
    v["adjacency_offset"] = off[1:n + 1]
    for j in range(att.shape[1] - 3):
        v[f"color_sh_{j}"] = att[:, 3 + j]
    header = ["ply", "format binary_little_endian 1.0", f"element vertex {n}"]
    header += [f"property {_PLY_TYPES[np.dtype(v.dtype[name].str)]} {name}" for name in v.dtype.names]
    header += [f"element adjacency {adj.shape[0]}", "property uint adjacency", "end_header"]
    with open(path, "wb") as f:
        f.write(("\n".join(header) + "\n").encode("ascii"))
        f.write(v.tobytes())
        f.write(adj.astype("<u4").tobytes())


def read_ply(path) -> dict:
    """Reads a binary little-endian PLY of scalar properties (the layout
    save_ply and the reference write) into {element name: structured array}."""
    with open(path, "rb") as f:
        if f.readline().strip() != b"ply":
            raise ValueError("not a PLY file")
        elements = []
        fmt = None
        while True:
            line = f.readline()
            if not line:
                raise ValueError("PLY header without end_header")
            tok = line.decode("ascii").split()
            if not tok or tok[0] in ("comment", "obj_info"):
                continue
            if tok[0] == "format":
                fmt = tok[1]
            elif tok[0] == "element":
                elements.append((tok[1], int(tok[2]), []))
            elif tok[0] == "property":
                if tok[1] == "list":
                    raise ValueError("list properties are not supported")
                elements[-1][2].append((tok[2], _PLY_NUMPY[tok[1]]))
            elif tok[0] == "end_header":
                break
        if fmt != "binary_little_endian":
            raise ValueError(f"unsupported PLY format {fmt}")
        out = {}
        for name, count, props in elements:
            dt = np.dtype(props)
            out[name] = np.frombuffer(f.read(dt.itemsize * count), dtype=dt, count=count)
        return out


def load_ply(path):
    """(points [N,3], color attributes [N, 3 + K] with the DC colour
    recovered from its 8-bit value, last channel [N], adjacency [E] uint32,
    offsets [N+1] uint32) from a scene.ply.  The 8-bit DC colour is lossy:
    model.pt is the exact checkpoint."""
    d = read_ply(path)
    v, a = d["vertex"], d["adjacency"]["adjacency"]
    pts = np.stack([v["x"], v["y"], v["z"]], 1).astype(np.float32)
    dc = np.stack([(v[c].astype(np.float32) / 255.0 - 0.5) / SH_C0 for c in ("red", "green", "blue")], 1)
    sh_names = sorted((n for n in v.dtype.names if n.startswith("color_sh_")), key=lambda s: int(s.split("_")[-1]))
    sh = np.stack([v[n] for n in sh_names], 1).astype(np.float32) if sh_names else np.zeros((len(v), 0), np.float32)
    off = np.concatenate([[0], v["adjacency_offset"].astype(np.uint32)]).astype(np.uint32)
    return pts, np.concatenate([dc, sh], 1), v["density"].astype(np.float32), a.astype(np.uint32), off
