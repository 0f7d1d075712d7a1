"""Generates tests/golden/sdfnet256_eikonal_golden.npz from the reference
SDFNetwork at the benchmarked width (8 x 256, skip at 4, multires 6, weight
normalisation): the SDF, its input gradient and the eikonal term's loss and
parameter gradients (sdfoam_model/sdfnet.py:120-152, train.py:293-326).

Run in a container that has the reference checkout (read-only) at
REFERENCE_ROOT (default /root/reference):

    python tests/golden/make_sdfnet256_eikonal_golden.py

The reference module is plain PyTorch and is imported directly.  Its weights
are replaced by values drawn from numpy's default_rng(SEED) in a fixed order
(weight_g, weight_v, bias per layer; see fill_params), which the tests
redraw, so the fixture holds only the 512 points and the outputs; the
parameter gradients are stored as float16 (the fused path they check is
bf16).
"""
import os
import sys

import numpy as np
import torch

SEED = 20261202
OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "sdfnet256_eikonal_golden.npz")


def fill_params(named_params, seed=SEED):
    """Draws every parameter of the network from default_rng(seed), in the
    sorted order of the names in named_params: weight_g ~ U(0.8, 1.2), weight_v ~ N(0, 1 / fan_in),
    bias ~ N(0, 0.05)."""
    rng = np.random.default_rng(seed)
    out = {}
    for name, shape in sorted(named_params):
        if name.endswith("weight_v"):
            v = rng.standard_normal(shape) / np.sqrt(shape[1])
        elif name.endswith("weight_g"):
            v = rng.uniform(0.8, 1.2, shape)
        else:
            v = rng.normal(0.0, 0.05, shape)
        out[name] = v.astype(np.float32)
    return out


def main():
    ref = os.environ.get("REFERENCE_ROOT", "/root/reference")
    sys.path.insert(0, ref)
    from sdfoam_model.sdfnet import SDFNetwork  # noqa: E402
    rng = np.random.default_rng(SEED + 1)
    cloud = rng.uniform(-1, 1, (512, 3)).astype(np.float32)
    net = SDFNetwork(d_in=3, d_out=1, d_hidden=256, n_layers=8, skip_in=(4,), multires=6, bias=0.5, scale=1.0,
                     geometric_init=True, weight_norm=True, point_cloud=torch.from_numpy(cloud))
    params = fill_params([(k, tuple(v.shape)) for k, v in net.named_parameters()])
    with torch.no_grad():
        for k, v in net.named_parameters():
            v.copy_(torch.from_numpy(params[k]))
    pts = torch.from_numpy(rng.uniform(-1.1, 1.1, (512, 3)).astype(np.float32))
    arrays = {"cloud": cloud, "points": pts.numpy()}
    x = pts.clone().requires_grad_(True)
    y = net(x)
    (g,) = torch.autograd.grad(y.sum(), x)
    arrays["sdf"] = y.detach().numpy()
    arrays["grad_points"] = g.numpy()
    grads = net.gradient(pts.clone())
    loss = net.eikonal_loss(grads)
    net.zero_grad()
    loss.backward()
    arrays["eik_grad"] = grads.detach().numpy()
    arrays["eik_loss"] = np.array(loss.item(), np.float64)
    for k, v in net.named_parameters():
        gv = v.grad if v.grad is not None else torch.zeros_like(v)
        arrays[f"eik_wgrad/{k}"] = gv.detach().numpy().astype(np.float16)
        arrays[f"eik_wgrad_scale/{k}"] = np.array(float(gv.abs().max()), np.float64)
    np.savez_compressed(OUT, **arrays)
    print(OUT, os.path.getsize(OUT), "bytes")


if __name__ == "__main__":
    main()
