"""Generates tests/golden/sdfnet_golden.npz from the reference SDFNetwork.

Run in a container that has the reference checkout (read-only) at
REFERENCE_ROOT (default /root/reference):

    python tests/golden/make_sdfnet_golden.py

The reference module (sdfoam_model/sdfnet.py) is plain PyTorch, so it is
imported directly: a small network of the reference architecture (hidden
width 64 instead of 256 to keep the fixture small; same PE, skip layer,
Softplus(100), weight normalisation, point-cloud centring) is seeded, its
weights are perturbed so no initialisation pattern is special, and its SDF
outputs and input gradients on 256 points are stored with the weights.
For the eikonal term (sdfnet.py:144-152) it also stores gradient(x), the
eikonal loss and the loss's parameter gradients (the double backward).
"""
import os
import sys

import numpy as np
import torch

REF = os.environ.get("REFERENCE_ROOT", "/root/reference")
sys.path.insert(0, REF)
from sdfoam_model.sdfnet import SDFNetwork  # noqa: E402

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "sdfnet_golden.npz")


def main():
    torch.manual_seed(0)
    rng = np.random.default_rng(0)
    cloud = rng.uniform(-1, 1, (512, 3)).astype(np.float32)
    net = SDFNetwork(d_in=3, d_out=1, d_hidden=64, n_layers=8, skip_in=(4,), multires=6, bias=0.5, scale=1.0,
                     geometric_init=True, weight_norm=True, point_cloud=torch.from_numpy(cloud))
    with torch.no_grad():
        for name, p in net.named_parameters():
            p.add_(0.05 * torch.randn_like(p))
    pts = torch.from_numpy(rng.uniform(-1.2, 1.2, (256, 3)).astype(np.float32)).requires_grad_(True)
    y = net(pts)
    (g,) = torch.autograd.grad(y.sum(), pts)
    arrays = {f"param/{k}": v.detach().numpy() for k, v in net.state_dict().items()}
    arrays["points"] = pts.detach().numpy()
    arrays["sdf"] = y.detach().numpy()
    arrays["grad_points"] = g.numpy()
    # eikonal term: d sdf / d x with a graph, its loss and the loss's
    # parameter gradients
    x_eik = pts.detach().clone()
    grads = net.gradient(x_eik)
    loss = net.eikonal_loss(grads)
    net.zero_grad()
    loss.backward()
    arrays["eik_grad"] = grads.detach().numpy()
    arrays["eik_loss"] = np.array(loss.item(), np.float64)
    for k, v in net.named_parameters():
        # parameters the input gradient does not depend on (the output bias)
        # get no gradient
        arrays[f"eik_wgrad/{k}"] = (v.grad if v.grad is not None else torch.zeros_like(v)).detach().numpy()
    np.savez_compressed(OUT, **arrays)
    print(OUT, {k: v.shape for k, v in arrays.items() if not k.startswith("param/")})


if __name__ == "__main__":
    main()
