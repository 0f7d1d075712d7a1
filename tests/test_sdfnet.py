"""The SDF MLP against golden vectors of the reference SDFNetwork
(tests/golden/sdfnet_golden.npz, made by tests/golden/make_sdfnet_golden.py
from sdfoam_model/sdfnet.py)."""
import os

import numpy as np
import torch

from sdfoam_b200.sdfnet import SDFNetwork, mlp_flops_per_site

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "sdfnet_golden.npz")


def _golden_net(dtype=torch.float32, device="cpu"):
    z = np.load(GOLDEN)
    net = SDFNetwork(d_in=3, d_out=1, d_hidden=64, n_layers=8, skip_in=(4,), multires=6, bias=0.5, scale=1.0,
                     point_cloud=np.zeros((1, 3), np.float32), dtype=dtype)
    state = {k[len("param/"):]: torch.from_numpy(z[k]) for k in z.files if k.startswith("param/")}
    missing, unexpected = net.load_state_dict(state, strict=True)
    assert not missing and not unexpected
    return net.to(device), z


def test_sdfnet_matches_reference_fp32():
    net, z = _golden_net()
    pts = torch.from_numpy(z["points"]).requires_grad_(True)
    y = net(pts)
    (g,) = torch.autograd.grad(y.sum(), pts)
    np.testing.assert_allclose(y.detach().numpy(), z["sdf"], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(g.numpy(), z["grad_points"], rtol=1e-4, atol=1e-4 * np.abs(z["grad_points"]).max())


def test_sdfnet_bf16_within_bf16_tolerance():
    net, z = _golden_net(dtype=torch.bfloat16)
    y = net(torch.from_numpy(z["points"])).detach().numpy()
    ref = z["sdf"]
    assert np.abs(y - ref).max() <= 0.05 * np.abs(ref).max() + 1e-2


def test_full_size_flops_match_survey():
    net = SDFNetwork(d_hidden=256, n_layers=8, multires=6, init="xavier")
    # 459,008 multiply-adds per site (39->256, 2x 256->256, 256->217, 256->256 after the skip, 3x 256->256, 256->1)
    assert mlp_flops_per_site(net) == 2 * 459008


def test_eikonal_gradient_and_double_backward_match_reference():
    """gradient(x), the eikonal loss and the loss's parameter gradients (a
    double backward through the network) against the reference's."""
    net, z = _golden_net()
    pts = torch.from_numpy(z["points"]).clone()
    grads = net.gradient(pts)
    np.testing.assert_allclose(grads.detach().numpy(), z["eik_grad"], rtol=1e-4,
                               atol=1e-4 * np.abs(z["eik_grad"]).max())
    loss = net.eikonal_loss(grads)
    assert abs(loss.item() - float(z["eik_loss"])) <= 1e-4 * abs(float(z["eik_loss"]))
    net.zero_grad()
    loss.backward()
    for name, p in net.named_parameters():
        ref = z[f"eik_wgrad/{name}"]
        got = p.grad.detach().numpy() if p.grad is not None else np.zeros_like(ref)
        np.testing.assert_allclose(got, ref, rtol=1e-3, atol=1e-4 * max(1e-6, np.abs(ref).max()), err_msg=name)


def test_layer_give_up_flag_raises_naming_the_layer():
    """A tcgen05 layer that gives up its bounded waits sets its launch's flag;
    the host turns it into a RuntimeError naming the layer (host logic, CPU
    flags standing in for the device ones)."""
    import pytest
    from sdfoam_b200 import sdfnet

    sdfnet.check_layer_flags()
    ok = sdfnet.LayerFlags(torch.device("cpu"))
    ok.post()
    sdfnet.check_layer_flags()  # all clear
    bad = sdfnet.LayerFlags(torch.device("cpu"))
    bad.flags[8 + 7 - 3] = 1  # the dgrad of hidden layer 3
    bad.post()
    with pytest.raises(RuntimeError, match="backward dgrad of layer 3"):
        sdfnet.check_layer_flags()
    sdfnet.check_layer_flags()  # reported once
    late = sdfnet.LayerFlags(torch.device("cpu"))
    late.flags[2] = 1
    late.post()
    with pytest.raises(RuntimeError, match="forward hidden layer 2"):
        sdfnet.check_layer_flags(wait=False)
