"""The eikonal term (sdfoam_model/sdfnet.py:144-152, train.py:293-326) at the
benchmarked width, against golden outputs of the reference SDFNetwork
(tests/golden/sdfnet256_eikonal_golden.npz, made by
tests/golden/make_sdfnet256_eikonal_golden.py): the plain float32 layers on
the CPU, and the fused bf16 tcgen05 path (FusedSDFGradient) on the GPU."""
import importlib.util
import os

import numpy as np
import pytest
import torch

from sdfoam_b200.sdfnet import FusedSDFGradient, SDFNetwork

HERE = os.path.dirname(os.path.abspath(__file__))
GOLDEN = os.path.join(HERE, "golden", "sdfnet256_eikonal_golden.npz")


def _maker():
    spec = importlib.util.spec_from_file_location("make_golden",
                                                  os.path.join(HERE, "golden", "make_sdfnet256_eikonal_golden.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _net(dtype, device):
    z = np.load(GOLDEN)
    net = SDFNetwork(d_hidden=256, n_layers=8, skip_in=(4,), multires=6, point_cloud=z["cloud"], dtype=dtype)
    params = _maker().fill_params([(k, tuple(v.shape)) for k, v in net.named_parameters()])
    with torch.no_grad():
        for k, v in net.named_parameters():
            v.copy_(torch.from_numpy(params[k]))
    return net.to(device), z


def _eikonal(net, pts):
    g = net.gradient(pts.clone())
    loss = net.eikonal_loss(g)
    net.zero_grad(set_to_none=True)
    loss.backward()
    return g.detach().float().cpu(), float(loss), {k: v.grad.float().cpu() for k, v in net.named_parameters()
                                                   if v.grad is not None}


def test_plain_layers_match_the_reference_eikonal():
    net, z = _net(torch.float32, "cpu")
    pts = torch.from_numpy(z["points"])
    y = net(pts)
    np.testing.assert_allclose(y.detach().numpy(), z["sdf"], rtol=1e-4, atol=1e-5)
    g, loss, wg = _eikonal(net, pts)
    np.testing.assert_allclose(g.numpy(), z["eik_grad"], rtol=1e-4, atol=1e-4)
    assert abs(loss - float(z["eik_loss"])) <= 1e-4 * abs(float(z["eik_loss"]))
    for k, v in wg.items():
        ref = z[f"eik_wgrad/{k}"].astype(np.float32)
        scale = float(z[f"eik_wgrad_scale/{k}"])
        # float16 storage of the golden: 2^-11 of the largest entry
        assert np.abs(v.numpy() - ref).max() <= 2e-3 * scale + 1e-6, k


@pytest.mark.gpu
def test_fused_eikonal_matches_the_reference_at_bf16_tolerance():
    """bf16 weights and activations against the reference's float32.  The
    bf16 network itself differs from the float32 one (nine layers of bf16
    rounding, forward and both backward sweeps), so the tolerance of each
    tensor is set by the same bf16 network evaluated as plain PyTorch layers
    with autograd's double backward: the fused path may deviate from the
    reference by at most twice that, or 2 % of the tensor's largest entry."""
    dev = torch.device("cuda:0")
    net, z = _net(torch.bfloat16, dev)
    pts = torch.from_numpy(z["points"]).to(dev)
    assert net.fused_ok(pts)
    g, loss, wg = _eikonal(net, pts)

    x2 = pts.clone().requires_grad_(True)
    y2 = net.forward_layers(x2)[:, :1]
    (g2,) = torch.autograd.grad(y2, x2, torch.ones_like(y2), create_graph=True)
    l2 = net.eikonal_loss(g2)
    net.zero_grad(set_to_none=True)
    l2.backward()
    wp = {k: v.grad.float().cpu() for k, v in net.named_parameters() if v.grad is not None}

    def check(got, plain, ref, scale, what):
        bound = max(2.0 * float(np.abs(plain - ref).max()), 2e-2 * scale) + 1e-4
        err = float(np.abs(got - ref).max())
        assert err <= bound, (what, err, bound)

    ref_g = z["eik_grad"]
    check(g.numpy(), g2.detach().float().cpu().numpy(), ref_g, float(np.abs(ref_g).max()), "input gradient")
    ref_l = float(z["eik_loss"])
    assert abs(loss - ref_l) <= max(2.0 * abs(float(l2) - ref_l), 2e-2 * abs(ref_l))
    for k in z.files:
        if not k.startswith("eik_wgrad/"):
            continue
        name = k[len("eik_wgrad/"):]
        ref = z[k].astype(np.float32)
        got = wg[name].numpy() if name in wg else np.zeros_like(ref)
        plain = wp[name].numpy() if name in wp else np.zeros_like(ref)
        check(got, plain, ref, float(z[f"eik_wgrad_scale/{name}"]), name)


@pytest.mark.gpu
def test_fused_eikonal_matches_plain_layers_on_many_points():
    """The fused double backward against autograd's double backward of the
    same bf16 network as plain layers, on 65,536 points (rows past one tile
    and a partial last tile), and gradients that reach the points."""
    dev = torch.device("cuda:0")
    net, _ = _net(torch.bfloat16, dev)
    gen = torch.Generator(device="cpu").manual_seed(3)
    pts = (torch.rand((65536 + 77, 3), generator=gen) * 2.2 - 1.1).to(dev)

    x1 = pts.clone().requires_grad_(True)
    g1 = FusedSDFGradient.apply(x1, net.pc_center, 1.0, *__import__("sdfoam_b200.sdfnet").sdfnet.augmented_weights(net))
    l1 = net.eikonal_loss(g1)
    net.zero_grad(set_to_none=True)
    l1.backward()
    w1 = {k: v.grad.float().clone() for k, v in net.named_parameters() if v.grad is not None}
    dx1 = x1.grad.clone()

    x2 = pts.clone().requires_grad_(True)
    y2 = net.forward_layers(x2)[:, :1]
    (g2,) = torch.autograd.grad(y2, x2, torch.ones_like(y2), create_graph=True)
    l2 = net.eikonal_loss(g2)
    net.zero_grad(set_to_none=True)
    l2.backward()
    w2 = {k: v.grad.float().clone() for k, v in net.named_parameters() if v.grad is not None}
    dx2 = x2.grad.clone()

    def rel(a, b):
        return float((a.float() - b.float()).abs().max() / b.float().abs().max().clamp_min(1e-12))

    assert rel(g1, g2) < 5e-2 and abs(float(l1) - float(l2)) <= 5e-2 * abs(float(l2))
    for k in w2:
        assert rel(w1[k], w2[k]) < 8e-2, (k, rel(w1[k], w2[k]))
    assert rel(dx1, dx2) < 8e-2
