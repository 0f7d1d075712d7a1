"""The eikonal term's double backward written out layer by layer, in the
form a fused implementation evaluates it, against autograd (float64).

For the sdfnet f(x) (positional encoding, softplus-100 hidden layers with a
skip concatenation, linear output) and g = d f / d x, the loss's gradient
for any upstream gbar = dL/dg is the gradient of the directional
derivative h = <gbar, g> = J_f(x) gbar.  Its pieces:

  primal     z_l = W_l in_l + b_l, a_l = sp(z_l); sp' = sigmoid(100 z),
             sp'' = 100 sp' (1 - sp') (sp' = 1, sp'' = 0 past torch's
             softplus threshold 100 z > 20)
  backward   da_7 = W_8[0]; dz_l = da_l * sp'(z_l); d in_l = W_l^T dz_l
             (the first-order chain that gives g = J_enc^T d enc)
  tangent    t_enc = J_enc gbar; tz_l = W_l t_in_l; ta_l = sp'(z_l) tz_l
             (a forward sweep: GEMM + sp' epilogue)
  second     dz2_l = dz_l * tz_l * sp''(z_l) / sp'(z_l)
             S_7 = dz2_7; S_l = sp'(z_l) * [W_{l+1}^T S_{l+1}]_a + dz2_l
             (a backward sweep: GEMM + sp' epilogue + the injected term)
  gradients  dL/dW_l = dz_l^T t_in_l + S_l^T in_l, dL/db_l = sum S_l,
             dL/dW_8 = sum ta_7, dL/db_8 = 0,
             dL/dx = J_enc^T d enc_S + H_enc[d enc](gbar)

so each layer needs one forward-tangent GEMM and one backward GEMM with the
first-order dz of the same layer in its epilogue, plus the weight-gradient
GEMMs over [dz | S] against [t_in ; in]."""
import math

import torch

from sdfoam_b200.sdfnet import SDFNetwork, positional_encoding

SKIP = 4


def _weights(net):
    Ws, bs = [], []
    for l in range(net.num_layers - 1):
        lin = getattr(net, f"lin{l}")
        Ws.append(lin.weight().detach().double().clone().requires_grad_(True))
        bs.append(lin.bias.detach().double().clone().requires_grad_(True))
    return Ws, bs


def _f(x, Ws, bs, center):
    enc = positional_encoding(x - center, 6)
    a = enc
    for l in range(len(Ws)):
        inp = torch.cat([a, enc], 1) / math.sqrt(2.0) if l == SKIP else a
        z = inp @ Ws[l].t() + bs[l]
        a = torch.nn.functional.softplus(z, beta=100) if l < len(Ws) - 1 else z
    return a[:, 0]


def _enc_jvp_hvp(x, center, v, denc):
    """J_enc v and H_enc[denc](v) of the positional encoding."""
    u = x - center
    t = [v]
    h = torch.zeros_like(x)
    for k in range(6):
        w = 2.0 * math.pi * (2.0 ** k)
        s, c = torch.sin(w * u), torch.cos(w * u)
        t += [w * c * v, -w * s * v]
        ds, dc = denc[:, 3 + 6 * k:6 + 6 * k], denc[:, 6 + 6 * k:9 + 6 * k]
        h = h + ds * (-w * w * s) * v + dc * (-w * w * c) * v
    return torch.cat(t, 1), h


def _enc_vjp(x, center, denc):
    u = x - center
    g = denc[:, :3].clone()
    for k in range(6):
        w = 2.0 * math.pi * (2.0 ** k)
        g = g + denc[:, 3 + 6 * k:6 + 6 * k] * w * torch.cos(w * u) - denc[:, 6 + 6 * k:9 + 6 * k] * w * torch.sin(w * u)
    return g


def _chain(x, Ws, bs, center, gbar):
    L = len(Ws)  # 9: 8 hidden + output
    enc = positional_encoding(x - center, 6)
    d_skip = enc.shape[1]
    ins, zs, sp1 = [], [], []
    a = enc
    for l in range(L - 1):
        inp = torch.cat([a, enc], 1) / math.sqrt(2.0) if l == SKIP else a
        z = inp @ Ws[l].t() + bs[l]
        ins.append(inp)
        zs.append(z)
        # torch's Softplus(beta=100) is linear past beta z > 20 (threshold):
        # there sp' = 1 and sp'' = 0 exactly
        sp1.append(torch.where(100.0 * z > 20.0, torch.ones_like(z), torch.sigmoid(100.0 * z)))
        a = torch.nn.functional.softplus(z, beta=100)
    ins.append(a)
    # first-order backward
    dz = [None] * (L - 1)
    da = Ws[L - 1][0].expand(x.shape[0], -1)
    denc = torch.zeros_like(enc)
    for l in range(L - 2, -1, -1):
        dz[l] = da * sp1[l]
        din = dz[l] @ Ws[l]
        if l == SKIP:
            da = din[:, :-d_skip] / math.sqrt(2.0)
            denc = denc + din[:, -d_skip:] / math.sqrt(2.0)
        elif l == 0:
            denc = denc + din
        else:
            da = din
    g = _enc_vjp(x, center, denc)
    # tangent sweep along gbar
    tenc, henc = _enc_jvp_hvp(x, center, gbar, denc)
    tins, tzs = [], []
    ta = tenc
    for l in range(L - 1):
        tin = torch.cat([ta, tenc], 1) / math.sqrt(2.0) if l == SKIP else ta
        tz = tin @ Ws[l].t()
        tins.append(tin)
        tzs.append(tz)
        ta = sp1[l] * tz
    tins.append(ta)
    # second backward with the injected sp'' terms
    dz2 = [dz[l] * tzs[l] * 100.0 * (1.0 - sp1[l]) for l in range(L - 1)]  # (1 - sp') is 0 past the threshold
    S = [None] * (L - 1)
    S[L - 2] = dz2[L - 2]
    denc_S = torch.zeros_like(enc)
    for l in range(L - 2, -1, -1):
        din = S[l] @ Ws[l]
        if l == SKIP:
            upper = din[:, :-d_skip] / math.sqrt(2.0)
            denc_S = denc_S + din[:, -d_skip:] / math.sqrt(2.0)
        elif l == 0:
            denc_S = denc_S + din
            upper = None
        else:
            upper = din
        if l > 0:
            S[l - 1] = sp1[l - 1] * upper + dz2[l - 1]
    dW = [dz[l].t() @ tins[l] + S[l].t() @ ins[l] for l in range(L - 1)]
    db = [S[l].sum(0) for l in range(L - 1)]
    dW.append(torch.zeros_like(Ws[L - 1]))
    dW[L - 1][0] = tins[L - 1].sum(0)
    db.append(torch.zeros_like(bs[L - 1]))
    dx = _enc_vjp(x, center, denc_S) + henc
    return g, dW, db, dx


def test_eikonal_double_backward_chain_matches_autograd():
    torch.manual_seed(0)
    n = 64
    cloud = torch.rand(256, 3) * 2 - 1
    net = SDFNetwork(d_hidden=64, n_layers=8, multires=6, init="xavier", point_cloud=cloud,
                     generator=torch.Generator().manual_seed(4))
    Ws, bs = _weights(net)
    center = net.pc_center.double()
    x = (torch.rand(n, 3, dtype=torch.float64) * 2 - 1).requires_grad_(True)
    gbar = torch.randn(n, 3, dtype=torch.float64)

    f = _f(x, Ws, bs, center)
    (g_auto,) = torch.autograd.grad(f.sum(), x, create_graph=True)
    h = (g_auto * gbar).sum()
    grads = torch.autograd.grad(h, Ws + bs + [x], allow_unused=True)
    W_auto, b_auto, x_auto = grads[:len(Ws)], grads[len(Ws):2 * len(Ws)], grads[-1]

    with torch.no_grad():
        g, dW, db, dx = _chain(x.detach(), [w.detach() for w in Ws], [b.detach() for b in bs], center, gbar)
    assert torch.allclose(g, g_auto.detach(), rtol=1e-10, atol=1e-12)
    for l in range(len(Ws)):
        ref_w = W_auto[l] if W_auto[l] is not None else torch.zeros_like(dW[l])
        ref_b = b_auto[l] if b_auto[l] is not None else torch.zeros_like(db[l])
        assert torch.allclose(dW[l], ref_w, rtol=1e-9, atol=1e-10 * max(1.0, float(ref_w.abs().max()))), l
        assert torch.allclose(db[l], ref_b, rtol=1e-9, atol=1e-10 * max(1.0, float(ref_b.abs().max()))), l
    assert torch.allclose(dx, x_auto, rtol=1e-9, atol=1e-10 * float(x_auto.abs().max()))
