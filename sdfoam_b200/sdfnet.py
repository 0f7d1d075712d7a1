"""SDF MLP evaluated at every site (drop-in for sdfoam_model/sdfnet.py:43-161).

Architecture of the reference SDFNetwork: positional encoding
[x, sin(2 pi 2^k x), cos(2 pi 2^k x)] for k < multires (sdfnet.py:21-40),
n_layers hidden layers of d_hidden with Softplus(beta=100), a skip connection
that concatenates the encoded input and divides by sqrt(2) before the
layers in skip_in (sdfnet.py:128-134), weight normalisation w = g v / |v| per
output row, and the first output channel divided by `scale`.  Parameter names
(lin{l}.weight_g, lin{l}.weight_v, lin{l}.bias, pc_center) match the
reference's state_dict, so its checkpoints load unchanged.

`dtype=torch.bfloat16` keeps weights and activations in bf16 with fp32
accumulation (the benchmark configuration: "bf16 weights, Xavier init").
The dense layers run as cuBLAS GEMMs through torch here.
"""
from __future__ import annotations

import math

import torch
import torch.nn as nn
import torch.nn.functional as F


def positional_encoding(x: torch.Tensor, multires: int) -> torch.Tensor:
    """[x, sin(2 pi f x), cos(2 pi f x)] for f = 2^0 .. 2^(multires-1)
    (reference sdfnet.py:28-36)."""
    outs = [x]
    for k in range(multires):
        w = 2.0 * math.pi * (2.0 ** k)
        outs += [torch.sin(x * w), torch.cos(x * w)]
    return torch.cat(outs, dim=-1)


class WeightNormLinear(nn.Module):
    """Linear layer with weight normalisation over each output row (the
    parametrisation nn.utils.weight_norm(..., dim=0) applies)."""

    def __init__(self, weight: torch.Tensor, bias: torch.Tensor, dtype):
        super().__init__()
        v = weight.detach().clone()
        g = v.norm(dim=1, keepdim=True)
        self.weight_g = nn.Parameter(g.to(dtype))
        self.weight_v = nn.Parameter(v.to(dtype))
        self.bias = nn.Parameter(bias.detach().clone().to(dtype))

    def weight(self) -> torch.Tensor:
        v = self.weight_v
        return v * (self.weight_g / v.float().norm(dim=1, keepdim=True).to(v.dtype))

    def forward(self, x):
        return F.linear(x, self.weight(), self.bias)


class SDFNetwork(nn.Module):
    def __init__(self, d_in=3, d_out=1, d_hidden=256, n_layers=8, skip_in=(4,), multires=6, bias=0.5,
                 scale=1.0, geometric_init=True, weight_norm=True, inside_outside=False, point_cloud=None,
                 init="geometric", dtype=torch.float32, device=None, generator=None):
        super().__init__()
        dims = [d_in] + [d_hidden] * n_layers + [d_out]
        self.multires = multires
        if multires > 0:
            dims[0] = d_in + 2 * multires * d_in
        self.num_layers = len(dims)
        self.skip_in = tuple(skip_in)
        self.scale = scale
        self.dtype = dtype
        self.weight_norm = weight_norm
        if point_cloud is not None:
            pc = torch.as_tensor(point_cloud, dtype=torch.float32).reshape(-1, d_in)
            self.register_buffer("pc_center", pc.mean(dim=0, keepdim=True))
        else:
            self.register_buffer("pc_center", None)
        if not geometric_init:
            init = "xavier"
        for l in range(self.num_layers - 1):
            out_dim = dims[l + 1] - dims[0] if (l + 1) in self.skip_in else dims[l + 1]
            w = torch.empty(out_dim, dims[l])
            b = torch.zeros(out_dim)
            if init == "geometric":
                # sdfnet.py:96-114
                if l == self.num_layers - 2:
                    mean = math.sqrt(math.pi) / math.sqrt(dims[l])
                    w.normal_(-mean if inside_outside else mean, 0.0001, generator=generator)
                    b.fill_(bias if inside_outside else -bias)
                elif multires > 0 and l == 0:
                    w.zero_()
                    w[:, :3].normal_(0.0, math.sqrt(2) / math.sqrt(out_dim), generator=generator)
                elif multires > 0 and l in self.skip_in:
                    w.normal_(0.0, math.sqrt(2) / math.sqrt(out_dim), generator=generator)
                    w[:, -(dims[0] - 3):] = 0.0
                else:
                    w.normal_(0.0, math.sqrt(2) / math.sqrt(out_dim), generator=generator)
            else:  # Xavier (Glorot) uniform
                a = math.sqrt(6.0 / (dims[l] + out_dim))
                w.uniform_(-a, a, generator=generator)
            if weight_norm:
                lin = WeightNormLinear(w, b, dtype)
            else:
                lin = nn.Linear(dims[l], out_dim, dtype=dtype)
                with torch.no_grad():
                    lin.weight.copy_(w)
                    lin.bias.copy_(b)
            setattr(self, f"lin{l}", lin)
        if device is not None:
            self.to(device)

    def forward(self, inputs: torch.Tensor) -> torch.Tensor:
        if self.pc_center is not None:
            inputs = inputs - self.pc_center
        inputs = inputs * self.scale
        if self.multires > 0:
            inputs = positional_encoding(inputs, self.multires)
        inputs = inputs.to(self.dtype)
        x = inputs
        for l in range(self.num_layers - 1):
            lin = getattr(self, f"lin{l}")
            if l in self.skip_in:
                x = torch.cat([x, inputs], 1) / math.sqrt(2.0)
            x = lin(x)
            if l < self.num_layers - 2:
                x = F.softplus(x, beta=100)
        x = x.float()
        return torch.cat([x[:, :1] / self.scale, x[:, 1:]], dim=-1)

    def sdf(self, x):
        return self.forward(x)[:, :1]


class SingleVarianceNetwork(nn.Module):
    """Learnable sharpness inv_s = exp(variance) (sdfnet.py:155-161)."""

    def __init__(self, init_val, device=None):
        super().__init__()
        self.register_parameter("variance", nn.Parameter(torch.tensor(float(init_val), device=device)))

    def forward(self, x):
        return torch.ones([len(x), 1], device=x.device) * torch.exp(self.variance * 1.0)


def mlp_flops_per_site(net: SDFNetwork) -> int:
    """Multiply-adds x 2 of one forward evaluation."""
    macs = 0
    for l in range(net.num_layers - 1):
        lin = getattr(net, f"lin{l}")
        w = lin.weight_v if isinstance(lin, WeightNormLinear) else lin.weight
        macs += w.shape[0] * w.shape[1]
    return 2 * macs
