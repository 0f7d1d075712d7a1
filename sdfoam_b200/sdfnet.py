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
On a CUDA device the reference architecture (8 x 256, skip at 4, multires 6,
one output) runs as FusedSDFMLP: every GEMM is padded to multiples of 8 with
its bias folded in as an extra input column of ones (no separate bias
kernels).  Each forward hidden layer is one tcgen05 GEMM of
libsdfoam_b200.so whose TMEM epilogue applies softplus, the skip
concatenation and the bias column (sdfoam_mlp_layer); each backward hidden
layer's dgrad is a tcgen05 GEMM with the softplus derivative (recomputed
from the stored activation) and the skip split fused into its epilogue
(sdfoam_mlp_layer_backward); the last hidden layer's epilogue also applies
the single-output final layer (sdfoam_mlp_layer_dot); every layer's weight
gradient is a tcgen05 GEMM reducing over the rows with both operands
MN-major (sdfoam_mlp_wgrad), and the encoding's gradient a tcgen05 GEMM with
the skip connection's gradient added in its epilogue (sdfoam_mlp_input_grad).
Other shapes and the CPU use the plain PyTorch layers below.
"""
from __future__ import annotations

import ctypes
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

    def fused_ok(self, inputs: torch.Tensor) -> bool:
        """The reference architecture on a CUDA device, bf16, weight norm."""
        return (inputs.is_cuda and self.dtype == torch.bfloat16 and self.weight_norm and self.multires == 6
                and self.num_layers == 10 and self.skip_in == (4,) and inputs.dim() == 2 and inputs.shape[1] == 3
                and getattr(self, "lin8").weight_v.shape[0] == 1 and getattr(self, "lin1").weight_v.shape == (256, 256)
                and float(self.scale) == 1.0)

    def forward(self, inputs: torch.Tensor) -> torch.Tensor:
        if self.fused_ok(inputs):
            return FusedSDFMLP.apply(inputs.float().contiguous(), self.pc_center, float(self.scale),
                                     *augmented_weights(self))
        return self.forward_layers(inputs)

    def forward_layers(self, inputs: torch.Tensor) -> torch.Tensor:
        """The network as plain PyTorch layers (sdfnet.py:120-136)."""
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

    def sdf_hidden_appearance(self, x):
        return self.forward(x)

    def gradient(self, x: torch.Tensor) -> torch.Tensor:
        """d sdf / d x with its graph kept, for the eikonal loss
        (sdfnet.py:144-148).  On the reference architecture on a CUDA device
        (fused_ok) it is FusedSDFGradient: the input gradient and, when the
        loss is differentiated, its double backward on the library's tcgen05
        kernels.  Otherwise the plain PyTorch layers, whose double backward
        autograd provides."""
        x = x.requires_grad_(True)
        if self.fused_ok(x):
            return FusedSDFGradient.apply(x.float().contiguous(), self.pc_center, float(self.scale),
                                          *augmented_weights(self))
        with torch.enable_grad():
            y = self.forward_layers(x)[:, :1]
            (grad,) = torch.autograd.grad(y, x, torch.ones_like(y), create_graph=True, retain_graph=True)
        return grad

    @staticmethod
    def eikonal_loss(grads: torch.Tensor) -> torch.Tensor:
        """mean((|grad| - 1)^2) (sdfnet.py:150-152)."""
        return ((grads.norm(2, dim=-1) - 1) ** 2).mean()


class SingleVarianceNetwork(nn.Module):
    """Learnable sharpness inv_s = exp(variance) (sdfnet.py:155-161)."""

    def __init__(self, init_val, device=None):
        super().__init__()
        self.register_parameter("variance", nn.Parameter(torch.tensor(float(init_val), device=device)))

    def forward(self, x):
        return torch.ones([len(x), 1], device=x.device) * torch.exp(self.variance * 1.0)


ENC_LD = 48    # 39 encoding features + bias column + padding
HID_LD = 264   # 256 hidden (or 217 + 39 skip) + bias column + padding
SKIP_OUT = 217


def _aug(w: torch.Tensor, b: torch.Tensor, ld: int, rows: int | None = None) -> torch.Tensor:
    """[w | b | 0] with `ld` columns (and zero rows up to `rows`)."""
    out, k = w.shape
    parts = [w, b.reshape(out, 1)]
    if ld > k + 1:
        parts.append(w.new_zeros(out, ld - k - 1))
    a = torch.cat(parts, 1)
    if rows is not None and rows > out:
        a = torch.cat([a, a.new_zeros(rows - out, ld)], 0)
    return a


def augmented_weights(net: "SDFNetwork"):
    """Bias-augmented, 8-aligned weights of the fused path (tracked by autograd
    back to weight_g, weight_v and bias)."""
    ws = []
    for l in range(9):
        lin = getattr(net, f"lin{l}")
        w, b = lin.weight(), lin.bias
        if l == 0:
            ws.append(_aug(w, b, ENC_LD))
        elif l == 3:
            ws.append(_aug(w, b, HID_LD, rows=224))
        elif l == 8:
            ws.append(_aug(w, b, HID_LD, rows=8))
        else:
            ws.append(_aug(w, b, HID_LD))
    return ws


def _p(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


# Launches of one fused evaluation that carry a give-up flag, in flag order:
# the 8 forward hidden layers (the last one with the output layer), the 8
# backward dgrads, the 9 weight gradients and the encoding's gradient.
FLAG_NAMES = (tuple(f"forward hidden layer {l}" for l in range(8))
              + tuple(f"backward dgrad of layer {l}" for l in range(7, -1, -1))
              + tuple(f"weight gradient of layer {l}" for l in range(8, -1, -1))
              + ("gradient of the positional encoding",))
FLAG_WGRAD = 16
FLAG_INPUT = 25


class LayerFlags:
    """Give-up flags of the tcgen05 layers of one evaluation.

    Every layer kernel bounds its waits on the tensor-core pipeline; a tile
    that gives up writes NaN rows and sets its launch's flag.  The flags are
    copied to pinned host memory behind the launches (no synchronisation) and
    read when they have arrived: at the next fused call, or in check_layer_flags(),
    which waits for them.  A raised flag becomes a RuntimeError naming the
    layer, so a stalled layer cannot pass for a normal step (TraceRays zeroes
    non-finite gradients)."""

    def __init__(self, device, names=None):
        self.device = device
        self.names = FLAG_NAMES if names is None else names
        self.flags = torch.zeros(len(self.names), dtype=torch.int32, device=device)
        self.host = None
        self.event = None

    def ptr(self, i: int):
        return ctypes.c_void_p(self.flags.data_ptr() + 4 * i)

    def post(self):
        """Queues the copy of the flags to the host behind the launches."""
        if self.flags.is_cuda:
            self.host = torch.empty(self.flags.shape, dtype=torch.int32, pin_memory=True)
            self.host.copy_(self.flags, non_blocking=True)
            self.event = torch.cuda.Event()
            self.event.record(torch.cuda.current_stream(self.device))
        else:
            self.host = self.flags.clone()
        _pending.append(self)

    def ready(self) -> bool:
        return self.event is None or self.event.query()

    def raise_if_set(self):
        if self.event is not None:
            self.event.synchronize()
        bad = [self.names[i] for i, v in enumerate(self.host.tolist()) if v]
        if bad:
            raise RuntimeError("sdfnet tcgen05 layer gave up waiting on the tensor-core pipeline and wrote NaN "
                               "rows: " + ", ".join(bad))


_pending: list = []


def check_layer_flags(wait: bool = True):
    """Raises RuntimeError if a fused sdfnet layer of an earlier call gave up.
    wait=False only reads the flags that have already reached the host."""
    keep = []
    while _pending:
        f = _pending.pop(0)
        if wait or f.ready():
            f.raise_if_set()
        else:
            keep.append(f)
    _pending.extend(keep)


def _wgrad(lib, stream, dz, m, act, k, bias_col, flag):
    """dW = dz[:, :m]^T act[:, :k] (+ the column sums of dz at bias_col) on
    the tensor cores, fp32 accumulation, returned as bf16 [m, act.shape[1]]."""
    from . import _lib
    dw = torch.zeros((m, act.shape[1]), dtype=torch.float32, device=dz.device)
    _lib.check(lib.sdfoam_mlp_wgrad(_p(dz), dz.shape[1], m, dz.shape[0], _p(act), act.shape[1], k, _p(dw),
                                    dw.shape[1], bias_col, flag, stream))
    return dw.to(torch.bfloat16)


class FusedSDFMLP(torch.autograd.Function):
    """sdfnet forward / backward on the library's tcgen05 kernels: hidden
    layers with fused activations (the last one also applies the output
    layer), dgrads with the softplus derivative fused, the weight gradients
    of every layer and the gradient of the positional encoding
    (libsdfoam_b200.so)."""

    @staticmethod
    def forward(ctx, points, center, scale, *wa):
        from . import _lib
        check_layer_flags(wait=False)
        lib = _lib.load()
        dev = points.device
        n = points.shape[0]
        stream = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
        c = center.reshape(3).float().contiguous() if center is not None else None
        bf = torch.bfloat16
        enc = torch.empty((n, ENC_LD), dtype=bf, device=dev)
        z = torch.empty((n, 4), dtype=torch.float32, device=dev)  # per 64-column block
        w_out = wa[8][0].contiguous()  # the output layer's row: 256 weights, bias at 256
        with torch.cuda.device(dev):
            _lib.check(lib.sdfoam_mlp_encode(_p(points), _p(c), n, 6, ENC_LD, _p(enc), stream))
            acts = [enc]
            x = enc
            flags = LayerFlags(dev)
            for l in range(8):
                # tcgen05 GEMM with softplus, skip and bias column fused; the
                # last hidden layer also applies the output layer
                nxt = torch.empty((n, HID_LD), dtype=bf, device=dev)
                w = wa[l]
                skip = l == 3
                args = (_p(x), x.shape[1], x.shape[1], n, _p(w), w.shape[1], w.shape[0],
                        _p(enc) if skip else None, ENC_LD, 39 if skip else 0, SKIP_OUT if skip else 256,
                        1.0 / math.sqrt(2.0) if skip else 1.0, _p(nxt), HID_LD)
                if l == 7:
                    _lib.check(lib.sdfoam_mlp_layer_dot(*args, _p(w_out), _p(z), 1.0 / scale, flags.ptr(l), stream))
                else:
                    _lib.check(lib.sdfoam_mlp_layer(*args, flags.ptr(l), stream))
                acts.append(nxt)
                x = nxt
        flags.post()
        ctx.flags = flags
        ctx.scale = scale
        ctx.has_center = c is not None
        ctx.save_for_backward(points, c if c is not None else points.new_empty(0), *acts, *wa)
        return ((z[:, 0:1] + z[:, 1:2]) + z[:, 2:3]) + z[:, 3:4]

    @staticmethod
    def backward(ctx, g):
        if torch.is_grad_enabled():
            # create_graph=True: the kernels below leave no graph behind
            raise RuntimeError("the fused sdfnet backward is not differentiable (double backward); take input "
                               "gradients for the eikonal term with SDFNetwork.gradient()")
        from . import _lib
        lib = _lib.load()
        saved = ctx.saved_tensors
        points, c = saved[0], (saved[1] if ctx.has_center else None)
        acts, wa = saved[2:11], saved[11:20]
        dev = points.device
        n = points.shape[0]
        bf = torch.bfloat16
        stream = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
        dw = [None] * 9
        dz = torch.zeros((n, 8), dtype=bf, device=dev)
        dz[:, 0] = (g.reshape(n) / ctx.scale).to(bf)
        flags = ctx.flags
        with torch.cuda.device(dev):
            dw[8] = _wgrad(lib, stream, dz, 8, acts[8], 256, 256, flags.ptr(FLAG_WGRAD))
            skip = torch.empty((n, ENC_LD), dtype=bf, device=dev)
            dz_next = dz
            for l in range(7, -1, -1):
                # tcgen05 dgrad of layer l + 1 fused with this layer's softplus derivative
                wt = wa[l + 1].t().contiguous()  # [inputs of layer l + 1, its outputs]
                skip_layer = l == 3
                ldz = 224 if skip_layer else 256
                dzl = torch.empty((n, ldz), dtype=bf, device=dev)
                _lib.check(lib.sdfoam_mlp_layer_backward(
                    _p(dz_next), dz_next.shape[1], dz_next.shape[1], n, _p(wt), wt.shape[1], 256, _p(acts[l + 1]),
                    HID_LD, SKIP_OUT if skip_layer else 256, 1.0 / math.sqrt(2.0) if skip_layer else 1.0,
                    _p(dzl), ldz, _p(skip) if skip_layer else None, ENC_LD, flags.ptr(8 + 7 - l), stream))
                # this layer's weight gradient (bias: the ones column at 256;
                # layer 0's input carries its ones column at 39)
                if l == 0:
                    dw[0] = _wgrad(lib, stream, dzl, 256, acts[0], ENC_LD, -1, flags.ptr(FLAG_WGRAD + 8))
                else:
                    dw[l] = _wgrad(lib, stream, dzl, ldz, acts[l], 256, 256, flags.ptr(FLAG_WGRAD + 8 - l))
                dz_next = dzl
            # gradient of the encoding: dz0 W0 plus the skip connection's
            w0t = wa[0].t().contiguous()  # [48, 256]
            denc = torch.empty((n, ENC_LD), dtype=bf, device=dev)
            _lib.check(lib.sdfoam_mlp_input_grad(_p(dz_next), dz_next.shape[1], 256, n, _p(w0t), w0t.shape[1],
                                                 w0t.shape[0], _p(skip), ENC_LD, 39, _p(denc), ENC_LD,
                                                 flags.ptr(FLAG_INPUT), stream))
            dpoints = torch.zeros((n, 3), dtype=torch.float32, device=dev)
            _lib.check(lib.sdfoam_mlp_decode(_p(points), _p(c), n, 6, _p(denc), ENC_LD, _p(dpoints), stream))
        flags.post()
        return (dpoints, None, None, *dw)


# Give-up flags of one eikonal evaluation (FusedSDFGradient), in flag order.
EIK_FLAG_NAMES = (tuple(f"eikonal: forward hidden layer {l}" for l in range(8))
                  + tuple(f"eikonal: dgrad of layer {l}" for l in range(7, -1, -1))
                  + ("eikonal: gradient of the positional encoding",)
                  + tuple(f"eikonal: tangent of layer {l}" for l in range(8))
                  + tuple(f"eikonal: second sweep of layer {l}" for l in range(7, -1, -1))
                  + ("eikonal: second sweep's encoding gradient",)
                  + tuple(f"eikonal: weight gradient of layer {l}" for l in range(8, -1, -1))
                  + tuple(f"eikonal: tangent weight gradient of layer {l}" for l in range(7, -1, -1)))


class FusedSDFGradient(torch.autograd.Function):
    """g = d sdf / d x of the sdfnet (the eikonal term's input gradient,
    sdfoam_model/sdfnet.py:144-148) on the library's tcgen05 kernels, with a
    backward that is the eikonal loss's double backward (train.py:293-326).

    forward: the forward sweep (stored activations), the first-order
    backward sweep (dgrads with the softplus derivative fused, stored as
    dz_l) and the encoding's chain rule give g.
    backward (given gbar = dL/dg), layer by layer:
      tangent   t_enc = J_enc gbar; ta_l = sp'(z_l) * (W_l t_in_l), also
                keeping tz_l = W_l t_in_l (sdfoam_mlp_layer_tangent)
      second    S_7 = dz_7 tz_7 sp''/sp'; S_l = sp'(z_l) * [W_{l+1}^T
                S_{l+1}] + dz_l tz_l sp''(z_l)/sp'(z_l) (sdfoam_mlp_layer_second;
                sp''/sp' = 100 (1 - sp'))
      weights   dL/dW_l = dz_l^T t_in_l + S_l^T in_l (bias: sum S_l),
                dL/dW_8 = sum ta_7 / scale (sdfoam_mlp_wgrad, twice into one
                accumulator)
      input     dL/dx = J_enc^T denc_S + H_enc[denc](gbar)
                (sdfoam_mlp_input_grad, sdfoam_mlp_decode_hessian)
    The layer-by-layer form is checked against autograd in float64 by
    tests/test_eikonal_chain.py."""

    @staticmethod
    def forward(ctx, points, center, scale, *wa):
        from . import _lib
        check_layer_flags(wait=False)
        lib = _lib.load()
        dev = points.device
        n = points.shape[0]
        bf = torch.bfloat16
        stream = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
        c = center.reshape(3).float().contiguous() if center is not None else None
        flags = LayerFlags(dev, EIK_FLAG_NAMES)
        enc = torch.empty((n, ENC_LD), dtype=bf, device=dev)
        with torch.cuda.device(dev):
            _lib.check(lib.sdfoam_mlp_encode(_p(points), _p(c), n, 6, ENC_LD, _p(enc), stream))
            acts = [enc]
            x = enc
            for l in range(8):
                nxt = torch.empty((n, HID_LD), dtype=bf, device=dev)
                w = wa[l]
                skip = l == 3
                _lib.check(lib.sdfoam_mlp_layer(_p(x), x.shape[1], x.shape[1], n, _p(w), w.shape[1], w.shape[0],
                                                _p(enc) if skip else None, ENC_LD, 39 if skip else 0,
                                                SKIP_OUT if skip else 256, 1.0 / math.sqrt(2.0) if skip else 1.0,
                                                _p(nxt), HID_LD, flags.ptr(l), stream))
                acts.append(nxt)
                x = nxt
            # first-order backward of sdf = z_8 / scale
            dz_next = torch.zeros((n, 8), dtype=bf, device=dev)
            dz_next[:, 0] = 1.0 / scale
            dzs = [None] * 8
            skip = torch.empty((n, ENC_LD), dtype=bf, device=dev)
            for l in range(7, -1, -1):
                wt = wa[l + 1].t().contiguous()
                skip_layer = l == 3
                ldz = 224 if skip_layer else 256
                dzl = torch.empty((n, ldz), dtype=bf, device=dev)
                _lib.check(lib.sdfoam_mlp_layer_backward(
                    _p(dz_next), dz_next.shape[1], dz_next.shape[1], n, _p(wt), wt.shape[1], 256, _p(acts[l + 1]),
                    HID_LD, SKIP_OUT if skip_layer else 256, 1.0 / math.sqrt(2.0) if skip_layer else 1.0,
                    _p(dzl), ldz, _p(skip) if skip_layer else None, ENC_LD, flags.ptr(8 + 7 - l), stream))
                dzs[l] = dzl
                dz_next = dzl
            w0t = wa[0].t().contiguous()
            denc = torch.empty((n, ENC_LD), dtype=bf, device=dev)
            _lib.check(lib.sdfoam_mlp_input_grad(_p(dz_next), dz_next.shape[1], 256, n, _p(w0t), w0t.shape[1],
                                                 w0t.shape[0], _p(skip), ENC_LD, 39, _p(denc), ENC_LD,
                                                 flags.ptr(16), stream))
            g = torch.zeros((n, 3), dtype=torch.float32, device=dev)
            _lib.check(lib.sdfoam_mlp_decode(_p(points), _p(c), n, 6, _p(denc), ENC_LD, _p(g), stream))
        flags.post()
        ctx.flags = flags
        ctx.scale = scale
        ctx.has_center = c is not None
        ctx.save_for_backward(points, c if c is not None else points.new_empty(0), denc, *acts, *dzs, *wa)
        return g

    @staticmethod
    def backward(ctx, gbar):
        if torch.is_grad_enabled():
            raise RuntimeError("the fused eikonal backward is not differentiable again")
        from . import _lib
        lib = _lib.load()
        saved = ctx.saved_tensors
        points, c, denc = saved[0], (saved[1] if ctx.has_center else None), saved[2]
        acts, dzs, wa = saved[3:12], saved[12:20], saved[20:29]
        dev = points.device
        n = points.shape[0]
        bf = torch.bfloat16
        stream = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
        flags = LayerFlags(dev, EIK_FLAG_NAMES)
        gb = gbar.float().contiguous()
        rs2 = 1.0 / math.sqrt(2.0)
        with torch.cuda.device(dev):
            # tangent sweep along gbar
            tenc = torch.empty((n, ENC_LD), dtype=bf, device=dev)
            _lib.check(lib.sdfoam_mlp_encode_jvp(_p(points), _p(c), n, 6, _p(gb), ENC_LD, _p(tenc), stream))
            t_ins, tzs = [tenc], []
            t_in = tenc
            for l in range(8):
                w = wa[l]
                skip = l == 3
                ta = torch.empty((n, 256), dtype=bf, device=dev)
                tz = torch.empty((n, 256), dtype=bf, device=dev)
                _lib.check(lib.sdfoam_mlp_layer_tangent(
                    _p(t_in), t_in.shape[1], 48 if l == 0 else 256, n, _p(w), w.shape[1], w.shape[0],
                    _p(acts[l + 1]), HID_LD, SKIP_OUT if skip else 256, rs2 if skip else 1.0,
                    _p(tenc) if skip else None, ENC_LD, 39 if skip else 0, _p(ta), 256, _p(tz), 256,
                    flags.ptr(17 + l), stream))
                t_ins.append(ta)
                tzs.append(tz)
                t_in = ta
            # second sweep: S_l with the softplus curvature along the tangent
            s_next = torch.zeros((n, 8), dtype=bf, device=dev)
            skip_s = torch.empty((n, ENC_LD), dtype=bf, device=dev)
            Ss = [None] * 8
            for l in range(7, -1, -1):
                wt = wa[l + 1].t().contiguous()
                skip_layer = l == 3
                ldz = 224 if skip_layer else 256
                sl = torch.empty((n, ldz), dtype=bf, device=dev)
                _lib.check(lib.sdfoam_mlp_layer_second(
                    _p(s_next), s_next.shape[1], s_next.shape[1], n, _p(wt), wt.shape[1], 256, _p(acts[l + 1]),
                    HID_LD, SKIP_OUT if skip_layer else 256, rs2 if skip_layer else 1.0, _p(dzs[l]),
                    dzs[l].shape[1], _p(tzs[l]), 256, _p(sl), ldz, _p(skip_s) if skip_layer else None, ENC_LD,
                    flags.ptr(25 + 7 - l), stream))
                Ss[l] = sl
                s_next = sl
            w0t = wa[0].t().contiguous()
            denc_s = torch.empty((n, ENC_LD), dtype=bf, device=dev)
            _lib.check(lib.sdfoam_mlp_input_grad(_p(s_next), s_next.shape[1], 256, n, _p(w0t), w0t.shape[1],
                                                 w0t.shape[0], _p(skip_s), ENC_LD, 39, _p(denc_s), ENC_LD,
                                                 flags.ptr(33), stream))
            dx = torch.zeros((n, 3), dtype=torch.float32, device=dev)
            _lib.check(lib.sdfoam_mlp_decode_hessian(_p(points), _p(c), n, 6, _p(denc_s), _p(denc), ENC_LD, _p(gb),
                                                     _p(dx), stream))
            # weight gradients: dz_l^T t_in_l + S_l^T in_l, and sum ta_7 / scale for the output layer
            dw = [None] * 9
            ones = torch.zeros((n, 8), dtype=bf, device=dev)
            ones[:, 0] = 1.0 / ctx.scale
            d8 = torch.zeros((8, HID_LD), dtype=torch.float32, device=dev)
            _lib.check(lib.sdfoam_mlp_wgrad(_p(ones), 8, 8, n, _p(t_ins[8]), 256, 256, _p(d8), HID_LD, -1,
                                            flags.ptr(34), stream))
            dw[8] = d8.to(bf)
            for l in range(8):
                m = Ss[l].shape[1]
                ld_in = acts[l].shape[1]
                k = ENC_LD if l == 0 else 256
                acc = torch.zeros((m, ld_in), dtype=torch.float32, device=dev)
                _lib.check(lib.sdfoam_mlp_wgrad(_p(Ss[l]), m, m, n, _p(acts[l]), ld_in, k, _p(acc), ld_in,
                                                -1 if l == 0 else 256, flags.ptr(35 + 7 - l), stream))
                _lib.check(lib.sdfoam_mlp_wgrad(_p(dzs[l]), m, m, n, _p(t_ins[l]), t_ins[l].shape[1], k, _p(acc),
                                                ld_in, -1, flags.ptr(43 + 7 - l), stream))
                dw[l] = acc.to(bf)
        flags.post()
        return (dx, None, None, *dw)


def mlp_flops_per_site(net: SDFNetwork) -> int:
    """Multiply-adds x 2 of one forward evaluation."""
    macs = 0
    for l in range(net.num_layers - 1):
        lin = getattr(net, f"lin{l}")
        w = lin.weight_v if isinstance(lin, WeightNormLinear) else lin.weight
        macs += w.shape[0] * w.shape[1]
    return 2 * macs
