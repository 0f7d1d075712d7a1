"""The tcgen05 sdfnet layer (sdfoam_mlp_layer) against the same layer as a
float32 GEMM followed by the library's activation rule, on the shapes the
fused MLP uses: the encoding layer (K 48), hidden layers (K 264), the layer
feeding the skip connection (224 weight rows, encoding appended, 1/sqrt 2),
and row counts that end in a partial 128-row tile."""
import ctypes
import math

import pytest
import torch

pytestmark = pytest.mark.gpu


def _ref(x, w, enc, enc_cols, zc, scale, ld):
    z = x.float() @ w.float().t()
    n = x.shape[0]
    out = torch.zeros((n, ld), dtype=torch.float32, device=x.device)
    out[:, :zc] = scale * torch.nn.functional.softplus(z[:, :zc], beta=100.0)
    if enc_cols:
        out[:, zc:zc + enc_cols] = scale * enc[:, :enc_cols].float()
    out[:, zc + enc_cols] = 1.0
    return out


def _run(x, w, enc, enc_cols, zc, scale, ld):
    from sdfoam_b200 import _lib
    lib = _lib.load()
    n, kx = x.shape[0], x.shape[1]
    out = torch.full((n, ld), float("nan"), dtype=torch.bfloat16, device=x.device)
    err = torch.zeros(1, dtype=torch.int32, device=x.device)
    p = lambda t: None if t is None else ctypes.c_void_p(t.data_ptr())
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    _lib.check(lib.sdfoam_mlp_layer(p(x), x.stride(0), kx, n, p(w), w.stride(0), w.shape[0], p(enc),
                                    enc.stride(0) if enc is not None else 0, enc_cols, zc, scale, p(out), ld,
                                    p(err), stream))
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    return out


@pytest.mark.parametrize("n", [1, 127, 128, 1000, 70001])
@pytest.mark.parametrize("kind", ["encoding", "hidden", "skip"])
def test_layer_matches_gemm_and_activation(n, kind):
    g = torch.Generator(device="cuda").manual_seed(n)
    dev = torch.device("cuda:0")
    bf = torch.bfloat16
    if kind == "encoding":
        kx, nw, zc, enc_cols, scale = 48, 256, 256, 0, 1.0
    elif kind == "hidden":
        kx, nw, zc, enc_cols, scale = 264, 256, 256, 0, 1.0
    else:
        kx, nw, zc, enc_cols, scale = 264, 224, 217, 39, 1.0 / math.sqrt(2.0)
    x = (torch.randn((n, kx), generator=g, device=dev) * 0.5).to(bf)
    x[:, kx - 8:] = 0
    x[:, kx - 8] = 1.0  # the bias column
    w = (torch.randn((nw, kx), generator=g, device=dev) / math.sqrt(kx)).to(bf)
    if kind == "skip":
        w[zc:] = 0
    enc = (torch.randn((n, 48), generator=g, device=dev)).to(bf) if enc_cols else None
    got = _run(x, w, enc, enc_cols, zc, scale, 264).float()
    ref = _ref(x, w, enc, enc_cols, zc, scale, 264)
    assert torch.isfinite(got).all()
    # bf16 outputs: one rounding (2^-8 relative) plus fp32 accumulation order
    err = (got - ref).abs() - 8e-3 * ref.abs()
    assert err.max().item() < 2e-3, (err.max().item(), (err > 2e-3).sum().item())


def _run_backward(dz_next, wt, act, cols, scale, ldz, with_skip):
    from sdfoam_b200 import _lib
    lib = _lib.load()
    n, k = dz_next.shape
    dz = torch.full((n, ldz), float("nan"), dtype=torch.bfloat16, device=dz_next.device)
    skip = torch.full((n, 48), float("nan"), dtype=torch.bfloat16, device=dz_next.device) if with_skip else None
    err = torch.zeros(1, dtype=torch.int32, device=dz_next.device)
    p = lambda t: None if t is None else ctypes.c_void_p(t.data_ptr())
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    _lib.check(lib.sdfoam_mlp_layer_backward(p(dz_next), dz_next.stride(0), k, n, p(wt), wt.stride(0), 256, p(act),
                                             act.stride(0), cols, scale, p(dz), ldz, p(skip), 48, p(err), stream))
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    return dz, skip


@pytest.mark.parametrize("n", [1, 1000, 70001])
@pytest.mark.parametrize("kind", ["first", "hidden", "skip"])
def test_layer_backward_matches_gemm_and_derivative(n, kind):
    """dz = scale * (dz_next Wt^T)[:, :cols] * sigmoid(100 z) with the
    sigmoid recomputed from the stored activation; the skip columns' gradient
    goes to its own buffer."""
    g = torch.Generator(device="cuda").manual_seed(n + 7)
    dev = torch.device("cuda:0")
    bf = torch.bfloat16
    k = {"first": 8, "hidden": 256, "skip": 256}[kind]
    cols, scale, ldz = (217, 1.0 / math.sqrt(2.0), 224) if kind == "skip" else (256, 1.0, 256)
    dz_next = torch.randn((n, k), generator=g, device=dev).to(bf)
    wt = (torch.randn((264, k), generator=g, device=dev) / math.sqrt(k)).to(bf)
    z = torch.randn((n, 264), generator=g, device=dev) * 0.05
    act = (scale * torch.nn.functional.softplus(z, beta=100.0)).to(bf)
    dz, skip = _run_backward(dz_next, wt, act, cols, scale, ldz, kind == "skip")
    da = dz_next.float() @ wt.float()[:256].t()
    deriv = 1.0 - torch.exp(-100.0 * act[:, :cols].float() / scale)
    ref = scale * da[:, :cols] * deriv
    got = dz.float()
    assert torch.isfinite(got).all()
    e = (got[:, :cols] - ref).abs() - 1e-2 * ref.abs()
    assert e.max().item() < 2e-3 * max(1.0, ref.abs().max().item()), e.max().item()
    assert (got[:, cols:] == 0).all()
    if kind == "skip":
        sref = scale * da[:, cols:256]
        es = (skip.float()[:, :256 - cols] - sref).abs() - 1e-2 * sref.abs()
        assert es.max().item() < 2e-3 * max(1.0, sref.abs().max().item())


def _p(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


@pytest.mark.parametrize("n", [1, 63, 1000, 70001, 600000])
@pytest.mark.parametrize("kind", ["hidden", "skip", "first", "output"])
def test_weight_gradient_matches_fp32_gemm(n, kind):
    """sdfoam_mlp_wgrad: dw = dz^T act (+ the column sums of dz at the bias
    column) against a float32 GEMM of the same bf16 operands, on the shapes
    of the sdfnet's layers: hidden (256 x 264, bias at 256), the skip layer
    (224 rows), the first layer (input = the 48-column encoding whose ones
    column is at 39, no separate bias column) and the output layer (dz with 8
    columns)."""
    from sdfoam_b200 import _lib
    lib = _lib.load()
    g = torch.Generator(device="cuda").manual_seed(n + 11)
    dev = torch.device("cuda:0")
    bf = torch.bfloat16
    m, lda, k, bias_col = {"hidden": (256, 264, 256, 256), "skip": (224, 264, 256, 256),
                           "first": (256, 48, 48, -1), "output": (8, 264, 256, 256)}[kind]
    dz = torch.randn((n, m), generator=g, device=dev).to(bf)
    act = (torch.rand((n, lda), generator=g, device=dev) * 0.2).to(bf)
    act[:, k:] = 0
    if bias_col >= 0:
        act[:, bias_col] = 1.0
    dw = torch.zeros((m, lda), dtype=torch.float32, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    _lib.check(lib.sdfoam_mlp_wgrad(_p(dz), m, m, n, _p(act), lda, k, _p(dw), lda, bias_col, _p(err), _stream()))
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    ref = dz.double().t() @ act.double()
    ref_abs = dz.double().abs().t() @ act.double().abs()
    # fp32 accumulation of bf16 products: relative 1e-4 of the sum of |terms|
    bad = (dw.double() - ref).abs() > 1e-4 * ref_abs + 1e-6
    assert not bad.any(), (bad.sum().item(), (dw.double() - ref).abs().max().item())


@pytest.mark.parametrize("n", [1, 1000, 70001])
def test_input_gradient_matches_fp32_gemm(n):
    """sdfoam_mlp_input_grad: denc = dz0 W0 + the skip connection's gradient
    on the first 39 columns, against a float32 GEMM (bf16 output)."""
    from sdfoam_b200 import _lib
    lib = _lib.load()
    g = torch.Generator(device="cuda").manual_seed(n + 5)
    dev = torch.device("cuda:0")
    bf = torch.bfloat16
    dz = torch.randn((n, 256), generator=g, device=dev).to(bf)
    w0 = (torch.randn((256, 48), generator=g, device=dev) / 16).to(bf)
    skip = torch.randn((n, 48), generator=g, device=dev).to(bf)
    w0t = w0.t().contiguous()
    out = torch.full((n, 48), float("nan"), dtype=bf, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    _lib.check(lib.sdfoam_mlp_input_grad(_p(dz), 256, 256, n, _p(w0t), 256, 48, _p(skip), 48, 39, _p(out), 48,
                                         _p(err), _stream()))
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    ref = dz.float() @ w0.float()
    ref[:, :39] += skip[:, :39].float()
    e = (out.float() - ref).abs() - 1e-2 * ref.abs()
    assert e.max().item() < 2e-3 * max(1.0, ref.abs().max().item()), e.max().item()


@pytest.mark.parametrize("n", [1, 1000, 70001])
def test_layer_with_output_dot(n):
    """sdfoam_mlp_layer_dot: the hidden layer's bf16 output as
    sdfoam_mlp_layer, plus the single-output final layer applied to it
    (z = (out[:, :256] . w + w[256]) * dot_scale) in the same kernel."""
    from sdfoam_b200 import _lib
    lib = _lib.load()
    g = torch.Generator(device="cuda").manual_seed(n + 3)
    dev = torch.device("cuda:0")
    bf = torch.bfloat16
    x = (torch.randn((n, 264), generator=g, device=dev) * 0.5).to(bf)
    x[:, 256:] = 0
    x[:, 256] = 1.0
    w = (torch.randn((256, 264), generator=g, device=dev) / 16).to(bf)
    wdot = (torch.randn((264,), generator=g, device=dev) / 16).to(bf)
    out = torch.full((n, 264), float("nan"), dtype=bf, device=dev)
    z4 = torch.full((n, 4), float("nan"), dtype=torch.float32, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    _lib.check(lib.sdfoam_mlp_layer_dot(_p(x), 264, 264, n, _p(w), 264, 256, None, 0, 0, 256, 1.0, _p(out), 264,
                                        _p(wdot), _p(z4), 0.5, _p(err), _stream()))
    torch.cuda.synchronize()
    z = z4.sum(1)
    assert int(err.item()) == 0
    ref_out = _ref(x, w, None, 0, 256, 1.0, 264)
    e = (out.float() - ref_out).abs() - 8e-3 * ref_out.abs()
    assert e.max().item() < 2e-3
    zref = 0.5 * (out.float()[:, :256] @ wdot.float()[:256] + wdot.float()[256])
    zabs = 0.5 * (out.float()[:, :256].abs() @ wdot.float()[:256].abs() + wdot.float()[256].abs())
    assert ((z - zref).abs() <= 1e-5 * zabs + 1e-6).all()
