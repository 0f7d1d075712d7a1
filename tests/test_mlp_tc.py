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
