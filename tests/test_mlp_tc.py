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
