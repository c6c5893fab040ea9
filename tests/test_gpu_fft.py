"""Parity of the FFT convolution kernels with the oracle: the reference's own
FFT route outputs (tests/golden) at small sizes, the float64 numpy
restatement of that route at other sizes, and at the BASELINE size a slice of
the full-size output (the per-channel computation is independent of the
others, so a slice checks the full-size launch).  FFT-route bar: rel-L2 <= 5e-3."""
from __future__ import annotations

import math

import numpy as np
import pytest
import torch

import oracle
from conftest import load_golden, torch_dtype

pytestmark = pytest.mark.gpu

FFT_TOL = 5e-3


def _np(t):
    return t.detach().float().cpu().numpy()


def _kaiming(shape, g):
    bound = 1.0 / math.sqrt(math.prod(shape[1:]))
    return (torch.rand(*shape, generator=g) * 2 - 1) * bound


@pytest.mark.parametrize("case", list(load_golden("fftconv1d")))
def test_fftconv1d_golden(cuda, case):
    from amd_tuned_torch import fftconv_ops
    d = load_golden("fftconv1d")[case]
    dt = torch_dtype(d["dtype"])
    B, C, L, K, pad = (int(v) for v in d["meta"])
    x = torch.as_tensor(d["x"]).to(cuda, dt)
    w = torch.as_tensor(d["w"]).to(cuda, dt)
    b = torch.as_tensor(d["b"]).to(cuda, dt)
    y = fftconv_ops.fftconv1d(x, w, b, pad)
    assert y is not None and tuple(y.shape) == d["y"].shape
    tol = 1e-5 if d["dtype"] == "f32" else FFT_TOL
    assert oracle.rel_l2(_np(y), d["y_fft"]) <= tol   # the reference's FFT route
    assert oracle.rel_l2(_np(y), d["y"]) <= tol       # and direct convolution


@pytest.mark.parametrize("B,C,L,K,pad,dt", [
    (1, 3, 1000, 257, 128, "f32"), (3, 2, 4000, 64, 0, "bf16"), (2, 4, 5000, 999, 499, "f16"),
    (5, 1, 100, 100, 99, "f32"), (4, 8, 16384, 2048, 1024, "f16"),
])
def test_fftconv1d_shapes(cuda, B, C, L, K, pad, dt):
    from amd_tuned_torch import fftconv_ops
    g = torch.Generator().manual_seed(L + K)
    x = torch.randn(B, C, L, generator=g).to(torch_dtype(dt))
    w = _kaiming((C, 1, K), g).to(torch_dtype(dt))
    b = torch.randn(C, generator=g).to(torch_dtype(dt))
    y = fftconv_ops.fftconv1d(x.to(cuda), w.to(cuda), b.to(cuda), pad)
    ref = oracle.fft_conv_np(x.float().numpy(), w.float().numpy(), b.float().numpy(), (pad,),
                             groups=C)
    tol = 1e-5 if dt == "f32" else FFT_TOL
    assert oracle.rel_l2(_np(y), ref) <= tol


# Overlap-save segments (b200_fftconv1d_fwd_os) against the whole-row
# transform and the float64 oracle: several segments with a ragged last one,
# pad 0 / pad > K, an odd batch, and a row longer than one transform holds.
@pytest.mark.parametrize("B,C,L,K,pad,nfft,dt", [
    (3, 2, 20000, 1000, 500, 4096, "f32"), (2, 3, 9000, 257, 0, 2048, "bf16"),
    (1, 2, 5000, 100, 300, 1024, "f16"), (2, 2, 40000, 2048, 1024, 8192, "f16"),
    (2, 3, 30000, 3000, 1500, 16384, "f32"), (3, 2, 3000, 500, 250, 2048, "f32"),
    (5, 3, 30000, 2048, 1024, 8192, "f32"), (2, 2, 9000, 700, 0, 4096, "bf16"),
])
def test_fftconv1d_overlap_save(cuda, B, C, L, K, pad, nfft, dt):
    from amd_tuned_torch import ops
    g = torch.Generator().manual_seed(L + K + nfft)
    x = torch.randn(B, C, L, generator=g).to(torch_dtype(dt))
    w = _kaiming((C, 1, K), g).to(torch_dtype(dt))
    b = torch.randn(C, generator=g).to(torch_dtype(dt))
    y = ops.fftconv1d(x.to(cuda), w.to(cuda), b.to(cuda), pad, nfft, segmented=True)
    assert y is not None and tuple(y.shape) == (B, C, L + 2 * pad - K + 1)
    ref = oracle.fft_conv_np(x.float().numpy(), w.float().numpy(), b.float().numpy(), (pad,),
                             groups=C)
    tol = 1e-5 if dt == "f32" else FFT_TOL
    assert oracle.rel_l2(_np(y), ref) <= tol
    assert ops.read_device_flags() == 0


# Whole-row transforms at the register-resident lengths (2048 ... 16384)
# and at lengths that take the shared-memory pass-per-radix plan.
@pytest.mark.parametrize("nfft", [2048, 4096, 8192, 16384, 6144, 10240])
@pytest.mark.parametrize("dt", ["f32", "bf16"])
def test_fftconv1d_whole_row_lengths(cuda, nfft, dt):
    from amd_tuned_torch import ops
    g = torch.Generator().manual_seed(nfft)
    B, C, K = 3, 2, nfft // 8 + 1
    L, pad = nfft - 2 * (K // 2) - 5, K // 2
    x = torch.randn(B, C, L, generator=g).to(torch_dtype(dt))
    w = _kaiming((C, 1, K), g).to(torch_dtype(dt))
    b = torch.randn(C, generator=g).to(torch_dtype(dt))
    y = ops.fftconv1d(x.to(cuda), w.to(cuda), b.to(cuda), pad, nfft, segmented=False)
    assert y is not None and tuple(y.shape) == (B, C, L + 2 * pad - K + 1)
    ref = oracle.fft_conv_np(x.float().numpy(), w.float().numpy(), b.float().numpy(), (pad,),
                             groups=C)
    tol = 1e-5 if dt == "f32" else FFT_TOL
    assert oracle.rel_l2(_np(y), ref) <= tol


def test_fftconv1d_length_contest(cuda, monkeypatch):
    """The transform-length contest times every plan once, caches the
    winner, and the winner's output meets the FFT bar; a second call runs
    the cached plan."""
    from amd_tuned_torch import fftconv_ops, kernel_select
    monkeypatch.setattr(kernel_select, "_ENABLED", True)
    kernel_select.reset()
    g = torch.Generator().manual_seed(12)
    B, C, L, K, pad = 4, 8, 12000, 700, 350
    x = torch.randn(B, C, L, generator=g).half()
    w = _kaiming((C, 1, K), g).half()
    b = torch.randn(C, generator=g).half()
    xd, wd, bd = x.to(cuda), w.to(cuda), b.to(cuda)
    ref = oracle.fft_conv_np(x.float().numpy(), w.float().numpy(), b.float().numpy(), (pad,),
                             groups=C)
    y = fftconv_ops.fftconv1d(xd, wd, bd, pad)
    assert oracle.rel_l2(_np(y), ref) <= FFT_TOL
    plans = dict(fftconv_ops.fftconv1d_plans(L, K, pad))
    assert len(plans) > 1
    won = [v for k, v in kernel_select.debug_winners().items()
           if "fftconv_len" in str(k)]
    assert len(won) == 1 and won[0] in plans
    assert fftconv_ops.fftconv1d_chosen_plan(xd, wd, pad) == plans[won[0]]
    y2 = fftconv_ops.fftconv1d(xd, wd, bd, pad)
    assert oracle.rel_l2(_np(y2), ref) <= FFT_TOL
    kernel_select.reset()


def test_fftconv1d_cfg4b_full_size(cuda):
    """BASELINE cfg 4b: x[16,1024,16384] fp16 ~N(0,1), w[1024,1,2048] kaiming-U,
    bias, groups 1024, padding 1024 -> L_out 16385.  Checked on a slice of
    batches/channels against the float64 oracle."""
    from amd_tuned_torch import fftconv_ops, ops
    g = torch.Generator().manual_seed(44)
    x = torch.randn(16, 1024, 16384, generator=g).half()
    w = _kaiming((1024, 1, 2048), g).half()
    b = _kaiming((1024, 2048), g)[:, 0].half()
    y = fftconv_ops.fftconv1d(x.to(cuda), w.to(cuda), b.to(cuda), 1024)
    assert tuple(y.shape) == (16, 1024, 16385)
    bs, cs = [0, 7, 15], [0, 1, 511, 1023]
    xs = x[bs][:, cs].float().numpy()
    ref = oracle.fft_conv_np(xs, w[cs].float().numpy(), b[cs].float().numpy(), (1024,),
                             groups=len(cs))
    got = y[bs][:, cs]
    assert oracle.rel_l2(_np(got), ref) <= FFT_TOL
    assert torch.isfinite(y).all()
    assert ops.read_device_flags() == 0


def test_fftconv1d_spectrum_cache_follows_weight(cuda):
    """A new weight at a reused address must get its own spectrum."""
    from amd_tuned_torch import fftconv_ops
    g = torch.Generator().manual_seed(3)
    x = torch.randn(2, 4, 500, generator=g).to(cuda)
    for s in range(3):
        w = torch.randn(4, 1, 65, generator=torch.Generator().manual_seed(s)).to(cuda)
        y = fftconv_ops.fftconv1d(x, w, None, 32)
        ref = oracle.fft_conv_np(x.cpu().numpy(), w.cpu().numpy(), None, (32,), groups=4)
        assert oracle.rel_l2(_np(y), ref) <= 1e-5
        del w


# ----------------------------------------------------------- FFT conv3d ---
@pytest.mark.parametrize("case", list(load_golden("fftconv3d")))
def test_fftconv3d_golden(cuda, case):
    from amd_tuned_torch import fftconv_ops
    d = load_golden("fftconv3d")[case]
    dt = torch_dtype(d["dtype"])
    m = [int(v) for v in d["meta"]]
    p = tuple(m[9:12])
    x = torch.as_tensor(d["x"]).to(cuda, dt)
    w = torch.as_tensor(d["w"]).to(cuda, dt)
    b = torch.as_tensor(d["b"]).to(cuda, dt)
    y = fftconv_ops.fft_conv3d(x, w, b, padding=p)
    assert y is not None and tuple(y.shape) == d["y"].shape
    tol = 1e-5 if d["dtype"] == "f32" else FFT_TOL
    assert oracle.rel_l2(_np(y), d["y_fft"]) <= tol
    assert oracle.rel_l2(_np(y), d["y"]) <= tol


@pytest.mark.parametrize("N,Cin,D,H,W,Cout,k,p,dt", [
    (3, 5, 7, 9, 10, 3, (5, 6, 7), (2, 3, 3), "f32"),
    (1, 16, 8, 12, 12, 70, (7, 7, 7), (3, 3, 3), "bf16"),
    (2, 8, 6, 20, 6, 8, (6, 9, 6), (0, 4, 2), "f16"),
    # depth transform of 30 points (the register depth kernels): channel
    # counts that are not multiples of the 16-channel tile, an odd batch
    (3, 20, 16, 12, 12, 24, (15, 5, 5), (7, 2, 2), "f16"),
    (1, 6, 10, 8, 8, 10, (21, 3, 3), (10, 1, 1), "f32"),
    # input channels past one 64-channel block, narrow (Cout <= 16) and wide
    # contraction variants, output-channel counts off the lane-group widths
    (1, 70, 6, 8, 8, 16, (3, 3, 3), (1, 1, 1), "bf16"),
    (2, 72, 5, 6, 6, 13, (3, 3, 3), (1, 1, 1), "f32"),
    (1, 130, 4, 6, 6, 40, (3, 3, 3), (1, 1, 1), "f16"),
    # Cout a multiple of 64 with even input rows: the bulk-copy contraction
    (2, 24, 5, 8, 8, 64, (3, 3, 3), (1, 1, 1), "f16"),
    (3, 10, 4, 6, 6, 128, (3, 3, 3), (1, 1, 1), "bf16"),
    (2, 16, 5, 6, 8, 64, (3, 3, 3), (1, 1, 1), "f32"),
    # 80 x 80 planes (the compile-time 16 x 5 plane kernels), ragged data
    # rows inside the plane, an odd batch
    (3, 4, 4, 70, 66, 6, (3, 11, 15), (1, 5, 7), "f16"),
])
def test_fftconv3d_shapes(cuda, N, Cin, D, H, W, Cout, k, p, dt):
    from amd_tuned_torch import fftconv_ops
    g = torch.Generator().manual_seed(Cin * Cout)
    x = torch.randn(N, Cin, D, H, W, generator=g).to(torch_dtype(dt))
    w = _kaiming((Cout, Cin) + k, g).to(torch_dtype(dt))
    b = torch.randn(Cout, generator=g).to(torch_dtype(dt)) * 0.1
    y = fftconv_ops.fft_conv3d(x.to(cuda), w.to(cuda), b.to(cuda), padding=p)
    ref = oracle.fft_conv_np(x.float().numpy(), w.float().numpy(), b.float().numpy(), p)
    tol = 1e-5 if dt == "f32" else FFT_TOL
    assert oracle.rel_l2(_np(y), ref) <= tol


def test_fftconv3d_cfg4a_full_size(cuda):
    """BASELINE cfg 4a: x[2,64,16,64,64] fp16, w[64,64,15,15,15] kaiming-U, bias,
    padding 7; checked on a slice of output channels against the float64 oracle."""
    from amd_tuned_torch import fftconv_ops, ops
    g = torch.Generator().manual_seed(41)
    x = torch.randn(2, 64, 16, 64, 64, generator=g).half()
    w = _kaiming((64, 64, 15, 15, 15), g).half()
    b = _kaiming((64, 64 * 3375), g)[:, 0].half()
    y = fftconv_ops.fft_conv3d(x.to(cuda), w.to(cuda), b.to(cuda), padding=7)
    assert tuple(y.shape) == (2, 64, 16, 64, 64)
    cs = [0, 17, 63]
    ref = oracle.fft_conv_np(x.float().numpy(), w[cs].float().numpy(), b[cs].float().numpy(),
                             (7, 7, 7))
    assert oracle.rel_l2(_np(y[:, cs]), ref) <= FFT_TOL
    assert torch.isfinite(y).all()
    assert ops.read_device_flags() == 0
