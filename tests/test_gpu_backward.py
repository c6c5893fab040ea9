"""Backward kernels on the GPU: GroupNorm (b200_gn_bwd), depthwise conv1d
(b200_dwconv1d_bwd_weight + the tap-reversed forward), the differentiable FFT
conv1d route, and the custom ops under torch.compile.  Gradients are
compared with the float64 oracle restatements (oracle.np_*_backward, pinned
to torch autograd by tests/test_oracle.py) and with stock torch CPU fp32
autograd through the patched F.* entry points.  Bars: rel-L2 <= 1e-5 fp32,
<= 2e-3 fp16/bf16 direct kernels, <= 5e-3 FFT routes."""
from __future__ import annotations

import pytest
import torch
import torch.nn.functional as F

import oracle

pytestmark = pytest.mark.gpu

TOL = {torch.float32: 1e-5, torch.float16: 2e-3, torch.bfloat16: 2e-3}
FFT_TOL = {torch.float32: 1e-5, torch.float16: 5e-3, torch.bfloat16: 5e-3}


def _np(t):
    return t.detach().double().cpu().numpy()


def _ok(got, ref, dt, tol) -> bool:
    """rel-L2(got, ref) within `tol` plus what rounding the exact result to
    the output dtype costs by itself (a handful of bf16 parameter gradients
    already differ from fp64 by ~2e-3 when rounded correctly)."""
    rounded = torch.as_tensor(ref).to(dt).double().numpy()
    return oracle.rel_l2(_np(got), ref) <= tol + oracle.rel_l2(rounded, ref)


@pytest.fixture
def patched():
    import amd_tuned_torch
    from amd_tuned_torch import kernel_select
    kernel_select.reset()
    amd_tuned_torch.enable()
    yield amd_tuned_torch
    amd_tuned_torch.disable()
    kernel_select.reset()


# ------------------------------------------------------------- GroupNorm ---
@pytest.mark.parametrize("dt", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("shape,G,affine", [
    ((2, 64, 16, 16), 32, True), ((3, 12, 7, 5), 4, True), ((2, 32, 9), 1, False),
    ((1, 128, 4, 16, 16), 32, True), ((4, 512, 128, 128), 32, True)])
def test_group_norm_backward_kernel(cuda, dt, shape, G, affine):
    from amd_tuned_torch import ops
    g = torch.Generator().manual_seed(sum(shape) + G)
    x = (torch.randn(*shape, generator=g) * 2 + 0.5).to(dt)
    dy = torch.randn(*shape, generator=g).to(dt)
    C = shape[1]
    w = (torch.rand(C, generator=g) + 0.5).to(dt) if affine else None
    dx, dw, db = ops.group_norm_backward(dy.to(cuda), x.to(cuda), G,
                                         w.to(cuda) if affine else None, 1e-5,
                                         (True, affine, True), affine_dtype=dt)
    rx, rw, rb = oracle.np_group_norm_backward(_np(x), _np(dy), G, _np(w) if affine else None,
                                               1e-5)
    assert _ok(dx, rx, dt, TOL[dt])
    assert _ok(db, rb, dt, TOL[dt])
    if affine:
        assert _ok(dw, rw, dt, TOL[dt])
    else:
        assert dw is None


def test_group_norm_backward_fp16_large_group_stays_finite(cuda):
    from amd_tuned_torch import ops
    g = torch.Generator().manual_seed(7)
    x = (torch.randn(1, 32, 128, 128, generator=g) * 4).half()
    dy = torch.randn(1, 32, 128, 128, generator=g).half()
    dx, dw, db = ops.group_norm_backward(dy.to(cuda), x.to(cuda), 1,
                                         torch.ones(32, dtype=torch.half, device=cuda), 1e-5,
                                         (True, True, True))
    for t in (dx, dw, db):
        assert torch.isfinite(t.float()).all()
    rx, rw, rb = oracle.np_group_norm_backward(_np(x), _np(dy), 1, None, 1e-5)
    assert oracle.rel_l2(_np(dx), rx) <= 2e-3
    assert oracle.rel_l2(_np(db), rb) <= 2e-3


@pytest.mark.parametrize("dt", [torch.float32, torch.bfloat16])
def test_group_norm_training_through_patch(cuda, patched, dt):
    g = torch.Generator().manual_seed(3)
    x = (torch.randn(2, 64, 12, 12, generator=g) * 2).to(dt)
    w = (torch.rand(64, generator=g) + 0.5).to(dt)
    b = (torch.randn(64, generator=g) * 0.1).to(dt)
    dy = torch.randn(2, 64, 12, 12, generator=g).to(dt)
    xs, ws, bs = (t.to(cuda).requires_grad_() for t in (x, w, b))
    F.group_norm(xs, 32, ws, bs, 1e-6).backward(dy.to(cuda))
    rx, rw, rb = oracle.stock_group_norm_backward(_np(x), _np(dy), 32, _np(w), _np(b), 1e-6)
    assert _ok(xs.grad, rx, dt, TOL[dt])
    assert _ok(ws.grad, rw, dt, TOL[dt])
    assert _ok(bs.grad, rb, dt, TOL[dt])
    assert xs.grad.dtype == dt and ws.grad.dtype == dt


# ------------------------------------------------------ depthwise conv1d ---
@pytest.mark.parametrize("dt", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("K,pad,L", [(3, 1, 2048), (1, 0, 64), (2, 1, 100), (4, 1, 257),
                                     (5, 2, 96), (7, 6, 50), (9, 4, 1000), (16, 7, 300),
                                     (33, 16, 700), (3, 5, 40)])
def test_dwconv1d_backward_kernels(cuda, dt, K, pad, L):
    from amd_tuned_torch import ops
    B, C = 3, 6
    g = torch.Generator().manual_seed(K * 31 + pad + L)
    x = torch.randn(B, C, L, generator=g).to(dt)
    w = (torch.randn(C, K, generator=g) * 0.5).to(dt)
    dy = torch.randn(B, C, L + 2 * pad - K + 1, generator=g).to(dt)
    dx, dw, db = ops.depthwise_conv1d_backward(dy.to(cuda), x.to(cuda), w.to(cuda), pad)
    rx, rw, rb = oracle.np_dwconv1d_backward(_np(x), _np(dy), _np(w), pad)
    assert dx.shape == x.shape and dw.shape == w.shape and db.shape == (C,)
    assert _ok(dx, rx, dt, TOL[dt])
    assert _ok(dw, rw, dt, TOL[dt])
    assert _ok(db, rb, dt, TOL[dt])


def test_dwconv1d_weight_gradient_is_deterministic(cuda):
    from amd_tuned_torch import ops
    g = torch.Generator().manual_seed(5)
    x = torch.randn(8, 256, 2048, generator=g).to(cuda)
    w = torch.randn(256, 3, generator=g).to(cuda)
    dy = torch.randn(8, 256, 2048, generator=g).to(cuda)
    a = ops.depthwise_conv1d_backward(dy, x, w, 1)
    b = ops.depthwise_conv1d_backward(dy, x, w, 1)
    for u, v in zip(a, b):
        assert torch.equal(u, v)


@pytest.mark.parametrize("dt", [torch.float32, torch.bfloat16])
def test_depthwise_candidate_backward_matches_autograd(cuda, dt):
    from amd_tuned_torch import depthwise_conv1d_ops
    g = torch.Generator().manual_seed(11)
    x = torch.randn(4, 32, 512, generator=g).to(dt)
    w = (torch.randn(32, 1, 3, generator=g) * 0.5).to(dt)
    b = torch.randn(32, generator=g).to(dt)
    dy = torch.randn(4, 32, 512, generator=g).to(dt)
    xs, ws, bs = (t.to(cuda).requires_grad_() for t in (x, w, b))
    y = depthwise_conv1d_ops.depthwise_conv1d_candidate(xs, ws, bs, 1, 1, 1, 32)
    y.backward(dy.to(cuda))
    rx, rw, rb = oracle.stock_dwconv1d_backward(_np(x), _np(dy), _np(w).reshape(32, 3),
                                                _np(b), 1)
    assert _ok(xs.grad, rx, dt, TOL[dt])
    assert _ok(ws.grad.reshape(32, 3), rw.reshape(32, 3), dt, TOL[dt])
    assert _ok(bs.grad, rb, dt, TOL[dt])


# ------------------------------------------------- patched F.conv1d grads ---
def _conv1d_case(dt, B, C, L, K, pad, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(B, C, L, generator=g).to(dt)
    bound = 1.0 / K ** 0.5
    w = ((torch.rand(C, 1, K, generator=g) * 2 - 1) * bound).to(dt)
    b = ((torch.rand(C, generator=g) * 2 - 1) * bound).to(dt)
    dy = torch.randn(B, C, L + 2 * pad - K + 1, generator=g).to(dt)
    return x, w, b, dy


def _stock_grads(x, w, b, dy, pad, C):
    xs, ws, bs = (t.float().requires_grad_() for t in (x, w, b))
    F.conv1d(xs, ws, bs, padding=pad, groups=C).backward(dy.float())
    return xs.grad.double().numpy(), ws.grad.double().numpy(), bs.grad.double().numpy()


@pytest.mark.parametrize("route", ["contest", "fftconv", "depthwise"])
@pytest.mark.parametrize("dt,B,C,L,K,pad", [
    (torch.float32, 8, 16, 2048, 3, 1),            # cfg 1 slice
    (torch.float16, 2, 8, 16384, 2048, 1024),       # cfg 4b slice (long filter)
    (torch.bfloat16, 3, 5, 1000, 64, 31)])
def test_patched_conv1d_gradients(cuda, patched, monkeypatch, route, dt, B, C, L, K, pad):
    """Training through the patched F.conv1d keeps its gradients whichever
    candidate serves the call (the FFT route used to return a graph-less
    tensor)."""
    from amd_tuned_torch import conv1d_dispatch, depthwise_conv1d_ops, fftconv_ops, kernel_select
    x, w, b, dy = _conv1d_case(dt, B, C, L, K, pad, seed=K + L)
    xs, ws, bs = (t.to(cuda).requires_grad_() for t in (x, w, b))
    if route == "contest":
        y = F.conv1d(xs, ws, bs, padding=pad, groups=C)
    elif route == "fftconv":
        y = fftconv_ops.fftconv1d_candidate(xs, ws, bs, 1, pad, 1, C)
    else:
        y = depthwise_conv1d_ops.depthwise_conv1d_candidate(xs, ws, bs, 1, pad, 1, C)
    assert y is not None and y.requires_grad and y.grad_fn is not None
    y.backward(dy.to(cuda))
    rx, rw, rb = _stock_grads(x, w, b, dy, pad, C)
    tol = FFT_TOL[dt] if route != "depthwise" else TOL[dt]
    assert _ok(xs.grad, rx, dt, tol)
    assert _ok(ws.grad, rw, dt, tol)
    assert _ok(bs.grad, rb, dt, tol)
    _ = (conv1d_dispatch, kernel_select, monkeypatch)


def test_fft_backward_without_bias_and_input_only(cuda):
    from amd_tuned_torch import fftconv_ops
    x, w, _b, dy = _conv1d_case(torch.float32, 2, 4, 3000, 257, 128, seed=9)
    xs = x.to(cuda).requires_grad_()
    y = fftconv_ops.fftconv1d_candidate(xs, w.to(cuda), None, 1, 128, 1, 4)
    y.backward(dy.to(cuda))
    xr = x.clone().requires_grad_()
    F.conv1d(xr, w, None, padding=128, groups=4).backward(dy)
    assert oracle.rel_l2(_np(xs.grad), xr.grad.double().numpy()) <= 1e-5


# ------------------------------------------------------- torch.compile ---
def test_custom_ops_compile_fullgraph(cuda, patched):
    """The three patched ops trace as custom-op nodes (fullgraph: no graph
    break) and match eager; compiled training runs the registered backward."""
    torch._dynamo.reset()
    g = torch.Generator().manual_seed(21)
    x = torch.randn(2, 64, 8, 16, 16, generator=g).bfloat16().to(cuda)
    gw = (torch.rand(64, generator=g) + 0.5).bfloat16().to(cuda)
    gb = (torch.randn(64, generator=g) * 0.1).bfloat16().to(cuda)
    cw = (torch.randn(64, 64, 3, 3, 3, generator=g) * 0.02).bfloat16().to(cuda)
    cb = (torch.randn(64, generator=g) * 0.1).bfloat16().to(cuda)
    s = torch.randn(4, 32, 256, generator=g).to(cuda)
    sw = (torch.randn(32, 1, 3, generator=g) * 0.5).to(cuda)
    sb = torch.randn(32, generator=g).to(cuda)

    def f(x, s):
        h = F.group_norm(x, 32, gw, gb, 1e-6)
        h = F.conv3d(h, cw, cb, padding=1)
        return h, F.conv1d(s, sw, sb, padding=1, groups=32)

    compiled = torch.compile(f, fullgraph=True)
    with torch.no_grad():
        h1, c1 = compiled(x, s)
        h0, c0 = f(x, s)
    assert oracle.rel_l2(_np(h1), _np(h0)) <= 2e-3
    assert oracle.rel_l2(_np(c1), _np(c0)) <= 1e-5

    xg = x.clone().requires_grad_()
    sg = s.clone().requires_grad_()
    h, c = compiled(xg, sg)
    (h.float().square().mean() + c.square().mean()).backward()
    xe = x.clone().requires_grad_()
    se = s.clone().requires_grad_()
    he, ce = f(xe, se)
    (he.float().square().mean() + ce.square().mean()).backward()
    assert oracle.rel_l2(_np(sg.grad), _np(se.grad)) <= 1e-5
    assert oracle.rel_l2(_np(xg.grad), _np(xe.grad)) <= 5e-3
    torch._dynamo.reset()
