"""Dispatch logic on CPU with the native ops replaced by fakes (the reference
does the same with MagicMock natives, tests/conftest.py:44-95 there): install
set, routing, eligibility and the autograd wrappers."""
from __future__ import annotations

import pytest
import torch
import torch.nn.functional as F

import amd_tuned_torch
from amd_tuned_torch import _dispatch, conv1d_dispatch, kernel_select, ops

STOCK = (F.conv1d, F.conv3d, F.group_norm)
STOCK_CONV2D = F.conv2d
STOCK_SEQ_FORWARD = torch.nn.Sequential.forward


@pytest.fixture
def patched():
    amd_tuned_torch.enable()
    yield
    amd_tuned_torch.disable()


@pytest.fixture
def force_eligible(monkeypatch):
    """CPU tensors reach the native branches; natives are recording fakes."""
    calls = []
    monkeypatch.setattr(_dispatch, "_usable", lambda *a, **k: True)
    monkeypatch.setattr(_dispatch._lib, "available", lambda: True)
    monkeypatch.setattr(kernel_select, "_ENABLED", False)

    def fake_gn(x, G, w, b, eps, variant=0, out=None):
        calls.append(("group_norm", variant))
        return STOCK[2](x, G, w, b, eps)

    def fake_conv3d(x, w, b, stride, padding, dilation, variant=0, x_channels_last=False,
                    out_channels_last=False, out=None, gate=None, weight_key=None):
        calls.append(("conv3d", x_channels_last))
        if x_channels_last:
            x = x.permute(0, 4, 1, 2, 3)
        y = STOCK[1](x, w, b, stride, padding, dilation)
        return y.permute(0, 2, 3, 4, 1).contiguous() if out_channels_last else y

    monkeypatch.setattr(ops, "group_norm", fake_gn)
    monkeypatch.setattr(ops, "conv3d", fake_conv3d)
    return calls


def test_enable_disable_install_set():
    assert not amd_tuned_torch.is_enabled()
    amd_tuned_torch.enable()
    try:
        assert amd_tuned_torch.is_enabled()
        assert F.conv3d is _dispatch._patched_conv3d
        assert F.group_norm is _dispatch._patched_group_norm
        assert getattr(F.conv1d, "_amd_tuned_torch_wrapper", False)
        amd_tuned_torch.enable()                    # idempotent
        assert F.conv3d is _dispatch._patched_conv3d
        assert F.conv2d is _dispatch._patched_conv2d
        assert torch.nn.Sequential.forward is _dispatch._patched_sequential_forward
    finally:
        amd_tuned_torch.disable()
    assert (F.conv1d, F.conv3d, F.group_norm) == STOCK
    assert F.conv2d is STOCK_CONV2D
    assert torch.nn.Sequential.forward is STOCK_SEQ_FORWARD
    assert not amd_tuned_torch.is_enabled()
    amd_tuned_torch.disable()                       # idempotent


def test_cpu_conv2d_and_sequential_blocks_go_to_stock(patched):
    x = torch.randn(2, 8, 6, 6)
    w = torch.randn(4, 8, 3, 3)
    torch.testing.assert_close(F.conv2d(x, w, padding=1), STOCK_CONV2D(x, w, padding=1))
    torch.manual_seed(0)
    for conv in (torch.nn.Conv3d(8, 8, 3, padding=1), torch.nn.Conv2d(8, 8, 3, padding=1)):
        blk = torch.nn.Sequential(torch.nn.GroupNorm(4, 8), torch.nn.SiLU(), conv).eval()
        xi = torch.randn(1, 8, 3, 5, 5) if isinstance(conv, torch.nn.Conv3d) else x
        with torch.no_grad():
            torch.testing.assert_close(blk(xi), STOCK_SEQ_FORWARD(blk, xi))
    other = torch.nn.Sequential(torch.nn.Linear(4, 4), torch.nn.ReLU(), torch.nn.Linear(4, 2))
    xl = torch.randn(3, 4)
    torch.testing.assert_close(other(xl), STOCK_SEQ_FORWARD(other, xl))


def test_conv2d_routes_as_depth1_conv3d(patched, force_eligible):
    x = torch.randn(2, 8, 6, 7)
    w = torch.randn(4, 8, 3, 3)
    b = torch.randn(4)
    torch.testing.assert_close(F.conv2d(x, w, b, padding=1), STOCK_CONV2D(x, w, b, padding=1))
    xc = x.contiguous(memory_format=torch.channels_last)
    torch.testing.assert_close(F.conv2d(xc, w, b, padding=(1, 2), dilation=(1, 2)),
                               STOCK_CONV2D(x, w, b, padding=(1, 2), dilation=(1, 2)))
    assert force_eligible == [("conv3d", False), ("conv3d", True)]
    F.conv2d(x, torch.randn(8, 4, 3, 3), padding=1, groups=2)   # grouped -> stock
    F.conv2d(x, torch.randn(4, 8, 1, 1))                          # pointwise -> stock
    assert force_eligible == [("conv3d", False), ("conv3d", True)]
    F.conv2d(x, w, padding=1, stride=2)                           # strided -> the conv3d route
    F.conv2d(x, w, padding="same")
    F.conv2d(x, torch.randn(4, 8, 2, 2), padding="same")          # uneven 'same' -> stock
    assert force_eligible == [("conv3d", False), ("conv3d", True), ("conv3d", False),
                              ("conv3d", False)]


def test_conv1d_fallback_toggle_is_independent():
    conv1d_dispatch.enable_conv1d_fallback()
    try:
        assert conv1d_dispatch.is_conv1d_fallback_enabled()
        amd_tuned_torch.enable()                    # does not double-wrap
        amd_tuned_torch.disable()
        assert conv1d_dispatch.is_conv1d_fallback_enabled()
    finally:
        conv1d_dispatch.disable_conv1d_fallback()
    assert F.conv1d is STOCK[0]


def test_cpu_tensors_go_to_stock(patched):
    x = torch.randn(2, 8, 4, 4)
    torch.testing.assert_close(F.group_norm(x, 4), STOCK[2](x, 4))
    x3 = torch.randn(1, 4, 3, 5, 5)
    w3 = torch.randn(2, 4, 3, 3, 3)
    torch.testing.assert_close(F.conv3d(x3, w3, padding=1), STOCK[1](x3, w3, padding=1))
    x1 = torch.randn(2, 4, 16)
    w1 = torch.randn(4, 1, 3)
    torch.testing.assert_close(F.conv1d(x1, w1, padding=1, groups=4),
                               STOCK[0](x1, w1, padding=1, groups=4))


def test_group_norm_routes_to_native(patched, force_eligible):
    x = torch.randn(2, 8, 4, 4)
    F.group_norm(x, 4, torch.ones(8), torch.zeros(8))
    assert force_eligible[0][0] == "group_norm"


def test_group_norm_non_contiguous_goes_to_stock(patched, force_eligible):
    x = torch.randn(2, 4, 4, 8).permute(0, 3, 1, 2)
    y = F.group_norm(x, 4)
    assert not force_eligible
    torch.testing.assert_close(y, STOCK[2](x, 4))


def test_conv3d_routes_to_tensor_cores_and_channels_last(patched, force_eligible):
    x = torch.randn(1, 8, 3, 4, 4)
    w = torch.randn(8, 8, 3, 3, 3)
    y = F.conv3d(x, w, None, 1, 1)
    assert force_eligible == [("conv3d", False)]
    xcl = x.contiguous(memory_format=torch.channels_last_3d)
    y2 = F.conv3d(xcl, w, None, 1, 1)
    assert force_eligible[-1] == ("conv3d", True)
    assert y2.is_contiguous(memory_format=torch.channels_last_3d)
    torch.testing.assert_close(y2, y)


def test_grouped_conv3d_goes_to_stock(patched, force_eligible):
    x = torch.randn(1, 8, 3, 4, 4)
    w = torch.randn(8, 4, 3, 3, 3)
    F.conv3d(x, w, None, 1, 1, 1, 2)
    assert not force_eligible


def test_conv3d_with_grad_uses_autograd_wrapper(patched, force_eligible):
    x = torch.randn(1, 4, 3, 4, 4, requires_grad=True)
    w = torch.randn(4, 4, 3, 3, 3, requires_grad=True)
    y = F.conv3d(x, w, None, 1, 1)
    assert y.grad_fn is not None and "Conv3dFn" in type(y.grad_fn).__name__
    y.sum().backward()
    x2 = x.detach().requires_grad_()
    w2 = w.detach().requires_grad_()
    STOCK[1](x2, w2, None, 1, 1).sum().backward()
    torch.testing.assert_close(x.grad, x2.grad)
    torch.testing.assert_close(w.grad, w2.grad)


def test_tensor_subclass_is_not_plain():
    class Sub(torch.Tensor):
        pass
    t = torch.zeros(2).as_subclass(Sub)
    assert not _dispatch._is_plain_tensor(t)
    assert _dispatch._is_plain_tensor(torch.zeros(2))
    assert _dispatch._is_plain_tensor(torch.nn.Parameter(torch.zeros(2)))


def test_grad_safe():
    a = torch.zeros(2, requires_grad=True)
    assert not _dispatch._grad_safe(a)
    with torch.no_grad():
        assert _dispatch._grad_safe(a)
    with torch.inference_mode():
        assert _dispatch._grad_safe(torch.zeros(2))


def test_depthwise_eligibility():
    elig = conv1d_dispatch._is_depthwise_conv1d_eligible
    x = torch.randn(2, 8, 32)
    w = torch.randn(8, 1, 4)
    assert not elig(x, w, 1, 1, 8)     # CPU tensor
    x.is_cuda  # noqa: B018
    meta = torch.empty(2, 8, 32, device="meta")
    assert not elig(meta, w, 1, 1, 8)


# ------------------------------------------------ GroupNorm backward route
def test_group_norm_backward_routes_to_native_kernel(monkeypatch):
    """_GroupNormFn's backward is the native b200_gn_bwd (ops.group_norm_backward,
    faked here); each gradient comes back in its parameter's dtype.  The
    numerics are checked on the GPU (tests/test_gpu_backward.py)."""
    seen = []

    def fake(dy, x, G, w, eps, needs, affine_dtype=None):
        seen.append((G, needs, affine_dtype))
        C = x.shape[1]
        return (torch.zeros_like(x) if needs[0] else None,
                torch.zeros(C, dtype=affine_dtype) if needs[1] else None,
                torch.zeros(C, dtype=torch.float64) if needs[2] else None)

    monkeypatch.setattr(ops, "group_norm_backward", fake)
    x = torch.randn(2, 8, 5, 3)
    dy = torch.randn_like(x)
    w = torch.rand(8).half()
    gx, gw, gb = _dispatch._group_norm_backward(dy, x, 4, w, 1e-5, (True, True, True),
                                                bias_dtype=torch.float32)
    assert seen == [(4, (True, True, True), torch.float16)]
    assert gx.shape == x.shape and gw.dtype == torch.float16 and gb.dtype == torch.float32
    gx, gw, gb = _dispatch._group_norm_backward(dy, x, 4, None, 1e-5, (True, True, False))
    assert seen[-1] == (4, (True, False, False), torch.float32) and gw is None and gb is None


def test_cpu_training_through_patches_stays_stock(patched):
    """CPU tensors with live gradients go to stock torch in the forward AND
    the backward (the native backward kernels take CUDA tensors only; a host
    pointer handed to them would be an illegal address on the GPU)."""
    g = torch.Generator().manual_seed(4)
    x = torch.randn(2, 8, 5, 5, generator=g, requires_grad=True)
    w = (torch.rand(8, generator=g) + 0.5).requires_grad_()
    b = torch.randn(8, generator=g).requires_grad_()
    F.group_norm(x, 4, w, b, 1e-5).sum().backward()
    x2, w2, b2 = (t.detach().clone().requires_grad_() for t in (x, w, b))
    STOCK[2](x2, 4, w2, b2, 1e-5).sum().backward()
    for a, r in ((x, x2), (w, w2), (b, b2)):
        torch.testing.assert_close(a.grad, r.grad)
    s = torch.randn(2, 4, 32, generator=g, requires_grad=True)
    k = torch.randn(4, 1, 3, generator=g, requires_grad=True)
    F.conv1d(s, k, None, 1, 1, 1, 4).sum().backward()
    assert s.grad is not None and k.grad is not None


def test_ops_refuse_host_tensors():
    """Every op that launches a kernel checks its tensors are on the GPU
    before anything is launched."""
    x = torch.randn(2, 8, 4, 4)
    with pytest.raises(ValueError, match="CUDA tensors required"):
        ops._on_gpu(x)
    with pytest.raises(ValueError, match="CUDA tensors required"):
        ops.group_norm_backward(x, x, 4, None, 1e-5, (True, False, False))
    with pytest.raises(ValueError, match="CUDA tensors required"):
        ops.depthwise_conv1d_backward(x[:, :, 0], x[:, :, 0], torch.randn(8, 3), 1)
