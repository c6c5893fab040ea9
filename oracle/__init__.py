"""CPU oracle for the conv/norm hot path -- TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may
import this package, and only as the checker.  The product path
(amd_tuned_torch) never imports it.

Three layers, each citing what it restates:

1. `stock_*` -- the reference's CPU behaviour.  On CPU tensors the reference
   package routes F.conv1d / F.conv3d / F.group_norm to stock torch (every
   accelerated tier requires CUDA tensors: amd_tuned_torch/_dispatch.py:651-659,
   miopen_fallback.py:280, :325), so stock torch CPU fp32 on the (cast) inputs
   IS the reference's output.  The BASELINE parity bar is stated against it.
2. `c_*` -- plain-C restatements of the reference's kernels in double
   precision (oracle/c/oracle.c: group_norm.cu:40-104, conv1d_bhl.cu:53-98,
   conv3d_fp32.cu:33-149), built by oracle/Makefile into oracle/_build/.
3. `fft_conv_np` -- numpy restatement of the reference's FFT route
   (fftconv_ops.py:603-746: pad -> rfftn -> multiply by the conjugated kernel
   spectrum, per-bin channel contraction (complex_matmul :480-543) -> irfftn
   -> crop -> + bias), in float64.

Pinning: tests/golden/*.npz were produced by the reference package itself
(tests/golden/make_golden.py); tests/test_oracle.py checks all three layers
against them.  The reference's own kernels cannot serve as a compiled oracle
here: they are HIP (hipcc is absent) or CUDA device code, not CPU programs.
"""
from __future__ import annotations

import ctypes
import subprocess
import threading
from pathlib import Path
from typing import Optional, Sequence

import numpy as np

_DIR = Path(__file__).resolve().parent
_LIB = _DIR / "_build" / "liboracle.so"
_lock = threading.Lock()
_clib: Optional[ctypes.CDLL] = None


def build() -> Path:
    """Compiles oracle/c/oracle.c with gcc (make) if needed."""
    src = _DIR / "c" / "oracle.c"
    if not _LIB.exists() or _LIB.stat().st_mtime < src.stat().st_mtime:
        subprocess.run(["make", "-s", "-C", str(_DIR)], check=True)
    return _LIB


def _c() -> ctypes.CDLL:
    global _clib
    with _lock:
        if _clib is None:
            build()
            lib = ctypes.CDLL(str(_LIB))
            f, i64, vp, d = ctypes.c_float, ctypes.c_int64, ctypes.c_void_p, ctypes.c_double
            lib.oracle_group_norm.argtypes = [vp, vp, vp, vp, i64, i64, i64, i64, d]
            lib.oracle_dwconv1d.argtypes = [vp, vp, vp, vp, i64, i64, i64, i64, i64]
            lib.oracle_conv3d.argtypes = [vp, vp, vp, vp] + [i64] * 9 + [vp]
            del f
            _clib = lib
        return _clib


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.float32))


def _p(a: Optional[np.ndarray]):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


# ------------------------------------------------------------ C restatement
def c_group_norm(x, G: int, gamma=None, beta=None, eps: float = 1e-5) -> np.ndarray:
    x = _f32(x)
    N, C = x.shape[0], x.shape[1]
    S = x.size // (N * C)
    g = _f32(gamma) if gamma is not None else None
    b = _f32(beta) if beta is not None else None
    y = np.empty_like(x)
    _c().oracle_group_norm(_p(x), _p(g), _p(b), _p(y), N, C, S, G, float(eps))
    return y


def c_dwconv1d(x, w, bias, pad: int) -> np.ndarray:
    """x [B, C, L], w [C, 1, K] or [C, K], bias [C] or None."""
    x = _f32(x)
    B, C, L = x.shape
    w = _f32(w).reshape(C, -1)
    K = w.shape[1]
    b = _f32(bias) if bias is not None else None
    y = np.empty((B, C, L + 2 * pad - K + 1), dtype=np.float32)
    _c().oracle_dwconv1d(_p(x), _p(w), _p(b), _p(y), B, C, L, K, pad)
    return y


def c_conv3d(x, w, bias, stride: Sequence[int], pad: Sequence[int],
             dil: Sequence[int]) -> np.ndarray:
    x, w = _f32(x), _f32(w)
    N, Cin, D, H, W = x.shape
    Cout, _, KD, KH, KW = w.shape
    prm = np.array([*stride, *pad, *dil], dtype=np.int64)
    Do = (D + 2 * pad[0] - dil[0] * (KD - 1) - 1) // stride[0] + 1
    Ho = (H + 2 * pad[1] - dil[1] * (KH - 1) - 1) // stride[1] + 1
    Wo = (W + 2 * pad[2] - dil[2] * (KW - 1) - 1) // stride[2] + 1
    b = _f32(bias) if bias is not None else None
    y = np.empty((N, Cout, Do, Ho, Wo), dtype=np.float32)
    _c().oracle_conv3d(_p(x), _p(w), _p(b), _p(y), N, Cin, D, H, W, Cout, KD, KH, KW,
                       prm.ctypes.data_as(ctypes.c_void_p))
    return y


# ------------------------------------------------------- numpy FFT route
def fft_conv_np(x, w, bias, pad: Sequence[int], groups: int = 1,
                fft_sizes: Optional[Sequence[int]] = None) -> np.ndarray:
    """Cross-correlation through the FFT, float64, stride 1 / dilation 1.
    x [N, Cin, *S], w [Cout, Cin/groups, *K]."""
    x = np.asarray(x, dtype=np.float64)
    w = np.asarray(w, dtype=np.float64)
    nd = x.ndim - 2
    xp = np.pad(x, [(0, 0), (0, 0)] + [(p, p) for p in pad])
    if xp.shape[-1] % 2:
        xp = np.pad(xp, [(0, 0)] * (xp.ndim - 1) + [(0, 1)])
    sizes = tuple(fft_sizes) if fft_sizes is not None else xp.shape[2:]
    axes = tuple(range(2, 2 + nd))
    X = np.fft.rfftn(xp, s=sizes, axes=axes)
    Wf = np.conj(np.fft.rfftn(w, s=sizes, axes=axes))
    N, Cin = x.shape[:2]
    Cout = w.shape[0]
    Xg = X.reshape(N, groups, Cin // groups, -1)
    Wg = Wf.reshape(groups, Cout // groups, w.shape[1], -1)
    Y = np.einsum("ngif,goif->ngof", Xg, Wg).reshape((N, Cout) + X.shape[2:])
    y = np.fft.irfftn(Y, s=sizes, axes=axes)
    out_sz = [x.shape[2 + i] + 2 * pad[i] - w.shape[2 + i] + 1 for i in range(nd)]
    y = y[(slice(None), slice(None)) + tuple(slice(0, n) for n in out_sz)]
    if bias is not None:
        y = y + np.asarray(bias, dtype=np.float64).reshape((1, -1) + (1,) * nd)
    return y


# --------------------------------------------- stock torch CPU (fp32)
def stock_conv1d(x, w, bias, pad: int, groups: int):
    import torch
    import torch.nn.functional as F
    t = lambda a: None if a is None else torch.as_tensor(np.asarray(a, dtype=np.float32))
    return F.conv1d(t(x), t(w), t(bias), 1, pad, 1, groups).numpy()


def stock_conv3d(x, w, bias, pad, dil=(1, 1, 1)):
    import torch
    import torch.nn.functional as F
    t = lambda a: None if a is None else torch.as_tensor(np.asarray(a, dtype=np.float32))
    return F.conv3d(t(x), t(w), t(bias), 1, tuple(pad), tuple(dil), 1).numpy()


def stock_group_norm(x, G: int, gamma=None, beta=None, eps: float = 1e-5):
    import torch
    import torch.nn.functional as F
    t = lambda a: None if a is None else torch.as_tensor(np.asarray(a, dtype=np.float32))
    return F.group_norm(t(x), G, t(gamma), t(beta), eps).numpy()


# ------------------------------------------------------------ backward
def np_group_norm_backward(x, dy, G: int, gamma=None, eps: float = 1e-5):
    """(dx, dgamma, dbeta) of GroupNorm in float64: the derivative the
    reference's _group_norm_backward computes (amd_tuned_torch/_dispatch.py:
    2212-2302): xhat = (x - mean) * rstd per (n, g); dbeta = sum dy;
    dgamma = sum dy * xhat; dx = rstd * (gamma dy - mean_g(gamma dy)
    - xhat * mean_g(gamma dy xhat))."""
    x = np.asarray(x, dtype=np.float64)
    dy = np.asarray(dy, dtype=np.float64)
    N, C = x.shape[:2]
    xg = x.reshape(N, G, C // G, -1)
    dg = dy.reshape(N, G, C // G, -1)
    mean = xg.mean(axis=(2, 3), keepdims=True)
    rstd = 1.0 / np.sqrt(((xg - mean) ** 2).mean(axis=(2, 3), keepdims=True) + eps)
    xhat = (xg - mean) * rstd
    gm = (np.ones(C) if gamma is None else np.asarray(gamma, dtype=np.float64))
    gdy = dg * gm.reshape(1, G, C // G, 1)
    dx = rstd * (gdy - gdy.mean(axis=(2, 3), keepdims=True)
                 - xhat * (gdy * xhat).mean(axis=(2, 3), keepdims=True))
    dgamma = (dg * xhat).sum(axis=(0, 3)).reshape(C)
    dbeta = dg.sum(axis=(0, 3)).reshape(C)
    return dx.reshape(x.shape), dgamma, dbeta


def np_dwconv1d_backward(x, dy, w, pad: int):
    """(dx, dw [C, K], dbias) of the depthwise conv1d
    y[b,c,o] = bias[c] + sum_k w[c,k] x[b,c,o-pad+k] in float64 -- the
    gradients the reference's vendored backward kernel produces
    (amd_tuned_torch/_vendor/flashfftconv_depthwise_conv1d/
    conv1d_bwd_cuda_bhl.cu:34-72: du[j] = sum_k dout[j-pad+k] w[K-1-k]
    (valid there for L_out = L), dk[k] = sum_j u[k-pad+j] dout[j]; dbias =
    sum of dout), here for any padding and output length."""
    x = np.asarray(x, dtype=np.float64)
    dy = np.asarray(dy, dtype=np.float64)
    B, C, L = x.shape
    w = np.asarray(w, dtype=np.float64).reshape(C, -1)
    K = w.shape[1]
    Lout = dy.shape[-1]
    xp = np.pad(x, [(0, 0), (0, 0), (pad, pad)])
    dxp = np.zeros_like(xp)
    dw = np.zeros((C, K))
    for k in range(K):
        dxp[:, :, k:k + Lout] += dy * w[None, :, k, None]
        dw[:, k] = (dy * xp[:, :, k:k + Lout]).sum(axis=(0, 2))
    return dxp[:, :, pad:pad + L], dw, dy.sum(axis=(0, 2))


def stock_group_norm_backward(x, dy, G: int, gamma=None, beta=None, eps: float = 1e-5):
    """Stock torch CPU fp32 autograd of F.group_norm: (dx, dgamma, dbeta)."""
    import torch
    import torch.nn.functional as F
    t = lambda a: None if a is None else torch.tensor(np.asarray(a, dtype=np.float32),
                                                      requires_grad=True)
    xt, gt, bt = t(x), t(gamma), t(beta)
    F.group_norm(xt, G, gt, bt, eps).backward(torch.as_tensor(np.asarray(dy, np.float32)))
    g = lambda a: None if a is None else a.grad.numpy()
    return g(xt), g(gt), g(bt)


def stock_dwconv1d_backward(x, dy, w, bias, pad: int):
    """Stock torch CPU fp32 autograd of the depthwise F.conv1d: (dx, dw, dbias)."""
    import torch
    import torch.nn.functional as F
    t = lambda a: None if a is None else torch.tensor(np.asarray(a, dtype=np.float32),
                                                      requires_grad=True)
    xt, wt, bt = t(x), t(w), t(bias)
    C = xt.shape[1]
    F.conv1d(xt, wt.reshape(C, 1, -1), bt, 1, pad, 1, C).backward(
        torch.as_tensor(np.asarray(dy, np.float32)))
    return xt.grad.numpy(), wt.grad.numpy(), None if bt is None else bt.grad.numpy()


def rel_l2(y, ref) -> float:
    """||y - ref||_2 / ||ref||_2 in float64 (the BASELINE parity metric)."""
    y = np.asarray(y, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    den = np.linalg.norm(ref.ravel())
    return float(np.linalg.norm((y - ref).ravel()) / (den if den > 0 else 1.0))
