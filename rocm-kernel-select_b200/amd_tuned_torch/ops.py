"""Tensor-level wrappers around the C ABI of libb200conv.so.

Each function takes torch CUDA tensors, allocates the output with torch (the
library itself never allocates), passes raw pointers plus the current stream,
and returns the output -- or None when the kernel declines the problem
(status > 0), which is the kernel_select decline convention
(amd_tuned_torch/kernel_select.py:541-544 in the reference).  A status < 0 is
a real error and raises `_lib.NativeError`.

Reference counterparts: `ops.group_norm` <-> `_C.group_norm`
(src/main_rocm.cpp:556-599); `ops.depthwise_conv1d` <->
`_native_depthwise_conv1d.conv1d_forward` (host.cpp:7-11); `ops.conv3d` <->
`_C.conv3d` (src/main_rocm.cpp:798-854); `ops.fftconv1d` / `ops.fftconv3d` <->
`fftconv_ops.fft_conv` (amd_tuned_torch/fftconv_ops.py:603-746).
"""
from __future__ import annotations

import ctypes
import threading
import weakref
from collections import OrderedDict
from typing import Optional, Sequence

import torch

from . import _lib

DTYPE_CODE = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}


def _code(dtype: torch.dtype) -> int:
    try:
        return DTYPE_CODE[dtype]
    except KeyError:
        raise TypeError(f"unsupported dtype {dtype}") from None


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _on_gpu(*tensors: Optional[torch.Tensor]) -> None:
    """Every tensor handed to a kernel is a CUDA tensor on the first one's
    device.  A host pointer given to a kernel would be an illegal address on
    the GPU, so this is checked before anything launches."""
    dev = None
    for t in tensors:
        if t is None:
            continue
        if not t.is_cuda:
            raise ValueError("amd_tuned_torch.ops: CUDA tensors required (got a "
                             f"{t.device.type} tensor)")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise ValueError(f"amd_tuned_torch.ops: tensors on {dev} and {t.device}")


_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def _stream(device: torch.device) -> int:
    """cudaStream_t of torch's current stream on `device` (raw pointer)."""
    idx = device.index
    if idx is None:
        idx = torch.cuda.current_device()
    if _raw_stream is not None:
        return _raw_stream(idx)
    return torch.cuda.current_stream(idx).cuda_stream


# ------------------------------------------------------------ workspaces ---
# One growable scratch buffer per (device, stream): launches on one stream are
# ordered, so consecutive ops on it may reuse the same bytes.
_ws_lock = threading.Lock()
_workspaces: dict = {}


def workspace(device: torch.device, nbytes: int,
              stream: Optional[int] = None) -> Optional[torch.Tensor]:
    if nbytes <= 0:
        return None
    key = (device.index, stream if stream is not None else _stream(device))
    buf = _workspaces.get(key)
    if buf is not None and buf.numel() >= nbytes:
        return buf
    with _ws_lock:
        buf = _workspaces.get(key)
        if buf is None or buf.numel() < nbytes:
            buf = torch.empty(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
            _workspaces[key] = buf
        return buf


def clear_workspaces() -> None:
    with _ws_lock:
        _workspaces.clear()


class _DerivedCache:
    """Small LRU of tensors derived from a weight (packed conv3d operand, FFT
    spectra).  An entry belongs to one live weight OBJECT: it is dropped when
    that tensor is garbage collected (weakref callback), and ignored when the
    tensor's version counter, storage pointer, shape or dtype changed since
    (in-place update, .data swap).  Keying on the storage pointer alone would
    hand a new weight the stale entry of a freed one whose memory the caching
    allocator reused."""

    def __init__(self, cap: int = 32):
        self.cap = cap
        self.d: OrderedDict = OrderedDict()
        self.lock = threading.RLock()   # weakref callbacks may fire under the lock

    @staticmethod
    def _sig(w: torch.Tensor):
        return (w._version, w.data_ptr(), tuple(w.shape), w.dtype, w.device.index)

    def get(self, w: torch.Tensor, extra=()):
        key = (id(w),) + tuple(extra)
        with self.lock:
            ent = self.d.get(key)
            if ent is None:
                return None
            ref, sig, val = ent
            if ref() is not w or sig != self._sig(w):
                del self.d[key]
                return None
            self.d.move_to_end(key)
            return val

    def put(self, w: torch.Tensor, extra, val) -> None:
        key = (id(w),) + tuple(extra)

        def _drop(_ref, key=key, d=self.d, lock=self.lock):
            with lock:
                ent = d.get(key)
                if ent is not None and ent[0] is _ref:
                    del d[key]

        with self.lock:
            self.d[key] = (weakref.ref(w, _drop), self._sig(w), val)
            self.d.move_to_end(key)
            while len(self.d) > self.cap:
                self.d.popitem(last=False)

    def clear(self) -> None:
        with self.lock:
            self.d.clear()


_packed_weights = _DerivedCache()
_spectra = _DerivedCache(cap=8)


def clear_caches() -> None:
    _packed_weights.clear()
    _spectra.clear()
    _conv_plans.clear()
    clear_workspaces()


# ------------------------------------------------------------ GroupNorm ---
# auto; stats+apply; two-pass L2-resident; three-kernel streaming (persistent grids)
GN_AUTO, GN_SPLIT, GN_L2, GN_STREAM = 0, 1, 2, 3


def gn_cluster_variant(k: int) -> int:
    return 16 + k


def group_norm(x: torch.Tensor, num_groups: int, weight: Optional[torch.Tensor],
               bias: Optional[torch.Tensor], eps: float, variant: int = GN_AUTO,
               out: Optional[torch.Tensor] = None) -> Optional[torch.Tensor]:
    """F.group_norm forward on a contiguous [N, C, *] CUDA tensor (into `out`
    when given: same shape/dtype as x, contiguous)."""
    L = _lib.lib()
    _on_gpu(x, weight, bias, out)
    if not x.is_contiguous():
        return None
    N, C = x.shape[0], x.shape[1]
    S = x.numel() // max(1, N * C)
    if weight is not None:
        weight = weight.contiguous()
    if bias is not None:
        bias = bias.contiguous()
    adt = weight.dtype if weight is not None else (bias.dtype if bias is not None else x.dtype)
    if weight is not None and bias is not None and weight.dtype != bias.dtype:
        bias = bias.to(weight.dtype)
    y = torch.empty_like(x) if out is None else out
    if x.numel() == 0:
        return y
    dt = _code(x.dtype)
    wsb = L.b200_gn_workspace_bytes(N, C, S, num_groups, dt, variant)
    ws = workspace(x.device, wsb)
    rc = L.b200_gn_fwd(x.data_ptr(), _ptr(weight), _ptr(bias), y.data_ptr(), dt, _code(adt),
                       N, C, S, num_groups, float(eps), variant,
                       _ptr(ws), wsb, _stream(x.device))
    return y if _lib.check(rc, "b200_gn_fwd") else None


def group_norm_partial_stats(x: torch.Tensor, num_groups: int) -> torch.Tensor:
    """(count, mean, M2) per (n, g) of a contiguous [N, C, *] tensor, fp32 [N*G, 3]."""
    L = _lib.lib()
    _on_gpu(x)
    N, C = x.shape[0], x.shape[1]
    S = x.numel() // max(1, N * C)
    out = torch.empty(N * num_groups, 3, dtype=torch.float32, device=x.device)
    dt = _code(x.dtype)
    wsb = L.b200_gn_stats_workspace_bytes(N, C, S, num_groups, dt)
    ws = workspace(x.device, wsb)
    rc = L.b200_gn_partial_stats(x.data_ptr(), out.data_ptr(), dt, N, C, S, num_groups,
                                 _ptr(ws), wsb, _stream(x.device))
    if not _lib.check(rc, "b200_gn_partial_stats"):
        raise _lib.NativeError("GroupNorm statistics declined")
    return out


def group_norm_merge_ranks(parts: torch.Tensor) -> torch.Tensor:
    """[R, groups, 3] fp32 per-rank (count, mean, M2) -> [groups, 3], merged in
    rank order (fp64) on the device."""
    L = _lib.lib()
    _on_gpu(parts)
    parts = parts.contiguous()
    R, groups = parts.shape[0], parts.shape[1]
    out = torch.empty(groups, 3, dtype=torch.float32, device=parts.device)
    rc = L.b200_gn_merge_ranks(parts.data_ptr(), out.data_ptr(), R, groups, _stream(parts.device))
    if not _lib.check(rc, "b200_gn_merge_ranks"):
        raise _lib.NativeError("b200_gn_merge_ranks declined")
    return out


def group_norm_apply(x: torch.Tensor, stats: torch.Tensor, num_groups: int,
                     weight: Optional[torch.Tensor], bias: Optional[torch.Tensor], eps: float,
                     silu: bool = False, channels_last_out: bool = False) -> torch.Tensor:
    """Normalise [N, C, *] with precomputed (count, mean, M2) stats, optional
    SiLU, output NC[*] or channels-last [N, *, C] (returned as an [N, S, C]
    contiguous tensor in that case)."""
    L = _lib.lib()
    _on_gpu(x, stats, weight, bias)
    N, C = x.shape[0], x.shape[1]
    S = x.numel() // max(1, N * C)
    if channels_last_out:
        y = torch.empty(N, S, C, dtype=x.dtype, device=x.device)
    else:
        y = torch.empty_like(x)
    adt = weight.dtype if weight is not None else (bias.dtype if bias is not None else x.dtype)
    if weight is not None and bias is not None and weight.dtype != bias.dtype:
        bias = bias.to(weight.dtype)
    rc = L.b200_gn_apply(x.data_ptr(), stats.data_ptr(), _ptr(weight), _ptr(bias),
                         y.data_ptr(), _code(x.dtype), _code(adt), N, C, S, num_groups,
                         float(eps), int(silu), int(channels_last_out), _stream(x.device))
    if not _lib.check(rc, "b200_gn_apply"):
        raise _lib.NativeError("GroupNorm apply declined")
    return y


def group_norm_backward(grad_out: torch.Tensor, x: torch.Tensor, num_groups: int,
                        weight: Optional[torch.Tensor], eps: float, needs,
                        affine_dtype: Optional[torch.dtype] = None):
    """(dx, dgamma, dbeta) of F.group_norm on contiguous [N, C, *] CUDA
    tensors; `needs` = (dx, dgamma, dbeta) flags, an unneeded gradient is
    None.  The group statistics are recomputed from x (one read)."""
    L = _lib.lib()
    _on_gpu(grad_out, x, weight)
    need_x, need_w, need_b = needs
    N, C = x.shape[0], x.shape[1]
    S = x.numel() // max(1, N * C)
    x = x.contiguous()
    dy = grad_out.contiguous()
    if weight is not None:
        weight = weight.contiguous()
    adt = weight.dtype if weight is not None else (affine_dtype or x.dtype)
    dx = torch.empty_like(x) if need_x else None
    dg = torch.empty(C, dtype=adt, device=x.device) if need_w else None
    db = torch.empty(C, dtype=adt, device=x.device) if need_b else None
    if x.numel() == 0:
        if dg is not None:
            dg.zero_()
        if db is not None:
            db.zero_()
        return dx, dg, db
    stats = group_norm_partial_stats(x, num_groups)
    wsb = L.b200_gn_bwd_workspace_bytes(N, C, S, num_groups)
    ws = workspace(x.device, wsb)
    rc = L.b200_gn_bwd(x.data_ptr(), dy.data_ptr(), stats.data_ptr(), _ptr(weight), _ptr(dx),
                       _ptr(dg), _ptr(db), _code(x.dtype), _code(adt), N, C, S, num_groups,
                       float(eps), _ptr(ws), wsb, _stream(x.device))
    if not _lib.check(rc, "b200_gn_bwd"):
        raise _lib.NativeError("GroupNorm backward declined")
    return dx, dg, db


# ---------------------------------------------------- depthwise conv1d ---
def depthwise_conv1d(x: torch.Tensor, weight2d: torch.Tensor, bias: Optional[torch.Tensor],
                     padding: int, out: Optional[torch.Tensor] = None,
                     flip_taps: bool = False) -> Optional[torch.Tensor]:
    """x [B, C, L] contiguous, weight2d [C, K], bias [C] or None -> [B, C, L + 2p - K + 1].
    flip_taps: tap k uses weight2d[:, K-1-k] (the input-gradient form)."""
    L_ = _lib.lib()
    _on_gpu(x, weight2d, bias, out)
    B, C, L = x.shape
    K = weight2d.shape[1]
    Lout = L + 2 * padding - K + 1
    if Lout <= 0:
        return None
    x = x.contiguous()
    w = weight2d.contiguous()
    b = bias.contiguous() if bias is not None else None
    if b is not None and b.dtype != w.dtype:
        b = b.to(w.dtype)
    y = torch.empty(B, C, Lout, dtype=x.dtype, device=x.device) if out is None else out
    rc = L_.b200_dwconv1d_fwd(x.data_ptr(), w.data_ptr(), _ptr(b), y.data_ptr(),
                              _code(x.dtype), _code(w.dtype), B, C, L, K, padding, Lout,
                              1 if flip_taps else 0, _stream(x.device))
    return y if _lib.check(rc, "b200_dwconv1d_fwd") else None


def _crop_for_negative_padding(dy: torch.Tensor, K: int, padding: int):
    """(source, padding) of the input-gradient correlation: dy itself at
    padding K-1-p, or -- when p > K-1 -- dy cropped by p-K+1 on both ends at
    padding 0 (the same sums without a negative padding)."""
    back = K - 1 - padding
    if back >= 0:
        return dy, back
    cut = -back
    return dy[..., cut:dy.shape[-1] - cut].contiguous(), 0


def depthwise_conv1d_backward(grad_out: torch.Tensor, x: torch.Tensor, weight2d: torch.Tensor,
                              padding: int, needs=(True, True, True)):
    """(dx, dweight [C, K], dbias [C]) of depthwise_conv1d on the sm_100a
    kernels: dx = the forward kernel on dy with flipped taps, dweight/dbias =
    b200_dwconv1d_bwd_weight (fixed-order reduction)."""
    L_ = _lib.lib()
    _on_gpu(grad_out, x, weight2d)
    need_x, need_w, need_b = needs
    B, C, L = x.shape
    K = weight2d.shape[1]
    dy = grad_out.contiguous()
    Lout = dy.shape[-1]
    w = weight2d.contiguous()
    dx = dw = db = None
    if need_x:
        src, back = _crop_for_negative_padding(dy, K, padding)
        dx = depthwise_conv1d(src, w, None, back, flip_taps=True)
        if dx is None or dx.shape[-1] != L:
            raise _lib.NativeError("dwconv1d input gradient declined")
    if need_w or need_b:
        dw = torch.empty(C, K, dtype=w.dtype, device=x.device)
        db = torch.empty(C, dtype=w.dtype, device=x.device) if need_b else None
        wsb = L_.b200_dwconv1d_bwd_workspace_bytes(B, C, K, Lout)
        ws = workspace(x.device, wsb)
        rc = L_.b200_dwconv1d_bwd_weight(x.contiguous().data_ptr(), dy.data_ptr(), dw.data_ptr(),
                                         _ptr(db), _code(x.dtype), _code(w.dtype), B, C, L, K,
                                         padding, Lout, _ptr(ws), wsb, _stream(x.device))
        if not _lib.check(rc, "b200_dwconv1d_bwd_weight"):
            raise _lib.NativeError("dwconv1d weight gradient declined")
        if not need_w:
            dw = None
    return dx, dw, db


# --------------------------------------------------------------- conv3d ---
def conv3d_packed_weight(w: torch.Tensor, key: Optional[torch.Tensor] = None) -> torch.Tensor:
    """[Cout, Cin, KD, KH, KW] -> packed K-major GEMM operand, cached on `key`
    (default: w itself).  A caller that passes a fresh view of a longer-lived
    tensor (a conv2d weight seen as depth 1) keys on that tensor instead, so
    the cache hits on every call."""
    key = w if key is None else key
    hit = _packed_weights.get(key)
    if hit is not None:
        return hit
    L = _lib.lib()
    _on_gpu(w)
    Cout, Cin, KD, KH, KW = w.shape
    nbytes = L.b200_conv3d_packed_weight_bytes_for(Cout, Cin, KD, KH, KW, _code(w.dtype))
    # fp32 weights pack as bf16 hi/lo blocks; 16-bit weights keep their dtype.
    pdt = torch.bfloat16 if w.dtype == torch.float32 else w.dtype
    wp = torch.empty(nbytes // 2, dtype=pdt, device=w.device)
    rc = L.b200_conv3d_pack_weight(w.contiguous().data_ptr(), wp.data_ptr(), _code(w.dtype),
                                   Cout, Cin, KD, KH, KW, _stream(w.device))
    if not _lib.check(rc, "b200_conv3d_pack_weight"):
        raise _lib.NativeError("conv3d weight packing declined")
    _packed_weights.put(key, (), wp)
    return wp


def conv3d(x: torch.Tensor, w: torch.Tensor, bias: Optional[torch.Tensor],
           stride: Sequence[int], padding: Sequence[int], dilation: Sequence[int],
           variant: int = 0, x_channels_last: bool = False,
           out_channels_last: bool = False, out: Optional[torch.Tensor] = None,
           gate: Optional[Sequence[int]] = None,
           weight_key: Optional[torch.Tensor] = None,
           scratch: Optional[torch.Tensor] = None) -> Optional[torch.Tensor]:
    """Dense conv3d on tensor cores (fp16 / bf16; fp32 through bf16 hi/lo
    splits with fp32 accumulation).  x NCDHW (or [N, D, H, W, C] contiguous
    when x_channels_last), w [Cout, Cin, KD, KH, KW].  Returns NCDHW, or an
    [N, Do, Ho, Wo, Cout] contiguous tensor when out_channels_last.
    gate = (epoch, lo, hi, scale) device addresses (lo/hi may be 0) for
    b200_conv3d_fwd_gated: the edge output frames wait for halo arrivals.
    weight_key: the tensor the packed-weight cache is keyed on when w is a
    per-call view of it (conv2d weights seen as depth 1).
    scratch: a caller-owned uint8 workspace used instead of the per-stream
    one (with variant bit 23 it must hold x staged by an earlier call)."""
    key = (x.shape, x.dtype, w.shape, w.dtype, tuple(stride), tuple(padding), tuple(dilation),
           variant, x_channels_last, out_channels_last)
    plan = _conv_plans.get(key)
    if plan is None:
        plan = _conv3d_plan(x, w, stride, padding, dilation, x_channels_last, out_channels_last)
        _conv_plans[key] = plan
    if plan is False:
        return None
    dims, out_shape, prm, wsb, dcode, _problems = plan
    if not (x.is_cuda and w.is_cuda and (bias is None or bias.is_cuda)):
        _on_gpu(x, w, bias)
    if not x.is_contiguous():
        x = x.contiguous()
    wp = conv3d_packed_weight(w, weight_key)
    if bias is not None and not bias.is_contiguous():
        bias = bias.contiguous()
    dev = x.device
    st = _stream(dev)
    if out is None:
        out = torch.empty(out_shape, dtype=x.dtype, device=dev)
    if scratch is not None:
        if scratch.numel() < wsb:
            raise ValueError(f"conv3d scratch holds {scratch.numel()} bytes, needs {wsb}")
        ws = scratch
    else:
        ws = workspace(dev, wsb, st) if wsb > 0 else None
    if gate is None:
        bcode = DTYPE_CODE[bias.dtype] if bias is not None else 0
        rc = _lib.lib().b200_conv3d_fwd_call(
            _conv3d_problem(plan, bcode, x_channels_last, out_channels_last, variant),
            x.data_ptr(), wp.data_ptr(), bias.data_ptr() if bias is not None else None,
            out.data_ptr(), ws.data_ptr() if ws is not None else None, st)
        return out if (rc == 0 or _lib.check(rc, "b200_conv3d_fwd")) else None
    g_epoch, g_lo, g_hi, g_scale = gate
    rc = _lib.lib().b200_conv3d_fwd_gated(
        x.data_ptr(), wp.data_ptr(), bias.data_ptr() if bias is not None else None,
        out.data_ptr(), dcode, DTYPE_CODE[bias.dtype] if bias is not None else 0, *dims, prm,
        int(x_channels_last), int(out_channels_last), variant,
        ws.data_ptr() if ws is not None else None, ws.numel() if ws is not None else 0,
        g_epoch or None, g_lo or None,
        g_hi or None, g_scale, st)
    return out if (rc == 0 or _lib.check(rc, "b200_conv3d_fwd")) else None


def conv3d_scratch_bytes(x: torch.Tensor, w: torch.Tensor, stride: Sequence[int],
                         padding: Sequence[int], dilation: Sequence[int],
                         x_channels_last: bool = False) -> int:
    """Workspace bytes ops.conv3d needs for this problem (either kernel)."""
    plan = _conv3d_plan(x, w, tuple(stride), tuple(padding), tuple(dilation), x_channels_last,
                        False)
    return 0 if plan is False else plan[3]


CONV3D_SLAB, CONV3D_NO_SLAB, CONV3D_SLAB_NO_PAIRS, CONV3D_STAGED = 1 << 20, 1 << 21, 1 << 22, 1 << 23


def conv3d_uses_slab(x: torch.Tensor, w: torch.Tensor, stride: Sequence[int],
                     padding: Sequence[int], dilation: Sequence[int], variant: int = 0,
                     x_channels_last: bool = False) -> bool:
    """Whether ops.conv3d runs this problem on the slab kernel."""
    if x_channels_last:
        N, D, H, W, Cin = x.shape
    else:
        N, Cin, D, H, W = x.shape
    Cout, _, KD, KH, KW = w.shape
    prm = (ctypes.c_int64 * 9)(*stride, *padding, *dilation)
    return bool(_lib.lib().b200_conv3d_uses_slab(N, Cin, D, H, W, Cout, KD, KH, KW, prm,
                                                 _code(x.dtype), variant))


# Per call signature (shapes, dtypes, conv parameters, layout flags): the
# derived sizes, output shape and packed parameter array, or False when the
# kernel cannot take it.  Keeps the per-call host work to a dict lookup.
_conv_plans: dict = {}


def _conv3d_plan(x, w, stride, padding, dilation, x_channels_last, out_channels_last):
    L = _lib.lib()
    if x.dtype not in (torch.float16, torch.bfloat16, torch.float32) or w.dtype != x.dtype:
        return False
    if x_channels_last:
        N, D, H, W, Cin = x.shape
    else:
        N, Cin, D, H, W = x.shape
    Cout, Cin_w, KD, KH, KW = w.shape
    if Cin_w != Cin:
        return False
    sd, sh, sw = stride
    pd, ph, pw = padding
    dd, dh, dw = dilation
    Do = (D + 2 * pd - dd * (KD - 1) - 1) // sd + 1
    Ho = (H + 2 * ph - dh * (KH - 1) - 1) // sh + 1
    Wo = (W + 2 * pw - dw * (KW - 1) - 1) // sw + 1
    if min(Do, Ho, Wo) <= 0:
        return False
    out_shape = (N, Do, Ho, Wo, Cout) if out_channels_last else (N, Cout, Do, Ho, Wo)
    prm = (ctypes.c_int64 * 9)(sd, sh, sw, pd, ph, pw, dd, dh, dw)
    wsb = int(L.b200_conv3d_fwd_workspace_bytes(N, Cin, D, H, W, KD, KH, KW, prm,
                                                _code(x.dtype), int(x_channels_last)))
    return (N, Cin, D, H, W, Cout, KD, KH, KW), out_shape, prm, wsb, _code(x.dtype), {}


def _conv3d_problem(plan, bias_code: int, x_channels_last: bool, out_channels_last: bool,
                    variant: int) -> int:
    """Address of the plan's packed B200Conv3dProblem for this bias dtype
    (built once; b200_conv3d_fwd_call then takes only the per-call pointers)."""
    dims, _shape, prm, wsb, dcode, problems = plan
    addr = problems.get(bias_code)
    if addr is None:
        pr = _lib.Conv3dProblem(*dims, prm, dcode, bias_code, int(x_channels_last),
                                int(out_channels_last), variant, 0, wsb)
        addr = ctypes.addressof(pr)
        problems[bias_code] = addr
        problems[("keep", bias_code)] = pr   # the struct lives as long as the plan
    return addr


def to_channels_last(x: torch.Tensor) -> torch.Tensor:
    """[N, C, *] contiguous -> [N, S, C] contiguous copy (S = prod(*))."""
    L = _lib.lib()
    _on_gpu(x)
    N, C = x.shape[0], x.shape[1]
    S = x.numel() // max(1, N * C)
    y = torch.empty(N, S, C, dtype=x.dtype, device=x.device)
    rc = L.b200_to_channels_last(x.contiguous().data_ptr(), y.data_ptr(), _code(x.dtype), N, C,
                                 S, _stream(x.device))
    if not _lib.check(rc, "b200_to_channels_last"):
        raise _lib.NativeError("to_channels_last declined")
    return y


# ------------------------------------------------------------------ FFT ---
def fftconv1d_spectrum(w: torch.Tensor, nfft: int, cache: bool = True) -> Optional[torch.Tensor]:
    """Conjugated spectrum (nfft complex64 per channel, transform-position
    order) of a depthwise kernel given as [C, 1, K] or [C, K]; cached on the
    caller's weight object (pass the parameter itself, not a fresh view, or
    every call recomputes it).  cache=False for one-off filters (gradients
    used as filters in the backward pass), which would only evict weights."""
    hit = _spectra.get(w, ("fft1d", nfft)) if cache else None
    if hit is not None:
        return hit
    L = _lib.lib()
    _on_gpu(w)
    C, K = w.shape[0], w.shape[-1]
    w2d = w.reshape(C, K).contiguous()
    spec = torch.empty(L.b200_fftconv1d_spectrum_bytes(C, nfft) // 4, dtype=torch.float32,
                       device=w.device)
    rc = L.b200_fftconv1d_prepare(w2d.data_ptr(), spec.data_ptr(), _code(w.dtype), C, K, nfft,
                                  _stream(w.device))
    if not _lib.check(rc, "b200_fftconv1d_prepare"):
        return None
    if cache:
        _spectra.put(w, ("fft1d", nfft), spec)
    return spec


def fftconv1d(x: torch.Tensor, w2d: torch.Tensor, bias: Optional[torch.Tensor], padding: int,
              nfft: int, segmented: bool = False, cache: bool = True) -> Optional[torch.Tensor]:
    """Depthwise FFT conv1d; `w2d` is the kernel as [C, 1, K] or [C, K].
    segmented: overlap-save segments of nfft - K + 1 outputs (nfft >= K)
    instead of one transform of the whole padded row (nfft >= L + 2p)."""
    L_ = _lib.lib()
    _on_gpu(x, w2d, bias)
    if not L_.b200_fft_supported_length(nfft):
        return None
    B, C, L = x.shape
    K = w2d.shape[-1]
    Lout = L + 2 * padding - K + 1
    spec = fftconv1d_spectrum(w2d, nfft, cache=cache)
    if spec is None:
        return None
    x = x.contiguous()
    b = bias.contiguous() if bias is not None else None
    y = torch.empty(B, C, Lout, dtype=x.dtype, device=x.device)
    if segmented:
        rc = L_.b200_fftconv1d_fwd_os(x.data_ptr(), spec.data_ptr(), _ptr(b), y.data_ptr(),
                                      _code(x.dtype), _code(b.dtype) if b is not None else 0,
                                      B, C, L, K, padding, Lout, nfft, _stream(x.device))
    else:
        rc = L_.b200_fftconv1d_fwd(x.data_ptr(), spec.data_ptr(), _ptr(b), y.data_ptr(),
                                   _code(x.dtype), _code(b.dtype) if b is not None else 0,
                                   B, C, L, padding, Lout, nfft, _stream(x.device))
    return y if _lib.check(rc, "b200_fftconv1d_fwd") else None


def fftconv3d_spectrum(w: torch.Tensor, fsize: Sequence[int]) -> Optional[torch.Tensor]:
    hit = _spectra.get(w, ("fft3d",) + tuple(fsize))
    if hit is not None:
        return hit
    L = _lib.lib()
    _on_gpu(w)
    Cout, Cin, KD, KH, KW = w.shape
    fd, fh, fw = fsize
    nbytes = L.b200_fftconv3d_spectrum_bytes(Cout, Cin, fd, fh, fw, _code(w.dtype))
    spec = torch.empty(nbytes // 4, dtype=torch.float32, device=w.device)
    wsb = L.b200_fftconv3d_workspace_bytes(1, Cin, Cout, fd, fh, fw)
    ws = workspace(w.device, wsb)
    rc = L.b200_fftconv3d_prepare(w.contiguous().data_ptr(), spec.data_ptr(), _code(w.dtype),
                                  Cout, Cin, KD, KH, KW, fd, fh, fw, _ptr(ws), wsb,
                                  _stream(w.device))
    if not _lib.check(rc, "b200_fftconv3d_prepare"):
        return None
    _spectra.put(w, ("fft3d",) + tuple(fsize), spec)
    return spec


def fftconv3d(x: torch.Tensor, w: torch.Tensor, bias: Optional[torch.Tensor],
              pad: Sequence[int], fsize: Sequence[int]) -> Optional[torch.Tensor]:
    L_ = _lib.lib()
    _on_gpu(x, w, bias)
    N, Cin, D, H, W = x.shape
    Cout, _, KD, KH, KW = w.shape
    fd, fh, fw = fsize
    if not all(L_.b200_fft_supported_length(n) for n in fsize):
        return None
    if w.dtype != x.dtype:   # the spectrum's storage type follows the weight dtype
        return None
    spec = fftconv3d_spectrum(w, fsize)
    if spec is None:
        return None
    Do, Ho, Wo = D + 2 * pad[0] - KD + 1, H + 2 * pad[1] - KH + 1, W + 2 * pad[2] - KW + 1
    x = x.contiguous()
    b = bias.contiguous() if bias is not None else None
    y = torch.empty(N, Cout, Do, Ho, Wo, dtype=x.dtype, device=x.device)
    wsb = L_.b200_fftconv3d_workspace_bytes(N, Cin, Cout, fd, fh, fw)
    ws = workspace(x.device, wsb)
    p3 = (ctypes.c_int64 * 3)(*pad)
    rc = L_.b200_fftconv3d_fwd(x.data_ptr(), spec.data_ptr(), _ptr(b), y.data_ptr(),
                               _code(x.dtype), _code(b.dtype) if b is not None else 0,
                               N, Cin, D, H, W, Cout, KD, KH, KW, p3, fd, fh, fw,
                               _ptr(ws), wsb, _stream(x.device))
    return y if _lib.check(rc, "b200_fftconv3d_fwd") else None


def read_device_flags(device: Optional[torch.device] = None) -> int:
    """Reads and clears the kernels' device-side fault word (0 = no fault)."""
    device = device or torch.device("cuda", torch.cuda.current_device())
    out = ctypes.c_int(0)
    _lib.check(_lib.lib().b200_read_device_flags(_stream(device), ctypes.byref(out)),
               "b200_read_device_flags")
    return out.value
