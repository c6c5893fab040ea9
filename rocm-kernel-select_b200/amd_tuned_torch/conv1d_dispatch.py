"""The patched F.conv1d: depthwise-direct / FFT / stock contest.

Role of the reference's amd_tuned_torch/miopen_fallback.py (:312-398
eligibility + `_try_fftconv1d_fastpath`, :434-501 the wrapper), minus its
MIOpen retry and CPU fallback (there is no MIOpen here, and this build never
falls back to the CPU) and minus the causal-conv1d and sparse fast paths
(other projects' kernels).  One kernel_select contest per shape over
{"fftconv", "depthwise", "stock"} -- stock last as the verification
reference -- with the FFT verification bar, exactly as the reference folds
its depthwise candidate into the fftconv contest.

Eligibility for "depthwise" (reference `_is_depthwise_conv1d_eligible`):
CUDA 3-D input, groups == C == Cout, one input channel per group, stride 1,
dilation 1.  The reference additionally requires an odd kernel width because
its vendored kernel does (conv1d.h:76); this kernel handles any width, so
that restriction is dropped.
"""
from __future__ import annotations

from typing import Any, Callable, Optional

import torch
import torch.nn.functional as F

from . import _lib, depthwise_conv1d_ops, fftconv_ops, kernel_select


def _scalar(v: Any) -> Any:
    return v[0] if isinstance(v, (tuple, list)) else v


def _is_depthwise_conv1d_eligible(input: torch.Tensor, weight: torch.Tensor, stride: Any,
                                  dilation: Any, groups: int) -> bool:
    if not (input.is_cuda and input.dim() == 3 and weight.dim() == 3):
        return False
    if type(input) not in (torch.Tensor, torch.nn.Parameter):
        return False
    dim = input.shape[1]
    out_channels, in_per_group, _width = weight.shape
    if groups != dim or out_channels != dim or in_per_group != 1:
        return False
    if input.dtype not in (torch.float16, torch.bfloat16, torch.float32):
        return False
    return _scalar(stride) == 1 and _scalar(dilation) == 1


def _try_fftconv1d_fastpath(input, weight, bias, stride, padding, dilation, groups,
                            orig_fn: Callable) -> Optional[torch.Tensor]:
    """The {fftconv, depthwise, stock} contest, or None when no own candidate
    applies (the caller then calls stock directly)."""
    if not input.is_cuda or not _lib.available() or isinstance(_scalar(padding), str):
        return None
    if input.numel() == 0 or weight.numel() == 0:   # empty: stock's own result
        return None
    depthwise = (depthwise_conv1d_ops.available()
                 and _is_depthwise_conv1d_eligible(input, weight, stride, dilation, groups))
    if torch.compiler.is_compiling():
        # While Dynamo traces: the depthwise custom op (one graph node with a
        # registered backward), no contest; anything else goes to stock.
        if not depthwise or not isinstance(_scalar(padding), int):
            return None
        b = bias if bias is not None else torch.zeros(weight.shape[0], device=input.device,
                                                      dtype=weight.dtype)
        return depthwise_conv1d_ops.conv1d_forward(input, weight.squeeze(1), b,
                                                   int(_scalar(padding)))
    fft = (fftconv_ops.fft_conv1d_enabled()
           and fftconv_ops._is_depthwise(input, weight, groups)
           and _scalar(stride) == 1 and _scalar(dilation) == 1)
    if not (depthwise or fft):
        return None
    s, p, d = _scalar(stride), _scalar(padding), _scalar(dilation)
    candidates = []
    if fft:
        candidates.append(("fftconv", lambda: fftconv_ops.fftconv1d_candidate(
            input, weight, bias, s, p, d, groups)))
    if depthwise:
        candidates.append(("depthwise", lambda: depthwise_conv1d_ops.depthwise_conv1d_candidate(
            input, weight, bias, stride, padding, dilation, groups)))
    candidates.append(("stock", lambda: orig_fn(input, weight, bias, stride, padding,
                                                dilation, groups)))
    if kernel_select.enabled():
        return kernel_select.pick("conv1d", input, weight, stride, padding, dilation,
                                  candidates, tolerance=fftconv_ops.fftconv_tolerance(input.dtype))
    for _name, thunk in candidates:  # contest off: fixed order, own kernels first
        out = thunk()
        if out is not None:
            return out
    return None


def make_wrapper(get_orig: Callable[[], Callable]) -> Callable:
    def conv1d(input: torch.Tensor, weight: torch.Tensor, bias: Optional[torch.Tensor] = None,
               stride: Any = 1, padding: Any = 0, dilation: Any = 1,
               groups: int = 1) -> torch.Tensor:
        orig = get_orig()
        out = _try_fftconv1d_fastpath(input, weight, bias, stride, padding, dilation, groups,
                                      orig)
        if out is not None:
            return out
        return orig(input, weight, bias, stride, padding, dilation, groups)
    conv1d._amd_tuned_torch_wrapper = True
    return conv1d


_original_conv1d: Optional[Callable] = None


def enable_conv1d_fallback() -> None:
    """Install only the F.conv1d wrapper (idempotent)."""
    global _original_conv1d
    if getattr(F.conv1d, "_amd_tuned_torch_wrapper", False):
        return
    _original_conv1d = F.conv1d
    F.conv1d = make_wrapper(lambda: _original_conv1d)


def disable_conv1d_fallback() -> None:
    global _original_conv1d
    if _original_conv1d is not None and getattr(F.conv1d, "_amd_tuned_torch_wrapper", False):
        F.conv1d = _original_conv1d
        _original_conv1d = None


def is_conv1d_fallback_enabled() -> bool:
    return bool(getattr(F.conv1d, "_amd_tuned_torch_wrapper", False))
