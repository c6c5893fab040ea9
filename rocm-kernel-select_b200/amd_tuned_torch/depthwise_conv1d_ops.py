"""Depthwise conv1d candidate for the F.conv1d contest.

Same surface as the reference's amd_tuned_torch/depthwise_conv1d_ops.py
(`available`, `maybe_contiguous`, `_out_len`, `conv1d_forward`,
`DepthwiseConv1dFn`, `depthwise_conv1d_candidate`, the
`amd_tuned_torch::depthwise_conv1d_forward` custom op with a fake for
torch.compile), now backed by the sm_100a kernel `b200_dwconv1d_fwd`
(register/shared-memory tiled, fp32 accumulation, current stream).

Layout: only BHL ([B, C, L], the nn.Conv1d layout) -- the reference's
candidate always passes is_bhl=True (depthwise_conv1d_ops.py:247); the
`is_bhl=False` path raises here.  Backward: the reference calls its vendored
backward kernel (conv1d_bwd_cuda_bhl.cu:19-114); here du is the forward
kernel run on dy with the taps reversed (b200_dwconv1d_fwd,
B200_DWCONV1D_FLIP_TAPS) and dweight / dbias come from
b200_dwconv1d_bwd_weight (per-tile partial sums, fixed-order reduction).
"""
from __future__ import annotations

from typing import Any, List, Optional

import torch

from . import _lib, ops


def available() -> bool:
    return _lib.available()


def maybe_contiguous(x: Optional[torch.Tensor]) -> Optional[torch.Tensor]:
    """Copy only when the last dimension is not unit-stride."""
    return x.contiguous() if x is not None and x.stride(-1) != 1 else x


def _out_len(length: int, padding: int, width: int) -> int:
    """l_out = l + 2 * padding - k + 1 (stride 1, dilation 1)."""
    return length + 2 * padding - width + 1


def _forward_native(input_: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor,
                    padding: int, is_bhl: bool) -> torch.Tensor:
    if not is_bhl:
        raise RuntimeError("depthwise conv1d: only the [B, C, L] layout is supported")
    out = ops.depthwise_conv1d(input_, weight, bias, int(padding))
    if out is None:
        raise RuntimeError("depthwise conv1d kernel declined this problem")
    return out


if not (hasattr(torch.ops, "amd_tuned_torch")
        and hasattr(torch.ops.amd_tuned_torch, "depthwise_conv1d_forward")):

    @torch.library.custom_op("amd_tuned_torch::depthwise_conv1d_forward", mutates_args=())
    def _depthwise_conv1d_forward_op(input_: torch.Tensor, weight: torch.Tensor,
                                     bias: torch.Tensor, padding: int,
                                     is_bhl: bool) -> torch.Tensor:
        return _forward_native(input_, weight, bias, padding, is_bhl)

    @_depthwise_conv1d_forward_op.register_fake
    def _depthwise_conv1d_forward_fake(input_, weight, bias, padding, is_bhl):
        del bias
        if is_bhl:
            b, d, length = input_.shape
            return input_.new_empty(b, d, _out_len(length, padding, weight.shape[1]))
        b, length, d = input_.shape
        return input_.new_empty(b, _out_len(length, padding, weight.shape[0]), d)

    @torch.library.custom_op("amd_tuned_torch::depthwise_conv1d_backward", mutates_args=())
    def _depthwise_conv1d_backward_op(dout: torch.Tensor, input_: torch.Tensor,
                                      weight: torch.Tensor, padding: int, need_x: bool,
                                      need_w: bool, need_b: bool) -> List[torch.Tensor]:
        du, dw, db = ops.depthwise_conv1d_backward(dout, input_, weight, padding,
                                                   (need_x, need_w, need_b))
        none = lambda dt: torch.empty(0, dtype=dt, device=input_.device)  # noqa: E731
        return [du if du is not None else none(input_.dtype),
                dw if dw is not None else none(weight.dtype),
                db if db is not None else none(weight.dtype)]

    @_depthwise_conv1d_backward_op.register_fake
    def _depthwise_conv1d_backward_fake(dout, input_, weight, padding, need_x, need_w, need_b):
        return [torch.empty_like(input_, memory_format=torch.contiguous_format) if need_x
                else input_.new_empty(0),
                weight.new_empty(weight.shape if need_w else (0,)),
                weight.new_empty(weight.shape[0] if need_b else 0)]

    def _dw_setup(ctx, inputs, output):
        input_, weight, bias, padding, is_bhl = inputs
        ctx.save_for_backward(input_, weight)
        ctx.padding, ctx.is_bhl = padding, is_bhl
        ctx.bias_dtype = bias.dtype

    def _dw_backward(ctx, dout):
        input_, weight = ctx.saved_tensors
        if not ctx.is_bhl:
            raise RuntimeError("depthwise conv1d: only the [B, C, L] layout is supported")
        nx, nw, nb = ctx.needs_input_grad[:3]
        du, dw, db = torch.ops.amd_tuned_torch.depthwise_conv1d_backward(
            dout.contiguous(), input_, weight, ctx.padding, nx, nw, nb)
        return (du if nx else None, dw if nw else None,
                db.to(ctx.bias_dtype) if nb else None, None, None)

    _depthwise_conv1d_forward_op.register_autograd(_dw_backward, setup_context=_dw_setup)

_conv1d_forward_impl = torch.ops.amd_tuned_torch.depthwise_conv1d_forward


def conv1d_forward(input: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor,
                   padding: int, is_bhl: bool = True) -> torch.Tensor:
    """`weight` is the squeezed [C, K] depthwise kernel; `bias` is required."""
    input, weight, bias = maybe_contiguous(input), maybe_contiguous(weight), maybe_contiguous(bias)
    if torch.compiler.is_compiling():
        return _conv1d_forward_impl(input, weight, bias, padding, is_bhl)
    return _forward_native(input, weight, bias, padding, is_bhl)


def conv1d_backward(dout: torch.Tensor, input: torch.Tensor, weight: torch.Tensor,
                    bias: torch.Tensor, padding: int, is_bhl: bool = True, needs=None):
    """(du, dweight, dbias) of y = bias + corr(x, w) for the BHL layout, on
    the sm_100a kernels.  `weight` is the squeezed [C, K] kernel; `needs`
    (three flags, default all) skips gradients nobody asked for."""
    if not is_bhl:
        raise RuntimeError("depthwise conv1d: only the [B, C, L] layout is supported")
    du, dweight, dbias = ops.depthwise_conv1d_backward(
        dout, maybe_contiguous(input), weight, int(padding),
        tuple(needs) if needs is not None else (True, True, True))
    if dbias is not None and bias is not None and dbias.dtype != bias.dtype:
        dbias = dbias.to(bias.dtype)
    return du, dweight, dbias


class DepthwiseConv1dFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, input, weight, bias, padding, is_bhl):
        ctx.padding = padding
        ctx.is_bhl = is_bhl
        ctx.save_for_backward(input, weight, bias)
        return conv1d_forward(input, weight, bias, padding, is_bhl)

    @staticmethod
    def backward(ctx, dout):
        input, weight, bias = ctx.saved_tensors
        needs = ctx.needs_input_grad[:3]
        if not any(needs):
            return None, None, None, None, None
        du, dweight, dbias = conv1d_backward(dout.contiguous(), input, weight, bias,
                                             ctx.padding, ctx.is_bhl, needs=needs)
        return du, dweight, dbias, None, None


def depthwise_conv1d_candidate(input: torch.Tensor, weight: torch.Tensor,
                               bias: Optional[torch.Tensor], stride: Any, padding: Any,
                               dilation: Any, groups: int) -> Optional[torch.Tensor]:
    """kernel_select candidate with F.conv1d's calling convention (weight
    [C, 1, K], bias may be None); the caller has checked depthwise
    eligibility.  Returns None (declines) instead of raising."""
    channels = weight.shape[0]
    squeezed = weight.squeeze(1)
    if bias is None:
        bias = torch.zeros(channels, device=input.device, dtype=weight.dtype)
    pad = padding[0] if isinstance(padding, (tuple, list)) else padding
    if not isinstance(pad, int):
        return None
    try:
        return DepthwiseConv1dFn.apply(input, squeezed, bias, pad, True)
    except _lib.NativeError:
        raise
    except RuntimeError:
        return None
