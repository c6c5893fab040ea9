"""torch.library custom ops so the native kernels stay single graph nodes
under torch.compile (no graph break), with fake (meta) implementations for
shape propagation and autograd formulas so compiled training works.

Reference: amd_tuned_torch/compile_ops.py:168-235 (`group_norm`,
`conv3d_native` custom ops + register_fake) and :369-415 (the Python entry
points).  The eager dispatch path calls ops.* directly (a custom op costs
dispatcher overhead per call) and switches to these only while Dynamo traces
(`_dispatch._patched_group_norm` / `_patched_conv3d`, the conv1d wrapper),
the same split the reference makes in _dispatch._group_norm_native
(:2100-2115).  Backward: GroupNorm and the depthwise conv1d run their native
backward kernels as custom ops of their own; conv3d's backward is
aten.convolution_backward (stock, as in eager mode).
"""
from __future__ import annotations

from typing import List, Optional

import torch

from . import ops


def _registered(name: str) -> bool:
    return hasattr(torch.ops, "amd_tuned_torch") and hasattr(torch.ops.amd_tuned_torch, name)


if not _registered("group_norm"):

    @torch.library.custom_op("amd_tuned_torch::group_norm", mutates_args=())
    def _group_norm_op(input: torch.Tensor, num_groups: int, weight: Optional[torch.Tensor],
                       bias: Optional[torch.Tensor], eps: float) -> torch.Tensor:
        out = ops.group_norm(input.contiguous(), num_groups, weight, bias, eps)
        if out is None:
            raise RuntimeError("amd_tuned_torch::group_norm: kernel declined")
        return out

    @_group_norm_op.register_fake
    def _group_norm_fake(input, num_groups, weight, bias, eps):
        return torch.empty_like(input, memory_format=torch.contiguous_format)

    @torch.library.custom_op("amd_tuned_torch::group_norm_backward", mutates_args=())
    def _group_norm_bwd_op(grad: torch.Tensor, input: torch.Tensor, num_groups: int,
                           weight: Optional[torch.Tensor], eps: float, need_x: bool,
                           need_w: bool, need_b: bool,
                           affine_dtype: torch.dtype) -> List[torch.Tensor]:
        gx, gw, gb = ops.group_norm_backward(grad, input, num_groups, weight, eps,
                                             (need_x, need_w, need_b), affine_dtype=affine_dtype)
        empty = lambda dt: torch.empty(0, dtype=dt, device=input.device)  # noqa: E731
        return [gx if gx is not None else empty(input.dtype),
                gw if gw is not None else empty(affine_dtype),
                gb if gb is not None else empty(affine_dtype)]

    @_group_norm_bwd_op.register_fake
    def _group_norm_bwd_fake(grad, input, num_groups, weight, eps, need_x, need_w, need_b,
                             affine_dtype):
        C = input.shape[1]
        return [torch.empty_like(input, memory_format=torch.contiguous_format) if need_x
                else input.new_empty(0),
                input.new_empty(C if need_w else 0, dtype=affine_dtype),
                input.new_empty(C if need_b else 0, dtype=affine_dtype)]

    def _gn_setup(ctx, inputs, output):
        input, num_groups, weight, bias, eps = inputs
        ctx.save_for_backward(input, weight)
        ctx.num_groups, ctx.eps = num_groups, eps
        ctx.has_bias = bias is not None
        ctx.affine_dtype = (weight.dtype if weight is not None else
                            bias.dtype if bias is not None else input.dtype)

    def _gn_backward(ctx, grad):
        input, weight = ctx.saved_tensors
        need_x = ctx.needs_input_grad[0]
        need_w = weight is not None and ctx.needs_input_grad[2]
        need_b = ctx.has_bias and ctx.needs_input_grad[3]
        gx, gw, gb = torch.ops.amd_tuned_torch.group_norm_backward(
            grad, input, ctx.num_groups, weight, ctx.eps, need_x, need_w, need_b,
            ctx.affine_dtype)
        return (gx if need_x else None, None, gw if need_w else None, gb if need_b else None,
                None)

    _group_norm_op.register_autograd(_gn_backward, setup_context=_gn_setup)


if not _registered("conv3d_native"):

    @torch.library.custom_op("amd_tuned_torch::conv3d_native", mutates_args=())
    def _conv3d_op(input: torch.Tensor, weight: torch.Tensor, bias: Optional[torch.Tensor],
                   stride: List[int], padding: List[int], dilation: List[int]) -> torch.Tensor:
        out = ops.conv3d(input.contiguous(), weight, bias, stride, padding, dilation)
        if out is None:
            raise RuntimeError("amd_tuned_torch::conv3d_native: kernel declined")
        return out

    @_conv3d_op.register_fake
    def _conv3d_fake(input, weight, bias, stride, padding, dilation):
        N, _, D, H, W = input.shape
        Cout, _, KD, KH, KW = weight.shape
        size = [N, Cout]
        for n, k, s, p, d in zip((D, H, W), (KD, KH, KW), stride, padding, dilation):
            size.append((n + 2 * p - d * (k - 1) - 1) // s + 1)
        return input.new_empty(size)

    def _conv3d_setup(ctx, inputs, output):
        input, weight, bias, stride, padding, dilation = inputs
        ctx.save_for_backward(input, weight)
        ctx.conv = (list(stride), list(padding), list(dilation))
        ctx.bias_sizes = [bias.shape[0]] if bias is not None else None

    def _conv3d_backward(ctx, grad):
        input, weight = ctx.saved_tensors
        stride, padding, dilation = ctx.conv
        needs = [ctx.needs_input_grad[0], ctx.needs_input_grad[1],
                 ctx.bias_sizes is not None and ctx.needs_input_grad[2]]
        gi, gw, gb = torch.ops.aten.convolution_backward(
            grad.contiguous(), input, weight, ctx.bias_sizes, stride, padding, dilation, False,
            [0, 0, 0], 1, needs)
        return gi, gw, gb, None, None, None

    _conv3d_op.register_autograd(_conv3d_backward, setup_context=_conv3d_setup)


def group_norm(input, num_groups, weight=None, bias=None, eps=1e-5):
    return torch.ops.amd_tuned_torch.group_norm(input, num_groups, weight, bias, eps)


def conv3d_native(input, weight, bias=None, stride=1, padding=0, dilation=1):
    def trip(v):
        return [v] * 3 if isinstance(v, int) else list(v) * (3 if len(v) == 1 else 1)
    return torch.ops.amd_tuned_torch.conv3d_native(input, weight, bias, trip(stride),
                                                   trip(padding), trip(dilation))


def conv3d_native_eligible(input, weight, bias, stride, padding, dilation, groups) -> bool:
    """Shape-only test (no device work, safe while tracing) for the problems
    the tensor-core kernel takes: groups 1, numeric padding, stride 1,
    fp16/bf16 with matching weight, Cin a multiple of 8."""
    if groups != 1 or isinstance(padding, str) or input.dim() != 5 or weight.dim() != 5:
        return False
    if input.dtype not in (torch.float16, torch.bfloat16) or weight.dtype != input.dtype:
        return False
    s = [stride] * 3 if isinstance(stride, int) else list(stride)
    return all(v == 1 for v in s) and input.shape[1] % 8 == 0 and input.numel() > 0
