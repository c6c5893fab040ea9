"""torch.library custom ops so the native kernels stay single graph nodes
under torch.compile (no graph break), with fake (meta) implementations for
shape propagation.

Reference: amd_tuned_torch/compile_ops.py:168-235 (`group_norm`,
`conv3d_native` custom ops + register_fake) and :369-415 (the Python entry
points).  The eager dispatch path calls ops.* directly (a custom op costs
dispatcher overhead per call) and switches to these only while Dynamo traces,
the same split the reference makes in _dispatch._group_norm_native
(:2100-2115).
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
        out = ops.group_norm(input, num_groups, weight, bias, eps)
        if out is None:
            raise RuntimeError("amd_tuned_torch::group_norm: kernel declined")
        return out

    @_group_norm_op.register_fake
    def _group_norm_fake(input, num_groups, weight, bias, eps):
        return torch.empty_like(input)


if not _registered("conv3d_native"):

    @torch.library.custom_op("amd_tuned_torch::conv3d_native", mutates_args=())
    def _conv3d_op(input: torch.Tensor, weight: torch.Tensor, bias: Optional[torch.Tensor],
                   stride: List[int], padding: List[int], dilation: List[int]) -> torch.Tensor:
        out = ops.conv3d(input, weight, bias, stride, padding, dilation)
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


def group_norm(input, num_groups, weight=None, bias=None, eps=1e-5):
    return torch.ops.amd_tuned_torch.group_norm(input, num_groups, weight, bias, eps)


def conv3d_native(input, weight, bias=None, stride=1, padding=0, dilation=1):
    def trip(v):
        return [v] * 3 if isinstance(v, int) else list(v)
    return torch.ops.amd_tuned_torch.conv3d_native(input, weight, bias, trip(stride),
                                                   trip(padding), trip(dilation))
