"""GroupNorm -> SiLU fusion and GroupNorm -> SiLU -> conv blocks.

Reference: amd_tuned_torch/conv_fusion_ops.py:301-353 (group_norm_silu:
SiLU(GroupNorm(x)) decided per shape by a kernel_select contest between fused
kernels and stock, forward only) and _dispatch.py:2683-2738
(_patched_sequential_forward: an nn.Sequential of GroupNorm(affine), SiLU and
Conv2d runs group_norm_silu, then the conv).

Here the fused GroupNorm + SiLU is this package's statistics kernel
(b200_gn_partial_stats) and normalise kernel (b200_gn_apply with SiLU).  For
a block, the normalise kernel writes its result channels-last, which is
exactly the tcgen05 conv kernel's operand layout: the conv runs on it
directly (no NC[D]HW intermediate of the activation, no SiLU pass, no layout
transposition).  Conv3d blocks run as they are; Conv2d blocks run as a
depth-1 Conv3d.  Each fused path contests stock per shape (kernel_select),
so a shape where fusion loses keeps the unfused chain.
"""
from __future__ import annotations

from typing import Optional

import torch
import torch.nn.functional as F

from . import _lib, kernel_select, ops

_DTYPES = (torch.float16, torch.bfloat16)


def _orig(name: str):
    from . import _dispatch
    return _dispatch._ORIGINALS.get((F, name), getattr(F, name))


def _stock_group_norm_silu(x, num_groups, weight, bias, eps):
    return F.silu(_orig("group_norm")(x, num_groups, weight, bias, eps))


def _grad_live(*tensors) -> bool:
    return torch.is_grad_enabled() and any(
        isinstance(t, torch.Tensor) and t.requires_grad for t in tensors)


def _fused_group_norm_silu(x, num_groups, weight, bias, eps, channels_last_out=False):
    stats = ops.group_norm_partial_stats(x, num_groups)        # (count, mean, M2) per (n, g)
    return ops.group_norm_apply(x, stats, num_groups, weight, bias, eps, silu=True,
                                channels_last_out=channels_last_out)


def group_norm_silu(x: torch.Tensor, num_groups: int, weight: Optional[torch.Tensor] = None,
                    bias: Optional[torch.Tensor] = None, eps: float = 1e-5) -> torch.Tensor:
    """SiLU(GroupNorm(x)) in two kernels (statistics, normalise + SiLU) where
    that wins the per-shape contest, stock otherwise.  Forward only: stock
    whenever a gradient is live."""
    if (not _lib.available() or not isinstance(x, torch.Tensor) or not x.is_cuda
            or x.dim() < 3 or x.dtype not in _DTYPES or x.numel() == 0 or num_groups <= 0
            or x.shape[1] % num_groups != 0 or not x.is_contiguous()
            or _grad_live(x, weight, bias)):
        return _stock_group_norm_silu(x, num_groups, weight, bias, eps)
    cands = [("fused", lambda: _fused_group_norm_silu(x, num_groups, weight, bias, eps)),
             ("stock", lambda: _stock_group_norm_silu(x, num_groups, weight, bias, eps))]
    key = (x.dtype, tuple(x.shape), int(num_groups), "nchw")
    out = kernel_select.pick_key("group_norm_silu", key, cands)
    if out is not None:
        return out
    for _name, thunk in cands:        # contest off: fused first
        out = thunk()
        if out is not None:
            return out
    return _stock_group_norm_silu(x, num_groups, weight, bias, eps)


def _weight5(w: torch.Tensor) -> torch.Tensor:
    """A Conv2d weight [Co, Ci, KH, KW] as the depth-1 Conv3d weight (a view;
    ops.conv3d keys its packed-weight cache on the original tensor)."""
    return w if w.dim() == 5 else w.unsqueeze(2)


def _triple(v, fill):
    if isinstance(v, int):
        return (v, v, v)
    v = tuple(v)
    return v if len(v) == 3 else (fill,) + v


def _fused_block(x, norm, conv) -> Optional[torch.Tensor]:
    """GN + SiLU written channels-last, then the tensor-core conv on it."""
    N, C = x.shape[0], x.shape[1]
    two_d = x.dim() == 4
    y = _fused_group_norm_silu(x, norm.num_groups, norm.weight, norm.bias, norm.eps,
                               channels_last_out=True)            # [N, S, C]
    spatial = (1,) + tuple(x.shape[2:]) if two_d else tuple(x.shape[2:])
    xcl = y.view((N,) + spatial + (C,))
    stride = _triple(conv.stride, 1)
    pad = _triple(conv.padding, 0)
    dil = _triple(conv.dilation, 1)
    out = ops.conv3d(xcl, _weight5(conv.weight), conv.bias, stride, pad, dil,
                     x_channels_last=True, weight_key=conv.weight)
    if out is None:
        return None
    return out.squeeze(2) if two_d else out


def _block_ok(x, norm, conv) -> bool:
    conv3 = isinstance(conv, torch.nn.Conv3d)
    if not (conv3 or isinstance(conv, torch.nn.Conv2d)):
        return False
    if x.dim() != (5 if conv3 else 4) or not x.is_cuda or x.dtype not in _DTYPES:
        return False
    if not x.is_contiguous() or x.numel() == 0 or x.shape[1] % norm.num_groups != 0:
        return False
    if conv.groups != 1 or conv.padding_mode != "zeros" or isinstance(conv.padding, str):
        return False
    if conv.weight.dtype != x.dtype or any(s != 1 for s in conv.stride):
        return False
    return not _grad_live(x, norm.weight, norm.bias, conv.weight, conv.bias)


def gn_silu_conv(x: torch.Tensor, norm, conv, stock) -> torch.Tensor:
    """The block GroupNorm -> SiLU -> conv: fused where it wins the per-shape
    contest against the unfused chain (`stock`, the Sequential's own forward)."""
    if not _lib.available() or not _block_ok(x, norm, conv):
        return stock()
    key = (x.dtype, tuple(x.shape), int(norm.num_groups), tuple(conv.weight.shape),
           tuple(conv.padding) if not isinstance(conv.padding, str) else conv.padding,
           tuple(conv.dilation))
    cands = [("fused", lambda: _fused_block(x, norm, conv)), ("stock", stock)]
    out = kernel_select.pick_key("gn_silu_conv", key, cands)
    if out is not None:
        return out
    out = _fused_block(x, norm, conv)
    return out if out is not None else stock()
