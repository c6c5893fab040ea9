"""amd_tuned_torch -- B200-native build of rocm-kernel-select's conv/norm hot path.

`import amd_tuned_torch` patches torch.nn.functional.conv1d (depthwise),
conv3d and group_norm unless AMD_TUNED_TORCH_AUTOPATCH=0, exactly like the
reference package (amd_tuned_torch/__init__.py:606-610).  `enable()`,
`disable()` and `is_enabled()` toggle the patches.  Each patched op holds a
first-call benchmark-then-cache contest (`kernel_select`) between this
project's own sm_100a kernels (libb200conv.so, C ABI in include/b200conv.h),
with stock torch as the verification reference.

On a machine with a CUDA device the native library must load, otherwise the
import fails (no silent fallback); see `_lib`.
"""
from __future__ import annotations

import os

import torch

from . import _lib

if torch.cuda.is_available() and not _lib.available():
    raise ImportError(
        "amd_tuned_torch: CUDA is available but libb200conv.so could not be loaded "
        f"({_lib.load_error()}). Build it with `python rocm-kernel-select_b200/csrc/build.py`.")

from . import kernel_select, ops, compile_ops, depthwise_conv1d_ops, fftconv_ops  # noqa: E402
from . import conv1d_dispatch  # noqa: E402
from ._dispatch import *  # noqa: E402,F401,F403
from ._dispatch import enable, disable, is_enabled  # noqa: E402

__version__ = "0.1.0"


def native_available() -> bool:
    """True when libb200conv.so is loaded."""
    return _lib.available()


if os.environ.get("AMD_TUNED_TORCH_AUTOPATCH", "1") != "0":
    enable()
