"""Loader for libb200conv.so, the sm_100a kernels behind this package.

Plays the role of the reference's amd_tuned_torch/_native_loader.py:56-147
(which dlopens per-torch-build pybind11 modules); here there is exactly one
shared library with a plain C ABI (include/b200conv.h), loaded with ctypes.

Failure policy: on a machine with a CUDA device the library is REQUIRED --
`import amd_tuned_torch` raises ImportError if it cannot be loaded, so no call
can silently run on some other implementation.  On a CPU-only machine the
import succeeds (the dispatch logic is still importable and testable) and
`available()` reports False; every patched op then leaves CPU tensors to stock
torch exactly as the reference does (its tiers all require CUDA tensors,
amd_tuned_torch/_dispatch.py:651-659).
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path
from typing import Optional

_LIB_NAME = "libb200conv.so"
_LIB_PATH = Path(os.environ.get("AMD_TUNED_TORCH_LIB", Path(__file__).with_name(_LIB_NAME)))

c_int, c_int64, c_float, c_size_t, c_vp = (ctypes.c_int, ctypes.c_int64, ctypes.c_float,
                                           ctypes.c_size_t, ctypes.c_void_p)
c_i64p = ctypes.POINTER(ctypes.c_int64)
c_intp = ctypes.POINTER(ctypes.c_int)

class Conv3dProblem(ctypes.Structure):
    """Mirror of B200Conv3dProblem (include/b200conv.h)."""
    _fields_ = ([(n, ctypes.c_int64) for n in ("N", "Cin", "D", "H", "W", "Cout", "KD", "KH",
                                                 "KW")]
                + [("params9", ctypes.c_int64 * 9)]
                + [(n, ctypes.c_int32) for n in ("dtype", "bias_dtype", "x_channels_last",
                                                 "y_channels_last", "variant", "reserved")]
                + [("workspace_bytes", ctypes.c_uint64)])


# name -> (restype, argtypes).  Mirrors include/b200conv.h one to one; the CPU
# test suite checks that every function declared there is exported and listed.
SIGNATURES = {
    "b200_version": (c_int, []),
    "b200_last_error": (ctypes.c_char_p, []),
    "b200_read_device_flags": (c_int, [c_vp, c_intp]),
    "b200_sm_count": (c_int, []),
    "b200_gn_workspace_bytes": (c_size_t, [c_int64, c_int64, c_int64, c_int64, c_int, c_int]),
    "b200_gn_fwd": (c_int, [c_vp, c_vp, c_vp, c_vp, c_int, c_int, c_int64, c_int64, c_int64,
                            c_int64, c_float, c_int, c_vp, c_size_t, c_vp]),
    "b200_gn_fwd_static_scratch": (c_int, [c_vp, c_vp, c_vp, c_vp, c_int, c_int, c_int64,
                                           c_int64, c_int64, c_int64, c_float, c_vp]),
    "b200_gn_merge_ranks": (c_int, [c_vp, c_vp, c_int64, c_int64, c_vp]),
    "b200_gn_stats_workspace_bytes":(c_size_t, [c_int64, c_int64, c_int64, c_int64, c_int]),
    "b200_gn_partial_stats": (c_int, [c_vp, c_vp, c_int, c_int64, c_int64, c_int64, c_int64,
                                      c_vp, c_size_t, c_vp]),
    "b200_gn_apply": (c_int, [c_vp, c_vp, c_vp, c_vp, c_vp, c_int, c_int, c_int64, c_int64,
                              c_int64, c_int64, c_float, c_int, c_int, c_vp]),
    "b200_dwconv1d_fwd": (c_int, [c_vp, c_vp, c_vp, c_vp, c_int, c_int, c_int64, c_int64,
                                  c_int64, c_int64, c_int64, c_int64, c_int, c_vp]),
    "b200_dwconv1d_bwd_workspace_bytes": (c_size_t, [c_int64] * 4),
    "b200_dwconv1d_bwd_weight": (c_int, [c_vp, c_vp, c_vp, c_vp, c_int, c_int] + [c_int64] * 6
                                 + [c_vp, c_size_t, c_vp]),
    "b200_gn_bwd_workspace_bytes": (c_size_t, [c_int64] * 4),
    "b200_gn_bwd": (c_int, [c_vp] * 7 + [c_int, c_int] + [c_int64] * 4
                    + [c_float, c_vp, c_size_t, c_vp]),
    "b200_conv3d_packed_weight_bytes": (c_size_t, [c_int64] * 5),
    "b200_conv3d_pack_weight": (c_int, [c_vp, c_vp, c_int, c_int64, c_int64, c_int64, c_int64,
                                        c_int64, c_vp]),
    "b200_conv3d_workspace_bytes": (c_size_t, [c_int64] * 5 + [c_int]),
    "b200_conv3d_fwd_workspace_bytes": (c_size_t, [c_int64] * 8 + [c_i64p, c_int, c_int]),
    "b200_conv3d_uses_slab": (c_int, [c_int64] * 9 + [c_i64p, c_int, c_int]),
    "b200_conv3d_packed_weight_bytes_for": (c_size_t, [c_int64] * 5 + [c_int]),
    "b200_conv3d_fwd": (c_int, [c_vp, c_vp, c_vp, c_vp, c_int, c_int] + [c_int64] * 9
                        + [c_i64p, c_int, c_int, c_int, c_vp, c_size_t, c_vp]),
    "b200_conv3d_fwd_call": (c_int, [c_vp] * 7),
    "b200_conv3d_fwd_gated": (c_int, [c_vp, c_vp, c_vp, c_vp, c_int, c_int] + [c_int64] * 9
                              + [c_i64p, c_int, c_int, c_int, c_vp, c_size_t, c_vp, c_vp, c_vp,
                                 c_int64, c_vp]),
    "b200_to_channels_last": (c_int, [c_vp, c_vp, c_int, c_int64, c_int64, c_int64, c_vp]),
    "b200_fft_supported_length": (c_int, [c_int64]),
    "b200_fftconv1d_spectrum_bytes": (c_size_t, [c_int64, c_int64]),
    "b200_fftconv1d_prepare": (c_int, [c_vp, c_vp, c_int, c_int64, c_int64, c_int64, c_vp]),
    "b200_fftconv1d_fwd": (c_int, [c_vp, c_vp, c_vp, c_vp, c_int, c_int] + [c_int64] * 6
                           + [c_vp]),
    "b200_fftconv1d_fwd_os": (c_int, [c_vp, c_vp, c_vp, c_vp, c_int, c_int] + [c_int64] * 7
                              + [c_vp]),
    "b200_fftconv3d_spectrum_bytes": (c_size_t, [c_int64] * 5 + [c_int]),
    "b200_fftconv3d_prepare": (c_int, [c_vp, c_vp, c_int] + [c_int64] * 8
                               + [c_vp, c_size_t, c_vp]),
    "b200_fftconv3d_workspace_bytes": (c_size_t, [c_int64] * 6),
    "b200_fftconv3d_fwd": (c_int, [c_vp, c_vp, c_vp, c_vp, c_int, c_int] + [c_int64] * 9
                           + [c_i64p, c_int64, c_int64, c_int64, c_vp, c_size_t, c_vp]),
    "b200_peer_window_xp_offset": (c_int64, [c_int64, c_int64]),
    "b200_peer_window_bytes": (c_int64, [c_int64, c_int64, c_int64]),
    "b200_peer_window_alloc": (c_int, [c_int64, ctypes.POINTER(c_vp), c_vp]),
    "b200_peer_window_open": (c_int, [c_vp, ctypes.POINTER(c_vp)]),
    "b200_peer_window_close": (c_int, [c_vp]),
    "b200_peer_window_free": (c_int, [c_vp]),
    "b200_peer_stats_publish": (c_int, [c_vp, c_vp, c_int64, c_int64, c_int64, c_vp, c_vp]),
    "b200_peer_stats_merge": (c_int, [c_vp, c_vp, c_int64, c_int64, c_vp]),
    "b200_peer_halo_push": (c_int, [c_vp, c_vp, c_vp, c_vp, c_int64, c_int64, c_vp, c_vp, c_vp,
                                    c_int64, c_int64, c_int64, c_int64, c_vp]),
    "b200_peer_halo_wait": (c_int, [c_vp, c_int, c_int, c_vp]),
}

_lib: Optional[ctypes.CDLL] = None
_load_error: Optional[str] = None


def _load() -> None:
    global _lib, _load_error
    try:
        lib = ctypes.CDLL(str(_LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    except (OSError, AttributeError) as exc:
        _lib = None
        _load_error = f"{_LIB_PATH}: {exc}"


def available() -> bool:
    return _lib is not None


def load_error() -> Optional[str]:
    return _load_error


def lib() -> ctypes.CDLL:
    """The loaded library; raises RuntimeError (never a silent fallback)."""
    if _lib is None:
        raise RuntimeError(f"libb200conv.so is not loaded ({_load_error}); "
                           "build it with `python rocm-kernel-select_b200/csrc/build.py`")
    return _lib


def path() -> Path:
    return _LIB_PATH


class NativeError(RuntimeError):
    """A CUDA or argument error reported by the C ABI (status < 0)."""


def check(status: int, what: str) -> bool:
    """True if launched, False if the kernel declined (status > 0), raises on error."""
    if status == 0:
        return True
    msg = lib().b200_last_error()
    text = msg.decode(errors="replace") if msg else ""
    if status > 0:
        return False
    raise NativeError(f"{what}: status {status}: {text}")


_load()
