"""The drop-in boundary: libb200conv.so loads without a GPU and exports every
function include/b200conv.h declares, with a ctypes signature for each.
No kernel is launched here (CPU only)."""
from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

from amd_tuned_torch import _lib

HEADER = Path(__file__).resolve().parents[1] / "include" / "b200conv.h"


def declared_functions() -> list[str]:
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(b200_[a-z0-9_]+)\s*\(", text)))


def test_library_loads():
    assert _lib.available(), _lib.load_error()
    assert _lib.lib().b200_version() >= 10000


def test_header_declares_the_expected_entry_points():
    names = declared_functions()
    for must in ("b200_gn_fwd", "b200_dwconv1d_fwd", "b200_conv3d_fwd", "b200_conv3d_pack_weight",
                 "b200_fftconv1d_fwd", "b200_fftconv3d_fwd", "b200_version"):
        assert must in names


@pytest.mark.parametrize("name", declared_functions())
def test_every_declared_symbol_is_exported_and_typed(name):
    lib = _lib.lib()
    assert hasattr(lib, name), f"{name} declared in b200conv.h but not exported"
    assert name in _lib.SIGNATURES, f"{name} has no ctypes signature in _lib.SIGNATURES"


def test_no_extra_signatures():
    assert set(_lib.SIGNATURES) <= set(declared_functions())


def test_size_queries_need_no_gpu():
    lib = _lib.lib()
    assert lib.b200_conv3d_packed_weight_bytes(64, 64, 3, 3, 3) == 27 * 64 * 64 * 2
    assert lib.b200_conv3d_packed_weight_bytes(8, 8, 3, 3, 3) == 27 * 8 * 64 * 2
    assert lib.b200_conv3d_workspace_bytes(1, 64, 16, 32, 32, 0) == 64 * 16 * 32 * 32 * 2
    assert lib.b200_conv3d_workspace_bytes(1, 64, 16, 32, 32, 1) == 0
    assert lib.b200_gn_workspace_bytes(4, 512, 128 * 128, 32, 2, 0) > 0


def test_argument_errors_are_reported_without_a_gpu():
    lib = _lib.lib()
    rc = lib.b200_gn_fwd(None, None, None, None, 0, 0, 1, 4, 4, 2, 1e-5, 0, None, 0, None)
    assert rc == -1
    assert b"NULL" in lib.b200_last_error()
    rc = lib.b200_dwconv1d_fwd(1, 1, None, 1, 0, 0, 1, 1, 8, 3, 1, 99, 0, None)
    assert rc == -1
    with pytest.raises(_lib.NativeError):
        _lib.check(-1, "b200_dwconv1d_fwd")
    assert _lib.check(1, "declined") is False


def test_conv3d_problem_struct_layout():
    """The ctypes mirror of B200Conv3dProblem has the C layout: 18 int64,
    6 int32, one uint64 -- 176 bytes, workspace_bytes at offset 168."""
    from amd_tuned_torch import _lib
    P = _lib.Conv3dProblem
    assert ctypes.sizeof(P) == 176
    assert P.params9.offset == 72 and P.dtype.offset == 144 and P.workspace_bytes.offset == 168
