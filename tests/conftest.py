"""Shared test setup.

* Puts the repository root (for `oracle`) and rocm-kernel-select_b200/ (for
  the `amd_tuned_torch` package) on sys.path.
* Like the reference suite (tests/conftest.py:58-95 there), importing the
  package must not patch torch as a side effect of collection:
  AMD_TUNED_TORCH_AUTOPATCH=0; tests opt in with enable().  The kernel_select
  disk cache goes to a temporary directory.
* Registers the `gpu` marker: tests that need a B200.  Everything else runs
  on CPU.
"""
from __future__ import annotations

import os
import sys
import tempfile
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
PKG = ROOT / "rocm-kernel-select_b200"
for p in (str(ROOT), str(PKG)):
    if p not in sys.path:
        sys.path.insert(0, p)

os.environ.setdefault("AMD_TUNED_TORCH_AUTOPATCH", "0")
os.environ.setdefault("AMD_TUNED_TORCH_KERNEL_SELECT_CACHE_DIR",
                      tempfile.mkdtemp(prefix="ks_cache_"))

GOLDEN = Path(__file__).resolve().parent / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (B200) device")


def load_golden(name: str) -> dict:
    """{case: {field: array}} from tests/golden/<name>.npz."""
    raw = np.load(GOLDEN / f"{name}.npz", allow_pickle=False)
    cases: dict = {}
    for key in raw.files:
        case, field = key.split("__", 1)
        val = raw[key]
        cases.setdefault(case, {})[field] = str(val) if val.dtype.kind == "U" else val
    return dict(sorted(cases.items()))


def torch_dtype(name: str):
    import torch
    return {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}[name]


@pytest.fixture
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    return torch.device("cuda", 0)
