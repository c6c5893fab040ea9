"""Generates tests/golden/*.npz from the REFERENCE implementation itself.

Run once, in a container where the reference checkout exists:

    python tests/golden/make_golden.py /path/to/rocm-kernel-select

It imports the reference package `amd_tuned_torch` from that checkout the way
the reference's own test suite does (tests/conftest.py:58-95 there: autopatch
off, contest off, its compiled ROCm extensions replaced by stub modules -- the
shipped binaries are never loaded), calls `enable()`, and then calls the
patched F.conv1d / F.conv3d / F.group_norm on seeded CPU tensors.  On CPU the
reference routes every one of these to stock torch (its tiers require CUDA
tensors, _dispatch.py:651-659, miopen_fallback.py:280/325), so the outputs
recorded are exactly the reference's behaviour for those inputs.  For the FFT
route it records the reference's own `fftconv_ops.fft_conv1d` / `fft_conv3d`
(pure torch, fftconv_ops.py:603-781).

Inputs are generated in fp32 with torch.Generator seeds, cast to the case's
dtype and stored after the cast (so fp16/bf16 cases hold exactly the values
the kernels see); outputs are computed in fp32 from those values, the
convention of the BASELINE configs.  Nothing here is needed at test time
except the .npz files it writes.
"""
from __future__ import annotations

import math
import os
import sys
import tempfile
import types
from pathlib import Path
from unittest.mock import MagicMock

import numpy as np

OUT = Path(__file__).resolve().parent


def _import_reference(ref_root: str):
    tmp = tempfile.mkdtemp(prefix="golden_")
    os.environ["AMD_TUNED_TORCH_AUTOPATCH"] = "0"
    os.environ["AMD_TUNED_TORCH_MEASURE_KERNELS"] = "0"
    os.environ["AMD_TUNED_TORCH_KERNEL_SELECT_CACHE_DIR"] = tmp
    os.environ["AMD_TUNED_TORCH_FFTCONV_CALIBRATION_DIR"] = tmp
    os.environ["AMD_TUNED_TORCH_KERNEL_SELECT_CACHE"] = "0"
    sys.path.insert(0, ref_root)
    native = types.ModuleType("amd_tuned_torch._native")
    for name in ("group_norm", "conv2d", "conv3d", "conv3d_fp16_winograd_bt8_bc8",
                 "iu4_gemm_supported", "iu4_gemm", "iu8_gemm", "dot4_i8_gemm",
                 "fast_block_diag_forward", "fast_block_diag_backward"):
        setattr(native, name, MagicMock(name=name))
    sys.modules["amd_tuned_torch._native"] = native
    for mod, fn in (("_native_ck", "has_ck"), ("_native_hipblaslt", "has_hipblaslt"),
                    ("_native_rocsparse", "has_rocsparse")):
        m = types.ModuleType(f"amd_tuned_torch.{mod}")
        setattr(m, fn, MagicMock(name=fn, return_value=False))
        sys.modules[f"amd_tuned_torch.{mod}"] = m
    import amd_tuned_torch  # noqa: PLC0415 -- the reference package
    from amd_tuned_torch import fftconv_ops  # noqa: PLC0415
    amd_tuned_torch.enable()
    return amd_tuned_torch, fftconv_ops


def _gen(shape, seed, kind="normal", std=1.0, lo=0.0, hi=1.0):
    import torch
    g = torch.Generator().manual_seed(seed)
    if kind == "normal":
        return torch.randn(*shape, generator=g) * std
    return torch.rand(*shape, generator=g) * (hi - lo) + lo


def _kaiming(shape, seed):
    import torch
    fan_in = math.prod(shape[1:])
    bound = 1.0 / math.sqrt(fan_in)  # kaiming_uniform_(a=sqrt(5)) on a conv weight
    g = torch.Generator().manual_seed(seed)
    return (torch.rand(*shape, generator=g) * 2 - 1) * bound


def _cast(t, dtype):
    return t.to(dtype).float()


def main(ref_root: str) -> None:
    import torch
    import torch.nn.functional as F
    _, fftconv_ops = _import_reference(ref_root)
    dts = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}

    # --------------------------------------------------- depthwise conv1d
    cases = {}
    dw = [  # (B, C, L, K, pad, dtype, bias)
        (2, 8, 64, 3, 1, "f32", True), (2, 8, 67, 5, 2, "f32", True),
        (1, 4, 33, 4, 1, "f32", False), (2, 8, 64, 3, 1, "f16", True),
        (2, 8, 64, 3, 1, "bf16", True), (1, 3, 7, 7, 3, "f32", True),
        (1, 2, 5, 7, 3, "f32", True), (3, 5, 130, 1, 0, "f32", True),
        (2, 6, 2100, 9, 4, "f32", True),
    ]
    for i, (B, C, L, K, pad, dt, has_b) in enumerate(dw):
        x = _cast(_gen((B, C, L), 100 + i), dts[dt])
        w = _cast(_kaiming((C, 1, K), 200 + i), dts[dt])
        b = _cast(_gen((C,), 300 + i, "uniform", lo=-0.5, hi=0.5), dts[dt]) if has_b else None
        y = F.conv1d(x, w, b, 1, pad, 1, C)   # the reference's patched F.conv1d (CPU -> stock)
        cases[f"dw{i}"] = dict(x=x.numpy(), w=w.numpy(), b=(b.numpy() if has_b else np.zeros(0)),
                               y=y.numpy(), meta=np.array([B, C, L, K, pad, has_b]), dtype=dt)
    np.savez_compressed(OUT / "dwconv1d.npz", **{f"{k}__{f}": v for k, d in cases.items()
                                                  for f, v in d.items()})

    # ------------------------------------------------ FFT conv1d (long k)
    cases = {}
    ff = [(2, 4, 256, 64, 32, "f32"), (1, 3, 300, 41, 20, "f32"), (2, 4, 256, 64, 32, "f16"),
          (1, 2, 1000, 128, 64, "f32")]
    for i, (B, C, L, K, pad, dt) in enumerate(ff):
        x = _cast(_gen((B, C, L), 400 + i), dts[dt])
        w = _cast(_kaiming((C, 1, K), 500 + i), dts[dt])
        b = _cast(_gen((C,), 600 + i, "uniform", lo=-0.5, hi=0.5), dts[dt])
        y_fft = fftconv_ops.fft_conv1d(x, w, bias=b, padding=pad, groups=C)  # reference FFT route
        y_dir = F.conv1d(x, w, b, 1, pad, 1, C)
        cases[f"ff{i}"] = dict(x=x.numpy(), w=w.numpy(), b=b.numpy(), y_fft=y_fft.numpy(),
                               y=y_dir.numpy(), meta=np.array([B, C, L, K, pad]), dtype=dt)
    np.savez_compressed(OUT / "fftconv1d.npz", **{f"{k}__{f}": v for k, d in cases.items()
                                                   for f, v in d.items()})

    # ------------------------------------------------------------ conv3d
    cases = {}
    c3 = [  # (N, Cin, D, H, W, Cout, k(d,h,w), pad(d,h,w), dil, dtype)
        (1, 8, 4, 6, 6, 8, (3, 3, 3), (1, 1, 1), (1, 1, 1), "f16"),
        (2, 16, 3, 5, 7, 8, (3, 3, 3), (1, 1, 1), (1, 1, 1), "bf16"),
        (1, 8, 3, 5, 9, 12, (1, 3, 3), (0, 1, 1), (1, 1, 1), "f16"),
        (1, 16, 5, 6, 6, 16, (3, 3, 3), (2, 2, 2), (2, 2, 2), "bf16"),
        (1, 64, 2, 8, 8, 64, (3, 3, 3), (1, 1, 1), (1, 1, 1), "f16"),
        (1, 8, 3, 4, 4, 4, (3, 3, 3), (0, 0, 0), (1, 1, 1), "f32"),
    ]
    for i, (N, Ci, D, H, W, Co, k, p, d, dt) in enumerate(c3):
        x = _cast(_gen((N, Ci, D, H, W), 700 + i), dts[dt])
        w = _cast(_kaiming((Co, Ci) + k, 800 + i), dts[dt])
        b = _cast(_gen((Co,), 900 + i, "uniform", lo=-0.2, hi=0.2), dts[dt])
        y = F.conv3d(x, w, b, 1, p, d, 1)   # the reference's patched F.conv3d (CPU -> stock)
        cases[f"c3_{i}"] = dict(x=x.numpy(), w=w.numpy(), b=b.numpy(), y=y.numpy(),
                                meta=np.array([N, Ci, D, H, W, Co, *k, *p, *d]), dtype=dt)
    np.savez_compressed(OUT / "conv3d.npz", **{f"{k}__{f}": v for k, d in cases.items()
                                                for f, v in d.items()})

    # -------------------------------------------------------- FFT conv3d
    cases = {}
    f3 = [(1, 4, 6, 8, 8, 4, (5, 5, 5), (2, 2, 2), "f32"),
          (2, 3, 5, 6, 7, 2, (3, 5, 4), (1, 2, 0), "f32"),
          (1, 4, 6, 8, 8, 4, (5, 5, 5), (2, 2, 2), "f16")]
    for i, (N, Ci, D, H, W, Co, k, p, dt) in enumerate(f3):
        x = _cast(_gen((N, Ci, D, H, W), 1000 + i), dts[dt])
        w = _cast(_kaiming((Co, Ci) + k, 1100 + i), dts[dt])
        b = _cast(_gen((Co,), 1200 + i, "uniform", lo=-0.2, hi=0.2), dts[dt])
        y_fft = fftconv_ops.fft_conv3d(x, w, bias=b, padding=p)   # reference FFT route
        y_dir = F.conv3d(x, w, b, 1, p, 1, 1)
        cases[f"f3_{i}"] = dict(x=x.numpy(), w=w.numpy(), b=b.numpy(), y_fft=y_fft.numpy(),
                                y=y_dir.numpy(), meta=np.array([N, Ci, D, H, W, Co, *k, *p]),
                                dtype=dt)
    np.savez_compressed(OUT / "fftconv3d.npz", **{f"{k}__{f}": v for k, d in cases.items()
                                                   for f, v in d.items()})

    # -------------------------------------------------------- group_norm
    cases = {}
    gn = [  # (shape, G, eps, affine, dtype, std)
        ((2, 8, 4, 4), 4, 1e-5, True, "f32", 1.0), ((1, 6, 5, 7), 3, 1e-5, False, "f32", 1.0),
        ((2, 32, 8, 8), 32, 1e-6, True, "bf16", 2.0), ((1, 8, 2, 4, 4), 4, 1e-5, True, "f16", 1.0),
        ((2, 16, 3, 3), 2, 1e-6, True, "f32", 2.0), ((1, 4, 1, 1), 2, 1e-5, True, "f32", 1.0),
        ((2, 64, 16, 16), 32, 1e-6, True, "f32", 2.0),
    ]
    for i, (shape, G, eps, affine, dt, std) in enumerate(gn):
        x = _cast(_gen(shape, 1300 + i, std=std) + 0.5, dts[dt])
        C = shape[1]
        wt = _cast(_gen((C,), 1400 + i, "uniform", lo=0.5, hi=1.5), dts[dt]) if affine else None
        bs = _cast(_gen((C,), 1500 + i, std=0.1), dts[dt]) if affine else None
        y = F.group_norm(x, G, wt, bs, eps)   # the reference's patched F.group_norm (CPU -> stock)
        cases[f"gn{i}"] = dict(x=x.numpy(), w=(wt.numpy() if affine else np.zeros(0)),
                               b=(bs.numpy() if affine else np.zeros(0)), y=y.numpy(),
                               meta=np.array([G, int(affine)]), eps=np.array(eps), dtype=dt)
    np.savez_compressed(OUT / "group_norm.npz", **{f"{k}__{f}": v for k, d in cases.items()
                                                    for f, v in d.items()})
    print("wrote", sorted(p.name for p in OUT.glob("*.npz")))


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py /path/to/rocm-kernel-select")
    main(sys.argv[1])
