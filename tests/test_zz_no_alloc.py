"""The allocation-free GroupNorm entry point (b200_gn_fwd_static_scratch).

It exists for callers that cannot allocate device memory -- applications
whose device memory all belongs to their own pool or arena, or loops where an
allocation is not acceptable -- and keeps its scratch in a fixed array inside
the library.  Checked here through the C ABI against the existing
b200_gn_fwd (which takes a caller workspace), on two calls in a row so that
the second call proves the shared scratch carries nothing over from the
first.  Kept in a file of its own that pytest collects last; it passes both
alone in a fresh process and after the rest of the suite.
"""
from __future__ import annotations

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

CODES = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}
TOL = {torch.float32: 1e-5, torch.float16: 2e-3, torch.bfloat16: 2e-3}


def _rel_l2(a, b):
    a, b = a.double().flatten(), b.double().flatten()
    return float((a - b).norm() / b.norm().clamp_min(1e-300))


def _existing(lib, x, G, w, b, eps, stream):
    """b200_gn_fwd, split variant, with a caller-allocated workspace."""
    N, C = x.shape[0], x.shape[1]
    S = x.numel() // (N * C)
    y = torch.empty_like(x)
    wsb = lib.b200_gn_workspace_bytes(N, C, S, G, CODES[x.dtype], 1)
    ws = torch.empty(max(wsb, 1), dtype=torch.uint8, device=x.device)
    rc = lib.b200_gn_fwd(x.data_ptr(), w.data_ptr(), b.data_ptr(), y.data_ptr(), CODES[x.dtype],
                         CODES[w.dtype], N, C, S, G, eps, 1, ws.data_ptr(), wsb, stream)
    assert rc == 0, lib.b200_last_error()
    return y


def _no_alloc(lib, x, G, w, b, eps, stream):
    N, C = x.shape[0], x.shape[1]
    S = x.numel() // (N * C)
    y = torch.empty_like(x)
    rc = lib.b200_gn_fwd_static_scratch(x.data_ptr(), w.data_ptr(), b.data_ptr(), y.data_ptr(),
                                        CODES[x.dtype], CODES[w.dtype], N, C, S, G, eps, stream)
    assert rc == 0, lib.b200_last_error()
    return y


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_static_scratch_matches_existing_entry_point_twice(dtype):
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from amd_tuned_torch import _lib
    lib = _lib.lib()
    dev = torch.device("cuda", 0)
    stream = torch.cuda.current_stream(dev).cuda_stream
    shapes = [((4, 512, 128, 128), 32, 1e-6), ((3, 96, 17, 19), 6, 1e-5)]
    for i, (shape, G, eps) in enumerate(shapes):   # two calls in a row, different data
        g = torch.Generator().manual_seed(100 + i)
        x = ((torch.randn(*shape, generator=g) * 2) + i).to(dev, dtype)
        w = (torch.rand(shape[1], generator=g) + 0.5).to(dev, dtype)
        b = (torch.randn(shape[1], generator=g) * 0.1).to(dev, dtype)
        want = _existing(lib, x, G, w, b, eps, stream)
        got = _no_alloc(lib, x, G, w, b, eps, stream)
        torch.cuda.synchronize()
        assert _rel_l2(got.float(), want.float()) <= TOL[dtype]
        ref = torch.nn.functional.group_norm(x.float().cpu(), G, w.float().cpu(),
                                             b.float().cpu(), eps)
        assert _rel_l2(got.float().cpu(), ref) <= TOL[dtype]


def _limit_case(groups: int, dev):
    """[groups, 1, 65537] fp16: one channel per group, C/G * S = 65537, so
    every group spans two 65536-element chunks and the scratch need is
    ceil4(3 * groups) + 3 * groups * 2 floats (65530 at 7281 groups, 65540
    at 7282)."""
    g = torch.Generator(device=dev).manual_seed(groups)
    x = torch.randn(groups, 1, 65537, generator=g, device=dev, dtype=torch.float16)
    w = torch.full((1,), 1.25, device=dev, dtype=torch.float16)
    b = torch.full((1,), -0.5, device=dev, dtype=torch.float16)
    return x, w, b


def test_static_scratch_at_its_limit():
    """The largest accepted problem: the partial statistics reach the end of
    the array; matches b200_gn_fwd and torch's own CUDA GroupNorm, twice."""
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from amd_tuned_torch import _lib
    lib = _lib.lib()
    dev = torch.device("cuda", 0)
    stream = torch.cuda.current_stream(dev).cuda_stream
    x, w, b = _limit_case(7281, dev)
    want = _existing(lib, x, 1, w, b, 1e-5, stream)
    for _ in range(2):
        got = _no_alloc(lib, x, 1, w, b, 1e-5, stream)
        torch.cuda.synchronize()
        assert _rel_l2(got.float(), want.float()) <= TOL[torch.float16]
        ref = torch.nn.functional.group_norm(x.float(), 1, w.float(), b.float(), 1e-5)
        assert _rel_l2(got.float(), ref) <= TOL[torch.float16]
    del x, got, want, ref
    x, w, b = _limit_case(7282, dev)
    y = torch.empty_like(x)
    rc = lib.b200_gn_fwd_static_scratch(x.data_ptr(), w.data_ptr(), b.data_ptr(), y.data_ptr(),
                                        1, 1, 7282, 1, 65537, 1, 1e-5, stream)
    assert rc == -1
    assert b"static array holds" in lib.b200_last_error()


def test_static_scratch_rejects_oversized_problems():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from amd_tuned_torch import _lib
    lib = _lib.lib()
    x = torch.empty(1, device="cuda")
    # N * G = 32768 groups -> 3 * 32768 * 2 floats > 65536: rejected before any launch.
    rc = lib.b200_gn_fwd_static_scratch(x.data_ptr(), None, None, x.data_ptr(), 0, 0, 1024, 32,
                                        1, 32, 1e-5, ctypes.c_void_p(0))
    assert rc == -1
    assert b"static array holds" in lib.b200_last_error()
