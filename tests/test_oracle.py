"""The oracle is pinned to the reference: every layer of it reproduces the
golden vectors that the reference package itself produced
(tests/golden/make_golden.py).  CPU only."""
from __future__ import annotations

import numpy as np
import pytest

import oracle
from conftest import load_golden

# fp32 restatements agree with the reference far inside the BASELINE fp32 bar
# (rel-L2 <= 1e-5); the golden outputs were computed in fp32 from the stored
# (already cast) inputs, so low-precision cases share the bar.
ORACLE_RTOL = 2e-6


def _bias(d):
    return d["b"] if d["b"].size else None


@pytest.mark.parametrize("case", list(load_golden("dwconv1d")))
def test_c_dwconv1d_matches_reference(case):
    d = load_golden("dwconv1d")[case]
    B, C, L, K, pad, has_b = (int(v) for v in d["meta"])
    y = oracle.c_dwconv1d(d["x"], d["w"], _bias(d), pad)
    assert y.shape == d["y"].shape
    assert oracle.rel_l2(y, d["y"]) < ORACLE_RTOL


@pytest.mark.parametrize("case", list(load_golden("dwconv1d")))
def test_stock_dwconv1d_matches_reference(case):
    d = load_golden("dwconv1d")[case]
    B, C, L, K, pad, has_b = (int(v) for v in d["meta"])
    y = oracle.stock_conv1d(d["x"], d["w"], _bias(d), pad, C)
    np.testing.assert_array_equal(y, d["y"])


@pytest.mark.parametrize("case", list(load_golden("group_norm")))
def test_c_group_norm_matches_reference(case):
    d = load_golden("group_norm")[case]
    G, affine = (int(v) for v in d["meta"])
    w = d["w"] if affine else None
    b = d["b"] if affine else None
    y = oracle.c_group_norm(d["x"], G, w, b, float(d["eps"]))
    assert oracle.rel_l2(y, d["y"]) < ORACLE_RTOL


@pytest.mark.parametrize("case", list(load_golden("conv3d")))
def test_c_conv3d_matches_reference(case):
    d = load_golden("conv3d")[case]
    m = [int(v) for v in d["meta"]]
    k, p, dil = m[6:9], m[9:12], m[12:15]
    y = oracle.c_conv3d(d["x"], d["w"], d["b"], (1, 1, 1), p, dil)
    assert y.shape == d["y"].shape
    assert oracle.rel_l2(y, d["y"]) < ORACLE_RTOL


@pytest.mark.parametrize("case", list(load_golden("fftconv1d")))
def test_numpy_fft_route_matches_reference_fft(case):
    d = load_golden("fftconv1d")[case]
    B, C, L, K, pad = (int(v) for v in d["meta"])
    y = oracle.fft_conv_np(d["x"], d["w"], d["b"], (pad,), groups=C)
    # The reference's FFT route rounds to the case dtype at the end.
    tol = 1e-6 if d["dtype"] == "f32" else 2e-3
    assert oracle.rel_l2(y, d["y_fft"]) < tol
    # ...and the FFT route agrees with direct convolution.
    assert oracle.rel_l2(y, d["y"]) < 1e-5


@pytest.mark.parametrize("case", list(load_golden("fftconv3d")))
def test_numpy_fft3d_route_matches_reference_fft(case):
    d = load_golden("fftconv3d")[case]
    m = [int(v) for v in d["meta"]]
    p = m[9:12]
    y = oracle.fft_conv_np(d["x"], d["w"], d["b"], p)
    tol = 1e-6 if d["dtype"] == "f32" else 2e-3
    assert oracle.rel_l2(y, d["y_fft"]) < tol
    assert oracle.rel_l2(y, d["y"]) < 1e-5


def test_fft_route_is_length_invariant():
    """Zero-padding the transform further never changes the result -- the
    property behind the reference's transform-length contest
    (fftconv_ops.py:381-460) and this build's 2/3/5-smooth lengths."""
    rng = np.random.default_rng(0)
    x = rng.standard_normal((1, 3, 50))
    w = rng.standard_normal((3, 1, 9))
    a = oracle.fft_conv_np(x, w, None, (4,), groups=3)
    b = oracle.fft_conv_np(x, w, None, (4,), groups=3, fft_sizes=(90,))
    np.testing.assert_allclose(a, b, rtol=1e-10, atol=1e-10)


def test_rel_l2_is_scale_free():
    a = np.array([1.0, 2.0, 3.0])
    assert oracle.rel_l2(a, a) == 0.0
    assert abs(oracle.rel_l2(a * 1.01, a) - 0.01) < 1e-12


@pytest.mark.parametrize("affine", [True, False])
def test_group_norm_backward_restatement_matches_autograd(affine):
    rng = np.random.default_rng(0)
    x = rng.normal(size=(2, 8, 5, 3)) * 2 + 1
    dy = rng.normal(size=x.shape)
    gamma = rng.uniform(0.5, 1.5, size=8) if affine else None
    beta = rng.normal(size=8) if affine else None
    dx, dg, db = oracle.np_group_norm_backward(x, dy, 4, gamma, 1e-5)
    sx, sg, sb = oracle.stock_group_norm_backward(x, dy, 4, gamma, beta, 1e-5)
    assert oracle.rel_l2(dx, sx) < 1e-5
    if affine:
        assert oracle.rel_l2(dg, sg) < 1e-5 and oracle.rel_l2(db, sb) < 1e-5


@pytest.mark.parametrize("K,pad,L", [(3, 1, 40), (4, 1, 33), (5, 0, 20), (7, 6, 9), (2, 3, 11)])
def test_dwconv1d_backward_restatement_matches_autograd(K, pad, L):
    rng = np.random.default_rng(K * 100 + pad)
    B, C = 3, 5
    x = rng.normal(size=(B, C, L))
    w = rng.normal(size=(C, K))
    b = rng.normal(size=C)
    dy = rng.normal(size=(B, C, L + 2 * pad - K + 1))
    dx, dw, db = oracle.np_dwconv1d_backward(x, dy, w, pad)
    sx, sw, sb = oracle.stock_dwconv1d_backward(x, dy, w, b, pad)
    assert oracle.rel_l2(dx, sx) < 1e-5
    assert oracle.rel_l2(dw, sw.reshape(C, K)) < 1e-5
    assert oracle.rel_l2(db, sb) < 1e-5
