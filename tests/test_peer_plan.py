"""Host-side planning (no GPU): the peer-memory exchange's halo sides and
window layout, and the FFT conv1d transform plan (whole row or overlap-save
segments)."""
from __future__ import annotations

import pytest

from amd_tuned_torch import _lib
from amd_tuned_torch.peer import HaloSide, halo_plan
from amd_tuned_torch.video_stack import t_partition


@pytest.mark.parametrize("T,world", [(64, 8), (17, 4), (5, 3), (2, 2)])
def test_halo_plan_targets_neighbour_halo_frames(T, world):
    fb = 1000 * 16
    sizes = t_partition(T, world)
    for r in range(world):
        lo, hi = halo_plan(r, sizes, fb)
        assert (lo is None) == (r == 0) and (hi is None) == (r == world - 1)
        if lo is not None:
            # my first interior frame -> previous rank's top halo frame T_prev + 1
            assert lo == HaloSide(r - 1, fb, (sizes[r] + 2) * fb, (sizes[r - 1] + 1) * fb,
                                  (sizes[r - 1] + 2) * fb)
        if hi is not None:
            # my last interior frame -> next rank's bottom halo frame 0
            assert hi == HaloSide(r + 1, sizes[r] * fb, (sizes[r] + 2) * fb, 0,
                                  (sizes[r + 1] + 2) * fb)


def test_halo_plan_is_a_permutation_of_neighbour_frames():
    """Every halo frame of every rank is written by exactly one push, and it
    is the neighbour's adjacent interior frame (global frame index check)."""
    sizes = t_partition(23, 5)
    start = [sum(sizes[:r]) for r in range(5)]
    written = {}
    for r in range(5):
        for side in halo_plan(r, sizes, 1):
            if side is None:
                continue
            src_global = start[r] + side.src_off - 1        # interior frame t -> global start+t-1
            dst_local = side.dst_off                        # frame index in the receiver's xp
            key = (side.peer, dst_local)
            assert key not in written
            written[key] = src_global
    for q in range(5):
        if q > 0:
            assert written[(q, 0)] == start[q] - 1           # frame just below q's slice
        if q < 4:
            assert written[(q, sizes[q] + 1)] == start[q] + sizes[q]   # frame just above


def test_window_layout():
    L = _lib.lib()
    off = L.b200_peer_window_xp_offset(8, 32)
    assert off > 0 and off % 65536 == 0
    assert off >= 2048 + 2 * 8 * 32 * 3 * 4
    assert L.b200_peer_window_bytes(8, 32, 100) == off + 65536
    assert L.b200_peer_window_xp_offset(65, 32) == -1
    assert L.b200_peer_window_xp_offset(2, 0) == -1


def test_fftconv1d_plan_choice():
    from amd_tuned_torch import fftconv_ops
    assert fftconv_ops.fftconv1d_plan(16384, 2048, 1024) == (8192, True)    # cfg 4b
    assert fftconv_ops.fftconv1d_plan(4000, 64, 0) == (4000, False)
    assert fftconv_ops.fftconv1d_plan(60000, 257, 128)[1] is True           # too long for one
    nfft, seg = fftconv_ops.fftconv1d_plan(1000, 257, 128)
    assert not seg and nfft >= 1000 + 2 * 128


def test_fftconv1d_length_contest_plans():
    """The transform plans contested per shape: distinct, valid for the row
    (whole-row lengths cover the padded signal, segments are >= 2K), the
    default rule's plan last as the verification reference."""
    from amd_tuned_torch import fftconv_ops
    plans = fftconv_ops.fftconv1d_plans(16384, 2048, 1024)                 # cfg 4b
    names = [n for n, _ in plans]
    assert names[-1] == "original" and plans[-1][1] == (8192, True)
    assert len({p for _, p in plans}) == len(plans)
    assert dict(plans)["5smooth"] == (18432, False)
    assert ("segments16384", (16384, True)) in plans and "pow2" not in names  # 32768 too long
    for L, K, pad in [(16384, 2048, 1024), (4000, 64, 0), (1000, 257, 128), (60000, 257, 128),
                      (5000, 999, 499)]:
        for name, (nfft, seg) in fftconv_ops.fftconv1d_plans(L, K, pad):
            if seg:
                assert nfft >= K
            else:
                assert nfft >= L + 2 * pad and nfft <= 24576
    # nothing else to try: a row whose only plan is the default one
    assert [n for n, _ in fftconv_ops.fftconv1d_plans(100, 3, 1)][-1] == "original"


def test_fftconv_length_contest_skips(monkeypatch):
    """The contest hands straight to the default plan when off, when a
    gradient is live, below the minimum length, or with one plan."""
    from amd_tuned_torch import fftconv_ops, kernel_select
    ran = []
    plans = [("pow2", (2,)), ("original", (1,))]
    key = ("conv1d", "probe")

    def run(p):
        ran.append(p)
        return p
    monkeypatch.setattr(kernel_select, "_ENABLED", True)
    assert fftconv_ops._length_contest(key, plans, run, None, True, 10 ** 6) == (1,)
    assert fftconv_ops._length_contest(key, plans, run, None, False, 10) == (1,)
    assert fftconv_ops._length_contest(key, plans[-1:], run, None, False, 10 ** 6) == (1,)
    monkeypatch.setattr(kernel_select, "_ENABLED", False)
    assert fftconv_ops._length_contest(key, plans, run, None, False, 10 ** 6) == (1,)
    assert ran == [(1,)] * 4
