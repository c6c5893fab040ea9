"""kernel_select policy, hardware-free: timing is stubbed with a name -> ms
table and candidates return sentinels, as in the reference's own
tests/test_kernel_select.py (:44-236 policy, :239-370 verification, :372-414
persistence, :416-590 out-of-memory handling).  CPU only."""
from __future__ import annotations

import json
import os

import pytest
import torch

from amd_tuned_torch import kernel_select


@pytest.fixture(autouse=True)
def _clean(monkeypatch, tmp_path):
    monkeypatch.setattr(kernel_select, "_ENABLED", True)
    monkeypatch.setattr(kernel_select, "_VERIFY_ENABLED", False)
    monkeypatch.setattr(kernel_select, "_REFERENCE_COMPETES", True)
    monkeypatch.setattr(kernel_select, "_CACHE_DIR", str(tmp_path))
    kernel_select.reset()
    yield
    kernel_select.reset()


@pytest.fixture
def timings(monkeypatch):
    calls: dict = {}

    def install(table):
        def fake_time(fn):
            calls[fn._name] = calls.get(fn._name, 0) + 1
            if fn() is None:
                return None
            return table.get(fn._name)
        monkeypatch.setattr(kernel_select, "_measure", fake_time)
        return calls
    return install


def cands(names, declines=(), outputs=None):
    out = []
    for n in names:
        def thunk(n=n):
            if n in declines:
                return None
            return outputs[n] if outputs else f"out:{n}"
        thunk._name = n
        out.append((n, thunk))
    return out


def args():
    return torch.zeros(1, 4, 8, 8, 8), torch.zeros(4, 4, 3, 3, 3), 1, 1, 1


def test_fastest_wins_not_first(timings):
    timings({"tcgen05": 5.0, "fftconv": 9.0, "stock": 1.0})
    x, w, s, p, d = args()
    assert kernel_select.pick("conv3d", x, w, s, p, d,
                              cands(["tcgen05", "fftconv", "stock"])) == "out:stock"
    assert kernel_select.cached("conv3d", x, w, s, p, d) == "stock"


def test_winner_is_cached_per_shape(timings):
    calls = timings({"a": 1.0, "stock": 2.0})
    x, w, s, p, d = args()
    for _ in range(3):
        assert kernel_select.pick("conv3d", x, w, s, p, d, cands(["a", "stock"])) == "out:a"
    assert calls == {"a": 1, "stock": 1}          # measured once
    x2 = torch.zeros(2, 4, 8, 8, 8)
    kernel_select.pick("conv3d", x2, w, s, p, d, cands(["a", "stock"]))
    assert calls["a"] == 2                         # a new shape is measured again


def test_declining_candidate_loses(timings):
    timings({"a": 0.1, "b": 3.0, "stock": 5.0})
    x, w, s, p, d = args()
    out = kernel_select.pick("conv3d", x, w, s, p, d, cands(["a", "b", "stock"], declines={"a"}))
    assert out == "out:b"


def test_kill_switch(monkeypatch, timings):
    monkeypatch.setattr(kernel_select, "_ENABLED", False)
    x, w, s, p, d = args()
    assert kernel_select.pick("conv3d", x, w, s, p, d, cands(["a", "stock"])) is None
    assert kernel_select.pick_key("group_norm", ("k",), cands(["a", "stock"])) is None
    assert kernel_select.cached("conv3d", x, w, s, p, d) is None


def test_pick_key(timings):
    timings({"native": 1.0, "stock": 2.0})
    key = (torch.bfloat16, (4, 512, 128, 128), 32, False)
    assert kernel_select.pick_key("group_norm", key, cands(["native", "stock"])) == "out:native"
    assert kernel_select.cached_key("group_norm", key) == "native"


def test_cached_winner_that_declines_is_evicted(timings):
    calls = timings({"a": 1.0, "stock": 2.0})
    x, w, s, p, d = args()
    kernel_select.pick("conv3d", x, w, s, p, d, cands(["a", "stock"]))
    out = kernel_select.pick("conv3d", x, w, s, p, d, cands(["a", "stock"], declines={"a"}))
    assert out == "out:stock"
    assert kernel_select.cached("conv3d", x, w, s, p, d) == "stock"
    assert calls["stock"] == 2


def test_reference_not_timed_by_default(monkeypatch, timings):
    """B200 build: own kernels compete, stock only verifies / serves as fallback."""
    monkeypatch.setattr(kernel_select, "_REFERENCE_COMPETES", False)
    calls = timings({"a": 5.0, "b": 3.0, "stock": 0.001})
    x, w, s, p, d = args()
    assert kernel_select.pick("conv3d", x, w, s, p, d, cands(["a", "b", "stock"])) == "out:b"
    assert "stock" not in calls
    kernel_select.reset()
    out = kernel_select.pick("conv3d", x, w, s, p, d, cands(["a", "stock"], declines={"a"}))
    assert out == "out:stock"      # nothing of ours applies: the reference serves it
    assert kernel_select.cached("conv3d", x, w, s, p, d) == "stock"


def test_pick_key_reference_competes_when_asked(monkeypatch, timings):
    """A contest whose reference is one of this package's own plans (the
    FFT transform-length contest) times the reference too, whatever the
    stock-competes setting."""
    monkeypatch.setattr(kernel_select, "_REFERENCE_COMPETES", False)
    calls = timings({"segments4096": 5.0, "original": 3.0})
    out = kernel_select.pick_key("fftconv_len", ("conv1d", 1), cands(["segments4096", "original"]),
                                 reference_competes=True)
    assert out == "out:original" and calls["original"] == 1
    assert kernel_select.cached_key("fftconv_len", ("conv1d", 1)) == "original"


# ------------------------------------------------------------ verification
def test_wrong_fast_candidate_is_blacklisted(monkeypatch, timings):
    monkeypatch.setattr(kernel_select, "_VERIFY_ENABLED", True)
    good = torch.ones(64, 64)
    outs = {"bad": good * 2, "good": good + 1e-6, "stock": good}
    timings({"bad": 1.0, "good": 2.0, "stock": 3.0})
    x, w, s, p, d = args()
    with pytest.warns(UserWarning, match="disagrees"):
        out = kernel_select.pick("conv3d", x, w, s, p, d,
                                 cands(["bad", "good", "stock"], outputs=outs))
    assert out is outs["good"]
    key = kernel_select.shape_key("conv3d", x, w, s, p, d)
    assert kernel_select.debug_bad_candidates()[key] == {"bad"}


def test_verification_bar_scales_with_output_rms():
    ref = torch.full((1000,), 300.0)
    ref[0] = 1e-3                     # one near-zero element
    cand = ref.clone()
    cand[0] = 2e-3                    # off by 1e-3: fails a plain atol of 1e-5
    assert kernel_select._agree(cand, ref, tolerance=(1e-4, 1e-5)) is True
    wrong = ref * 1.01
    assert kernel_select._agree(wrong, ref, tolerance=(1e-4, 1e-5)) is False


def test_verify_shape_mismatch_is_a_failure():
    assert kernel_select._agree(torch.zeros(3), torch.zeros(4)) is False


def test_verify_non_contiguous_pieces_and_nan(monkeypatch):
    monkeypatch.setattr(kernel_select, "_PIECE", 64)     # force several pieces
    ref = torch.randn(7, 5, 9).permute(2, 0, 1)          # non-contiguous view
    assert kernel_select._agree(ref.clone(), ref) is True
    bad = ref.clone()
    bad[8, 6, 4] += 1.0                                  # last element of the last piece
    assert kernel_select._agree(bad, ref) is False
    nan_ref = ref.clone()
    nan_ref[0, 0, 0] = float("nan")
    assert kernel_select._agree(nan_ref.clone(), nan_ref) is True


def test_key_string_round_trip_nested():
    key = ("conv3d", torch.bfloat16, (1, (2, 3)), 4, False, "x")
    text = kernel_select.key_string(key)
    assert kernel_select.parse_key(text) == key
    assert text.startswith('["conv3d", {"__dtype__": "torch.bfloat16"}, {"__tuple__": [1, ')


def test_all_candidates_wrong_falls_back_to_reference(monkeypatch, timings):
    monkeypatch.setattr(kernel_select, "_VERIFY_ENABLED", True)
    ref = torch.ones(8, 8)
    outs = {"a": ref * 3, "b": ref * -1, "stock": ref}
    timings({"a": 1.0, "b": 2.0, "stock": 3.0})
    x, w, s, p, d = args()
    with pytest.warns(UserWarning):
        out = kernel_select.pick("conv3d", x, w, s, p, d, cands(["a", "b", "stock"], outputs=outs))
    assert out is outs["stock"]
    assert kernel_select.cached("conv3d", x, w, s, p, d) == "stock"


# -------------------------------------------------------------- OOM handling
def test_oom_during_deciding_run_is_a_decline(monkeypatch, timings):
    timings({"a": 1.0, "stock": 2.0})

    def oom():
        raise torch.OutOfMemoryError("CUDA out of memory")
    oom._name = "a"
    x, w, s, p, d = args()
    stock = ("stock", lambda: "out:stock")
    stock[1]._name = "stock"
    monkeypatch.setattr(kernel_select, "_measure", lambda fn: {"a": 1.0, "stock": 2.0}[fn._name])
    assert kernel_select.pick("conv3d", x, w, s, p, d, [("a", oom), stock]) == "out:stock"


def test_non_oom_errors_propagate_in_the_deciding_run(monkeypatch):
    def boom():
        raise RuntimeError("kernel bug")
    boom._name = "a"
    ref = lambda: "out:stock"  # noqa: E731
    ref._name = "stock"
    monkeypatch.setattr(kernel_select, "_measure", lambda fn: 1.0)
    x, w, s, p, d = args()
    with pytest.raises(RuntimeError, match="kernel bug"):
        kernel_select.pick("conv3d", x, w, s, p, d, [("a", boom), ("stock", ref)])


def test_oom_while_verifying_records_nothing(monkeypatch, timings):
    monkeypatch.setattr(kernel_select, "_VERIFY_ENABLED", True)
    monkeypatch.setattr(kernel_select, "_agree", lambda *a, **k: None)
    timings({"a": 1.0, "stock": 2.0})
    x, w, s, p, d = args()
    with pytest.warns(UserWarning, match="out of memory"):
        out = kernel_select.pick("conv3d", x, w, s, p, d, cands(["a", "stock"]))
    assert out == "out:stock"
    assert kernel_select.debug_winners() == {}
    assert kernel_select.debug_bad_candidates() == {}


# --------------------------------------------------------------- persistence
def test_disk_cache_roundtrip_and_format(timings, monkeypatch):
    timings({"tcgen05": 1.0, "stock": 2.0})
    x, w, s, p, d = args()
    kernel_select.pick("conv3d", x, w, s, p, d, cands(["tcgen05", "stock"]))
    path = kernel_select.cache_file()
    raw = json.load(open(path))
    assert raw["verify_bar"] == kernel_select._VERIFY_BAR_VERSION
    (k, v), = raw["winners"].items()
    assert v == "tcgen05"
    assert json.loads(k)[1] == {"__dtype__": "torch.float32"}
    assert json.loads(k)[2] == {"__tuple__": [1, 4, 8, 8, 8]}
    kernel_select._book.clear()
    kernel_select.load_cache_file()
    assert kernel_select.cached("conv3d", x, w, s, p, d) == "tcgen05"


def test_stale_verify_bar_drops_blacklist_and_its_winners(tmp_path):
    key_a = kernel_select.key_string(("conv3d", torch.float16, (1,), (2,), (1,), (1,), (1,), False))
    key_b = kernel_select.key_string(("group_norm", torch.bfloat16, (4,), 32, False))
    raw = {"verify_bar": 1, "winners": {key_a: "x", key_b: "y"}, "bad": {key_a: ["z"]}}
    with open(kernel_select.cache_file(), "w") as f:
        json.dump(raw, f)
    kernel_select.load_cache_file()
    winners = kernel_select.debug_winners()
    assert list(winners.values()) == ["y"]
    assert kernel_select.debug_bad_candidates() == {}


def test_flat_legacy_file_and_corrupt_file(tmp_path):
    key = kernel_select.key_string(("conv1d", torch.float32, (1,), (1,), (1,), (1,), (1,), False))
    with open(kernel_select.cache_file(), "w") as f:
        json.dump({key: "depthwise"}, f)
    kernel_select.load_cache_file()
    assert "depthwise" in kernel_select.debug_winners().values()
    with open(kernel_select.cache_file(), "w") as f:
        f.write("{not json")
    kernel_select.load_cache_file()   # must not raise


def test_reset_removes_the_file(timings):
    timings({"a": 1.0, "stock": 2.0})
    x, w, s, p, d = args()
    kernel_select.pick("conv3d", x, w, s, p, d, cands(["a", "stock"]))
    assert os.path.exists(kernel_select.cache_file())
    kernel_select.reset()
    assert not os.path.exists(kernel_select.cache_file())
