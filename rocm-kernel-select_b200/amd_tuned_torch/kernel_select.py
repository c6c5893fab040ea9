"""First-call benchmark-then-cache kernel selection.

Behavioural contract of the reference's amd_tuned_torch/kernel_select.py
(:204-295 verification, :309-423 persistence, :454-693 the contest), kept so
that callers and cache files move over unchanged:

* `pick(kind, input, weight, stride, padding, dilation, candidates)` and
  `pick_key(kind, key, candidates)` run a contest the first time a shape key
  is seen and return the winning candidate's output; later calls run the
  cached winner directly.  `cached`/`cached_key` expose the winner so callers
  can skip building thunks.
* `candidates` is `[(name, thunk), ...]`, best guess first, the REFERENCE
  LAST.  A thunk returns None to decline.  During timing, RuntimeError /
  TypeError / AssertionError count as a decline; in the deciding run only an
  out-of-memory error does, anything else propagates.
* Timing: 2 warm-up calls, then the fastest of 3 individually CUDA-event-
  timed calls (a delayed call can only be slower, so the minimum is the
  least contaminated estimate).
* Verification: before a non-reference candidate is crowned it is compared
  with the reference's output.  The bar is allclose with
  atol' = max(atol, rtol * RMS(reference)) -- relative to the output's
  scale -- evaluated in slices so no full fp32 copy is made.  A candidate
  that fails is blacklisted for that exact key (in memory and on disk) and
  the next-fastest one is tried.  An out-of-memory during verification
  records nothing.
* Persistence: `{"verify_bar": 3, "winners": {...}, "bad": {...}}` JSON in
  `AMD_TUNED_TORCH_KERNEL_SELECT_CACHE_DIR` (default: `_kernel_select_cache`
  beside this file), one file per GPU model + torch + Python, written via a
  temp file and os.replace.  Keys are JSON lists with dtypes and tuples
  tagged ({"__dtype__": ...}, {"__tuple__": [...]}), the same encoding as
  the reference, so files are interchangeable.  A file with a different
  verify_bar drops its blacklist and those shapes' winners.

One deliberate difference (the B200 build contests only its own kernels):
by default the reference candidate -- stock torch -- is NOT timed as a
competitor.  It remains the verification reference and the answer when
every own candidate declines or fails verification ("if nothing else works,
stock is used").  `AMD_TUNED_TORCH_STOCK_COMPETES=1` restores the
reference's behaviour of timing stock like any other candidate.

Env switches (read at import): AMD_TUNED_TORCH_MEASURE_KERNELS (0 disables
the contest), AMD_TUNED_TORCH_KERNEL_SELECT_VERIFY, AMD_TUNED_TORCH_
KERNEL_SELECT_CACHE, AMD_TUNED_TORCH_KERNEL_SELECT_CACHE_DIR.
"""
from __future__ import annotations

import json
import math
import os
import re
import sys
import threading
import warnings
from typing import Callable, Optional

import torch

_ENABLED = (os.environ.get("AMD_TUNED_TORCH_MEASURE_KERNELS",
                           os.environ.get("AMD_TUNED_TORCH_CONV_MEASURE", "1")) != "0")
_VERIFY_ENABLED = os.environ.get("AMD_TUNED_TORCH_KERNEL_SELECT_VERIFY", "1") != "0"
_REFERENCE_COMPETES = os.environ.get("AMD_TUNED_TORCH_STOCK_COMPETES", "0") == "1"

_winners: dict = {}
_bad_candidates: dict = {}
_lock = threading.Lock()

# Per-dtype (rtol, atol) verification defaults, same values as the reference
# (kernel_select.py:150-155).
_TOLERANCES = {
    torch.float16: (1e-2, 1e-2),
    torch.bfloat16: (2e-2, 2e-2),
    torch.float32: (1e-4, 1e-5),
}
_DEFAULT_TOLERANCE = (2e-2, 2e-2)

_SCALE_SAMPLE = 1 << 20
_CHUNK_ELEMENTS = 1 << 23

_VERIFY_BAR_VERSION = 3
_DISK_CACHE_ENABLED = os.environ.get("AMD_TUNED_TORCH_KERNEL_SELECT_CACHE", "1") != "0"
_CACHE_DIR = os.environ.get(
    "AMD_TUNED_TORCH_KERNEL_SELECT_CACHE_DIR",
    os.path.join(os.path.dirname(os.path.abspath(__file__)), "_kernel_select_cache"),
)

_WARMUP = 2
_ITERS = 3


def enabled() -> bool:
    return _ENABLED


def _is_oom(exc: BaseException) -> bool:
    for cls in (getattr(torch, "OutOfMemoryError", None),
                getattr(getattr(torch, "cuda", None), "OutOfMemoryError", None)):
        if isinstance(cls, type) and isinstance(exc, cls):
            return True
    return "out of memory" in str(exc).lower()


def _reference_scale(ref) -> Optional[float]:
    """RMS of a strided sample of `ref` (a whole-tensor fp32 reduction could
    cost more than the op being verified); None if not measurable."""
    try:
        flat = ref.flatten()
        step = max(1, flat.numel() // _SCALE_SAMPLE)
        scale = float(flat[::step].float().pow(2).mean().sqrt())
    except (RuntimeError, TypeError, ValueError, AttributeError, ZeroDivisionError):
        return None
    return scale if math.isfinite(scale) and scale > 0.0 else None


def _verify(out, ref, tolerance=None):
    """True = agrees, False = disagrees (or cannot be compared), None = the
    comparison itself ran out of memory (no judgement)."""
    try:
        rtol, atol = tolerance if tolerance is not None else _TOLERANCES.get(
            out.dtype, _DEFAULT_TOLERANCE)
        scale = _reference_scale(ref)
        if scale is not None:
            atol = max(atol, rtol * scale)
        if out.shape != ref.shape:
            return False
        if out.dim() == 0:
            return bool(torch.allclose(out.float(), ref.float(), rtol=rtol, atol=atol,
                                       equal_nan=True))
        rows = out.shape[0]
        per_row = max(1, out.numel() // max(1, rows))
        step = max(1, _CHUNK_ELEMENTS // per_row)
        for a in range(0, rows, step):
            b = min(rows, a + step)
            if not torch.allclose(out[a:b].float(), ref[a:b].float(), rtol=rtol, atol=atol,
                                  equal_nan=True):
                return False
        return True
    except (RuntimeError, TypeError, ValueError, AttributeError) as exc:
        return None if _is_oom(exc) else False


# ----------------------------------------------------------- persistence ---
def _device_key() -> str:
    try:
        name = torch.cuda.get_device_name(0) if torch.cuda.is_available() else "cpu"
    except Exception:  # noqa: BLE001 -- any driver trouble just names the file "unknown"
        name = "unknown"
    safe = re.sub(r"[^A-Za-z0-9_.-]+", "_", name)
    tv = torch.__version__.replace("+", "_").replace("/", "_")
    return f"{safe}-torch-{tv}-cp{sys.version_info.major}{sys.version_info.minor}"


def _cache_path() -> str:
    return os.path.join(_CACHE_DIR, f"{_device_key()}.json")


def _encode(v):
    if isinstance(v, torch.dtype):
        return {"__dtype__": str(v)}
    if isinstance(v, tuple):
        return {"__tuple__": [_encode(e) for e in v]}
    return v


def _decode(v):
    if isinstance(v, dict):
        if "__dtype__" in v:
            return getattr(torch, v["__dtype__"].rsplit(".", 1)[-1])
        if "__tuple__" in v:
            return tuple(_decode(e) for e in v["__tuple__"])
    return v


def _key_to_str(key) -> str:
    return json.dumps([_encode(e) for e in key])


def _str_to_key(s: str):
    return tuple(_decode(e) for e in json.loads(s))


def _load_disk_cache() -> None:
    if not _DISK_CACHE_ENABLED:
        return
    try:
        with open(_cache_path()) as f:
            raw = json.load(f)
    except (OSError, ValueError):
        return
    if not isinstance(raw, dict):
        return
    if "winners" in raw or "bad" in raw:
        winners, bad = raw.get("winners", {}), raw.get("bad", {})
    else:
        winners, bad = raw, {}
    stale = raw.get("verify_bar") != _VERIFY_BAR_VERSION
    with _lock:
        for ks, name in winners.items():
            if stale and ks in bad:
                continue
            try:
                _winners.setdefault(_str_to_key(ks), name)
            except (ValueError, TypeError, AttributeError):
                continue
        if not stale:
            for ks, names in bad.items():
                try:
                    _bad_candidates.setdefault(_str_to_key(ks), set()).update(names)
                except (ValueError, TypeError, AttributeError):
                    continue


def _save_disk_cache() -> None:
    if not _DISK_CACHE_ENABLED:
        return
    path = _cache_path()
    try:
        os.makedirs(os.path.dirname(path), exist_ok=True)
        with _lock:
            raw = {
                "verify_bar": _VERIFY_BAR_VERSION,
                "winners": {_key_to_str(k): v for k, v in _winners.items()},
                "bad": {_key_to_str(k): sorted(v) for k, v in _bad_candidates.items() if v},
            }
        tmp = f"{path}.tmp"
        with open(tmp, "w") as f:
            json.dump(raw, f)
        os.replace(tmp, path)
    except OSError:
        pass


# ------------------------------------------------------------------ keys ---
def _norm(v):
    return (v,) if isinstance(v, int) else tuple(v)


def _key(kind, input, weight, stride, padding, dilation):
    cl = (input.is_contiguous(memory_format=torch.channels_last) if input.dim() == 4 else
          input.is_contiguous(memory_format=torch.channels_last_3d) if input.dim() == 5 else
          False)
    return (kind, input.dtype, tuple(input.shape), tuple(weight.shape), _norm(stride),
            _norm(padding), _norm(dilation), bool(cl))


# ---------------------------------------------------------------- timing ---
def _time(fn) -> Optional[float]:
    """Fastest of _ITERS CUDA-event-timed calls after _WARMUP warm-ups; None
    if the candidate declines or fails."""
    try:
        for _ in range(_WARMUP):
            if fn() is None:
                return None
        torch.cuda.synchronize()
        events = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                  for _ in range(_ITERS)]
        for a, b in events:
            a.record()
            fn()
            b.record()
        torch.cuda.synchronize()
        return min(a.elapsed_time(b) for a, b in events)
    except (RuntimeError, TypeError, AssertionError):
        return None


# --------------------------------------------------------------- contest ---
def cached(kind: str, input, weight, stride, padding, dilation) -> Optional[str]:
    if not _ENABLED:
        return None
    with _lock:
        return _winners.get(_key(kind, input, weight, stride, padding, dilation))


def cached_key(kind: str, key) -> Optional[str]:
    if not _ENABLED:
        return None
    with _lock:
        return _winners.get((kind,) + tuple(key))


def pick(kind: str, input, weight, stride, padding, dilation,
         candidates: "list[tuple[str, Callable]]", tolerance=None):
    if not _ENABLED:
        return None
    return _contest(_key(kind, input, weight, stride, padding, dilation), candidates,
                    tolerance=tolerance)


def pick_key(kind: str, key, candidates: "list[tuple[str, Callable]]", tolerance=None):
    if not _ENABLED:
        return None
    return _contest((kind,) + tuple(key), candidates, tolerance=tolerance)


def _record(key, name) -> None:
    with _lock:
        _winners[key] = name
    _save_disk_cache()


def _run_guarded(thunk):
    """(output, oom) -- only an out-of-memory error is swallowed."""
    try:
        return thunk(), False
    except (RuntimeError, TypeError, AssertionError) as exc:
        if not _is_oom(exc):
            raise
        return None, True


def _contest(key, candidates, tolerance=None):
    if not candidates:
        return None
    ref_name, ref_thunk = candidates[-1]

    with _lock:
        winner = _winners.get(key)
        bad = set(_bad_candidates.get(key, ()))

    if winner is not None and winner not in bad:
        for name, thunk in candidates:
            if name == winner:
                out = thunk()
                if out is not None:
                    return out
                break
        with _lock:
            _winners.pop(key, None)
        _save_disk_cache()

    ranked = []
    for name, thunk in candidates:
        if name in bad:
            continue
        if name == ref_name and not _REFERENCE_COMPETES:
            continue
        ms = _time(thunk)
        if ms is not None:
            ranked.append((ms, name, thunk))
    ranked.sort(key=lambda r: r[0])

    unset = object()
    ref_out = unset
    ref_oom = False
    for _, name, thunk in ranked:
        out, _oom = _run_guarded(thunk)
        if out is None:
            continue
        if name == ref_name or not _VERIFY_ENABLED:
            _record(key, name)
            return out
        if ref_out is unset:
            ref_out, ref_oom = _run_guarded(ref_thunk)
            if ref_out is None:
                if ref_oom:
                    return out  # nothing learned: serve, record nothing
                _record(key, name)
                return out
        verdict = _verify(out, ref_out, tolerance)
        if verdict:
            _record(key, name)
            return out
        if verdict is None:
            warnings.warn(
                f"amd_tuned_torch.kernel_select: out of memory while verifying '{name}' for "
                f"{key} against '{ref_name}'; no judgement recorded, using the reference "
                "for this call.", UserWarning)
            return ref_out
        warnings.warn(
            f"amd_tuned_torch.kernel_select: candidate '{name}' for {key} was fastest but "
            f"disagrees with '{ref_name}' beyond tolerance; excluding it for this shape and "
            "trying the next candidate.", UserWarning)
        with _lock:
            _bad_candidates.setdefault(key, set()).add(name)
        _save_disk_cache()

    # Nothing of ours won: the reference serves the call (and the shape).
    if ref_out is unset:
        ref_out, ref_oom = _run_guarded(ref_thunk)
    if ref_oom:
        return None
    if ref_out is not None:
        _record(key, ref_name)
        return ref_out
    return None


def debug_winners() -> dict:
    with _lock:
        return dict(_winners)


def debug_bad_candidates() -> dict:
    with _lock:
        return {k: set(v) for k, v in _bad_candidates.items()}


def reset() -> None:
    """Forget every winner and exclusion, in memory and this GPU's cache file."""
    with _lock:
        _winners.clear()
        _bad_candidates.clear()
    if _DISK_CACHE_ENABLED:
        try:
            os.remove(_cache_path())
        except OSError:
            pass


if _ENABLED:
    _load_disk_cache()
