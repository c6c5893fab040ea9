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
  timed calls.
* Verification: before a non-reference candidate is crowned it is compared
  with the reference's output under allclose with
  atol' = max(atol, rtol * RMS(reference)) -- relative to the output's
  scale -- in pieces, so no full fp32 copy of either tensor is made.  A
  candidate that fails is excluded for that exact key (in memory and on
  disk) and the next-fastest one is tried.  An out-of-memory during
  verification records nothing.
* Persistence: `{"verify_bar": 3, "winners": {...}, "bad": {...}}` JSON in
  `AMD_TUNED_TORCH_KERNEL_SELECT_CACHE_DIR` (default: `_kernel_select_cache`
  beside this file), one file per GPU model + torch + Python, replaced
  atomically.  Keys are JSON lists with dtypes and tuples tagged
  ({"__dtype__": ...}, {"__tuple__": [...]}), so the files are
  interchangeable with the reference's.  A file written under another
  verify_bar loses its exclusions and the winners of those keys.

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
import tempfile
import threading
import warnings
from typing import Callable, Iterator, Optional, Tuple

import torch

_ENABLED = (os.environ.get("AMD_TUNED_TORCH_MEASURE_KERNELS",
                           os.environ.get("AMD_TUNED_TORCH_CONV_MEASURE", "1")) != "0")
_VERIFY_ENABLED = os.environ.get("AMD_TUNED_TORCH_KERNEL_SELECT_VERIFY", "1") != "0"
_REFERENCE_COMPETES = os.environ.get("AMD_TUNED_TORCH_STOCK_COMPETES", "0") == "1"
_DISK_CACHE_ENABLED = os.environ.get("AMD_TUNED_TORCH_KERNEL_SELECT_CACHE", "1") != "0"
_CACHE_DIR = os.environ.get(
    "AMD_TUNED_TORCH_KERNEL_SELECT_CACHE_DIR",
    os.path.join(os.path.dirname(os.path.abspath(__file__)), "_kernel_select_cache"),
)
_VERIFY_BAR_VERSION = 3

# Per-dtype (rtol, atol) verification defaults -- the reference's values
# (kernel_select.py:150-155), part of the acceptance contract.
_TOLERANCES = {
    torch.float16: (1e-2, 1e-2),
    torch.bfloat16: (2e-2, 2e-2),
    torch.float32: (1e-4, 1e-5),
}
_DEFAULT_TOLERANCE = (2e-2, 2e-2)

_RMS_SAMPLE = 1 << 20        # elements sampled for the output scale
_PIECE = 1 << 23             # elements compared per allclose call
_WARMUP, _ITERS = 2, 3


def enabled() -> bool:
    return _ENABLED


# ------------------------------------------------------------ the book ---
class _Book:
    """Winners and exclusions per key, behind one lock."""

    def __init__(self) -> None:
        self.lock = threading.Lock()
        self.winners: dict = {}
        self.excluded: dict = {}

    def winner(self, key) -> Optional[str]:
        with self.lock:
            return self.winners.get(key)

    def state(self, key) -> Tuple[Optional[str], frozenset]:
        with self.lock:
            return self.winners.get(key), frozenset(self.excluded.get(key, ()))

    def crown(self, key, name: str) -> None:
        with self.lock:
            self.winners[key] = name

    def forget(self, key) -> None:
        with self.lock:
            self.winners.pop(key, None)

    def exclude(self, key, name: str) -> None:
        with self.lock:
            self.excluded.setdefault(key, set()).add(name)

    def clear(self) -> None:
        with self.lock:
            self.winners.clear()
            self.excluded.clear()


_book = _Book()


# ---------------------------------------------------------- cache file ---
def _json_value(v):
    """Key element -> JSON value with dtypes and tuples tagged."""
    if isinstance(v, torch.dtype):
        return {"__dtype__": str(v)}
    if isinstance(v, tuple):
        return {"__tuple__": [_json_value(e) for e in v]}
    return v


def _untag(obj: dict):
    """json object_hook: tagged dtypes / tuples back to Python values (inner
    objects are converted first, so nested tuples come back whole)."""
    if "__dtype__" in obj:
        return getattr(torch, obj["__dtype__"].split(".")[-1])
    if "__tuple__" in obj:
        return tuple(obj["__tuple__"])
    return obj


def key_string(key) -> str:
    return json.dumps([_json_value(e) for e in key])


def parse_key(text: str):
    return tuple(json.loads(text, object_hook=_untag))


def cache_file() -> str:
    """One file per GPU model, torch build and Python minor version."""
    try:
        gpu = torch.cuda.get_device_name(0) if torch.cuda.is_available() else "cpu"
    except Exception:  # noqa: BLE001 -- a driver problem only changes the file name
        gpu = "unknown"
    parts = (re.sub(r"[^A-Za-z0-9_.-]+", "_", gpu), "torch",
             torch.__version__.replace("+", "_").replace("/", "_"),
             "cp%d%d" % sys.version_info[:2])
    return os.path.join(_CACHE_DIR, "-".join(parts) + ".json")


def load_cache_file() -> None:
    """Merges the cache file into the book (entries already known win)."""
    if not _DISK_CACHE_ENABLED:
        return
    try:
        with open(cache_file()) as f:
            raw = json.load(f)
    except (OSError, ValueError):
        return
    if not isinstance(raw, dict):
        return
    structured = "winners" in raw or "bad" in raw
    winners = raw.get("winners", {}) if structured else raw
    bad = raw.get("bad", {}) if structured else {}
    same_bar = raw.get("verify_bar") == _VERIFY_BAR_VERSION
    decoded = []
    for text, name in winners.items():
        if not same_bar and text in bad:
            continue          # decided under another verification bar
        try:
            decoded.append((parse_key(text), name))
        except (ValueError, TypeError, AttributeError):
            pass
    exclusions = []
    if same_bar:
        for text, names in bad.items():
            try:
                exclusions.append((parse_key(text), set(names)))
            except (ValueError, TypeError, AttributeError):
                pass
    with _book.lock:
        for key, name in decoded:
            _book.winners.setdefault(key, name)
        for key, names in exclusions:
            _book.excluded.setdefault(key, set()).update(names)


def save_cache_file() -> None:
    if not _DISK_CACHE_ENABLED:
        return
    path = cache_file()
    with _book.lock:
        doc = {"verify_bar": _VERIFY_BAR_VERSION,
               "winners": {key_string(k): v for k, v in _book.winners.items()},
               "bad": {key_string(k): sorted(v) for k, v in _book.excluded.items() if v}}
    try:
        folder = os.path.dirname(path)
        os.makedirs(folder, exist_ok=True)
        fd, tmp = tempfile.mkstemp(dir=folder, suffix=".part")
        with os.fdopen(fd, "w") as f:
            json.dump(doc, f)
        os.replace(tmp, path)
    except OSError:
        pass


# -------------------------------------------------------- verification ---
def _out_of_memory(exc: BaseException) -> bool:
    oom = getattr(torch, "OutOfMemoryError", None)
    if isinstance(oom, type) and isinstance(exc, oom):
        return True
    return "out of memory" in str(exc).lower()


def _rms(t: torch.Tensor) -> Optional[float]:
    """Root-mean-square of an evenly strided sample of at most _RMS_SAMPLE
    elements (a full fp32 reduction could cost more than the op itself);
    None when it is zero or not finite."""
    try:
        flat = t.reshape(-1)
        n = flat.numel()
        if n == 0:
            return None
        sample = flat[::-(-n // _RMS_SAMPLE)].float()
        value = float(torch.linalg.vector_norm(sample)) / math.sqrt(sample.numel())
    except (RuntimeError, TypeError, ValueError, AttributeError):
        return None
    return value if math.isfinite(value) and value > 0.0 else None


def _pieces(a: torch.Tensor, b: torch.Tensor) -> Iterator[Tuple[torch.Tensor, torch.Tensor]]:
    """Matching pieces of two same-shape tensors of about _PIECE elements:
    flat slices when both are contiguous, else blocks of leading-dimension
    rows (views, no copies)."""
    if a.dim() == 0:
        yield a, b
        return
    if a.is_contiguous() and b.is_contiguous():
        fa, fb = a.view(-1), b.view(-1)
        for lo in range(0, fa.numel(), _PIECE):
            yield fa[lo:lo + _PIECE], fb[lo:lo + _PIECE]
        return
    row = max(1, a[0].numel())
    rows_per_piece = max(1, _PIECE // row)
    for lo in range(0, a.shape[0], rows_per_piece):
        yield a[lo:lo + rows_per_piece], b[lo:lo + rows_per_piece]


def _agree(out, ref, tolerance=None) -> Optional[bool]:
    """True if `out` matches the reference output within the scaled bar,
    False if not (or not comparable), None if the comparison itself ran out
    of memory (no verdict)."""
    try:
        if tuple(out.shape) != tuple(ref.shape):
            return False
        out, ref = out.detach(), ref.detach()
        rtol, atol = tolerance or _TOLERANCES.get(out.dtype, _DEFAULT_TOLERANCE)
        scale = _rms(ref)
        atol = max(atol, rtol * scale) if scale is not None else atol
        return all(torch.allclose(pa.float(), pb.float(), rtol=rtol, atol=atol, equal_nan=True)
                   for pa, pb in _pieces(out, ref))
    except (RuntimeError, TypeError, ValueError, AttributeError) as exc:
        return None if _out_of_memory(exc) else False


# --------------------------------------------------------------- timing ---
def _measure(thunk: Callable) -> Optional[float]:
    """Fastest of _ITERS CUDA-event-timed calls after _WARMUP untimed ones,
    in ms; None when the candidate declines or fails while being timed."""
    try:
        for _ in range(_WARMUP):
            if thunk() is None:
                return None
        best = math.inf
        for _ in range(_ITERS):
            begin = torch.cuda.Event(enable_timing=True)
            end = torch.cuda.Event(enable_timing=True)
            torch.cuda.synchronize()
            begin.record()
            thunk()
            end.record()
            end.synchronize()
            best = min(best, begin.elapsed_time(end))
        return best
    except (RuntimeError, TypeError, AssertionError):
        return None


# ----------------------------------------------------------------- keys ---
def _as_tuple(v):
    return (v,) if isinstance(v, int) else tuple(v)


def shape_key(kind, input, weight, stride, padding, dilation):
    """(kind, dtype, input shape, weight shape, stride, padding, dilation,
    channels_last) -- the reference's conv key (kernel_select.py:438-445)."""
    fmt = {4: torch.channels_last, 5: torch.channels_last_3d}.get(input.dim())
    channels_last = fmt is not None and input.is_contiguous(memory_format=fmt)
    return (kind, input.dtype, tuple(input.shape), tuple(weight.shape), _as_tuple(stride),
            _as_tuple(padding), _as_tuple(dilation), bool(channels_last))


# -------------------------------------------------------------- contest ---
def cached(kind: str, input, weight, stride, padding, dilation) -> Optional[str]:
    return _book.winner(shape_key(kind, input, weight, stride, padding, dilation)) \
        if _ENABLED else None


def cached_key(kind: str, key) -> Optional[str]:
    return _book.winner((kind,) + tuple(key)) if _ENABLED else None


def pick(kind: str, input, weight, stride, padding, dilation,
         candidates: "list[tuple[str, Callable]]", tolerance=None):
    if not _ENABLED:
        return None
    return _contest(shape_key(kind, input, weight, stride, padding, dilation), candidates,
                    tolerance=tolerance)


def pick_key(kind: str, key, candidates: "list[tuple[str, Callable]]", tolerance=None,
             reference_competes: Optional[bool] = None):
    """Contest under an explicit key.  reference_competes: time the last
    candidate too (default: the stock-competes setting; a contest whose
    reference is one of this package's own plans passes True)."""
    if not _ENABLED:
        return None
    return _contest((kind,) + tuple(key), candidates, tolerance=tolerance,
                    reference_competes=reference_competes)


def _record(key, name) -> None:
    _book.crown(key, name)
    save_cache_file()


def _run_guarded(thunk):
    """(output, oom) -- only an out-of-memory error is swallowed."""
    try:
        return thunk(), False
    except (RuntimeError, TypeError, AssertionError) as exc:
        if not _out_of_memory(exc):
            raise
        return None, True


def _contest(key, candidates, tolerance=None, reference_competes: Optional[bool] = None):
    if not candidates:
        return None
    if reference_competes is None:
        reference_competes = _REFERENCE_COMPETES
    ref_name, ref_thunk = candidates[-1]
    winner, bad = _book.state(key)

    if winner is not None and winner not in bad:
        for name, thunk in candidates:
            if name == winner:
                out = thunk()
                if out is not None:
                    return out
                break
        _book.forget(key)
        save_cache_file()

    ranked = []
    for name, thunk in candidates:
        if name in bad:
            continue
        if name == ref_name and not reference_competes:
            continue
        ms = _measure(thunk)
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
        verdict = _agree(out, ref_out, tolerance)
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
        _book.exclude(key, name)
        save_cache_file()

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
    with _book.lock:
        return dict(_book.winners)


def debug_bad_candidates() -> dict:
    with _book.lock:
        return {k: set(v) for k, v in _book.excluded.items()}


def reset() -> None:
    """Forget every winner and exclusion, in memory and this GPU's cache file."""
    _book.clear()
    if _DISK_CACHE_ENABLED:
        try:
            os.remove(cache_file())
        except OSError:
            pass


if _ENABLED:
    load_cache_file()
