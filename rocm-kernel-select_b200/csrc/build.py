"""Builds libb200conv.so (the sm_100a kernels + C ABI) in-tree.

Every .cu file in this directory is compiled with nvcc for sm_100a only
(`-gencode arch=compute_100a,code=sm_100a`), objects go to csrc/_build/, and
the shared library is linked next to the Python package that loads it
(amd_tuned_torch/libb200conv.so).  The CUDA runtime is linked statically; the
driver API entry point needed for TMA descriptors is resolved at run time, so
the library loads on a machine without a GPU driver (it only fails at the
first kernel launch there).

Usage: python csrc/build.py [--force] [--verbose-ptxas]
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

CSRC = Path(__file__).resolve().parent
PKG_ROOT = CSRC.parent
OUT_DIR = CSRC / "_build"
LIB_PATH = PKG_ROOT / "amd_tuned_torch" / "libb200conv.so"
INCLUDE = PKG_ROOT.parent / "include"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-O2",
                "--expt-relaxed-constexpr", f"-I{INCLUDE}"]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libb200conv.so")


def _sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _headers() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def _compile(src: Path, ptxas_verbose: bool) -> tuple[Path, str]:
    obj = OUT_DIR / (src.stem + ".o")
    cmd = [_nvcc(), *ARCH_FLAGS, *COMMON_FLAGS, "-c", str(src), "-o", str(obj)]
    if ptxas_verbose:
        cmd += ["-Xptxas", "-v"]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{proc.stdout}\n{proc.stderr}")
    return obj, proc.stdout + proc.stderr


def build(force: bool = False, ptxas_verbose: bool = False, quiet: bool = True) -> Path:
    """Compiles stale objects and relinks the library; returns its path."""
    OUT_DIR.mkdir(parents=True, exist_ok=True)
    srcs = _sources()
    hdrs = _headers()
    todo = [s for s in srcs if force or ptxas_verbose
            or _stale(OUT_DIR / (s.stem + ".o"), [s, *hdrs])]
    logs = []
    if todo:
        with cf.ThreadPoolExecutor(max_workers=min(8, len(todo))) as ex:
            for obj, log in ex.map(lambda s: _compile(s, ptxas_verbose), todo):
                logs.append((obj, log))
    objs = [OUT_DIR / (s.stem + ".o") for s in srcs]
    if todo or _stale(LIB_PATH, objs):
        cmd = [_nvcc(), *ARCH_FLAGS, "-shared", "-o", str(LIB_PATH), *map(str, objs)]
        proc = subprocess.run(cmd, capture_output=True, text=True)
        if proc.returncode != 0:
            raise RuntimeError(f"link failed:\n{proc.stdout}\n{proc.stderr}")
    if not quiet or ptxas_verbose:
        for obj, log in logs:
            if log.strip():
                print(f"--- {obj.name}\n{log}")
    return LIB_PATH


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose-ptxas", action="store_true")
    args = ap.parse_args()
    path = build(force=args.force, ptxas_verbose=args.verbose_ptxas, quiet=False)
    print(path)
    return 0


if __name__ == "__main__":
    sys.exit(main())
