"""Build libkrunch_b200.so (all CUDA sources, sm_100a) in-tree.

Objects go to krunch_b200/_build/, the shared library next to this file so it
travels with the source tree.  Rebuilds only what changed (source or header
mtime newer than the object).

    python -m krunch_b200.build [-j N] [--force]
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
LIB = PKG / "libkrunch_b200.so"
INCLUDE = PKG.parent / "include"

NVCC = os.environ.get("NVCC", "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-std=c++17", "-O3", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall",
         "--expt-relaxed-constexpr", f"-I{INCLUDE}"]


def _sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _headers() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))


def _stale(obj: Path, src: Path, hdr_mtime: float) -> bool:
    if not obj.exists():
        return True
    m = obj.stat().st_mtime
    return src.stat().st_mtime > m or hdr_mtime > m


def _compile(src: Path) -> Path:
    obj = BUILD / (src.stem + ".o")
    cmd = [NVCC, *ARCH, *FLAGS, "-c", str(src), "-o", str(obj)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src.name}:\n{res.stdout}\n{res.stderr}")
    return obj


def build(force: bool = False, jobs: int | None = None, verbose: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    srcs = _sources()
    hdr_mtime = max((h.stat().st_mtime for h in _headers()), default=0.0)
    todo = [s for s in srcs if force or _stale(BUILD / (s.stem + ".o"), s, hdr_mtime)]
    if todo:
        jobs = jobs or min(len(todo), os.cpu_count() or 4)
        with cf.ThreadPoolExecutor(jobs) as ex:
            for obj in ex.map(_compile, todo):
                if verbose:
                    print(f"compiled {obj.name}", file=sys.stderr)
    objs = [BUILD / (s.stem + ".o") for s in srcs]
    if force or todo or not LIB.exists() or any(o.stat().st_mtime > LIB.stat().st_mtime for o in objs):
        tmp = LIB.with_suffix(".so.tmp")
        cmd = [NVCC, *ARCH, "-shared", "-o", str(tmp), *map(str, objs)]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
        os.replace(tmp, LIB)
        if verbose:
            print(f"linked {LIB}", file=sys.stderr)
    return LIB


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-j", type=int, default=None)
    a = ap.parse_args()
    print(build(force=a.force, jobs=a.j, verbose=True))


if __name__ == "__main__":
    main()
