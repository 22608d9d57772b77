"""Builds liboxf.so (CUDA kernels + C ABI + C++ host layer) for sm_100a.

Every translation unit is compiled by nvcc with
``-gencode arch=compute_100a,code=sm_100a -lineinfo`` into ``_build/`` and
linked into ``oxide-forge_b200/liboxf.so`` (in-tree, so it travels with the
repository snapshot). Rebuilds only what changed. Usage::

    python oxide-forge_b200/build.py [--force] [-j N]
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
BUILD = PKG / "_build"
LIB = PKG / "liboxf.so"

NVCC = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-Wall",
          "--expt-relaxed-constexpr", f"-I{ROOT / 'include'}", f"-I{PKG / 'csrc'}",
          f"-I{PKG / 'host'}"]

SOURCES = sorted((PKG / "csrc").glob("*.cu")) + sorted((PKG / "host").glob("*.cu")) + \
    sorted((PKG / "host").glob("*.cpp"))
HEADERS = sorted((PKG / "csrc").glob("*.cuh")) + sorted((PKG / "host").glob("*.h*")) + \
    sorted((ROOT / "include").glob("*.h"))


def _obj(src: Path) -> Path:
    return BUILD / (src.parent.name + "_" + src.stem + ".o")


def _stale(out: Path, deps) -> bool:
    if not out.exists():
        return True
    t = out.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def _compile(src: Path, force: bool) -> Path:
    obj = _obj(src)
    if force or _stale(obj, [src, *HEADERS, Path(__file__)]):
        # .cpp host files go through nvcc too (same flags), so they may use
        # the CUDA runtime headers and types.
        cmd = [NVCC, *ARCH, *COMMON, "-c", str(src), "-o", str(obj)]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed for {src.name}:\n{r.stdout}\n{r.stderr}")
        if r.stderr.strip():
            sys.stderr.write(r.stderr)
    return obj


def build(force: bool = False, jobs: int | None = None) -> Path:
    BUILD.mkdir(exist_ok=True)
    jobs = jobs or min(8, os.cpu_count() or 2)
    with ThreadPoolExecutor(jobs) as ex:
        objs = list(ex.map(lambda s: _compile(s, force), SOURCES))
    if force or _stale(LIB, objs):
        cmd = [NVCC, *ARCH, "-shared", "-o", str(LIB), *map(str, objs), "-lpthread"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return LIB


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-j", type=int, default=None)
    a = ap.parse_args()
    print(build(a.force, a.j))


if __name__ == "__main__":
    main()
