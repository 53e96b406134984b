"""Builds the MatMulNBits CUDA library in-tree for sm_100a.

``build()`` compiles every ``csrc/*.cu`` into ``xrgpu_b200/libxrgpu_mmnb.so`` with nvcc
(``-gencode arch=compute_100a,code=sm_100a``), skipping the build when the library is
newer than all sources and headers.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = ROOT / "include"
BUILD_DIR = PKG / "_build"
LIBRARY = PKG / "libxrgpu_mmnb.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    found = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(found).exists():
        raise RuntimeError("nvcc not found: the CUDA toolkit is required to build xrgpu_b200")
    return found


def _sources():
    return sorted(CSRC.glob("*.cu"))


def _deps():
    return _sources() + sorted(CSRC.glob("*.h")) + sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))


def up_to_date() -> bool:
    if not LIBRARY.exists():
        return False
    newest = max(p.stat().st_mtime for p in _deps())
    return LIBRARY.stat().st_mtime >= newest


def compile_flags(verbose_ptxas: bool = False):
    flags = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
             "--expt-relaxed-constexpr", f"-I{CSRC}", f"-I{INCLUDE}", *ARCH]
    if verbose_ptxas:
        flags += ["-Xptxas", "-v"]
    return flags


def build(force: bool = False, verbose_ptxas: bool = False, jobs: int | None = None) -> Path:
    if not force and up_to_date():
        return LIBRARY
    BUILD_DIR.mkdir(exist_ok=True)
    compiler = nvcc()
    objects = []

    def one(src: Path):
        obj = BUILD_DIR / (src.stem + ".o")
        cmd = [compiler, "-c", str(src), "-o", str(obj), *compile_flags(verbose_ptxas)]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"nvcc failed for {src.name}:\n{res.stdout}\n{res.stderr}")
        if verbose_ptxas:
            sys.stderr.write(res.stderr)
        return obj

    with ThreadPoolExecutor(max_workers=jobs or min(8, os.cpu_count() or 1)) as pool:
        objects = list(pool.map(one, _sources()))
    tmp = LIBRARY.with_suffix(".so.tmp")
    # No -lcuda: driver entry points (the TMA descriptor encoder) are resolved at run time.
    cmd = [compiler, "-shared", *ARCH, "-o", str(tmp), *map(str, objects), "-Xcompiler", "-fPIC"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
    os.replace(tmp, LIBRARY)
    return LIBRARY


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose_ptxas="-v" in sys.argv))
