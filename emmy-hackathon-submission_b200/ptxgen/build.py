"""Builds the native launcher library in-tree (``ptxgen/_lib/libptxgen_b200.so``).

The launcher is host C++ over the CUDA driver API (``csrc/launcher.cpp``); the library also
holds one hand-written sm_100a kernel pair (``csrc/noalloc_sum.cu``, compiled by nvcc and linked
with the static CUDA runtime, which loads libcuda only at its first call). Both build on a
machine without a GPU.
"""

from __future__ import annotations

import os
import shutil
import subprocess
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent  # the emmy-hackathon-submission_b200 directory
CSRC = ROOT / "csrc"
LIB_DIR = PKG / "_lib"
LIB = LIB_DIR / "libptxgen_b200.so"
CUDA_HOME = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))


NVCC_ARCH = "-gencode=arch=compute_100a,code=sm_100a"


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cpp"))


def cuda_sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def stale() -> bool:
    if not LIB.exists():
        return True
    built = LIB.stat().st_mtime
    header = ROOT.parent / "include" / "ptxgen_b200.h"
    return any(p.stat().st_mtime > built for p in [*sources(), *cuda_sources(), header]
               if p.exists())


def build_library(force: bool = False) -> Path:
    """Compile the launcher when it is missing or older than its sources; return its path."""
    if not force and not stale():
        return LIB
    cxx = shutil.which("g++") or shutil.which("c++")
    if cxx is None:
        raise RuntimeError("no C++ compiler (g++) to build the ptxgen launcher")
    LIB_DIR.mkdir(exist_ok=True)
    tmp = LIB.with_suffix(f".so.tmp{os.getpid()}")
    nvcc = CUDA_HOME / "bin" / "nvcc"
    objs = []
    for cu in cuda_sources():
        obj = LIB_DIR / f"{cu.stem}.o.tmp{os.getpid()}"
        _run([str(nvcc), NVCC_ARCH, "-lineinfo", "-O3", "-std=c++17", "-Xcompiler", "-fPIC",
              "-c", str(cu), "-o", str(obj)])
        objs.append(obj)
    cmd = [cxx, "-O2", "-std=c++17", "-shared", "-fPIC", "-Wall", "-Wextra",
           f"-I{CUDA_HOME / 'include'}", *map(str, sources()), *map(str, objs), "-o", str(tmp),
           f"-L{CUDA_HOME / 'lib64'}", "-lcudart_static", "-lrt", "-lpthread", "-ldl"]
    try:
        _run(cmd)
    finally:
        for obj in objs:
            obj.unlink(missing_ok=True)
    os.replace(tmp, LIB)
    return LIB


def _run(cmd: list[str]) -> None:
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode:
        raise RuntimeError(f"{' '.join(cmd)} failed:\n{r.stderr}")


if __name__ == "__main__":
    print(build_library(force=True))
