"""Builds the native launcher library in-tree (``ptxgen/_lib/libptxgen_b200.so``).

The launcher is host C++ over the CUDA driver API (``csrc/launcher.cpp``); it needs only
``g++`` and the CUDA headers, so it builds on a machine without a GPU.
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


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cpp"))


def stale() -> bool:
    if not LIB.exists():
        return True
    built = LIB.stat().st_mtime
    header = ROOT.parent / "include" / "ptxgen_b200.h"
    return any(p.stat().st_mtime > built for p in [*sources(), header] if p.exists())


def build_library(force: bool = False) -> Path:
    """Compile the launcher when it is missing or older than its sources; return its path."""
    if not force and not stale():
        return LIB
    cxx = shutil.which("g++") or shutil.which("c++")
    if cxx is None:
        raise RuntimeError("no C++ compiler (g++) to build the ptxgen launcher")
    LIB_DIR.mkdir(exist_ok=True)
    tmp = LIB.with_suffix(f".so.tmp{os.getpid()}")
    cmd = [cxx, "-O2", "-std=c++17", "-shared", "-fPIC", "-Wall", "-Wextra",
           f"-I{CUDA_HOME / 'include'}", *map(str, sources()), "-o", str(tmp), "-ldl"]
    subprocess.run(cmd, check=True, capture_output=True, text=True)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build_library(force=True))
