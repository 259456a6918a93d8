"""Builds the in-tree C-ABI library ``libnvk_paged.so`` for sm_100a with nvcc.

Every ``csrc/*.cu`` file is compiled separately (``-gencode
arch=compute_100a,code=sm_100a -lineinfo -O3``) and linked into one shared
library next to this file, so the built object travels with the source tree.
A file is recompiled only when it, or a header it may include, is newer than
its object. ``python -m nano_vllm_ascend_b200._build [--verbose-ptxas]``.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
CSRC = PKG_DIR / "csrc"
INCLUDE = PKG_DIR.parent / "include"
BUILD_DIR = PKG_DIR / "_build"
LIB_NAME = "libnvk_paged.so"
LIB_PATH = PKG_DIR / LIB_NAME

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "--expt-relaxed-constexpr",
    "-Xcompiler",
    "-fPIC,-O3,-fvisibility=hidden",
    "-DNVK_BUILD",
]


def nvcc_path() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found; the CUDA toolkit is required to build libnvk_paged.so")
    return cand


def _sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _headers() -> list[Path]:
    return sorted(list(CSRC.glob("*.h")) + list(CSRC.glob("*.cuh")) + list(INCLUDE.glob("*.h")))


def build(verbose_ptxas: bool = False, force: bool = False) -> Path:
    """Compiles and links the library; returns its path."""
    nvcc = nvcc_path()
    BUILD_DIR.mkdir(exist_ok=True)
    newest_header = max((h.stat().st_mtime for h in _headers()), default=0.0)
    objects = []
    for src in _sources():
        obj = BUILD_DIR / (src.stem + ".o")
        objects.append(obj)
        stale = (
            force
            or verbose_ptxas
            or not obj.exists()
            or obj.stat().st_mtime < max(src.stat().st_mtime, newest_header)
        )
        if not stale:
            continue
        cmd = [nvcc, *ARCH_FLAGS, *NVCC_FLAGS, "-I", str(INCLUDE), "-c", str(src), "-o", str(obj)]
        if verbose_ptxas:
            cmd[1:1] = ["-Xptxas", "-v"]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if verbose_ptxas or res.returncode != 0:
            sys.stderr.write(res.stdout + res.stderr)
        if res.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src.name}")
    lib_stale = force or not LIB_PATH.exists() or any(o.stat().st_mtime > LIB_PATH.stat().st_mtime for o in objects)
    if lib_stale:
        tmp = LIB_PATH.with_suffix(".so.tmp")
        cmd = [nvcc, *ARCH_FLAGS, "-shared", "-o", str(tmp), *map(str, objects), "-lcudart_static", "-ldl", "-lrt",
               "-lpthread"]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            sys.stderr.write(res.stdout + res.stderr)
            raise RuntimeError("linking libnvk_paged.so failed")
        os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    path = build(verbose_ptxas="--verbose-ptxas" in sys.argv, force="--force" in sys.argv)
    print(path)
