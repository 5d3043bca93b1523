"""Builds the DCNv2 CUDA library in-tree: jasnamacos_b200/lib/libdcn_b200.so.

All sources are compiled for sm_100a only (``-gencode arch=compute_100a,code=sm_100a``)
with the CUDA runtime linked statically, so the library carries no dependency on
the CUDA runtime that PyTorch ships.  Runs without a GPU (nvcc cross-compiles).

Usage: ``python -m jasnamacos_b200.csrc.build [--verbose-ptxas]``.
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

CSRC = Path(__file__).resolve().parent
PKG = CSRC.parent
REPO = PKG.parent
INCLUDE = REPO / "include"
LIB_DIR = PKG / "lib"
LIB_PATH = LIB_DIR / "libdcn_b200.so"

SOURCES = [
    "dcn_api.cu",
    "dcn_direct.cu",
    "dcn_fused_sm100.cu",
    "dcn_slab_sm100.cu",
    "dcn_prepack.cu",
    "dcn_aux.cu",
    "dcn_static_scratch.cu",
    "dcn_host.cu",
    "dcn_temporal.cu",
    "dcn_nhwc.cu",
]
HEADERS = ["dcn_common.cuh"]

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: the DCNv2 library cannot be built")


def _stale() -> bool:
    if not LIB_PATH.exists():
        return True
    built = LIB_PATH.stat().st_mtime
    deps = [CSRC / s for s in SOURCES + HEADERS] + [INCLUDE / "dcn_b200.h", Path(__file__)]
    return any(d.stat().st_mtime > built for d in deps)


def build(force: bool = False, verbose_ptxas: bool = False) -> Path:
    """Compiles the library if a source changed (or ``force``); returns its path."""
    if not force and not verbose_ptxas and not _stale():
        return LIB_PATH
    LIB_DIR.mkdir(parents=True, exist_ok=True)
    tmp = LIB_PATH.with_suffix(".so.tmp")
    cmd = [
        nvcc_path(),
        *ARCH_FLAGS,
        "-O3",
        "-lineinfo",
        "-std=c++17",
        "-Xcompiler",
        "-fPIC,-O2",
        "-shared",
        "-cudart",
        "static",
        f"-I{INCLUDE}",
        f"-I{CSRC}",
        "-o",
        str(tmp),
        *[str(CSRC / s) for s in SOURCES],
    ]
    if verbose_ptxas:
        cmd[1:1] = ["-Xptxas", "-v"]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        sys.stderr.write(proc.stdout + proc.stderr)
        raise RuntimeError(f"nvcc failed ({proc.returncode}) building {LIB_PATH.name}")
    if verbose_ptxas:
        sys.stderr.write(proc.stderr)
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose-ptxas", action="store_true", help="print registers/spills/shared memory")
    args = ap.parse_args()
    print(build(force=args.force, verbose_ptxas=args.verbose_ptxas))


if __name__ == "__main__":
    main()
