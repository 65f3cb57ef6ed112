"""Builds libaspire_b200.so in-tree with nvcc for sm_100a.

Usage: ``python -m aspire_b200.build [--verbose-ptxas]``.  The library is
written next to this file so that it travels with the source tree.
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
CSRC = PKG_DIR / "csrc"
INCLUDE = PKG_DIR.parent / "include"
LIB_NAME = "libaspire_b200.so"
LIB_PATH = PKG_DIR / LIB_NAME

SOURCES = [
    "capi.cu",
    "planner.cpp",
    "attn_gather.cu",
    "attn_tc.cu",
    "attn_merge.cu",
    "append_kv.cu",
    "select_pages.cu",
    "unified_indices.cu",
    "qkv_prologue.cu",
    "plan_device.cu",
    "noalloc.cu",
    "draft_spill.cu",
    "dump_state.cu",
]

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc_path() -> str:
    cand = shutil.which("nvcc")
    if cand:
        return cand
    default = "/usr/local/cuda/bin/nvcc"
    if os.path.exists(default):
        return default
    raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libaspire_b200")


def _inputs() -> list[Path]:
    files = [CSRC / s for s in SOURCES]
    files += sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + [INCLUDE / "aspire_b200.h"]
    return files


def is_stale() -> bool:
    if not LIB_PATH.exists():
        return True
    lib_mtime = LIB_PATH.stat().st_mtime
    return any(f.exists() and f.stat().st_mtime > lib_mtime for f in _inputs())


def build(verbose_ptxas: bool = False, force: bool = False) -> Path:
    """Compiles every CUDA/C++ source of the library into one shared object."""
    if not force and not is_stale():
        return LIB_PATH
    tmp = LIB_PATH.with_suffix(".so.tmp")
    cmd = [
        nvcc_path(),
        "-O3",
        "-std=c++17",
        *ARCH_FLAGS,
        "-lineinfo",
        "-shared",
        "-Xcompiler",
        "-fPIC,-fvisibility=hidden",
        "--expt-relaxed-constexpr",
        "-I",
        str(INCLUDE),
        "-o",
        str(tmp),
        *[str(CSRC / s) for s in SOURCES],
    ]
    if verbose_ptxas:
        cmd[1:1] = ["-Xptxas", "-v"]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(
            "nvcc failed building libaspire_b200.so:\n" + " ".join(cmd) + "\n" + proc.stdout + proc.stderr
        )
    if verbose_ptxas:
        sys.stderr.write(proc.stdout + proc.stderr)
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--verbose-ptxas", action="store_true")
    ap.add_argument("--force", action="store_true")
    args = ap.parse_args()
    path = build(verbose_ptxas=args.verbose_ptxas, force=args.force or args.verbose_ptxas)
    print(path)


if __name__ == "__main__":
    main()
