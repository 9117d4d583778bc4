"""Build libaihost_attn.so (the C-ABI attention library) in-tree with nvcc for sm_100a.

Usage: python -m aihost_b200.build [--force] [--verbose]
The library is written next to this file; a build is skipped when it is newer than every source.
"""
from __future__ import annotations

import argparse
import os
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
LIB = PKG / "libaihost_attn.so"
SOURCES = ["api.cu", "rope_append.cu", "decode.cu", "prefill_sm100.cu", "noalloc.cu", "decode_mma.cu", "dist.cu",
           "matmul_sm100.cu"]
HEADERS = ["common.cuh", "kernels.h", "rows.cuh"]


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    return "nvcc"


def needs_build() -> bool:
    if not LIB.exists():
        return True
    mtime = LIB.stat().st_mtime
    deps = [CSRC / s for s in SOURCES + HEADERS] + [ROOT / "include" / "aihost_attn.h", Path(__file__)]
    return any(p.stat().st_mtime > mtime for p in deps)


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and not needs_build():
        return LIB
    cmd = [
        nvcc_path(), "-O3", "-std=c++17", "-lineinfo",
        "-gencode", "arch=compute_100a,code=sm_100a",
        "-Xcompiler", "-fPIC", "-shared",
        "-Xptxas", "-v" if verbose else "-O3",
        "-o", str(LIB) + ".tmp",
    ] + [str(CSRC / s) for s in SOURCES] + ["-ldl"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if verbose or res.returncode != 0:
        sys.stderr.write(res.stdout + res.stderr)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed ({res.returncode}) building {LIB.name}")
    os.replace(str(LIB) + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    args = ap.parse_args()
    print(build(force=args.force, verbose=args.verbose))
