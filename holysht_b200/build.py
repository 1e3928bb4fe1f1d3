"""Build ``libholysht_b200.so`` in-tree with nvcc for sm_100a.

    python -m holysht_b200.build [--verbose]

The library has no torch dependency: it links only the CUDA runtime, so any
host language can bind the C ABI declared in ``include/holysht_b200.h``.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
SOURCES = [PKG / "csrc" / "capi.cu"]
HEADERS = [*(PKG / "csrc").glob("*.cuh"), ROOT / "include" / "holysht_b200.h"]
LIB = PKG / "libholysht_b200.so"


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def command(verbose: bool = False) -> list[str]:
    cmd = [
        nvcc(),
        "-gencode", "arch=compute_100a,code=sm_100a",
        "-O3", "-lineinfo", "-std=c++17",
        "-shared", "-Xcompiler", "-fPIC",
        "-I", str(ROOT / "include"),
        "-o", str(LIB),
        *map(str, SOURCES),
        "-lcudart",
    ]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    return cmd


def up_to_date() -> bool:
    if not LIB.exists():
        return False
    t = LIB.stat().st_mtime
    return all(src.stat().st_mtime <= t for src in SOURCES + HEADERS)


def build(force: bool = False, verbose: bool = False) -> Path:
    if force or not up_to_date():
        res = subprocess.run(command(verbose), capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"nvcc failed:\n{res.stdout}\n{res.stderr}")
        if verbose:
            sys.stderr.write(res.stderr)
    return LIB


if __name__ == "__main__":
    build(force=True, verbose="--verbose" in sys.argv)
    print(LIB)
