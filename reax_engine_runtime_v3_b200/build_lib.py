"""Build ``libreax_b200.so`` (the C-ABI library of hand-written sm_100a kernels) in-tree with nvcc."""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
LIB = PKG / "libreax_b200.so"
SOURCES = [PKG / "csrc" / "abi.cu"]
HEADERS = sorted((PKG / "csrc").glob("*.cuh")) + [ROOT / "include" / "reax_b200.h"]


def nvcc() -> str:
    home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    path = Path(home) / "bin" / "nvcc"
    return str(path) if path.exists() else "nvcc"


def command(out: Path = LIB, extra: list[str] | None = None) -> list[str]:
    return [nvcc(), "-gencode", "arch=compute_100a,code=sm_100a", "-lineinfo", "-O3", "-std=c++17",
            "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden", "-shared",
            "-I", str(ROOT / "include"), "-I", str(PKG / "csrc"),
            *(extra or []), *[str(s) for s in SOURCES], "-o", str(out)]


def up_to_date() -> bool:
    if not LIB.exists():
        return False
    t = LIB.stat().st_mtime
    return all(p.stat().st_mtime <= t for p in SOURCES + HEADERS)


def build(force: bool = False, verbose: bool = False, extra: list[str] | None = None) -> Path:
    if force or not up_to_date():
        cmd = command(extra=extra)
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True, extra=["-Xptxas", "-v"] if "--ptxas-v" in sys.argv else None)
