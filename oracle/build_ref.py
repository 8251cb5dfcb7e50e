"""Compile the reference's own gate/up CUDA kernels from their sources into ``oracle/_ref/`` (checker only).

The reference ships CUDA sources for its INT8 gate/up, grouped-projection and rotated-quantizer
kernels; they are
self-contained (one .cu + one .cuh each, no external libraries), so they build directly with nvcc.  The
flags are the reference's own (``-O3 --cubin``, kernel-source/legacy-v2/manifest.json) with the
architecture changed from sm_120a to sm_100a.  Outputs go to ``oracle/_ref/`` only (git-ignored); the
GPU tests load them through the CUDA driver to compare our kernels with the reference's kernels on the
same B200 and inputs.  Nothing is copied out of the reference tree: nvcc reads the sources in place.
"""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "_ref"
SOURCES = {
    "native_hybrid8.cubin": "kernel-source/legacy-v2/src/native_hybrid8.cu",
    "sliced_linear8.cubin": "kernel-source/legacy-v2/src/sliced_linear8.cu",
    "block_rotation.cubin": "kernel-source/legacy-v2/src/block_rotation.cu",
}


def nvcc() -> str:
    p = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda")) / "bin" / "nvcc"
    return str(p) if p.exists() else "nvcc"


def build(reference_root: str = "/root/reference", verbose: bool = False) -> list[Path]:
    root = Path(reference_root)
    if not root.exists():
        return []
    OUT.mkdir(exist_ok=True)
    built = []
    for name, rel in SOURCES.items():
        src = root / rel
        dst = OUT / name
        if not src.exists():
            continue
        if dst.exists() and dst.stat().st_mtime >= src.stat().st_mtime:
            built.append(dst)
            continue
        cmd = [nvcc(), "-O3", "-arch=sm_100a", "--cubin", str(src), "-o", str(dst)]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
        built.append(dst)
    return built


if __name__ == "__main__":
    print(build(sys.argv[1] if len(sys.argv) > 1 else "/root/reference", verbose=True))
