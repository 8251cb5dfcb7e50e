"""Compile the reference's own gate/up kernels from their sources into ``oracle/_ref/`` (checker only).

TEST INFRASTRUCTURE: nothing in the product imports this module or what it builds.

CUDA.  The reference ships CUDA sources for its INT8 gate/up (legacy ``hybrid8_*`` and the v3
production ``addressed_*`` / ``band_*`` variants), grouped-projection and rotated-quantizer kernels.
Each is one .cu + one .cuh with no external libraries, so it builds directly with nvcc.  The flags are
the reference's own (``-O3 --cubin``, kernel-source/legacy-v2/manifest.json) with the architecture
changed from sm_120a to sm_100a.

Triton.  The reference's quantizers (``reaxv2/quantize.py``: ``_prepare`` and ``prepare_kernel``) are
Triton kernels JIT-compiled at their first call.  The GPU box has no copy of the reference tree, so
they are compiled here ahead of time, for sm_100, with the options the reference launches them with
(``num_warps=8``, ``enable_fp_fusion=False``, reaxv2/gate_up.py:34-36 and reaxv2/sliced.py:14-17) and
the specialisation Triton's JIT gives 16-byte aligned tensors (``tt.divisibility`` 16 on every pointer).
One cubin per set of constexpr arguments the GPU tests and the bench use, each beside a JSON file with
its kernel name, warps and shared memory; ``oracle/ref_gpu.py`` launches them through the CUDA driver
the way Triton's own launcher does (the kernel's arguments, then two null scratch pointers).

Outputs go to ``oracle/_ref/`` only (git-ignored).  Nothing is copied out of the reference tree: nvcc
and Triton read the sources in place.  The reference root is a required argument.
"""
from __future__ import annotations

import importlib.util
import json
import os
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "_ref"
TRITON_OUT = OUT / "triton"
SOURCES = {
    "native_hybrid8.cubin": "kernel-source/legacy-v2/src/native_hybrid8.cu",
    "sliced_linear8.cubin": "kernel-source/legacy-v2/src/sliced_linear8.cu",
    "block_rotation.cubin": "kernel-source/legacy-v2/src/block_rotation.cu",
    # v3 production gate/up at K=2432, KH=128, N=18432 (launched by the wide_warp_hybrid.py snapshots)
    "addressed_gate_up.cubin": "kernel-source/src/model-preaddressed-GUP-r1/addressed_gate_up.cu",
    "band_gate_up.cubin": "kernel-source/src/model-preaddressed-GUP-tail-bands-r2/band_gate_up.cu",
    "addressed_table_gate_up.cubin": "kernel-source/src/model-addressed-bulk-activation-table-r1/addressed_gate_up.cu",
}

# _prepare constexprs (K, KL, KH, CENTER): the golden cases (tests/golden/gen_golden.py), the BASELINE
# widths, a centred K = 4096 bank and the v3 production bank (K = 2560: 2432 INT8 + 128 BF16 columns).
PREPARE_CONFIGS = [
    (1024, 1024, 0, False), (512, 512, 0, False), (4096, 4096, 0, False), (1024, 896, 128, True),
    (256, 0, 64, True), (256, 256, 0, False), (8192, 8192, 0, False), (4096, 4096, 0, True),
    (2560, 2432, 128, True), (2560, 2432, 128, False),
]
# prepare_kernel constexprs (M, K, G, HP, P): the golden case and two wider grouped banks
GROUPS_CONFIGS = [(6, 1024, 512, 64, 2), (64, 2560, 1280, 64, 2), (300, 4096, 2048, 0, 2)]


def nvcc() -> str:
    p = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda")) / "bin" / "nvcc"
    return str(p) if p.exists() else "nvcc"


def prepare_name(K, KL, KH, center) -> str:
    return f"prepare_K{K}_KL{KL}_KH{KH}_C{int(center)}"


def groups_name(M, K, G, HP, P) -> str:
    return f"groups_M{M}_K{K}_G{G}_HP{HP}_P{P}"


def _next_pow2(n: int) -> int:
    return 1 if n <= 1 else 1 << (n - 1).bit_length()


def _compile_triton(fn, signature, constexprs, name, num_warps=8, verbose=False) -> Path:
    import triton
    from triton.backends.compiler import GPUTarget
    from triton.compiler import make_backend
    target = GPUTarget("cuda", 100, 32)
    aligned = make_backend(target).parse_attr("D")          # what the JIT gives a 16-byte aligned pointer
    attrs = {(i,): aligned for i, (arg, ty) in enumerate(signature.items()) if ty.startswith("*")}
    src = triton.compiler.ASTSource(fn=fn, signature=signature, constexprs=constexprs, attrs=attrs)
    k = triton.compile(src, target=target, options={"num_warps": num_warps, "enable_fp_fusion": False})
    TRITON_OUT.mkdir(parents=True, exist_ok=True)
    (TRITON_OUT / f"{name}.cubin").write_bytes(k.asm["cubin"])
    meta = {"kernel": k.name, "num_warps": k.metadata.num_warps, "shared": k.metadata.shared,
            "global_scratch_size": k.metadata.global_scratch_size,
            "profile_scratch_size": k.metadata.profile_scratch_size, "constexprs": {str(a): v for a, v in constexprs.items()},
            "args": [a for a, t in signature.items() if t != "constexpr"], "triton": triton.__version__}
    (TRITON_OUT / f"{name}.json").write_text(json.dumps(meta, indent=1))
    if verbose:
        print("triton", name, "shared", meta["shared"], flush=True)
    return TRITON_OUT / f"{name}.cubin"


def build_triton(root: Path, verbose: bool = False) -> list[Path]:
    """The reference's Triton quantizers, compiled ahead of time for sm_100 (see the module docstring)."""
    src = root / "reaxv2" / "quantize.py"
    if not src.exists():
        return []
    try:
        import triton  # noqa: F401
    except ImportError:
        return []
    stamp = TRITON_OUT / "source.stamp"
    want = f"{src.stat().st_mtime_ns} {len(PREPARE_CONFIGS)} {len(GROUPS_CONFIGS)}"
    names = [prepare_name(*c) for c in PREPARE_CONFIGS] + [groups_name(*c) for c in GROUPS_CONFIGS]
    if stamp.exists() and stamp.read_text() == want and all((TRITON_OUT / f"{n}.cubin").exists() for n in names):
        return [TRITON_OUT / f"{n}.cubin" for n in names]
    spec = importlib.util.spec_from_file_location("reference_quantize", src)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    built = []
    sig_prepare = {"x": "*bf16", "low_columns": "*i32", "high_columns": "*i32", "smoothing": "*fp32",
                   "centers": "*fp32", "low": "*i8", "high": "*bf16", "scales": "*fp32", "K": "constexpr",
                   "KL": "constexpr", "KH": "constexpr", "BL": "constexpr", "BH": "constexpr", "CENTER": "constexpr"}
    for K, KL, KH, center in PREPARE_CONFIGS:
        consts = {"K": K, "KL": KL, "KH": KH, "BL": _next_pow2(max(KL, 1)), "BH": _next_pow2(max(KH, 1)),
                  "CENTER": center}
        built.append(_compile_triton(mod._prepare, sig_prepare, consts, prepare_name(K, KL, KH, center), verbose=verbose))
    sig_groups = {"x": "*bf16", "low_columns": "*i32", "high_columns": "*i32", "center": "*fp32", "smoothing": "*fp32",
                  "low": "*i8", "high": "*bf16", "scales": "*fp32", "M": "constexpr", "K": "constexpr", "G": "constexpr",
                  "HP": "constexpr", "P": "constexpr", "B": "constexpr", "BH": "constexpr"}
    for M, K, G, HP, P in GROUPS_CONFIGS:
        consts = {"M": M, "K": K, "G": G, "HP": HP, "P": P, "B": _next_pow2(G), "BH": _next_pow2(max(1, HP))}
        built.append(_compile_triton(mod.prepare_kernel, sig_groups, consts, groups_name(M, K, G, HP, P),
                                     verbose=verbose))
    stamp.write_text(want)
    return built


def build(reference_root: str | None, verbose: bool = False) -> list[Path]:
    if not reference_root:
        return []
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
    built += build_triton(root, verbose=verbose)
    return built


if __name__ == "__main__":
    if len(sys.argv) < 2:
        sys.exit("usage: python -m oracle.build_ref <reference root>")
    print(build(sys.argv[1], verbose=True))
