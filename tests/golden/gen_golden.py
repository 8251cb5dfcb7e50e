"""Generate golden vectors by running the reference's own Triton kernels on the CPU.

Run in a container where the reference project is mounted (its root as the first argument).  The reference's ``reaxv2/quantize.py`` kernels (``_prepare``,
``prepare_kernel``, ``reduce_kernel``) and ``runtime/mixed_origin_bf16.py``'s ``fold`` are
executed unmodified by Triton's CPU interpreter (``TRITON_INTERPRET=1``).  The interpreter cannot
lower the two libdevice calls of ``quantize.py:20,44``; they are supplied with their documented
semantics: ``div_rn`` = IEEE float32 division rounded to nearest (``tl.math.div_rn``) and
``nearbyint`` = round half to even (exact for the |v| <= 2**22 range a quantizer produces).  In the
interpreter the plain ``/`` of ``quantize.py:18-19`` is numpy's IEEE float32 division.

The interpreter (Triton 3.6) also truncates float32 -> bfloat16 casts, while the GPU lowering of
``.to(tl.bfloat16)`` rounds to nearest even (Triton's default ``fp_downcast_rounding``).  The
generator replaces that one conversion with round-to-nearest-even so that ``reduce_kernel`` and
``fold`` (``quantize.py:61``, ``mixed_origin_bf16.py:17``) produce what the GPU produces.

Outputs ``tests/golden/reference_kernels.npz``.  The tests only read the ``.npz``; this script is
the record of how it was made.
"""
from __future__ import annotations

import os
import sys
from pathlib import Path

os.environ["TRITON_INTERPRET"] = "1"

import numpy as np  # noqa: E402
import torch  # noqa: E402
import triton  # noqa: E402
import triton.language as tl  # noqa: E402

HERE = Path(__file__).resolve().parent


@triton.jit
def _round_half_even(v):
    # 1.5 * 2**23: adding and subtracting it rounds float32 |v| <= 2**22 to an integer, ties to even
    return (v + 12582912.0) - 12582912.0


def _patch_interpreter_bf16_rounding() -> None:
    import triton.runtime.interpreter as interp
    original = interp._convert_float

    def convert(data, input_dtype, output_dtype, rounding_mode):
        if input_dtype == tl.float32 and output_dtype == tl.bfloat16:
            u = np.ascontiguousarray(data).view(np.uint32).astype(np.uint64)
            rounded = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
            nan = np.isnan(np.ascontiguousarray(data).view(np.float32))
            rounded[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)
            return rounded
        return original(data, input_dtype, output_dtype, rounding_mode)

    interp._convert_float = convert


class _Libdevice:
    """Stand-in for ``triton.language.extra.cuda.libdevice`` inside the interpreter."""
    div_rn = property(lambda self: tl.math.div_rn)
    nearbyint = property(lambda self: _round_half_even)


def bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16).copy()


def student_t_outliers(gen, M, K, channels=8, factor=50.0):
    """Student-t (df=3) activations with a few fixed channels scaled up."""
    normal = torch.randn(M, K, generator=gen)
    chi2 = torch.randn(M, K, 3, generator=gen).square().sum(-1)
    x = normal / torch.sqrt(chi2 / 3.0)
    idx = torch.arange(channels) * (K // channels) + 3
    x[:, idx] *= factor
    return x


def main(reference_root: str) -> None:
    sys.path.insert(0, reference_root)
    import reaxv2.quantize as quantize                       # reference: reaxv2/quantize.py
    import runtime.mixed_origin_bf16 as mixed                # reference: runtime/mixed_origin_bf16.py
    quantize.libdevice = _Libdevice()
    _patch_interpreter_bf16_rounding()

    gen = torch.Generator().manual_seed(20261201)
    out: dict[str, np.ndarray] = {}

    # ---- _prepare (quantize.py:5-29) -------------------------------------------------------------------------
    cases = []
    # (name, M, K, kind, KH, center, smoothing kind)
    cases.append(("cfg1", 16, 1024, "normal", 0, False, "one"))
    cases.append(("ragged17", 17, 512, "normal", 0, False, "one"))
    cases.append(("outlier", 8, 4096, "student", 0, False, "one"))
    cases.append(("hybrid", 12, 1024, "normal", 128, True, "pow2"))
    cases.append(("highonly", 5, 256, "normal", 64, True, "allhigh"))
    cases.append(("zerorow", 4, 256, "zeros", 0, False, "one"))
    for name, M, K, kind, KH, center, smooth_kind in cases:
        if kind == "normal":
            xf = torch.randn(M, K, generator=gen)
        elif kind == "student":
            xf = student_t_outliers(gen, M, K)
        else:
            xf = torch.randn(M, K, generator=gen)
            xf[1] = 0.0
            xf[3, :] = 1e-30
        x = xf.to(torch.bfloat16)
        perm = torch.randperm(K, generator=gen)
        if smooth_kind == "allhigh":
            high = perm[:KH].sort().values
            low = torch.zeros(0, dtype=torch.int64)
        else:
            high = perm[:KH].sort().values
            keep = torch.ones(K, dtype=torch.bool)
            keep[high] = False
            low = keep.nonzero().flatten()
        KL = len(low)
        if smooth_kind == "pow2":
            smoothing = 2.0 ** torch.randint(-3, 4, (KL,), generator=gen).float()
        else:
            smoothing = torch.ones(KL)
        centers = (torch.randn(KL, generator=gen) * 0.1) if center else torch.zeros(KL)
        lowt = torch.empty(M, KL, dtype=torch.int8)
        hight = torch.empty(M, KH, dtype=torch.bfloat16)
        scales = torch.empty(M)
        lc, hc = low.to(torch.int32), high.to(torch.int32)
        quantize._prepare[(M,)](x, lc, hc, smoothing, centers, lowt, hight, scales,
                                K=K, KL=KL, KH=KH, BL=triton.next_power_of_2(max(KL, 1)),
                                BH=triton.next_power_of_2(max(KH, 1)), CENTER=center,
                                num_warps=8, enable_fp_fusion=False)
        p = f"prepare_{name}_"
        out[p + "x"] = bits(x)
        out[p + "low_columns"] = lc.numpy()
        out[p + "high_columns"] = hc.numpy()
        out[p + "smoothing"] = smoothing.numpy()
        out[p + "centers"] = centers.numpy()
        out[p + "center"] = np.array(int(center))
        out[p + "low"] = lowt.numpy()
        out[p + "high"] = bits(hight)
        out[p + "scales"] = scales.numpy()

    # ---- prepare_kernel (quantize.py:31-52) ------------------------------------------------------------------
    M, K, P, G, HP = 6, 1024, 2, 512, 64
    x = torch.randn(M, K, generator=gen).to(torch.bfloat16)
    perm = torch.randperm(K, generator=gen)
    high = perm[:P * HP - 3]
    lowcols = perm[P * HP - 3:]
    low_columns = torch.full((P * G,), -1, dtype=torch.int32)
    low_columns[:len(lowcols) // 2] = lowcols[:len(lowcols) // 2].to(torch.int32)
    low_columns[G:G + len(lowcols) - len(lowcols) // 2] = lowcols[len(lowcols) // 2:].to(torch.int32)
    high_columns = torch.full((P * HP,), -1, dtype=torch.int32)
    high_columns[:len(high)] = high.to(torch.int32)
    centers = torch.randn(P * G, generator=gen) * 0.05
    smoothing = 2.0 ** torch.randint(-2, 3, (P * G,), generator=gen).float()
    lowt = torch.empty(M, P * G, dtype=torch.int8)
    hight = torch.empty(M, P * HP, dtype=torch.bfloat16)
    scales = torch.empty(P, M)
    quantize.prepare_kernel[(M, P)](x, low_columns, high_columns, centers, smoothing, lowt, hight, scales,
                                    M=M, K=K, G=G, HP=HP, P=P, B=triton.next_power_of_2(G),
                                    BH=triton.next_power_of_2(max(1, HP)), num_warps=8, enable_fp_fusion=False)
    for k, v in dict(x=bits(x), low_columns=low_columns.numpy(), high_columns=high_columns.numpy(),
                     centers=centers.numpy(), smoothing=smoothing.numpy(), low=lowt.numpy(), high=bits(hight),
                     scales=scales.numpy(), shape=np.array([M, K, P, G, HP])).items():
        out["groups_" + k] = v

    # ---- reduce_kernel (quantize.py:55-61) -------------------------------------------------------------------
    P, M, N = 3, 5, 96
    partials = (torch.randn(P, M, N, generator=gen) * 4).to(torch.bfloat16)
    red = torch.empty(M, N, dtype=torch.bfloat16)
    quantize.reduce_kernel[(triton.cdiv(M * N, 512),)](partials, red, TOTAL=M * N, P=P, B=512,
                                                       num_warps=4, enable_fp_fusion=False)
    out["reduce_partials"] = bits(partials)
    out["reduce_out"] = bits(red)

    # ---- fold (runtime/mixed_origin_bf16.py:8-17) ------------------------------------------------------------
    P0, P1, M, N, split = 2, 3, 9, 64, 5
    parts = (torch.randn(max(P0, P1), M, N, generator=gen) * 3).to(torch.bfloat16)
    split_t = torch.tensor([split], dtype=torch.int32)
    folded = torch.empty(M, N, dtype=torch.bfloat16)
    mixed.fold[(triton.cdiv(M * N, 512),)](parts, split_t, folded, M=M, N=N, P0=P0, P1=P1, B=512,
                                           num_warps=4, enable_fp_fusion=False)
    out["fold_parts"] = bits(parts)
    out["fold_out"] = bits(folded)
    out["fold_shape"] = np.array([P0, P1, M, N, split])

    np.savez_compressed(HERE / "reference_kernels.npz", **out)
    print("wrote", HERE / "reference_kernels.npz", len(out), "arrays")


if __name__ == "__main__":
    if len(sys.argv) < 2:
        sys.exit("usage: python tests/golden/gen_golden.py <reference root>")
    main(sys.argv[1])
