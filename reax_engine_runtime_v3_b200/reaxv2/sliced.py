"""Drop-in for ``reaxv2/sliced.py``: grouped ("sliced") INT8 projections.

``prepare`` runs the grouped quantizer (P groups of G columns, one scale per row and group) and
``project`` computes one bf16 partial per group with a tcgen05 kernel (``reax_sliced_i8``) and folds
the partials in order when P > 1 (reaxv2/sliced.py:10-47; kernel semantics
kernel-source/legacy-v2/src/sliced_linear8.cu:4-32).
"""
from __future__ import annotations

import torch

from .. import _native
from .driver import NativeInt8
from .quantize import prepare_kernel, reduce_kernel

# Kernel names and (big rows, small rows, N tile, threads) of the reference's slice_* kernels
# (reaxv2/sliced.py:7); only the N tile enters the precondition check.
CONFIGS = {
    "slice_m128n128": (128, 32, 128, 256),
    "slice_m64n128": (64, 32, 128, 256),
    "slice_m64n128w4": (64, 32, 128, 128),
    "slice_m128n256": (128, 32, 256, 256),
    "slice_m128n128k64": (128, 32, 128, 256),
}


def _next_pow2(n: int) -> int:
    return 1 << max(0, int(n) - 1).bit_length()


def sliced_i8(low, w, high, wh, scales, sw, bias, partials, group, hp, parts, static_weights=False):
    """bf16 partials [P, M, N] of a grouped INT8 projection on the current stream.

    ``static_weights=True`` promises that the kernel launched just before this one on the stream does not
    write ``w`` or ``wh``, so the GEMM may request its first weight tiles before it waits for that kernel
    (``reax_sliced_i8_static``)."""
    m, n = low.shape[0], w.shape[0]
    _native.require_cuda(low, w, scales, sw, bias, partials)
    for t in (low, w, high, wh, scales, sw, bias, partials):
        if t is not None and t.numel() and not t.is_contiguous():
            raise RuntimeError("sliced: operands must be contiguous")
    with torch.cuda.device(low.device):
        ws = _native.workspace(low.device)
        lib = _native.load()
        entry = lib.reax_sliced_i8_static if static_weights else lib.reax_sliced_i8
        _native.check(entry(
            low.data_ptr(), w.data_ptr(), _native.ptr(high) if hp else None, _native.ptr(wh) if hp else None,
            scales.data_ptr(), sw.data_ptr(), bias.data_ptr(), partials.data_ptr(), m, n, int(group), int(hp),
            int(parts), ws.data_ptr(), ws.numel(), _native.stream_handle(low.device)))
    return partials


class Native(NativeInt8):
    def prepare(self, x, p):
        low = torch.empty((len(x), p.parts * p.group), device=x.device, dtype=torch.int8)
        high = torch.empty((len(x), p.parts * p.hp), device=x.device, dtype=x.dtype)
        scales = torch.empty((p.parts, len(x)), device=x.device)
        prepare_kernel[(len(x), p.parts)](x, p.low_columns, p.high_columns, p.centers, p.smoothing,
                                          low, high, scales, M=len(x), K=p.width, G=p.group, HP=p.hp, P=p.parts,
                                          B=_next_pow2(p.group), BH=_next_pow2(max(1, p.hp)),
                                          num_warps=8, enable_fp_fusion=False)
        return low, high, scales

    def project(self, x, p, name, drop=0, reference=False):
        low, high, scales = self.prepare(x, p)
        m, n = len(x), len(p.low_weight)
        partials = torch.empty((p.parts, m, n), device=x.device, dtype=x.dtype)
        bm, sm, bn, threads = CONFIGS[name]
        assert n % bn == 0
        # the kernel just before the GEMM on the stream is prepare's quantizer, which writes no weights
        sliced_i8(low, p.low_weight, high, p.high_weight, scales, p.scales, p.bias, partials, p.group, p.hp, p.parts,
                  static_weights=True)
        if p.parts == 1:
            return partials[0]
        out = torch.empty((m, n), device=x.device, dtype=x.dtype)
        reduce_kernel[((m * n + 511) // 512,)](partials, out, TOTAL=m * n, P=p.parts, B=512,
                                               num_warps=4, enable_fp_fusion=False)
        return out
