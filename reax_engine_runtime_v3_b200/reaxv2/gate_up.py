"""Drop-in for ``reaxv2/gate_up.py``: the hybrid INT8/BF16 gate/up + SwiGLU operator.

``Native.project(x, p, name, drop)`` quantizes the activations and runs the product in one library call
(``reax_project_i8``); ``product`` launches one tcgen05 kernel (``reax_gate_up_i8``) that computes the int32 INT8 GEMM of the gate and
up rows, dequantizes ``((acc * sa[row]) * sw[col]) + bias[col]``, adds the BF16 outlier columns and
writes ``bf16(silu(g)) * u`` as bf16 (reference: reaxv2/gate_up.py:11-37 and
kernel-source/legacy-v2/src/native_hybrid8.cu:4-28).

``name`` selects one of the reference's tile configurations; every name in ``CONFIGS`` is accepted
(with the reference's divisibility assert on its N tile) and runs the same B200 kernel, whose own
tiling and split are planned from the shape.  ``drop`` (the count of big-tile row bands the reference
demotes to small tiles) is a scheduling hint of the old kernels and is accepted and ignored.
"""
from __future__ import annotations

import torch

from .. import _native
from .driver import NativeInt8
from .quantize import _prepare

# Kernel names and (big rows, small rows, N tile, dynamic smem) of the reference's hybrid8_* kernels
# (reaxv2/gate_up.py:8); only the N tile enters the precondition check below.
CONFIGS = {
    "hybrid8_b128n256_s64n256": (128, 64, 256, 98304),
    "hybrid8_b64n256_s32n256": (64, 32, 256, 81920),
    "hybrid8_b128n128_s32n128": (128, 32, 128, 98304),
    "hybrid8_b128n256k32_s32n256k32": (128, 32, 256, 73728),
    "hybrid8_b64n128k64_s32n128k64": (64, 32, 128, 49152),
    "hybrid8_b64n128k32_s32n128k32": (64, 32, 128, 36864),
    "hybrid8_b64n128k32_min2": (64, 32, 128, 36864),
    "hybrid8_b32n128k32w4_min3": (32, 16, 128, 30720),
}


# Banks known to be dense: their low columns are every column in order and their smoothing is all ones (every
# BASELINE bank).  Keyed by the maps' device addresses; checked once per bank, outside stream capture.
_DENSE: dict = {}
# rows per SM from which project() takes the dense quantizer (fewer rows keep the decode quantizer, one wide
# CTA per row, whose latency is shorter)
_DENSE_MIN_ROWS_PER_SM = 4


def _dense_bank(p) -> bool:
    """Whether the quantizer may treat the bank as dense (reax_quant_rows with NULL maps): no high columns, no
    centring, low columns 0..K-1 in order and unit smoothing.  The first call per bank compares the maps on
    the device (one synchronization); under stream capture an unchecked bank counts as not dense."""
    if len(p.high_columns) or p.centered or len(p.low_columns) != p.width:
        return False
    key = (p.low_columns.data_ptr(), p.smoothing.data_ptr(), p.width)
    hit = _DENSE.get(key)
    if hit is None:
        if torch.cuda.is_current_stream_capturing():
            return False
        cols = torch.arange(p.width, device=p.low_columns.device, dtype=p.low_columns.dtype)
        hit = bool(torch.equal(p.low_columns, cols)) and bool((p.smoothing == 1.0).all())
        _DENSE[key] = hit
    return hit


def _next_pow2(n: int) -> int:
    return 1 << max(0, int(n) - 1).bit_length()


def gate_up_i8(x, w, xh, wh, sa, sw, bias, out=None, static_weights=False):
    """INT8 gate/up + dequant + SwiGLU on the current stream; returns bf16 [M, N2/2] (or fills ``out``).

    ``static_weights=True`` promises that the kernel launched just before this one on the stream does not
    write ``w`` or ``wh``; the GEMM then starts its weight stream before waiting for that kernel
    (``reax_gate_up_i8_static``)."""
    m, kl = x.shape
    n2 = w.shape[0]
    kh = xh.shape[1] if xh is not None else 0
    _native.require_cuda(x, w, sa, sw, bias)
    if x.dtype != torch.int8 or w.dtype != torch.int8:
        raise RuntimeError("gate_up: codes and weights must be int8")
    for t in (x, w, xh, wh, sa, sw, bias):
        if t is not None and not t.is_contiguous():
            raise RuntimeError("gate_up: operands must be contiguous")
    if out is None:
        out = torch.empty((m, n2 // 2), device=x.device, dtype=torch.bfloat16)
    with torch.cuda.device(x.device):
        ws = _native.workspace(x.device)
        lib = _native.load()
        entry = lib.reax_gate_up_i8_static if static_weights else lib.reax_gate_up_i8
        _native.check(entry(
            x.data_ptr(), w.data_ptr(), _native.ptr(xh) if kh else None, _native.ptr(wh) if kh else None,
            sa.data_ptr(), sw.data_ptr(), bias.data_ptr(), out.data_ptr(), m, n2, kl, kh, out.stride(0),
            ws.data_ptr(), ws.numel(), _native.stream_handle(x.device)))
    return out


def quantize_rows(x, p):
    """``_prepare`` of ``Native.project`` (reaxv2/gate_up.py:30-36): returns (low int8, high bf16, scales f32)."""
    m = len(x)
    kl, kh = len(p.low_columns), len(p.high_columns)
    low = torch.empty((m, kl), device=x.device, dtype=torch.int8)
    high = torch.empty((m, kh), device=x.device, dtype=torch.bfloat16)
    scales = torch.empty(m, device=x.device)
    _prepare[(m,)](x, p.low_columns, p.high_columns, p.smoothing, p.centers, low, high, scales,
                   K=p.width, KL=kl, KH=kh, BL=_next_pow2(kl), BH=_next_pow2(kh),
                   CENTER=p.centered, num_warps=8, enable_fp_fusion=False)
    return low, high, scales


def project_quantizer(x, p):
    """The quantizer as ``Native.project`` runs it: the dense kernel (NULL maps) for many rows of a dense bank,
    else ``quantize_rows``.  Returns (low int8, high bf16, scales f32); the same bits either way."""
    m = len(x)
    if not _uses_dense(x, p, m):
        return quantize_rows(x, p)
    k = p.width
    low = torch.empty((m, k), device=x.device, dtype=torch.int8)
    high = torch.empty((m, 0), device=x.device, dtype=torch.bfloat16)
    scales = torch.empty(m, device=x.device)
    with torch.cuda.device(x.device):
        _native.check(_native.load().reax_quant_rows(x.data_ptr(), None, None, None, None, low.data_ptr(), None,
                                                     scales.data_ptr(), m, k, k, 0, 0, _native.stream_handle(x.device)))
    return low, high, scales


def _uses_dense(x, p, m) -> bool:
    """Whether project() quantizes these rows with the dense kernel."""
    return (m > _DENSE_MIN_ROWS_PER_SM * _native.sm_count(x.device) and p.width % 1024 == 0 and p.width <= 8192
            and _dense_bank(p))


class Native(NativeInt8):
    def tile_n(self, name):
        return CONFIGS[name][2]

    def product(self, x, w, xh, wh, sa, sw, bias, name, drop=0):
        m, k = x.shape
        n = len(w)
        kh = xh.shape[1]
        bn = self.tile_n(name)
        assert k % 128 == 0 and kh % 64 == 0 and n % bn == 0
        return gate_up_i8(x, w, xh, wh, sa, sw, bias)

    def project(self, x, p, name, drop=0):
        """quantize_rows + product in one library call (``reax_project_i8``), which lets the GEMM start
        loading weights while the quantizer runs; same results as the two calls."""
        m = len(x)
        kl, kh = len(p.low_columns), len(p.high_columns)
        n2 = len(p.low_weight)
        assert kl % 128 == 0 and kh % 64 == 0 and n2 % self.tile_n(name) == 0
        _native.require_cuda(x, p.low_weight, p.scales, p.bias)
        if x.dtype != torch.bfloat16:
            raise RuntimeError("project: x must be a bfloat16 tensor")
        for t in (x, p.low_columns, p.high_columns, p.smoothing, p.centers, p.low_weight, p.high_weight, p.scales,
                  p.bias):
            if t is not None and not t.is_contiguous():
                raise RuntimeError("project: operands must be contiguous")
        low = torch.empty((m, kl), device=x.device, dtype=torch.int8)
        high = torch.empty((m, kh), device=x.device, dtype=torch.bfloat16)
        scales = torch.empty(m, device=x.device)
        out = torch.empty((m, n2 // 2), device=x.device, dtype=torch.bfloat16)
        # many rows of a dense bank: the maps are passed as NULL, which selects the library's dense quantizer
        # (same codes and scales; plain 16-byte row loads instead of staged maps and gathers)
        dense = _uses_dense(x, p, m)
        with torch.cuda.device(x.device):
            ws = _native.workspace(x.device)
            _native.check(_native.load().reax_project_i8(
                x.data_ptr(), None if dense else p.low_columns.data_ptr(), _native.ptr(p.high_columns) if kh else None,
                None if dense else p.smoothing.data_ptr(), _native.ptr(p.centers), 1 if p.centered else 0,
                p.low_weight.data_ptr(),
                _native.ptr(p.high_weight) if kh else None, p.scales.data_ptr(), p.bias.data_ptr(), low.data_ptr(),
                _native.ptr(high) if kh else None, scales.data_ptr(), out.data_ptr(), m, p.width, kl, kh, n2,
                out.stride(0), ws.data_ptr(), ws.numel(), _native.stream_handle(x.device)))
        return out
