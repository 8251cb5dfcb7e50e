"""Drop-in for ``reaxv2/quantize.py``: the three Triton kernels, launched the Triton way.

``_prepare[(M,)](...)``, ``prepare_kernel[(M, P)](...)`` and ``reduce_kernel[(g,)](...)`` keep the
reference's positional arguments and keyword constants (reaxv2/quantize.py:5-61, call sites
reaxv2/gate_up.py:34-36 and reaxv2/sliced.py:14-17,45-46); each launch goes to a hand-written CUDA
kernel of ``libreax_b200.so`` on the current stream.  Block-size and compiler keywords (``BL``,
``BH``, ``B``, ``num_warps``, ``enable_fp_fusion``) are accepted and have no effect.
"""
from __future__ import annotations

import torch

from .. import _native


class _GridLaunch:
    """``kernel[grid](*args, **constexprs)`` call syntax of a Triton kernel."""

    def __init__(self, fn, name):
        self._fn = fn
        self.__name__ = name

    def __getitem__(self, grid):
        grid = tuple(grid) if isinstance(grid, (tuple, list)) else (grid,)
        return lambda *args, **kwargs: self._fn(grid, *args, **kwargs)


def _prepare_launch(grid, x, low_columns, high_columns, smoothing, centers, low, high, scales, K=None, KL=None,
                    KH=None, BL=None, BH=None, CENTER=False, **_compile_options):
    """Per-token INT8 quantization, one row per program (reaxv2/quantize.py:5-29)."""
    M = int(grid[0])
    _native.require_cuda(x, low, scales)
    if x.dtype != torch.bfloat16 or not x.is_contiguous():
        raise RuntimeError("_prepare: x must be a contiguous bfloat16 tensor")
    K = int(K) if K is not None else x.shape[1]
    KL = int(KL) if KL is not None else len(low_columns)
    KH = int(KH) if KH is not None else len(high_columns)
    if M > x.shape[0] or low.numel() < M * KL or scales.numel() < M or (KH and high.numel() < M * KH):
        raise RuntimeError("_prepare: output tensors smaller than the grid")
    with torch.cuda.device(x.device):
        _native.check(_native.load().reax_quant_rows(
            x.data_ptr(), _native.ptr(low_columns), _native.ptr(high_columns), _native.ptr(smoothing),
            _native.ptr(centers), _native.ptr(low), _native.ptr(high), scales.data_ptr(), M, K, KL, KH,
            1 if CENTER else 0, _native.stream_handle(x.device)))


def _prepare_groups_launch(grid, x, low_columns, high_columns, center, smoothing, low, high, scales, M=None, K=None,
                           G=None, HP=None, P=None, B=None, BH=None, **_compile_options):
    """Grouped quantization, grid (M, P) (reaxv2/quantize.py:31-52)."""
    _native.require_cuda(x, low, scales)
    if x.dtype != torch.bfloat16 or not x.is_contiguous():
        raise RuntimeError("prepare_kernel: x must be a contiguous bfloat16 tensor")
    M = int(M) if M is not None else int(grid[0])
    P = int(P) if P is not None else int(grid[1])
    with torch.cuda.device(x.device):
        _native.check(_native.load().reax_quant_groups(
            x.data_ptr(), _native.ptr(low_columns), _native.ptr(high_columns), _native.ptr(center),
            _native.ptr(smoothing), _native.ptr(low), _native.ptr(high), scales.data_ptr(), M, int(K), int(G),
            int(HP), P, _native.stream_handle(x.device)))


def _reduce_launch(grid, partials, out, TOTAL=None, P=None, B=None, **_compile_options):
    """Ordered float32 sum of P bf16 partials (reaxv2/quantize.py:55-61)."""
    _native.require_cuda(partials, out)
    with torch.cuda.device(out.device):
        _native.check(_native.load().reax_reduce_partials(
            partials.data_ptr(), out.data_ptr(), int(TOTAL), int(P), _native.stream_handle(out.device)))


_prepare = _GridLaunch(_prepare_launch, "_prepare")
prepare_kernel = _GridLaunch(_prepare_groups_launch, "prepare_kernel")
reduce_kernel = _GridLaunch(_reduce_launch, "reduce_kernel")
