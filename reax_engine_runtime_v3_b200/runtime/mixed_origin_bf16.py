"""Drop-in for ``runtime/mixed_origin_bf16.py``: the BF16-weight gate/up projection.

Rows below ``split[0]`` follow the ``left`` split-K plan and the others the ``right`` plan (each
``{parts, chunk, mode}``, from the engine's pinned cuBLASLt algorithm).  ``Native.partials`` writes
one bf16 partial per K slice (bf16 of a float32 accumulation over the slice) with a tcgen05 kernel,
``fold`` sums a row's partials in slice order in float32 (runtime/mixed_origin_bf16.py:8-48).
``gate_up`` is the BF16-weight variant of the fused gate/up: the projection of [Wg; Wu] followed by
the engine's ``silu_mul`` rounding (vendor/s1eng/s1eng/fused.py:145-164); with one slice on both
origins it is a single kernel (``reax_gate_up_bf16``).
"""
from __future__ import annotations

import torch

from .. import _native
from ..reaxv2.driver import NativeInt8
from ..reaxv2.quantize import _GridLaunch


def _fold_launch(grid, parts, split, out, M=None, N=None, P0=None, P1=None, B=None, **_compile_options):
    _native.require_cuda(parts, split, out)
    with torch.cuda.device(out.device):
        _native.check(_native.load().reax_fold_partials(
            parts.data_ptr(), split.data_ptr(), out.data_ptr(), int(M), int(N), int(P0), int(P1),
            _native.stream_handle(out.device)))


fold = _GridLaunch(_fold_launch, "fold")


def reduction(core, shape, L, rows):
    """Split plan of the engine's pinned GEMM for (shape, L, rows) (runtime/mixed_origin_bf16.py:19-29)."""
    a = core.pinned.algo_r.get((*shape, L, rows), core.pinned.algo[(*shape, L)])
    if hasattr(a, "split"):
        p = max(1, a.split)
        mode = a.red
        chunk = a.chunk
    else:
        import reax_public.lt as lt  # the engine's cuBLASLt pin table
        cfg = lt.cfg_of(a)
        p = max(1, cfg.get("splitK", 1))
        mode = cfg.get("reduction", 0)
        chunk = ((shape[1] + p - 1) // p + 63) // 64 * 64
    assert mode in (0, 4), (shape, L, rows, mode)
    if p == 1:
        chunk = shape[1]
    return dict(parts=p, chunk=chunk, mode=mode)


def silu_mul(g, u, out=None):
    """``bf16(bf16(silu_f32(g)) * u)`` element-wise over 2-D row-strided views (fused.py:145-164)."""
    rows, cols = g.shape
    if out is None:
        out = torch.empty((rows, cols), device=g.device, dtype=torch.bfloat16)
    with torch.cuda.device(g.device):
        _native.check(_native.load().reax_silu_mul(
            g.data_ptr(), u.data_ptr(), out.data_ptr(), rows, cols, g.stride(0), u.stride(0),
            _native.stream_handle(g.device)))
    return out


def _split_tensor(split, device):
    if isinstance(split, torch.Tensor):
        return split
    return torch.tensor([int(split)], device=device, dtype=torch.int32)


class Native(NativeInt8):
    shapes = {"origin_m64n128": (64, 128, 128), "origin_m128n128": (128, 128, 256),
              "origin_m64n256": (64, 256, 256), "origin_m32n32": (32, 32, 64)}

    def __init__(self, binary=None):
        super().__init__(binary)

    def partials(self, x, w, split, left, right, name="origin_m64n128"):
        m, k = x.shape
        n = len(w)
        bm, bn, threads = self.shapes[name]
        p0, p1 = left["parts"], right["parts"]
        assert n % bn == 0 and k % 64 == 0 and x.is_contiguous() and w.is_contiguous()
        out = torch.empty((max(p0, p1), m, n), device=x.device, dtype=torch.bfloat16)
        split = _split_tensor(split, x.device)
        with torch.cuda.device(x.device):
            ws = _native.workspace(x.device)
            _native.check(_native.load().reax_bf16_partials(
                x.data_ptr(), w.data_ptr(), split.data_ptr(), out.data_ptr(), m, n, k, int(left["chunk"]),
                int(right["chunk"]), p0, p1, ws.data_ptr(), ws.numel(), _native.stream_handle(x.device)))
        return out

    def project(self, x, w, split, left, right, name="origin_m64n128"):
        parts = self.partials(x, w, split, left, right, name)
        m, n = parts.shape[1:]
        out = torch.empty((m, n), device=x.device, dtype=x.dtype)
        fold[((m * n + 511) // 512,)](parts, _split_tensor(split, x.device), out, M=m, N=n, P0=left["parts"],
                                      P1=right["parts"], B=512, num_warps=4, enable_fp_fusion=False)
        return out

    def gate_up(self, x, w, split=0, left=None, right=None, name="origin_m64n128", out=None):
        """BF16 gate/up + SwiGLU: bf16 [M, N2/2] from x bf16 [M, K] and w = [Wg; Wu] bf16 [N2, K]."""
        left = left or dict(parts=1, chunk=x.shape[1], mode=0)
        right = right or left
        m, k = x.shape
        n2 = len(w)
        if left["parts"] == 1 and right["parts"] == 1:
            assert k % 64 == 0 and x.is_contiguous() and w.is_contiguous()
            if out is None:
                out = torch.empty((m, n2 // 2), device=x.device, dtype=torch.bfloat16)
            with torch.cuda.device(x.device):
                ws = _native.workspace(x.device)
                _native.check(_native.load().reax_gate_up_bf16(
                    x.data_ptr(), w.data_ptr(), out.data_ptr(), m, n2, k, out.stride(0), ws.data_ptr(), ws.numel(),
                    _native.stream_handle(x.device)))
            return out
        gu = self.project(x, w, split, left, right, name)
        h = n2 // 2
        return silu_mul(gu[:, :h], gu[:, h:], out)
