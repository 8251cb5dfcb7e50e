"""Drop-in for ``reaxv2/rotation.py``: the rotated INT8 projection of the down projection.

``Native(matrices, prep, threads)`` wraps a grouped-projection ``Native`` (``reaxv2.sliced``) and
replaces its quantizer with the rotated one (reaxv2/rotation.py:5-30): per row and part, the centred
input columns are sign-flipped by a column hash and Walsh-Hadamard transformed on blocks of
``p.block`` values before the per-part INT8 quantization (kernel-source/legacy-v2/src/block_rotation.cu).
The projection itself is the grouped INT8 GEMM and its ordered fold, unchanged (``reaxv2.sliced``).
``threads`` and the cubin loader ``prep`` are accepted and kept for the reference's attribute layout;
the B200 kernel picks its own thread count.
"""
from __future__ import annotations

import torch

from .. import _native
from .sliced import Native as SlicedNative


def quantize_rotated(x, centers, chunk, parts, group, block):
    """(low int8 [M, parts*group], scales float32 [parts, M]) of the rotated quantizer on the current stream."""
    if x.dtype != torch.bfloat16 or not x.is_contiguous() or not centers.is_contiguous():
        raise RuntimeError("rotation: x must be contiguous bf16 and centers contiguous")
    _native.require_cuda(x, centers)
    m, k = x.shape
    low = torch.empty((m, parts * group), device=x.device, dtype=torch.int8)
    scales = torch.empty((parts, m), device=x.device, dtype=torch.float32)
    with torch.cuda.device(x.device):
        _native.check(_native.load().reax_quant_rotated(
            x.data_ptr(), centers.data_ptr(), low.data_ptr(), scales.data_ptr(), m, k, int(chunk), int(parts),
            int(group), int(block), _native.stream_handle(x.device)))
    return low, scales


class Native(SlicedNative):
    def __init__(self, matrices, prep, threads=128):
        self.__dict__.update(matrices.__dict__)
        self.prep = prep
        self.threads = threads

    def kernel_name(self, p):
        return f"rotation_g{p.group}_b{p.block}_t{self.threads}"

    def project(self, x, p, name, drop=0, reference=False):
        return super().project(x, p, selected_kernel(name, p), drop, reference=reference)

    def prepare(self, x, p):
        low, scales = quantize_rotated(x, p.centers, p.chunk, p.parts, p.group, p.block)
        high = torch.empty((len(x), 0), device=x.device, dtype=x.dtype)
        return low, high, scales


def selected_kernel(name, projection):
    """The grouped-projection route for a rotated projection (reaxv2/rotation.py:33-43), with the
    reference's checks and messages."""
    allowed = ("slice_m128n128", "slice_m64n128", "slice_m64n128w4", "slice_m128n256", "slice_m128n128k64")
    if name not in allowed:
        raise ValueError(f"Missing inner-loop contract for {name}")
    # Each INT8 MMA pipeline step consumes twice the named BF16 depth.
    depth = 64 if name.endswith("k64") else 32
    if projection.group % (2 * depth) == 0 and (not projection.hp or projection.hp % depth == 0):
        return name
    if name.endswith("k64") and projection.group % 64 == 0 and (not projection.hp or projection.hp % 32 == 0):
        return name[:-3]
    raise ValueError(f"Unsupported projection inner-loop alignment: {name}, group={projection.group}, "
                     f"high={projection.hp}")
