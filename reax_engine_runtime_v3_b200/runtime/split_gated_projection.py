"""Drop-in for the gate/up-path parts of ``runtime/split_gated_projection.py``.

``Prepared.project_ready`` projects an already-quantized activation through one bank (optionally
straight into a caller-supplied ``out``), and ``split_bank`` slices a grouped bank by output rows so
the GDN qkv and z branches can be launched separately (runtime/split_gated_projection.py:22-43,56-65).
The router that hooks these into the engine's GDN layer (``SplitRouter.context``) belongs to the
serving engine and is not part of this package.
"""
from __future__ import annotations

import copy

import torch

from ..reaxv2.sliced import CONFIGS
from ..reaxv2.sliced import Native as Sliced
from ..reaxv2.sliced import sliced_i8


class Prepared(Sliced):
    def __init__(self, original=None):
        if original is not None:
            self.__dict__.update(original.__dict__)
        else:
            Sliced.__init__(self)
        self.ready = None

    def prepare(self, x, p):
        assert self.ready is not None
        return self.ready

    def project_ready(self, x, p, ready, name, drop, out=None):
        assert self.ready is None
        if out is not None:
            assert p.parts == 1
            m, n = len(x), len(p.low_weight)
            bm, small, bn, threads = CONFIGS[name]
            assert n % bn == 0
            low, high, scales = ready
            sliced_i8(low, p.low_weight, high, p.high_weight, scales, p.scales, p.bias, out, p.group, p.hp, 1)
            return out
        self.ready = ready
        try:
            return Sliced.project(self, x, p, name, drop)
        finally:
            self.ready = None


_banks: dict = {}


def split_bank(p, begin, end):
    """Rows [begin, end) of a grouped bank: weight rows, and the matching columns of the [parts, N]
    ``scales`` and ``bias`` (runtime/split_gated_projection.py:56-65).  Cached per (bank, range)."""
    key = id(p), begin, end
    if key not in _banks:
        b = copy.copy(p)
        b.low_weight = p.low_weight[begin:end]
        b.high_weight = p.high_weight[begin:end]
        b.scales = p.scales[:, begin:end].contiguous()
        b.bias = p.bias[:, begin:end].contiguous()
        _banks[key] = (p, b)
    return _banks[key][1]


def project_split(x, p, count, name, drop=0, matrix=None):
    """Quantize once, then project the first ``count`` rows (qkv) and the rest (z) of bank ``p``
    separately, as the split router does: returns (qkv bf16 [M, count], z bf16 [M, N - count])."""
    matrix = matrix or Prepared()
    ready = Sliced.prepare(matrix, x, p)
    qkv = matrix.project_ready(x, split_bank(p, 0, count), ready, name, drop)
    zb = split_bank(p, count, len(p.low_weight))
    z = torch.empty((len(x), len(zb.low_weight)), device=x.device, dtype=x.dtype)
    matrix.project_ready(x, zb, ready, name, drop, out=z)
    return qkv, z

