"""Drop-in for the v3 production gate/up launcher ``private/snapshots/*/wide_warp_hybrid.py``.

The reference subclasses ``reaxv2.gate_up.Native`` with shape-specialised kernels named
``addressed_<i>_m<bm>n<bn>k<bk>`` and ``band_k<bk>_t<rows>n<bn>k<bk>``, all asserting the model's fixed
shape K=2432, KH=128, N=18432 (model-preaddressed-GUP-r1/wide_warp_hybrid.py:15-35); the activation-
table variant also builds and checks a 65536-entry SiLU table (model-addressed-bulk-activation-
table-r1/wide_warp_hybrid.py:11-17,41-49).  Here every such name runs the same B200 kernel.
"""
from __future__ import annotations

import re

import torch

from .. import _native
from .gate_up import Native as Original
from .gate_up import gate_up_i8

_NAME = re.compile(r"^(addressed_\d+_m\d+n\d+k\d+|band_k\d+_t\d+n\d+k\d+)$")


class Native(Original):
    def __init__(self, binary=None):
        super().__init__(binary)

    def product(self, x, w, xh, wh, sa, sw, bias, name, drop=0):
        m, k = x.shape
        n = len(w)
        kh = xh.shape[1]
        assert k == 2432 and kh == 128 and n == 18432
        if not _NAME.match(name):
            raise KeyError(name)
        return gate_up_i8(x, w, xh, wh, sa, sw, bias)

    def domain_check(self):
        """The epilogue's SiLU path against the direct formula, for every bf16 input pattern, as the
        reference's ``check_silu_domain`` compares its table with direct evaluation.  ``reax_silu_table``
        evaluates bf16(silu_f32(x)) directly for all 65536 patterns; ``silu_mul`` (times one) goes through
        what the GEMM epilogue uses: the shared-memory table for |x| in [2^-10, 128) and the closed forms
        outside it (tiny, large, infinite and NaN inputs).  The formula itself is pinned separately to the
        CPU oracle's correctly rounded SiLU (within 1 bf16 ulp on every pattern)."""
        table = torch.empty(65536, device="cuda", dtype=torch.bfloat16)
        with torch.cuda.device(table.device):
            _native.check(_native.load().reax_silu_table(table.data_ptr(), _native.stream_handle(table.device)))
            x = torch.arange(65536, device="cuda", dtype=torch.int32).to(torch.int16).view(torch.bfloat16)
            one = torch.ones_like(x)
            direct = torch.empty_like(x)
            _native.check(_native.load().reax_silu_mul(x.data_ptr(), one.data_ptr(), direct.data_ptr(), 1, 65536,
                                                        65536, 65536, _native.stream_handle(table.device)))
        torch.cuda.synchronize()
        assert torch.equal(direct.view(torch.int16), table.view(torch.int16))
        return {"BF16_input_patterns": 65536, "bit_identical": True}
