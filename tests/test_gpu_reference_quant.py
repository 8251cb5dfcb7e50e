"""Our quantizers against the reference's own Triton quantizers run on the same B200.

``reaxv2/quantize.py``'s ``_prepare`` and ``prepare_kernel`` are compiled ahead of time for sm_100 by
``oracle/build_ref.py`` (unmodified source, the reference's launch options) and launched here on the
inputs our kernels get.  Codes, high columns and ``scales.view(uint32)`` must be bit-identical: no
ulp allowance.  Covered: every BASELINE config's rows (cfg1; cfg2 M = 1/8/32/64; cfg3 4096 x 4096;
cfg4 8192 x 8192; cfg5 Student-t buckets), the golden edge cases (ragged rows, zero rows, KL = 0,
BF16 outlier columns), a centred bank with power-of-two smoothing over [2^-8, 2^8], a bank with
non-power-of-two smoothing (so the reference's ``value /= sm`` division rounds), the v3 production
bank (K = 2560: 2432 INT8 + 128 BF16 columns), and the grouped quantizer.
"""
import os

import numpy as np
import pytest
import torch

from oracle import ref_gpu
from tests import helpers as H

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not ref_gpu.TritonQuantizer.available(ref_gpu.TritonQuantizer.prepare_name(4096, 4096, 0, 0)),
                                 reason="reference Triton quantizers not built (oracle/build_ref.py)")]

_Q = {}


def ref():
    if "q" not in _Q:
        _Q["q"] = ref_gpu.TritonQuantizer()
    return _Q["q"]


def bank_columns(g, K, KH, smoothing, centered):
    """low/high column maps and per-column smoothing/centres of a bank with KH BF16 columns."""
    perm = torch.randperm(K, generator=g)
    high = perm[:KH].sort().values
    keep = torch.ones(K, dtype=torch.bool)
    keep[high] = False
    low = keep.nonzero().flatten()
    KL = len(low)
    if smoothing == "one":
        sm = torch.ones(KL)
    elif smoothing == "pow2":          # the bank builder's 2^round(log2), clamped to [-8, 8]
        sm = 2.0 ** torch.randint(-8, 9, (KL,), generator=g).float()
    else:                              # not a power of two: the division rounds
        sm = 0.5 + 1.5 * torch.rand(KL, generator=g)
    centers = (torch.randn(KL, generator=g) * 0.1) if centered else torch.zeros(KL)
    dev = "cuda"
    return (low.to(torch.int32).to(dev), high.to(torch.int32).to(dev), sm.float().to(dev), centers.float().to(dev))


def ours_prepare(x, low_columns, high_columns, smoothing, centers, center):
    """The drop-in reaxv2.quantize._prepare, called exactly as reaxv2/gate_up.py:31-36 calls it."""
    from reax_engine_runtime_v3_b200.reaxv2 import quantize
    m, kl, kh = len(x), len(low_columns), len(high_columns)
    low = torch.empty((m, kl), device=x.device, dtype=torch.int8)
    high = torch.empty((m, kh), device=x.device, dtype=torch.bfloat16)
    scales = torch.empty(m, device=x.device)
    quantize._prepare[(m,)](x, low_columns, high_columns, smoothing, centers, low, high, scales, K=x.shape[1], KL=kl,
                            KH=kh, BL=None, BH=None, CENTER=center, num_warps=8, enable_fp_fusion=False)
    return low, high, scales


def assert_identical(x, low_columns, high_columns, smoothing, centers, center):
    got = ours_prepare(x, low_columns, high_columns, smoothing, centers, center)
    want = ref().prepare(x, low_columns, high_columns, smoothing, centers, center)
    torch.cuda.synchronize()
    assert torch.equal(got[0], want[0]), f"codes differ in {(got[0] != want[0]).sum().item()} places"
    assert torch.equal(got[1].view(torch.int16), want[1].view(torch.int16)), "high columns differ"
    d = (got[2].view(torch.int32) != want[2].view(torch.int32)).sum().item()
    assert d == 0, f"{d} scales differ"


@pytest.mark.parametrize("M,K,kind", [
    (16, 1024, "normal"),                                          # config 1
    (1, 4096, "normal"), (8, 4096, "normal"), (32, 4096, "normal"), (64, 4096, "normal"),   # config 2
    (4096, 4096, "normal"),                                        # config 3
    (8192, 8192, "normal"),                                        # config 4
    (128, 4096, "student"), (512, 4096, "student"), (2048, 4096, "student"),   # config 5
])
def test_prepare_matches_reference_triton_on_baseline_configs(M, K, kind):
    g = H.gen(M + K + len(kind))
    x = H.activations(g, M, K, kind).cuda()
    cols = bank_columns(g, K, 0, "one", False)
    assert_identical(x, *cols, False)


@pytest.mark.parametrize("smoothing,M", [("pow2", 64), ("pow2", 4096), ("real", 64), ("real", 1000)])
def test_prepare_matches_reference_triton_centred_smoothed(smoothing, M):
    """A centred bank whose smoothing spans [2^-8, 2^8] (exact division) or is not a power of two (the
    reference's '/' rounds: Triton's fp32 division)."""
    g = H.gen(900 + M + len(smoothing))
    x = H.activations(g, M, 4096, "student").cuda()
    assert_identical(x, *bank_columns(g, 4096, 0, smoothing, True), True)


@pytest.mark.parametrize("M,center", [(1, True), (37, True), (300, True), (2304, True), (64, False)])
def test_prepare_matches_reference_triton_production_bank(M, center):
    """The v3 production bank: K = 2560 of which 128 BF16 outlier columns (wide_warp_hybrid.py:17)."""
    g = H.gen(2560 + M)
    x = H.activations(g, M, 2560, "student").cuda()
    assert_identical(x, *bank_columns(g, 2560, 128, "pow2", center), center)


@pytest.mark.parametrize("case", ["cfg1", "ragged17", "outlier", "hybrid", "highonly", "zerorow"])
def test_prepare_matches_reference_triton_golden_cases(case):
    """The golden cases' inputs (tests/golden/gen_golden.py), through both kernels on the GPU."""
    gz = np.load(os.path.join(os.path.dirname(__file__), "golden", "reference_kernels.npz"))
    p = f"prepare_{case}_"
    x = H.from_bits(gz[p + "x"], "cuda")
    t = lambda k, dt: torch.from_numpy(np.ascontiguousarray(gz[p + k])).to(dt).cuda()
    assert_identical(x, t("low_columns", torch.int32), t("high_columns", torch.int32), t("smoothing", torch.float32),
                     t("centers", torch.float32), bool(gz[p + "center"]))


@pytest.mark.parametrize("M,K,G,HP,P", [(6, 1024, 512, 64, 2), (64, 2560, 1280, 64, 2), (300, 4096, 2048, 0, 2)])
def test_prepare_groups_matches_reference_triton(M, K, G, HP, P):
    """reaxv2.quantize.prepare_kernel with padded groups (-1 columns), centres and smoothing."""
    from reax_engine_runtime_v3_b200.reaxv2 import quantize
    g = H.gen(M + G + HP)
    x = H.activations(g, M, K, "student").cuda()
    perm = torch.randperm(K, generator=g)
    n_high = max(0, P * HP - 3)
    high = perm[:n_high]
    rest = perm[n_high:]
    low_columns = torch.full((P * G,), -1, dtype=torch.int32)
    half = min(len(rest) // 2, G - 5)
    low_columns[:half] = rest[:half].to(torch.int32)
    n2 = min(len(rest) - half, G - 7)
    low_columns[G:G + n2] = rest[half:half + n2].to(torch.int32)
    high_columns = torch.full((max(1, P * HP),), -1, dtype=torch.int32)[:P * HP]
    high_columns[:n_high] = high.to(torch.int32)
    centers = torch.randn(P * G, generator=g) * 0.05
    smoothing = 2.0 ** torch.randint(-4, 5, (P * G,), generator=g).float()
    low_columns, high_columns, centers, smoothing = (t.cuda() for t in (low_columns, high_columns, centers, smoothing))
    low = torch.empty(M, P * G, dtype=torch.int8, device="cuda")
    hi = torch.empty(M, P * HP, dtype=torch.bfloat16, device="cuda")
    scales = torch.empty(P, M, device="cuda")
    quantize.prepare_kernel[(M, P)](x, low_columns, high_columns, centers, smoothing, low, hi, scales, M=M, K=K, G=G,
                                    HP=HP, P=P, B=None, BH=None, num_warps=8, enable_fp_fusion=False)
    want = ref().prepare_groups(x, low_columns, high_columns, centers, smoothing, G, HP, P)
    torch.cuda.synchronize()
    assert torch.equal(low, want[0])
    assert torch.equal(hi.view(torch.int16), want[1].view(torch.int16))
    assert torch.equal(scales.view(torch.int32), want[2].view(torch.int32))
