"""GPU parity of the quantizers (a1, a2) against the CPU oracle and the reference-generated golden vectors.

Codes, high columns and scales are compared bit for bit.  The reference's Triton source divides with a
plain '/' where it computes the scale (reaxv2/quantize.py:19); on the GPU that division is done the way
Triton's NVIDIA backend lowers fp32 '/', while the oracle divides with IEEE rounding.  The helper
below therefore accepts a scale that differs from the oracle's only within the 2-ulp bound of that
division, and then requires the codes to equal the oracle's codes for the GPU's scale.
"""
import numpy as np
import pytest
import torch

from oracle import reax_oracle as ro
from tests import helpers as H

pytestmark = pytest.mark.gpu

GOLDEN = None


def golden():
    global GOLDEN
    if GOLDEN is None:
        import os
        GOLDEN = np.load(os.path.join(os.path.dirname(__file__), "golden", "reference_kernels.npz"))
    return GOLDEN


def f32_ulps(a, b):
    ia = np.asarray(a, np.float32).view(np.int32).astype(np.int64)
    ib = np.asarray(b, np.float32).view(np.int32).astype(np.int64)
    return np.abs(ia - ib)


def check_quant(low_gpu, high_gpu, scales_gpu, x_bits, low_columns, high_columns, smoothing, centers, center):
    low_o, high_o, scales_o = ro.prepare_rows(x_bits, low_columns, high_columns, smoothing, centers, center)
    assert np.array_equal(high_gpu, high_o)
    d = f32_ulps(scales_gpu, scales_o)
    assert d.max(initial=0) <= 2, f"scale differs by {d.max()} ulps"
    if len(low_columns):
        v = ro.bf16_to_f32(np.asarray(x_bits)[:, np.asarray(low_columns, np.int64)])
        if center:
            v = v - np.asarray(centers, np.float32)[None, :]
        v = (v / np.asarray(smoothing, np.float32)[None, :]).astype(np.float32)
        assert np.array_equal(low_gpu, ro.quant_codes(v, scales_gpu))
    exact_rows = int((d == 0).sum())
    return exact_rows, int(d.size)


def run_prepare(x, bank):
    from reax_engine_runtime_v3_b200.reaxv2.gate_up import quantize_rows
    low, high, scales = quantize_rows(x, bank)
    torch.cuda.synchronize()
    return low.cpu().numpy(), H.bits(high), scales.cpu().numpy()


@pytest.mark.parametrize("case", ["cfg1", "ragged17", "outlier", "hybrid", "highonly", "zerorow"])
def test_prepare_rows_vs_reference_golden(case):
    g = {k[len(f"prepare_{case}_"):]: golden()[k] for k in golden().files if k.startswith(f"prepare_{case}_")}
    from types import SimpleNamespace
    dev = torch.device("cuda")
    bank = SimpleNamespace(width=g["x"].shape[1], centered=bool(g["center"]),
                           low_columns=torch.from_numpy(g["low_columns"]).to(dev),
                           high_columns=torch.from_numpy(g["high_columns"]).to(dev),
                           smoothing=torch.from_numpy(g["smoothing"]).to(dev),
                           centers=torch.from_numpy(g["centers"]).to(dev))
    x = H.from_bits(g["x"], dev)
    low, high, scales = run_prepare(x, bank)
    assert np.array_equal(high, g["high"])
    check_quant(low, high, scales, g["x"], g["low_columns"], g["high_columns"], g["smoothing"], g["centers"],
                bool(g["center"]))


@pytest.mark.parametrize("M,K,kind", [(16, 1024, "normal"), (1, 4096, "normal"), (64, 4096, "normal"),
                                      (2048, 4096, "student"), (333, 8192, "normal")])
def test_prepare_rows_baseline_shapes(M, K, kind):
    gen = H.gen(100 + M)
    x = H.activations(gen, M, K, kind)
    bank = H.int8_bank(gen, K, 128)
    low, high, scales = run_prepare(x.cuda(), H.bank_to(bank, "cuda"))
    nb = H.bank_numpy(bank)
    exact, n = check_quant(low, high, scales, H.bits(x), nb.low_columns, nb.high_columns, nb.smoothing, nb.centers,
                           False)
    print(f"scales bit-equal to the IEEE oracle: {exact}/{n}")


@pytest.mark.parametrize("M,K,KH,centered", [(1, 4096, 128, True), (7, 2603, 40, True), (148, 4096, 0, False),
                                              (3, 9000, 16, False), (2, 40000, 0, False)])
def test_prepare_rows_few_rows_edges(M, K, KH, centered):
    """Decode-sized row counts with production-style banks: a ragged tail (KL % 8 != 0, unaligned x),
    centred power-of-two smoothing with BF16 high columns, and a row longer than the codes the
    registers hold (the second pass recomputes the values past them)."""
    gen = H.gen(300 + M + K)
    x = H.activations(gen, M, K)
    bank = H.int8_bank(gen, K, 128, KH=KH, centered=centered, pow2_smoothing=True)
    low, high, scales = run_prepare(x.cuda(), H.bank_to(bank, "cuda"))
    nb = H.bank_numpy(bank)
    check_quant(low, high, scales, H.bits(x), nb.low_columns, nb.high_columns, nb.smoothing, nb.centers, centered)


@pytest.mark.parametrize("M,K,KH,centered", [(1000, 4096, 128, True), (700, 6003, 16, True), (600, 9000, 0, False)])
def test_prepare_rows_many_rows(M, K, KH, centered):
    """Prefill-sized row counts take narrower CTAs (128 threads up to 4096 low columns, 256 up to 8192,
    512 past that), with BF16 high columns, a ragged tail and centring."""
    gen = H.gen(500 + M + K)
    x = H.activations(gen, M, K)
    bank = H.int8_bank(gen, K, 128, KH=KH, centered=centered, pow2_smoothing=True)
    low, high, scales = run_prepare(x.cuda(), H.bank_to(bank, "cuda"))
    nb = H.bank_numpy(bank)
    check_quant(low, high, scales, H.bits(x), nb.low_columns, nb.high_columns, nb.smoothing, nb.centers, centered)


@pytest.mark.parametrize("M", [3, 700])
def test_prepare_rows_rounding_ties(M):
    """Quotients on and next to half-integers: with absmax 127 the scale is 1, so k + 0.5 values are exact
    ties (round half to even) and values one bf16 step away sit just inside or outside them; rows with
    other absmax values put quotients within a few ulps of half-integers.  The codes must follow
    nearbyint(div_rn) exactly (the kernel multiplies by the reciprocal and divides only near ties)."""
    from types import SimpleNamespace
    K = 512
    half = np.arange(-126, 127, dtype=np.float32) + np.float32(0.5)
    base = np.concatenate([[127.0], half, np.nextafter(half, np.float32(200)), np.nextafter(half, np.float32(-200))])
    base = base.astype(np.float32)[:K]
    rows = []
    g = np.random.default_rng(M)
    for r in range(M):
        row = np.zeros(K, np.float32)
        row[:len(base)] = base * (1.0 if r % 2 == 0 else np.float32(1.0 + 2.0 ** -(8 + r % 7)))
        row[len(base):] = g.standard_normal(K - len(base)).astype(np.float32)
        rows.append(row)
    x_bits = ro.f32_to_bf16(np.stack(rows))
    dev = torch.device("cuda")
    bank = SimpleNamespace(width=K, centered=False, low_columns=torch.arange(K, dtype=torch.int32, device=dev),
                           high_columns=torch.zeros(0, dtype=torch.int32, device=dev),
                           smoothing=torch.ones(K, device=dev), centers=torch.zeros(K, device=dev))
    low, high, scales = run_prepare(H.from_bits(x_bits, dev), bank)
    check_quant(low, high, scales, x_bits, np.arange(K), np.zeros(0, np.int64), np.ones(K, np.float32),
                np.zeros(K, np.float32), False)


def test_prepare_groups_vs_reference_golden():
    G = golden()
    M, K, P, Gs, HP = (int(v) for v in G["groups_shape"])
    dev = torch.device("cuda")
    from reax_engine_runtime_v3_b200.reaxv2.quantize import prepare_kernel
    x = H.from_bits(G["groups_x"], dev)
    low = torch.empty(M, P * Gs, dtype=torch.int8, device=dev)
    high = torch.empty(M, P * HP, dtype=torch.bfloat16, device=dev)
    scales = torch.empty(P, M, device=dev)
    prepare_kernel[(M, P)](x, torch.from_numpy(G["groups_low_columns"]).to(dev),
                           torch.from_numpy(G["groups_high_columns"]).to(dev), torch.from_numpy(G["groups_centers"]).to(dev),
                           torch.from_numpy(G["groups_smoothing"]).to(dev), low, high, scales, M=M, K=K, G=Gs, HP=HP, P=P,
                           B=512, BH=64, num_warps=8, enable_fp_fusion=False)
    torch.cuda.synchronize()
    assert np.array_equal(H.bits(high), G["groups_high"])
    d = f32_ulps(scales.cpu().numpy(), G["groups_scales"])
    assert d.max() <= 2
    # codes for the GPU's own scales
    lc = G["groups_low_columns"].reshape(P, Gs)
    xb = G["groups_x"]
    want = np.zeros((M, P * Gs), np.int8)
    for p in range(P):
        src = lc[p]
        raw = ro.bf16_to_f32(xb[:, np.maximum(src, 0)])
        v = np.where(src[None, :] >= 0, (raw - G["groups_centers"].reshape(P, Gs)[p]) / G["groups_smoothing"].reshape(P, Gs)[p],
                     np.float32(0)).astype(np.float32)
        want[:, p * Gs:(p + 1) * Gs] = ro.quant_codes(v, scales.cpu().numpy()[p], clamp=False)
    assert np.array_equal(low.cpu().numpy(), want)


def test_quantizer_is_deterministic_and_batch_invariant():
    gen = H.gen(7)
    x = H.activations(gen, 300, 4096).cuda()
    bank = H.bank_to(H.int8_bank(gen, 4096, 128), "cuda")
    a = run_prepare(x, bank)
    b = run_prepare(x[:16].contiguous(), bank)
    assert np.array_equal(a[0][:16], b[0]) and np.array_equal(a[2][:16], b[2])


def test_scale_division_is_tritons_fp32_division_exhaustive():
    """The reference computes the scale as ``tl.maximum(amax, 1e-12) / 127.`` in Triton
    (reaxv2/quantize.py:19).  With smoothing 1 and no centre, amax is a bf16 value, so all 32768
    non-negative finite bf16 amax values cover the domain: one row per value, the quantizer's scale
    must equal Triton's fp32 '/' of the same expression on this GPU bit for bit.  (IEEE division
    differs on part of the domain; the count is printed.)"""
    triton = pytest.importorskip("triton")
    import triton.language as tl

    @triton.jit
    def scale_expr(a, o, n, B: tl.constexpr):
        i = tl.program_id(0) * B + tl.arange(0, B)
        m = i < n
        v = tl.load(a + i, mask=m, other=1.0)
        tl.store(o + i, tl.maximum(v, 1.e-12) / 127., mask=m)

    patterns = torch.arange(0, 0x7F80, dtype=torch.int32)        # +0 .. largest finite bf16
    amax = patterns.to(torch.int16).view(torch.bfloat16)
    M = amax.numel()
    x = torch.zeros(M, 8, dtype=torch.bfloat16)
    x[:, 3] = amax
    from types import SimpleNamespace
    dev = torch.device("cuda")
    bank = SimpleNamespace(width=8, centered=False, low_columns=torch.arange(8, dtype=torch.int32, device=dev),
                           high_columns=torch.zeros(0, dtype=torch.int32, device=dev),
                           smoothing=torch.ones(8, device=dev), centers=torch.zeros(8, device=dev))
    low, high, scales = run_prepare(x.to(dev), bank)
    a32 = amax.float().to(dev)
    tri = torch.empty_like(a32)
    scale_expr[(triton.cdiv(M, 1024),)](a32, tri, M, B=1024, enable_fp_fusion=False)
    torch.cuda.synchronize()
    tri = tri.cpu().numpy()
    assert np.array_equal(scales.view(np.uint32), tri.view(np.uint32))
    ieee = ro.quant_scale(amax.float().numpy())
    print(f"scales differing from IEEE division: {int((ieee != tri).sum())} of {M}")


@pytest.mark.parametrize("M,K", [(4096, 4096), (1000, 8192), (700, 3072), (5, 1024), (1500, 2048)])
def test_dense_quantizer_matches_the_mapped_one(M, K):
    """A dense bank (low column c is column c, unit smoothing, no centring) may be quantized with NULL
    maps, which selects the library's dense kernel; its codes and scales are the mapped quantizer's bit
    for bit, on rows of N(0,1) values, all-zero rows, rows with +-inf or NaN, huge and tiny values and
    exact half-integer quotients."""
    from reax_engine_runtime_v3_b200 import _native
    g = H.gen(41 * M + K)
    x = torch.randn(M, K, generator=g)
    x[1] = 0.0
    if M > 8:
        x[2, 7] = float("inf")
        x[3, 11] = float("-inf")
        x[4, 5] = float("nan")
        x[5] *= 1e30
        x[6] *= 1e-30
        x[7] = torch.arange(K, dtype=torch.float32) % 255 - 127.0 + 0.5
        x[7, 0] = 127.0
    xb = x.to(torch.bfloat16).cuda()
    dev = xb.device
    lib = _native.load()
    cols = torch.arange(K, dtype=torch.int32, device=dev)
    ones = torch.ones(K, device=dev)
    outs = []
    for dense in (False, True):
        low = torch.empty(M, K, dtype=torch.int8, device=dev)
        scales = torch.empty(M, device=dev)
        _native.check(lib.reax_quant_rows(xb.data_ptr(), None if dense else cols.data_ptr(), None,
                                          None if dense else ones.data_ptr(), None, low.data_ptr(), None,
                                          scales.data_ptr(), M, K, K, 0, 0, _native.stream_handle(dev)))
        outs.append((low, scales))
    torch.cuda.synchronize()
    (lm, sm), (ld, sd) = outs
    assert torch.equal(lm, ld)
    assert torch.equal(sm.view(torch.int32), sd.view(torch.int32))


def test_project_on_a_dense_bank_takes_the_dense_quantizer_with_the_same_bits():
    """Native.project on a dense bank with prefill-sized rows (the dense quantizer behind reax_project_i8)
    gives the bits of the mapped quantizer followed by the GEMM."""
    from reax_engine_runtime_v3_b200.reaxv2 import gate_up as G
    g = H.gen(8800)
    M, K, Hh = 1200, 4096, 1792
    x = H.activations(g, M, K).cuda()
    bank = H.bank_to(H.int8_bank(g, K, Hh), "cuda")
    assert G._dense_bank(bank)
    out = G.Native(None).project(x, bank, "hybrid8_b128n256_s64n256")
    low, high, sc = G.quantize_rows(x, bank)
    two = G.gate_up_i8(low, bank.low_weight, high, bank.high_weight, sc, bank.scales, bank.bias)
    torch.cuda.synchronize()
    assert torch.equal(out.view(torch.int16), two.view(torch.int16))
