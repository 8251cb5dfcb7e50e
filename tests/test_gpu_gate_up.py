"""GPU parity of the fused INT8 gate/up + dequant + SwiGLU kernel against the CPU oracle.

INT8 path (KH == 0): the int32 accumulation and the float32 dequant are exact restatements, so the
bf16 output must be bit-identical to the oracle evaluated with the GPU's own SiLU table (the only
transcendental, expf, is CUDA's on the device).  Against the oracle's own correctly-rounded SiLU the
bound is the one north_star states: at most 1 bf16 ulp, with the max abs/rel error reported.
Hybrid banks (KH > 0) add BF16 outlier columns into the dequantized values 16 columns at a time, as
the reference does; the oracle restates that association with exact block sums (not the tensor
cores' rounding inside a block): at most 1 bf16 ulp, with the count of differing elements printed.
"""
import numpy as np
import pytest
import torch

from oracle import reax_oracle as ro
from tests import helpers as H

pytestmark = pytest.mark.gpu


def gpu_silu_table():
    from reax_engine_runtime_v3_b200 import _native
    t = torch.empty(65536, dtype=torch.bfloat16, device="cuda")
    _native.check(_native.load().reax_silu_table(t.data_ptr(), _native.stream_handle()))
    torch.cuda.synchronize()
    return H.bits(t)


_TABLE = None


def table():
    global _TABLE
    if _TABLE is None:
        _TABLE = gpu_silu_table()
    return _TABLE


def run_project(x, bank, name="hybrid8_b128n256_s64n256"):
    from reax_engine_runtime_v3_b200.reaxv2.gate_up import Native
    out = Native(None).project(x, bank, name)
    torch.cuda.synchronize()
    return out


def compare_int8(x, bank, rows=None, exact=True):
    """GPU project (quantize + gate/up) against the oracle's product of the GPU's own codes and scales.

    The quantizer is checked separately against the oracle (test_gpu_quant.py): its scale division
    follows Triton's fp32 '/' on the GPU, which differs from the oracle's IEEE division by <= 2 ulps
    on some rows; feeding the GPU's codes and scales makes every later step comparable bit for bit."""
    from reax_engine_runtime_v3_b200.reaxv2.gate_up import quantize_rows
    xd, bd = x.cuda(), H.bank_to(bank, "cuda")
    out = run_project(xd, bd)
    low, high, scales = quantize_rows(xd, bd)
    torch.cuda.synchronize()
    nb = H.bank_numpy(bank)
    sel = np.arange(x.shape[0]) if rows is None else rows
    low_g, high_g, sc_g = low.cpu().numpy()[sel], H.bits(high)[sel], scales.cpu().numpy()[sel]
    # quantizer: scales within the 2-ulp bound of the oracle's IEEE scales, codes exact for the GPU scales
    lo_o, hi_o, sc_o = ro.prepare_rows(H.bits(x)[sel], nb.low_columns, nb.high_columns, nb.smoothing, nb.centers,
                                       nb.centered)
    ulps = np.abs(sc_g.view(np.int32).astype(np.int64) - sc_o.view(np.int32).astype(np.int64))
    assert ulps.max(initial=0) <= 2
    assert np.array_equal(low_g[ulps == 0], lo_o[ulps == 0]) and np.array_equal(high_g, hi_o)
    got = H.bits(out)[sel]
    want_t = ro.gate_up_product(low_g, nb.low_weight, high_g, nb.high_weight, sc_g, nb.scales, nb.bias, table())
    want_c = ro.gate_up_product(low_g, nb.low_weight, high_g, nb.high_weight, sc_g, nb.scales, nb.bias)
    rep_t = H.ulp_report(got, want_t)
    rep_c = H.ulp_report(got, want_c)
    print("vs oracle(GPU silu table):", rep_t, "vs oracle(CPU silu):", rep_c)
    if exact:
        assert rep_t["n_diff"] == 0, rep_t
    assert rep_c["max_ulp"] <= 1, rep_c
    return out


@pytest.mark.parametrize("M", [16, 1, 17])
def test_cfg1_shape(M):
    """X [16, 1024] ~ N(0,1), Wg/Wu int8 [2816, 1024], scales U(1e-3, 1e-2)."""
    g = H.gen(1 + M)
    compare_int8(H.activations(g, M, 1024), H.int8_bank(g, 1024, 2816))


@pytest.mark.parametrize("M", [1, 8, 32, 64])
def test_cfg2_decode_full_size(M):
    """BASELINE config 2 at full size: K=4096, H=14336 (stream-K split over all SMs)."""
    g = H.gen(20 + M)
    compare_int8(H.activations(g, M, 4096), H.int8_bank(g, 4096, 14336))


@pytest.mark.parametrize("M,K,Hh", [(129, 512, 1024), (300, 1024, 8192), (1024, 512, 4096), (2048, 256, 4096),
                                    (4096, 384, 2560)])
def test_split_and_wave_shapes(M, K, Hh):
    """Tile counts below, between and above the SM count (data-parallel waves + stream-K remainder)."""
    g = H.gen(M + K + Hh)
    compare_int8(H.activations(g, M, K), H.int8_bank(g, K, Hh))


@pytest.mark.parametrize("M,K,Hh", [(5, 512, 4096), (33, 512, 10240), (64, 512, 28672), (17, 256, 18944),
                                    (8, 16384, 1792)])
def test_weight_major_plans(M, K, Hh):
    """Few tokens (weight-major tiles): short tiles of ceil(H / SMs) rows (H = 4096, K = 512), balanced
    tiles of ceil(H / SMs) rows with a short last tile and 24 tokens per warp (H = 10240, M = 33),
    balanced tiles over two waves (H = 28672), 128-row tiles filling exactly one wave of 148 SMs
    (H = 18944), and a long K on a small H, whose tiles are split over 8 CTAs (7 partials gathered)."""
    g = H.gen(7 * M + K + Hh)
    compare_int8(H.activations(g, M, K), H.int8_bank(g, K, Hh))


@pytest.mark.parametrize("M,K,Hh,sms", [(1, 4096, 1792, 74), (64, 4096, 1792, 74), (33, 2432, 1792, 0),
                                         (8, 640, 3584, 74), (64, 4096, 3584, 0), (16, 16384, 896, 0),
                                         (40, 2432, 896, 37)])
def test_multi_kblock_stages(M, K, Hh, sms):
    """Weight-major tiles of at most 64 gate rows stream several K blocks per pipeline stage (one 4-D copy
    of the tile's gate and up rows, one 3-D copy of its activation rows): the H shards of an 8- and a
    4-GPU job on one lane's share of 74 SMs (reax_set_stream_sms) and on the whole GPU, K = 2432 and
    640 (19 and 5 K blocks, so the last stage reaches past K and reads zeros), a long K over a small H,
    whose tiles are split by K at boundaries that are not multiples of the stage, and a share of 37 SMs."""
    from reax_engine_runtime_v3_b200 import _native
    g = H.gen(5 * M + K + Hh + sms)
    stream = torch.cuda.current_stream()
    if sms:
        _native.set_stream_sms(stream, sms)
    try:
        compare_int8(H.activations(g, M, K), H.int8_bank(g, K, Hh))
    finally:
        _native.set_stream_sms(stream, 0)


@pytest.mark.parametrize("M", [8, 200])
def test_silu_range_edges(M):
    """Gate values on both sides of every edge of the epilogue's SiLU table: column scales log-uniform
    over 1e-9 .. 1e-1 with zero bias put gates below 2^-10, inside [2^-10, 128) and at or above 128,
    mixed within warps, in weight-major (M = 8) and token-major (M = 200) tiles."""
    g = H.gen(77 + M)
    bank = H.int8_bank(g, 1024, 2816, bias=False)
    bank.scales = (10.0 ** (-9.0 + 8.0 * torch.rand(bank.scales.shape, generator=g))).float().contiguous()
    compare_int8(H.activations(g, M, 1024), bank)


@pytest.mark.parametrize("M,K,Hh,KH", [(1, 4096, 14336, 0), (64, 4096, 14336, 0), (300, 1024, 4096, 0),
                                       (200, 2560, 1024, 128)])
def test_project_entry_matches_two_calls(M, K, Hh, KH):
    """reax_project_i8 (the quantizer, then the GEMM requesting its first weight tiles while the quantizer
    runs) gives the bits of quantize_rows followed by gate_up_i8."""
    from reax_engine_runtime_v3_b200.reaxv2.gate_up import Native, gate_up_i8, quantize_rows
    g = H.gen(31 * M + K + Hh + KH)
    x = H.activations(g, M, K).cuda()
    bank = H.bank_to(H.int8_bank(g, K, Hh, KH=KH, centered=KH > 0), "cuda")
    fused = Native(None).project(x, bank, "hybrid8_b128n256_s64n256")
    low, high, sc = quantize_rows(x, bank)
    two = gate_up_i8(low, bank.low_weight, high, bank.high_weight, sc, bank.scales, bank.bias)
    torch.cuda.synchronize()
    assert torch.equal(fused.view(torch.int16), two.view(torch.int16))


@pytest.mark.parametrize("M", [1, 8])
def test_project_entry_repeated_status_clean(M):
    """Back-to-back project calls (the GEMM's weight producers start before its dependency wait and may
    lag the activation producer by whole stages) stay equal to the two-call path with no expired wait."""
    from reax_engine_runtime_v3_b200 import _native
    from reax_engine_runtime_v3_b200.reaxv2.gate_up import Native, gate_up_i8, quantize_rows
    g = H.gen(77 * M)
    bank = H.bank_to(H.int8_bank(g, 4096, 14336), "cuda")
    ws = _native.workspace(torch.device("cuda"))
    _native.clear_status(ws)
    xs = [H.activations(g, M, 4096).cuda() for _ in range(12)]
    outs = [Native(None).project(x, bank, "hybrid8_b128n256_s64n256") for x in xs]
    torch.cuda.synchronize()
    assert _native.read_status(ws) == 0
    for x, out in zip(xs, outs):
        low, high, sc = quantize_rows(x, bank)
        two = gate_up_i8(low, bank.low_weight, high, bank.high_weight, sc, bank.scales, bank.bias)
        assert torch.equal(out.view(torch.int16), two.view(torch.int16))


@pytest.mark.parametrize("M,Hh,KH", [(1, 14336, 0), (64, 14336, 0), (33, 1792, 0), (300, 2560, 128)])
def test_static_weights_entry_back_to_back(M, Hh, KH):
    """reax_gate_up_i8_static launched back to back (each launch streams its weights under the previous
    one's tail, over rotating banks) gives the bits of reax_gate_up_i8 with no expired wait."""
    from reax_engine_runtime_v3_b200 import _native
    from reax_engine_runtime_v3_b200.reaxv2.gate_up import gate_up_i8, quantize_rows
    g = H.gen(53 * M + Hh + KH)
    banks = [H.bank_to(H.int8_bank(g, 4096, Hh, KH=KH, centered=KH > 0), "cuda") for _ in range(2)]
    x = H.activations(g, M, 4096).cuda()
    low, high, sc = quantize_rows(x, banks[0])
    ws = _native.workspace(torch.device("cuda"))
    _native.clear_status(ws)
    outs = [gate_up_i8(low, b.low_weight, high, b.high_weight, sc, b.scales, b.bias, static_weights=True)
            for b in banks * 4]
    torch.cuda.synchronize()
    assert _native.read_status(ws) == 0
    for i, b in enumerate(banks):
        plain = gate_up_i8(low, b.low_weight, high, b.high_weight, sc, b.scales, b.bias)
        torch.cuda.synchronize()
        for out in outs[i::2]:
            assert torch.equal(out.view(torch.int16), plain.view(torch.int16))


@pytest.mark.parametrize("M,Hh", [(1, 1792), (64, 1792), (8, 3584), (33, 3584), (64, 7168)])
def test_rank_shard_shapes(M, Hh):
    """cfg2 as one rank of an H-sharded job sees it (K = 4096; H / 2, H / 4, H / 8 of 14336): few tiles,
    each split by K over several CTAs, with the finisher gathering their int32 partials."""
    from reax_engine_runtime_v3_b200 import _native
    ws = _native.workspace(torch.device("cuda"))
    _native.clear_status(ws)
    g = H.gen(5 * M + Hh)
    compare_int8(H.activations(g, M, 4096), H.int8_bank(g, 4096, Hh))
    assert _native.read_status(ws) == 0, _native.describe_status(_native.read_status(ws))


@pytest.mark.parametrize("M,K,Hh", [(512, 1024, 128), (513, 1024, 1024), (1000, 512, 2816), (2304, 2560, 1536),
                                    (777, 4096, 384)])
def test_cta_pair_tiles(M, K, Hh):
    """Many tokens without BF16 columns take CTA-pair tiles (256 token rows over two SMs, tcgen05
    cta_group::2): ragged last pair (one CTA of it wholly past M), fewer tiles than pairs, one n-tile."""
    g = H.gen(M * 3 + K + Hh)
    compare_int8(H.activations(g, M, K), H.int8_bank(g, K, Hh))


def test_cfg3_prefill_rows_sample():
    """BASELINE config 3 (M=4096, K=4096, H=14336): full GPU run, oracle on a sample of rows."""
    g = H.gen(3)
    rows = np.concatenate([np.arange(0, 64), np.arange(2000, 2040), np.arange(4096 - 64, 4096)])
    compare_int8(H.activations(g, 4096, 4096), H.int8_bank(g, 4096, 14336), rows=rows)


def test_cfg4_rank_shard_rows_sample():
    """BASELINE config 4 as one rank of its 8-way job sees it: X [8192, 8192] (the 256-thread quantizer),
    3584 gate rows and their up rows of an int8 [28672, 8192] bank, scales U(5e-4, 5e-3); full GPU run,
    oracle on a sample of rows."""
    g = H.gen(4)
    rows = np.concatenate([np.arange(0, 24), np.arange(4090, 4106), np.arange(8192 - 24, 8192)])
    compare_int8(H.activations(g, 8192, 8192), H.int8_bank(g, 8192, 3584, scale_lo=5e-4, scale_hi=5e-3), rows=rows)


def test_empty_batch():
    """M = 0: every entry point returns an empty result without launching (the runtime may call a
    bucket with no rows)."""
    from reax_engine_runtime_v3_b200.reaxv2.gate_up import gate_up_i8, quantize_rows
    from reax_engine_runtime_v3_b200.reaxv2.rotation import quantize_rotated
    g = H.gen(0)
    bank = H.bank_to(H.int8_bank(g, 1024, 512), "cuda")
    x = torch.zeros(0, 1024, dtype=torch.bfloat16, device="cuda")
    out = run_project(x, bank)
    assert out.shape == (0, 512)
    low, high, sc = quantize_rows(x, bank)
    assert low.shape == (0, 1024) and sc.shape == (0,)
    out2 = gate_up_i8(low, bank.low_weight, high, bank.high_weight, sc, bank.scales, bank.bias)
    assert out2.shape == (0, 512)
    rl, rs = quantize_rotated(x, torch.zeros(1024, device="cuda"), 512, 2, 512, 64)
    torch.cuda.synchronize()
    assert rl.shape == (0, 1024) and rs.shape == (2, 0)


def test_cfg5_outliers():
    """BASELINE config 5a: Student-t activations with 8 channels x50, buckets 128 / 512 / 2048."""
    g = H.gen(5)
    bank = H.int8_bank(g, 4096, 14336)
    for M in (128, 512):
        compare_int8(H.activations(g, M, 4096, "student"), bank, rows=np.arange(0, M, 3))


@pytest.mark.parametrize("M,K,Hh", [(200, 2560, 1024), (8, 2560, 10240), (40, 1280, 10240)])
def test_hybrid_bank_with_outlier_columns(M, K, Hh):
    """Production-style bank: centred, power-of-two smoothing, bias, 128 BF16 outlier columns.  Few
    tokens with BF16 columns take token-major tiles with a short activation box, and at H = 10240
    balanced tiles of ceil(H / SMs) gate rows (N = 2 x 72 per MMA)."""
    from reax_engine_runtime_v3_b200.reaxv2.gate_up import quantize_rows
    g = H.gen(11 + M)
    x = H.activations(g, M, K)
    bank = H.int8_bank(g, K, Hh, KH=128, centered=True, pow2_smoothing=True, bias=True)
    bd = H.bank_to(bank, "cuda")
    out = run_project(x.cuda(), bd)
    low, high, scales = quantize_rows(x.cuda(), bd)
    torch.cuda.synchronize()
    nb = H.bank_numpy(bank)
    got = H.bits(out)
    ops = (low.cpu().numpy(), nb.low_weight, H.bits(high), nb.high_weight, scales.cpu().numpy(), nb.scales, nb.bias)
    want = ro.gate_up_product(*ops, table())
    # The reference's own kernel on the same operands (when built): bit for bit.
    from oracle import ref_gpu
    if ref_gpu.available("native_hybrid8.cubin"):
        ref = ref_gpu.Hybrid8().product(low, bd.low_weight, high, bd.high_weight, scales, bd.scales, bd.bias,
                                        "hybrid8_b128n256_s64n256")
        torch.cuda.synchronize()
        rep_ref = H.ulp_report(got, H.bits(ref))
        print("against the reference kernel", rep_ref)
        assert rep_ref["n_diff"] == 0, rep_ref
    # The oracle restates the association (16-column blocks added into the dequantized values) with exact
    # block sums, not the tensor cores' rounding inside a block.  So each output must be the SwiGLU of a
    # gate and an up value within 1 bf16 ulp of the oracle's (the SiLU's slope can turn one ulp of the
    # gate into several of the output), except where the gate or up value nearly cancels (its float32
    # rounding errors exceed half a bf16 ulp of the value).
    g_bits, u_bits = ro.gate_up_pre_bits(*ops)
    near = np.zeros(got.shape, bool)
    for dg in (-1, 0, 1):
        for du in (-1, 0, 1):
            near |= got == ro.swiglu_bits((g_bits.astype(np.int32) + dg).astype(np.uint16),
                                          (u_bits.astype(np.int32) + du).astype(np.uint16), table())
    ill = ro.gate_up_ill_conditioned(*ops)
    rep = H.ulp_report(got, want)
    rep["not_within_1ulp_gate_up"] = int((~near).sum())
    rep["ill_conditioned"] = int(ill.sum())
    print("against the oracle", rep)
    assert (near | ill).all(), rep


def test_batch_invariance_first16():
    """The reference's screen invariant (resident_gate_up_screen.py:25-31): the first 16 rows computed
    alone equal rows 0..15 of the full batch, bit for bit."""
    g = H.gen(16)
    bank = H.bank_to(H.int8_bank(g, 4096, 14336), "cuda")
    x = H.activations(g, 768, 4096).cuda()
    full = run_project(x, bank)
    first = run_project(x[:16].contiguous(), bank)
    assert torch.equal(full[:16].view(torch.int16), first.view(torch.int16))


def test_repeat_calls_identical_and_status_clean():
    from reax_engine_runtime_v3_b200 import _native
    g = H.gen(17)
    bank = H.bank_to(H.int8_bank(g, 1024, 8192), "cuda")
    x = H.activations(g, 300, 1024).cuda()
    a = run_project(x, bank)
    b = run_project(x, bank)
    assert torch.equal(a.view(torch.int16), b.view(torch.int16))
    assert _native.read_status(_native.workspace(x.device)) == 0


def test_rejects_unsupported_shape():
    from reax_engine_runtime_v3_b200.reaxv2.gate_up import gate_up_i8
    a = torch.zeros(4, 100, dtype=torch.int8, device="cuda")
    w = torch.zeros(512, 100, dtype=torch.int8, device="cuda")
    f = torch.zeros(512, device="cuda")
    with pytest.raises(RuntimeError, match="KL"):
        gate_up_i8(a, w, None, None, torch.ones(4, device="cuda"), f, f)
