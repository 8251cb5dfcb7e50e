"""Our kernels against the reference's own kernels, compiled from source for sm_100a (oracle/_ref) and
run on the same B200 with the same inputs.

INT8 gate/up with KH == 0 and the grouped projection with HP == 0: bit-identical outputs (same int32
sums, same float32 dequant, same bf16 rounding points, the same CUDA expf in the SiLU).  With BF16
outlier columns both kernels add the BF16 products into the dequantized float32 values 16 columns at a
time in ascending order (mma.sync.m16n8k16 there, tcgen05.mma kind::f16 here): at most 1 bf16 ulp,
with the count of differing elements printed.
"""
import numpy as np
import pytest
import torch

from oracle import ref_gpu
from oracle import reax_oracle as ro
from tests import helpers as H

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not ref_gpu.available("native_hybrid8.cubin"),
                                 reason="reference kernels not built (oracle/build_ref.py)")]

_REF = {}


def ref_hybrid():
    if "h" not in _REF:
        _REF["h"] = ref_gpu.Hybrid8()
    return _REF["h"]


def both(x, bank, name):
    from reax_engine_runtime_v3_b200.reaxv2.gate_up import Native, quantize_rows
    xd, bd = x.cuda(), H.bank_to(bank, "cuda")
    ours = Native(None).project(xd, bd, name)
    low, high, scales = quantize_rows(xd, bd)
    ref = ref_hybrid().product(low, bd.low_weight, high, bd.high_weight, scales, bd.scales, bd.bias, name)
    torch.cuda.synchronize()
    return H.bits(ours), H.bits(ref)


@pytest.mark.parametrize("M,K,Hh,name", [
    (16, 1024, 2816, "hybrid8_b128n256_s64n256"),        # config 1
    (64, 4096, 14336, "hybrid8_b64n256_s32n256"),        # config 2, M = 64
    (1, 4096, 14336, "hybrid8_b32n128k32w4_min3"),       # config 2, M = 1
    (300, 1024, 4096, "hybrid8_b128n128_s32n128"),
    (777, 512, 2048, "hybrid8_b64n128k32_min2"),
])
def test_int8_gate_up_bit_identical_to_reference_kernel(M, K, Hh, name):
    g = H.gen(M * 7 + K)
    ours, ref = both(H.activations(g, M, K), H.int8_bank(g, K, Hh), name)
    rep = H.ulp_report(ours, ref)
    print(rep)
    assert rep["n_diff"] == 0, rep


def test_int8_gate_up_prefill_matches_reference_kernel():
    """Config 3 shape (M = 4096, K = 4096, H = 14336), every row."""
    g = H.gen(33)
    ours, ref = both(H.activations(g, 4096, 4096), H.int8_bank(g, 4096, 14336), "hybrid8_b128n256_s64n256")
    assert np.array_equal(ours, ref)


def test_hybrid_outlier_columns_close_to_reference_kernel():
    g = H.gen(44)
    ours, ref = both(H.activations(g, 200, 2560),
                     H.int8_bank(g, 2560, 1024, KH=128, centered=True, pow2_smoothing=True, bias=True),
                     "hybrid8_b128n256_s64n256")
    rep = H.ulp_report(ours, ref)
    print(rep)
    assert rep["max_ulp"] <= 1, rep


@pytest.mark.skipif(not ref_gpu.available("sliced_linear8.cubin"), reason="reference sliced kernel not built")
@pytest.mark.parametrize("P,G,HP,M,N", [(2, 1280, 64, 200, 512), (1, 2432, 128, 33, 1024), (3, 512, 64, 8, 2560)])
def test_sliced_partials_with_bf16_columns_close_to_reference_kernel(P, G, HP, M, N):
    """Grouped partials with BF16 columns per group (sliced_linear8.cu:28-30): the BF16 products add
    into the dequantized values as in the reference."""
    from reax_engine_runtime_v3_b200.reaxv2.sliced import sliced_i8
    g = H.gen(P + G + M + HP)
    dev = torch.device("cuda")
    low = torch.randint(-127, 128, (M, P * G), generator=g, dtype=torch.int32).to(torch.int8).to(dev)
    w = torch.randint(-127, 128, (N, P * G), generator=g, dtype=torch.int32).to(torch.int8).to(dev)
    ah = H.activations(g, M, P * HP).to(dev)
    wh = (torch.randn(N, P * HP, generator=g) * 0.05).to(torch.bfloat16).to(dev)
    sa = (1e-3 + 1e-2 * torch.rand(P, M, generator=g)).to(dev)
    sw = (1e-3 + 9e-3 * torch.rand(P, N, generator=g)).to(dev)
    bias = (torch.randn(P, N, generator=g) * 0.05).to(dev)
    ours = torch.empty(P, M, N, dtype=torch.bfloat16, device=dev)
    sliced_i8(low, w, ah, wh, sa, sw, bias, ours, G, HP, P)
    ref = ref_gpu.Sliced8().partials(low, w, ah, wh, sa, sw, bias, G, HP, P)
    torch.cuda.synchronize()
    rep = H.ulp_report(H.bits(ours), H.bits(ref))
    print(rep)
    assert rep["max_ulp"] <= 1, rep


@pytest.mark.skipif(not ref_gpu.available("sliced_linear8.cubin"), reason="reference sliced kernel not built")
@pytest.mark.parametrize("P,G,M,N", [(1, 2560, 64, 12288), (2, 1280, 200, 512), (4, 512, 33, 1024),
                                     (2, 1024, 1, 1536), (2, 1024, 33, 1536), (3, 512, 64, 2560)])
def test_sliced_partials_bit_identical_to_reference_kernel(P, G, M, N):
    """Decode-sized and prefill-sized token counts, one to four groups, N from 1024 to 12288."""
    from reax_engine_runtime_v3_b200.reaxv2.sliced import sliced_i8
    g = H.gen(P + G + M)
    dev = torch.device("cuda")
    low = torch.randint(-127, 128, (M, P * G), generator=g, dtype=torch.int32).to(torch.int8).to(dev)
    w = torch.randint(-127, 128, (N, P * G), generator=g, dtype=torch.int32).to(torch.int8).to(dev)
    sa = (1e-3 + 1e-2 * torch.rand(P, M, generator=g)).to(dev)
    sw = (1e-3 + 9e-3 * torch.rand(P, N, generator=g)).to(dev)
    bias = (torch.randn(P, N, generator=g) * 0.05).to(dev)
    empty_a = torch.zeros(M, 0, dtype=torch.bfloat16, device=dev)
    empty_w = torch.zeros(N, 0, dtype=torch.bfloat16, device=dev)
    ours = torch.empty(P, M, N, dtype=torch.bfloat16, device=dev)
    sliced_i8(low, w, empty_a, empty_w, sa, sw, bias, ours, G, 0, P)
    ref = ref_gpu.Sliced8().partials(low, w, empty_a, empty_w, sa, sw, bias, G, 0, P)
    torch.cuda.synchronize()
    assert torch.equal(ours.view(torch.int16), ref.view(torch.int16))
