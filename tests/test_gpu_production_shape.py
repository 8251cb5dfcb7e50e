"""The v3 production gate/up shape against the reference's own production kernels on the same B200.

The deployed model runs gate/up at K = 2560 with 128 BF16 outlier columns (KL = 2432, KH = 128) and
N2 = 18432 through ``wide_warp_hybrid.Native.product`` (private/snapshots/model-preaddressed-GUP-r1/
wide_warp_hybrid.py:15-35), which launches the ``addressed_*`` kernels (kernel-source/src/
model-preaddressed-GUP-r1/addressed_gate_up.cu:75-112), the tail-band ``band_*`` kernels
(model-preaddressed-GUP-tail-bands-r2/band_gate_up.cu:76-143) or the activation-table build.  Those are
compiled from source for sm_100a (oracle/build_ref.py) and run here on a bank built the way the
reference builds it (``bank_builder.bank``, earlier_gate_up_screen.py:17-33) from a synthetic BF16
weight and calibration statistics, at the screens' row counts (resident_gate_up_screen.py:17: 32 to
1024; gup_tail_band_screen.py:15: 384 to 1024 in steps of 32), with the screens' first-16-row batch
invariance check (resident_gate_up_screen.py:25-31).

Bar: at most 1 bf16 ulp from the reference kernel on every element (north_star), with the number of
differing elements and the max abs / rel error printed; quantizer outputs are shared (bit-identical
to the reference's Triton quantizer, tests/test_gpu_reference_quant.py).
"""
import numpy as np
import pytest
import torch

from oracle import ref_gpu
from tests import helpers as H

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not ref_gpu.available("addressed_gate_up.cubin"),
                                 reason="reference production kernels not built (oracle/build_ref.py)")]

K, KH, N2 = 2560, 128, 18432
_CACHE = {}


def production_bank():
    """A bank of the production shape built by the reference's recipe from a synthetic BF16 weight."""
    if "bank" not in _CACHE:
        from reax_engine_runtime_v3_b200.bank_builder import bank, statistics_of
        g = H.gen(18432)
        w = torch.randn(N2, K, generator=g) * 0.02
        w[:, torch.randperm(K, generator=g)[:64]] *= 6.0
        w = w.to(torch.bfloat16).cuda()
        calib = calibration_rows(g, 1024).cuda()
        _CACHE["bank"] = bank(w, statistics_of(calib), KH)
        _CACHE["x"] = calibration_rows(g, 1024).to(torch.bfloat16).cuda()
    return _CACHE["bank"], _CACHE["x"]


def calibration_rows(g, rows):
    """Student-t activations with a few heavy channels and non-zero channel means."""
    x = H.activations(g, rows, K, "student").float()
    return x + torch.linspace(-0.3, 0.3, K)


def ours_and_operands(x, p):
    from reax_engine_runtime_v3_b200.reaxv2.gate_up import quantize_rows
    from reax_engine_runtime_v3_b200.reaxv2.wide_warp_hybrid import Native
    low, high, scales = quantize_rows(x, p)
    out = Native(None).product(low, p.low_weight, high, p.high_weight, scales, p.scales, p.bias,
                               "addressed_0_m128n256k32")
    return out, (low, p.low_weight, high, p.high_weight, scales, p.scales, p.bias)


def check_close(ours, ref, what):
    rep = H.ulp_report(H.bits(ours), H.bits(ref))
    print(what, rep)
    assert rep["max_ulp"] <= 1, (what, rep)
    return rep


def test_bank_shape():
    p, _ = production_bank()
    assert p.low_weight.shape == (N2, K - KH) and p.high_weight.shape == (N2, KH)
    assert p.low_columns.numel() == K - KH and p.high_columns.numel() == KH


@pytest.mark.parametrize("rows", [32, 128, 512, 640, 768, 896, 1024])
def test_addressed_kernels_at_resident_screen_rows(rows):
    p, xs = production_bank()
    x = xs[:rows].contiguous()
    ours, ops = ours_and_operands(x, p)
    ref = ref_gpu.Addressed()
    worst = 0
    for name in ref_gpu.ADDRESSED:
        for drop in (0, 1):
            r = ref.product(*ops, name, drop)
            torch.cuda.synchronize()
            worst = max(worst, check_close(ours, r, f"{name} drop={drop} rows={rows}")["n_diff"])
    # first-16-row batch invariance (resident_gate_up_screen.py:25-31)
    first, _ = ours_and_operands(x[:16].contiguous(), p)
    torch.cuda.synchronize()
    assert torch.equal(first.view(torch.int16), ours[:16].view(torch.int16))
    print("rows", rows, "most differing elements against one reference variant:", worst)


@pytest.mark.parametrize("rows", list(range(384, 1025, 32)))
def test_band_kernels_at_tail_screen_rows(rows):
    p, xs = production_bank()
    x = xs[:rows].contiguous()
    ours, ops = ours_and_operands(x, p)
    ref = ref_gpu.Addressed("band_gate_up.cubin")
    ran = 0
    for name, (bm, small, _, _, _) in ref_gpu.BANDS.items():
        for drop in (0, 1):
            tail = rows - max(0, rows // bm - drop) * bm
            if not tail or not (small - 64 < tail <= small):    # gup_tail_band_screen.py:20-21
                continue
            r = ref.product(*ops, name, drop)
            torch.cuda.synchronize()
            check_close(ours, r, f"{name} drop={drop} rows={rows}")
            ran += 1
    if ran == 0:
        pytest.skip(f"no band variant covers a tail of {rows} rows")


@pytest.mark.parametrize("rows", [1, 16, 64, 300, 1024, 2304])
def test_activation_table_kernel(rows):
    """The activation-table build (model-addressed-bulk-activation-table-r1), whose SwiGLU reads a
    65536-entry SiLU table built on the device; 2304 rows is the served maximum."""
    p, xs = production_bank()
    if rows > len(xs):
        g = H.gen(rows)
        x = calibration_rows(g, rows).to(torch.bfloat16).cuda()
    else:
        x = xs[:rows].contiguous()
    ours, ops = ours_and_operands(x, p)
    r = ref_gpu.Addressed("addressed_table_gate_up.cubin").product(*ops, "addressed_1_m128n256k32", 0)
    torch.cuda.synchronize()
    check_close(ours, r, f"table rows={rows}")


def test_wide_warp_names_and_assert():
    """Every reference production kernel name is accepted; a non-production shape fails the reference's
    assert."""
    from reax_engine_runtime_v3_b200.reaxv2.wide_warp_hybrid import Native
    p, xs = production_bank()
    _, ops = ours_and_operands(xs[:8].contiguous(), p)
    nat = Native(None)
    first = None
    for name in list(ref_gpu.ADDRESSED) + list(ref_gpu.BANDS):
        o = nat.product(*ops, name)
        first = o if first is None else first
        assert torch.equal(o.view(torch.int16), first.view(torch.int16))
    low, w, high, wh, sa, sw, b = ops
    with pytest.raises(AssertionError):
        nat.product(low[:, :2304].contiguous(), w[:, :2304].contiguous(), high, wh, sa, sw, b, "addressed_0_m128n256k32")
