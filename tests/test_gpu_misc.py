"""GPU checks of the remaining pieces: the SiLU domain table (all 65536 inputs), silu_mul, the ordered
reductions (against the reference-generated golden vectors), the grouped INT8 projection, and the
bounded device wait."""
import os

import numpy as np
import pytest
import torch

from oracle import reax_oracle as ro
from tests import helpers as H

pytestmark = pytest.mark.gpu

GOLDEN = np.load(os.path.join(os.path.dirname(__file__), "golden", "reference_kernels.npz"))


def lib():
    from reax_engine_runtime_v3_b200 import _native
    return _native


def test_silu_table_domain():
    """All 65536 bf16 inputs: GPU table == GPU element-wise silu_mul (reference's domain check,
    wide_warp_hybrid.py:41-49), and within 1 bf16 ulp of the oracle's correctly rounded formula."""
    from reax_engine_runtime_v3_b200.reaxv2.wide_warp_hybrid import Native
    assert Native(None).domain_check()["bit_identical"]
    n = lib()
    t = torch.empty(65536, dtype=torch.bfloat16, device="cuda")
    n.check(n.load().reax_silu_table(t.data_ptr(), n.stream_handle()))
    torch.cuda.synchronize()
    got = H.bits(t)
    want = ro.silu_table()
    finite = np.isfinite(ro.bf16_to_f32(np.arange(65536, dtype=np.uint32).astype(np.uint16)))
    d = ro.ulp_distance_bf16(got[finite], want[finite])
    print("silu table: patterns differing from the oracle:", int((d > 0).sum()), "max ulp", int(d.max()))
    assert d.max() <= 1


def test_silu_mul_strided_matches_oracle_with_gpu_table():
    from reax_engine_runtime_v3_b200.runtime.mixed_origin_bf16 import silu_mul
    g = H.gen(9)
    gu = (torch.randn(37, 2 * 300, generator=g) * 4).to(torch.bfloat16)
    d = gu.cuda()
    out = silu_mul(d[:, :300], d[:, 300:])
    n = lib()
    t = torch.empty(65536, dtype=torch.bfloat16, device="cuda")
    n.check(n.load().reax_silu_table(t.data_ptr(), n.stream_handle()))
    torch.cuda.synchronize()
    b = H.bits(gu)
    want = ro.swiglu_bits(b[:, :300], b[:, 300:], H.bits(t))
    assert np.array_equal(H.bits(out), want)


def test_reduce_kernel_vs_reference_golden():
    from reax_engine_runtime_v3_b200.reaxv2.quantize import reduce_kernel
    parts = H.from_bits(GOLDEN["reduce_partials"], "cuda")
    P, M, N = parts.shape
    out = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    reduce_kernel[((M * N + 511) // 512,)](parts, out, TOTAL=M * N, P=P, B=512, num_warps=4, enable_fp_fusion=False)
    torch.cuda.synchronize()
    assert np.array_equal(H.bits(out), GOLDEN["reduce_out"])


def test_fold_vs_reference_golden():
    from reax_engine_runtime_v3_b200.runtime.mixed_origin_bf16 import fold
    P0, P1, M, N, split = (int(v) for v in GOLDEN["fold_shape"])
    parts = H.from_bits(GOLDEN["fold_parts"], "cuda")
    out = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    fold[((M * N + 511) // 512,)](parts, torch.tensor([split], dtype=torch.int32, device="cuda"), out, M=M, N=N, P0=P0,
                                  P1=P1, B=512, num_warps=4, enable_fp_fusion=False)
    torch.cuda.synchronize()
    assert np.array_equal(H.bits(out), GOLDEN["fold_out"])


@pytest.mark.parametrize("P,G,HP,M,N", [(1, 2560, 0, 64, 12288), (2, 1280, 0, 200, 512), (2, 512, 64, 130, 768),
                                        (3, 1024, 0, 17, 1536), (2, 512, 64, 9, 768)])
def test_sliced_projection(P, G, HP, M, N):
    """Grouped INT8 projection (reaxv2/sliced.py): bit-exact when HP == 0, tolerance otherwise."""
    from types import SimpleNamespace
    from reax_engine_runtime_v3_b200.reaxv2.sliced import Native
    g = H.gen(P * 1000 + G + HP + M)
    K = P * G + P * HP
    x = H.activations(g, M, K)
    perm = torch.randperm(K, generator=g)
    low_columns = perm[:P * G].to(torch.int32)
    high_columns = perm[P * G:].to(torch.int32)
    bank = SimpleNamespace(
        width=K, parts=P, group=G, hp=HP, low_columns=low_columns, high_columns=high_columns,
        centers=(torch.randn(P * G, generator=g) * 0.05), smoothing=2.0 ** torch.randint(-1, 2, (P * G,), generator=g).float(),
        low_weight=torch.randint(-127, 128, (N, P * G), generator=g, dtype=torch.int32).to(torch.int8),
        high_weight=(torch.randn(N, P * HP, generator=g) * 0.02).to(torch.bfloat16),
        scales=(1e-3 + 9e-3 * torch.rand(P, N, generator=g)), bias=torch.randn(P, N, generator=g) * 0.05)
    out = Native(None).project(x.cuda(), H.bank_to(bank, "cuda"), "slice_m128n256")
    torch.cuda.synchronize()
    nb = H.bank_numpy(bank)
    want = ro.sliced_project(H.bits(x), nb)
    got = H.bits(out)
    rep = H.ulp_report(got, want)
    print(rep)
    if HP == 0:
        # quantizer scale division: codes follow the GPU's scales; compare through the GPU's own codes
        low_g, high_g, sc_g = Native(None).prepare(x.cuda(), H.bank_to(bank, "cuda"))
        torch.cuda.synchronize()
        parts = ro.sliced_partials(low_g.cpu().numpy(), nb.low_weight, H.bits(high_g), nb.high_weight,
                                   sc_g.cpu().numpy(), nb.scales, nb.bias, G, HP, P)
        want2 = parts[0] if P == 1 else ro.reduce_partials(parts)
        assert np.array_equal(got, want2)
    else:
        d = ro.ulp_distance_bf16(got, want)
        gf, wf = ro.bf16_to_f32(got), ro.bf16_to_f32(want)
        ok = (d <= 2) | (np.abs(gf - wf) <= 1e-3 * np.abs(wf).max(axis=1, keepdims=True))
        assert ok.all(), rep


@pytest.mark.parametrize("P,G,M,N,sms", [(4, 2304, 64, 2560, 74), (4, 2304, 1, 2560, 37), (3, 640, 33, 1536, 74),
                                         (1, 4096, 16, 256, 0), (2, 384, 64, 512, 148)])
def test_sliced_weight_major_tiles(P, G, M, N, sms):
    """Few tokens: the grouped projection runs weight-major tiles of ceil(P * N / SMs) output columns with
    stages of several K blocks (the last stage of a group reaches into the next group's K blocks, or
    past K, which are loaded but not multiplied), on a lane's share of the SMs and on the whole GPU;
    the partials are the oracle's bit for bit."""
    from reax_engine_runtime_v3_b200 import _native
    from reax_engine_runtime_v3_b200.reaxv2.sliced import sliced_i8
    g = H.gen(11 * M + P * G + N + sms)
    dev = torch.device("cuda")
    low = torch.randint(-127, 128, (M, P * G), generator=g, dtype=torch.int32).to(torch.int8)
    w = torch.randint(-127, 128, (N, P * G), generator=g, dtype=torch.int32).to(torch.int8)
    sa = 1e-3 + 9e-3 * torch.rand(P, M, generator=g)
    sw = 1e-3 + 9e-3 * torch.rand(P, N, generator=g)
    bias = torch.randn(P, N, generator=g) * 0.05
    stream = torch.cuda.current_stream()
    if sms:
        _native.set_stream_sms(stream, sms)
    try:
        out = torch.empty(P, M, N, dtype=torch.bfloat16, device=dev)
        sliced_i8(low.to(dev), w.to(dev), torch.zeros(M, 0, dtype=torch.bfloat16, device=dev),
                  torch.zeros(N, 0, dtype=torch.bfloat16, device=dev), sa.to(dev), sw.to(dev), bias.to(dev), out, G, 0, P)
        torch.cuda.synchronize()
    finally:
        _native.set_stream_sms(stream, 0)
    want = ro.sliced_partials(low.numpy(), w.numpy(), np.zeros((M, 0), np.uint16), np.zeros((N, 0), np.uint16),
                              sa.numpy(), sw.numpy(), bias.numpy(), G, 0, P)
    assert np.array_equal(H.bits(out), want)


@pytest.mark.parametrize("P,G,HP,M,N", [(4, 2304, 0, 1, 2560), (4, 2304, 0, 64, 2560), (2, 512, 64, 130, 768)])
def test_sliced_static_entry_back_to_back(P, G, HP, M, N):
    """reax_sliced_i8_static launched back to back (each launch streams its weights under the previous
    one's tail, over rotating banks) gives the bits of reax_sliced_i8 with no expired wait."""
    from reax_engine_runtime_v3_b200 import _native
    from reax_engine_runtime_v3_b200.reaxv2.sliced import sliced_i8
    g = H.gen(7 * M + P * G + HP + N)
    dev = torch.device("cuda")
    low = torch.randint(-127, 128, (M, P * G), generator=g, dtype=torch.int32).to(torch.int8).to(dev)
    high = (torch.randn(M, P * HP, generator=g)).to(torch.bfloat16).to(dev)
    sa = (1e-3 + 9e-3 * torch.rand(P, M, generator=g)).to(dev)
    banks = [dict(w=torch.randint(-127, 128, (N, P * G), generator=g, dtype=torch.int32).to(torch.int8).to(dev),
                  wh=(torch.randn(N, P * HP, generator=g) * 0.02).to(torch.bfloat16).to(dev),
                  sw=(1e-3 + 9e-3 * torch.rand(P, N, generator=g)).to(dev),
                  bias=(torch.randn(P, N, generator=g) * 0.05).to(dev)) for _ in range(2)]

    def run(b, static):
        out = torch.empty(P, M, N, dtype=torch.bfloat16, device=dev)
        return sliced_i8(low, b["w"], high, b["wh"], sa, b["sw"], b["bias"], out, G, HP, P, static_weights=static)

    ws = _native.workspace(dev)
    _native.clear_status(ws)
    outs = [run(b, True) for b in banks * 4]
    torch.cuda.synchronize()
    assert _native.read_status(ws) == 0
    for i, b in enumerate(banks):
        plain = run(b, False)
        torch.cuda.synchronize()
        for out in outs[i::2]:
            assert torch.equal(out.view(torch.int16), plain.view(torch.int16))


def test_split_gated_projection_out_path():
    from reax_engine_runtime_v3_b200.runtime.split_gated_projection import project_split
    from reax_engine_runtime_v3_b200.reaxv2.sliced import Native
    from types import SimpleNamespace
    g = H.gen(77)
    M, G, N, count = 96, 2560, 12288, 8192
    x = H.activations(g, M, G)
    bank = SimpleNamespace(
        width=G, parts=1, group=G, hp=0, low_columns=torch.arange(G, dtype=torch.int32),
        high_columns=torch.zeros(0, dtype=torch.int32), centers=torch.zeros(G), smoothing=torch.ones(G),
        low_weight=torch.randint(-127, 128, (N, G), generator=g, dtype=torch.int32).to(torch.int8),
        high_weight=torch.zeros(N, 0, dtype=torch.bfloat16), scales=1e-3 + 9e-3 * torch.rand(1, N, generator=g),
        bias=torch.zeros(1, N))
    b = H.bank_to(bank, "cuda")
    qkv, z = project_split(x.cuda(), b, count, "slice_m128n256")
    whole = Native(None).project(x.cuda(), b, "slice_m128n256")
    torch.cuda.synchronize()
    assert torch.equal(torch.cat([qkv, z], 1).view(torch.int16), whole.view(torch.int16))


def test_bounded_wait_reports_timeout():
    """A wait on a barrier nothing arrives on ends after its bound with a status bit; the context
    stays usable (a later kernel runs normally)."""
    n = lib()
    ws = torch.zeros(1024, dtype=torch.uint8, device="cuda")
    n.check(n.load().reax_selftest_wait(ws.data_ptr(), 20_000_000, n.stream_handle()))
    torch.cuda.synchronize()
    assert n.read_status(ws) == 0x20
    t = torch.ones(4, device="cuda") * 2
    assert float(t.sum()) == 8.0
