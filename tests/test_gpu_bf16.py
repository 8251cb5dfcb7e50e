"""GPU parity of the BF16-weight variant (runtime/mixed_origin_bf16.py) against the CPU oracle.

GEMM part (the partials kernel): the GPU accumulates each K slice in float32 in the tensor core's own
order, the oracle sums exactly (float64).  Every partial must satisfy the standard float32 dot-product
bound plus its bf16 rounding:  |got - exact| <= gamma_n * sum_k |x_k w_k| + ulp_bf16(exact),
gamma_n = n u / (1 - n u), u = 2**-24, n = slice length.
SwiGLU part: the fused kernel (one launch) must equal, bit for bit, the oracle SwiGLU of the gate and
up values that the unfused GPU pipeline (partials kernel) produced: same accumulation, exact epilogue.
The fold of partials is exact given the partials (float32 adds in slice order).
"""
import numpy as np
import pytest
import torch

from oracle import reax_oracle as ro
from tests import helpers as H

pytestmark = pytest.mark.gpu


def dot_bound_ok(got_bits, x_bits, w_bits, k0=0, k1=None):
    x = ro.bf16_to_f32(x_bits).astype(np.float64)[:, k0:k1]
    w = ro.bf16_to_f32(w_bits).astype(np.float64)[:, k0:k1]
    exact = x @ w.T
    mag = np.abs(x) @ np.abs(w).T
    n = x.shape[1]
    u = 2.0 ** -24
    gamma = n * u / (1 - n * u)
    ulp = np.abs(ro.bf16_to_f32(ro.f32_to_bf16(exact.astype(np.float32))).astype(np.float64)) * 2.0 ** -7
    ulp = np.maximum(ulp, 2.0 ** -133)
    err = np.abs(ro.bf16_to_f32(got_bits).astype(np.float64) - exact)
    ok = err <= gamma * mag + ulp
    return ok, float((err / np.maximum(gamma * mag + ulp, 1e-300)).max())


def weights(g, N2, K):
    return (torch.randn(N2, K, generator=g) * 0.02).to(torch.bfloat16)


def gpu_table():
    from reax_engine_runtime_v3_b200 import _native
    t = torch.empty(65536, dtype=torch.bfloat16, device="cuda")
    _native.check(_native.load().reax_silu_table(t.data_ptr(), _native.stream_handle()))
    torch.cuda.synchronize()
    return H.bits(t)


@pytest.mark.parametrize("M,K,H2", [(1, 1024, 512), (64, 4096, 2048), (8, 512, 10240), (128, 4096, 14336),
                                    (333, 1024, 4096), (600, 1024, 1024), (1024, 2048, 384)])
def test_gate_up_bf16_unsplit(M, K, H2):
    """The fused BF16 gate/up (CTA-pair tiles from 512 rows) against the unfused partials of the same
    GPU: the SwiGLU of those partials bit for bit, and each partial within the float32 dot-product bound."""
    from reax_engine_runtime_v3_b200.runtime.mixed_origin_bf16 import Native
    g = H.gen(M + K)
    x = H.activations(g, M, K, "student")
    w = weights(g, 2 * H2, K)
    nat = Native()
    xd, wd = x.cuda(), w.cuda()
    one = dict(parts=1, chunk=K, mode=0)
    out = nat.gate_up(xd, wd)
    gu = nat.project(xd, wd, 0, one, one)
    torch.cuda.synchronize()
    ok, worst = dot_bound_ok(H.bits(gu), H.bits(x), H.bits(w))
    print(f"GEMM error / bound, worst: {worst:.3f}")
    assert ok.all()
    gub = H.bits(gu)
    want = ro.swiglu_bits(gub[:, :H2], gub[:, H2:], gpu_table())
    assert np.array_equal(H.bits(out), want)
    print("vs float64 oracle:", H.ulp_report(H.bits(out), ro.gate_up_bf16(H.bits(x), H.bits(w), 0, one, one)))


def test_cfg5b_bucket_rows_sample():
    """BASELINE config 5b: Student-t X [2048, 4096], W ~ N(0, 0.02) [28672, 4096]; oracle on sampled rows."""
    from reax_engine_runtime_v3_b200.runtime.mixed_origin_bf16 import Native
    g = H.gen(55)
    x = H.activations(g, 2048, 4096, "student")
    w = weights(g, 28672, 4096)
    nat = Native()
    one = dict(parts=1, chunk=4096, mode=0)
    out = nat.gate_up(x.cuda(), w.cuda())
    gu = nat.project(x.cuda(), w.cuda(), 0, one, one)
    torch.cuda.synchronize()
    rows = np.arange(0, 2048, 37)
    ok, worst = dot_bound_ok(H.bits(gu)[rows], H.bits(x)[rows], H.bits(w))
    print(f"GEMM error / bound, worst: {worst:.3f}")
    assert ok.all()
    gub = H.bits(gu)
    assert np.array_equal(H.bits(out), ro.swiglu_bits(gub[:, :14336], gub[:, 14336:], gpu_table()))


@pytest.mark.parametrize("P0,c0,P1,c1,split", [(1, 1024, 1, 1024, 50), (2, 512, 3, 384, 70), (3, 384, 1, 1024, 0),
                                               (4, 256, 2, 512, 300), (2, 640, 2, 640, 129)])
def test_mixed_origin_partials_and_fold(P0, c0, P1, c1, split):
    from reax_engine_runtime_v3_b200.runtime.mixed_origin_bf16 import Native
    g = H.gen(P0 * 10 + P1 + split)
    M, K, N = 300, 1024, 512
    x = H.activations(g, M, K)
    w = weights(g, N, K)
    left, right = dict(parts=P0, chunk=c0, mode=4), dict(parts=P1, chunk=c1, mode=4)
    nat = Native()
    split_t = torch.tensor([split], dtype=torch.int32, device="cuda")
    parts = nat.partials(x.cuda(), w.cuda(), split_t, left, right)
    torch.cuda.synchronize()
    gp = H.bits(parts)
    xb, wb = H.bits(x), H.bits(w)
    for s in range(max(P0, P1)):
        for rows, P, c in ((slice(0, min(split, M)), P0, c0), (slice(min(split, M), M), P1, c1)):
            if s < P and rows.start < rows.stop:
                k0, k1 = ro.slice_bounds(K, P, c)[s]
                if k1 > k0:
                    ok, worst = dot_bound_ok(gp[s, rows], xb[rows], wb, k0, k1)
                    assert ok.all(), (s, worst)
                else:
                    assert not gp[s, rows].any()
    out = nat.project(x.cuda(), w.cuda(), split_t, left, right)
    torch.cuda.synchronize()
    assert np.array_equal(H.bits(out), ro.fold(gp, split, P0, P1))
