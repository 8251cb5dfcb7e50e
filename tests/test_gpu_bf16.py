"""GPU parity of the BF16-weight variant (runtime/mixed_origin_bf16.py) against the CPU oracle.

The oracle sums each K slice exactly (float64) and rounds once to float32, then to bf16; the GPU
accumulates in float32 in the tensor core's own order.  Tolerance, stated per element: at most 2 bf16
ulps, or an absolute error of at most 1e-3 of the largest magnitude in the row (cancellation makes
small outputs arbitrarily sensitive in ulps).  The fold of partials is exact given the partials.
"""
import numpy as np
import pytest
import torch

from oracle import reax_oracle as ro
from tests import helpers as H

pytestmark = pytest.mark.gpu


def within_tol(got, want, ulps=2, rel_row=1e-3):
    d = ro.ulp_distance_bf16(got, want)
    gf, wf = ro.bf16_to_f32(got).astype(np.float64), ro.bf16_to_f32(want).astype(np.float64)
    tol = rel_row * np.abs(wf).max(axis=-1, keepdims=True)
    ok = (d <= ulps) | (np.abs(gf - wf) <= tol)
    return ok, H.ulp_report(got, want)


def weights(g, N2, K):
    return (torch.randn(N2, K, generator=g) * 0.02).to(torch.bfloat16)


@pytest.mark.parametrize("M,K,H2", [(1, 1024, 512), (64, 4096, 2048), (128, 4096, 14336), (333, 1024, 4096)])
def test_gate_up_bf16_unsplit(M, K, H2):
    from reax_engine_runtime_v3_b200.runtime.mixed_origin_bf16 import Native
    g = H.gen(M + K)
    x = H.activations(g, M, K, "student")
    w = weights(g, 2 * H2, K)
    out = Native().gate_up(x.cuda(), w.cuda())
    torch.cuda.synchronize()
    want = ro.gate_up_bf16(H.bits(x), H.bits(w), 0, dict(parts=1, chunk=K), dict(parts=1, chunk=K))
    ok, rep = within_tol(H.bits(out), want)
    print(rep)
    assert ok.all(), rep


def test_cfg5b_bucket_rows_sample():
    """BASELINE config 5b: Student-t X [2048, 4096], W ~ N(0, 0.02) [28672, 4096]; oracle on sampled rows."""
    from reax_engine_runtime_v3_b200.runtime.mixed_origin_bf16 import Native
    g = H.gen(55)
    x = H.activations(g, 2048, 4096, "student")
    w = weights(g, 28672, 4096)
    out = Native().gate_up(x.cuda(), w.cuda())
    torch.cuda.synchronize()
    rows = np.arange(0, 2048, 37)
    want = ro.gate_up_bf16(H.bits(x)[rows], H.bits(w), 0, dict(parts=1, chunk=4096), dict(parts=1, chunk=4096))
    ok, rep = within_tol(H.bits(out)[rows], want)
    print(rep)
    assert ok.all(), rep


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
    want = ro.bf16_partials(H.bits(x), H.bits(w), split, left, right)
    gp = H.bits(parts)
    for s in range(max(P0, P1)):
        for rows, P in ((slice(0, min(split, M)), P0), (slice(min(split, M), M), P1)):
            if s < P:
                ok, rep = within_tol(gp[s, rows], want[s, rows])
                assert ok.all(), (s, rep)
    # the fold itself is exact given the partials
    out = nat.project(x.cuda(), w.cuda(), split_t, left, right)
    torch.cuda.synchronize()
    folded = ro.fold(H.bits(nat.partials(x.cuda(), w.cuda(), split_t, left, right)), split, P0, P1)
    assert np.array_equal(H.bits(out), folded)
