"""The CPU oracle against golden vectors produced by the reference's own Triton kernels.

The vectors in ``golden/reference_kernels.npz`` were made by ``golden/gen_golden.py``, which runs
``reaxv2/quantize.py`` and ``runtime/mixed_origin_bf16.py`` of the reference under Triton's CPU
interpreter.  Every comparison here is bit-exact.
"""
import os

import numpy as np
import pytest

from oracle import reax_oracle as ro

GOLDEN = np.load(os.path.join(os.path.dirname(__file__), "golden", "reference_kernels.npz"))
PREPARE_CASES = sorted({k[len("prepare_"):-len("_x")] for k in GOLDEN.files if k.startswith("prepare_") and k.endswith("_x")})


@pytest.mark.parametrize("case", PREPARE_CASES)
def test_prepare_rows_matches_reference(case):
    g = {k[len(f"prepare_{case}_"):]: GOLDEN[k] for k in GOLDEN.files if k.startswith(f"prepare_{case}_")}
    low, high, scales = ro.prepare_rows(g["x"], g["low_columns"], g["high_columns"], g["smoothing"], g["centers"],
                                        bool(g["center"]))
    assert np.array_equal(low, g["low"])
    assert np.array_equal(high, g["high"])
    assert np.array_equal(scales.view(np.uint32), g["scales"].view(np.uint32))


def test_prepare_cases_cover_edges():
    assert {"cfg1", "ragged17", "outlier", "hybrid", "highonly", "zerorow"} <= set(PREPARE_CASES)


def test_prepare_groups_matches_reference():
    M, K, P, G, HP = GOLDEN["groups_shape"]
    low, high, scales = ro.prepare_groups(GOLDEN["groups_x"], GOLDEN["groups_low_columns"],
                                          GOLDEN["groups_high_columns"], GOLDEN["groups_centers"],
                                          GOLDEN["groups_smoothing"], int(G), int(HP), int(P))
    assert np.array_equal(low, GOLDEN["groups_low"])
    assert np.array_equal(high, GOLDEN["groups_high"])
    assert np.array_equal(scales.view(np.uint32), GOLDEN["groups_scales"].view(np.uint32))


def test_reduce_matches_reference():
    assert np.array_equal(ro.reduce_partials(GOLDEN["reduce_partials"]), GOLDEN["reduce_out"])


def test_fold_matches_reference():
    P0, P1, M, N, split = (int(v) for v in GOLDEN["fold_shape"])
    assert np.array_equal(ro.fold(GOLDEN["fold_parts"], split, P0, P1), GOLDEN["fold_out"])
