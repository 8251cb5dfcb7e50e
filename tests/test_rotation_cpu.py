"""Host side of the rotated down projection (no GPU): the route checks of reaxv2/rotation.py and the
oracle's rotated quantizer against golden vectors made by the reference's own rotation_* kernels."""
import os
from types import SimpleNamespace

import numpy as np
import pytest

from oracle import reax_oracle as ro

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "rotation_reference.npz")


def test_rotated_route_checks():
    """selected_kernel keeps the reference's route names and alignment errors (reaxv2/rotation.py:33-43)."""
    from reax_engine_runtime_v3_b200.reaxv2.rotation import selected_kernel
    p = SimpleNamespace(group=1344, hp=0)
    assert selected_kernel("slice_m128n256", p) == "slice_m128n256"
    assert selected_kernel("slice_m128n128k64", p) == "slice_m128n128"
    with pytest.raises(ValueError, match="Missing inner-loop contract"):
        selected_kernel("slice_m256", p)
    with pytest.raises(ValueError, match="Unsupported projection inner-loop alignment"):
        selected_kernel("slice_m128n256", SimpleNamespace(group=1000, hp=0))


def test_rotation_signs_follow_the_column_hash():
    """Bit 16 of column * 1103515245 + 12345 in uint32 arithmetic, including columns whose product wraps."""
    cols = np.array([0, 1, 2, 3, 4095, 9215, 4000000], dtype=np.int64)
    want = np.array([((c * 1103515245 + 12345) & 0xFFFFFFFF) & 65536 != 0 for c in cols.tolist()])
    assert np.array_equal(ro.rotation_negated(cols), want)


@pytest.mark.skipif(not os.path.exists(GOLDEN), reason="rotation golden vectors not generated")
def test_prepare_rotated_vs_reference_golden():
    g = np.load(GOLDEN)
    n = int(g["cases"])
    for i in range(n):
        M, K, chunk, parts, group, block, threads = (int(v) for v in g[f"c{i}_shape"])
        low, scales = ro.prepare_rotated(g[f"c{i}_x"], g[f"c{i}_centers"], chunk, parts, group, block)
        assert np.array_equal(scales.view(np.int32), g[f"c{i}_scales"].view(np.int32)), (i, "scales")
        assert np.array_equal(low, g[f"c{i}_low"]), (i, "codes")
