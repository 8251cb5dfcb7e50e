"""The offline bank builder (a13) against golden vectors made by the reference's own ``bank()``
(tests/golden/gen_bank_golden.py): the CPU oracle's numpy restatement and the package's torch builder."""
import os

import numpy as np
import pytest
import torch

from oracle import reax_oracle as ro

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "bank_reference.npz")
FIELDS = ("low_columns", "high_columns", "low_weight", "high_weight", "smoothing", "centers", "scales", "bias")


def load(case):
    z = np.load(GOLDEN)
    return {k[len(case) + 1:]: z[k] for k in z.files if k.startswith(case + "_")}


@pytest.mark.parametrize("case", ["small", "edges"])
def test_oracle_bank_matches_reference_golden(case):
    g = load(case)
    b = ro.build_bank(g["weight"], int(g["count"]), g["sum"], g["square"], g["maximum"], int(g["protected"]))
    for f in ("low_columns", "high_columns", "low_weight", "high_weight", "smoothing", "centers", "scales"):
        assert np.array_equal(getattr(b, f), g[f]), f
    # float64 dot products in another order: at most one float32 rounding apart
    d = np.abs(b.bias.view(np.int32).astype(np.int64) - g["bias"].view(np.int32).astype(np.int64))
    assert d.max() <= 1


@pytest.mark.parametrize("case", ["small", "edges"])
def test_bank_builder_matches_reference_golden(case):
    from reax_engine_runtime_v3_b200.bank_builder import bank
    g = load(case)
    w = torch.from_numpy(g["weight"].view(np.int16)).view(torch.bfloat16)
    stats = {"count": int(g["count"]), "sum": torch.from_numpy(g["sum"]), "square": torch.from_numpy(g["square"]),
             "maximum": torch.from_numpy(g["maximum"])}
    b = bank(w, stats, int(g["protected"]))
    assert b.centered and b.width == w.shape[1]
    for f in FIELDS:
        v = getattr(b, f)
        got = v.view(torch.int16).numpy().view(np.uint16) if v.dtype == torch.bfloat16 else v.numpy()
        assert np.array_equal(got, g[f]), f


def test_bank_layout_feeds_the_gate_up_oracle():
    """A built bank runs through the quantize + gate/up oracle with the layout the kernels read."""
    from reax_engine_runtime_v3_b200.bank_builder import bank, statistics_of
    gen = torch.Generator().manual_seed(3)
    w = (torch.randn(512, 320, generator=gen) * 0.02).to(torch.bfloat16)
    x = torch.randn(40, 320, generator=gen) + 0.2
    b = bank(w, statistics_of(x), 64)
    assert b.low_weight.shape == (512, 256) and b.high_weight.shape == (512, 64)
    assert set(b.low_columns.tolist()) | set(b.high_columns.tolist()) == set(range(320))
    xb = x.to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    nb = {k: (v.view(torch.int16).numpy().view(np.uint16) if isinstance(v, torch.Tensor) and v.dtype == torch.bfloat16
              else (v.numpy() if isinstance(v, torch.Tensor) else v)) for k, v in vars(b).items()}
    from types import SimpleNamespace
    out = ro.gate_up_project(xb, SimpleNamespace(**nb))
    assert out.shape == (40, 256)
    # the bank approximates the BF16 projection: compare with the unquantized gate/up + SwiGLU
    ref = x.to(torch.bfloat16).float() @ w.float().T
    want = torch.nn.functional.silu(ref[:, :256]) * ref[:, 256:]
    got = torch.from_numpy(ro.bf16_to_f32(out))
    assert (got - want).abs().max() < 0.05 * want.abs().max()
