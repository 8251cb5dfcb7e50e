"""Generate golden vectors for the offline bank builder by running the reference's own ``bank()``.

Run where the reference project is mounted (its root as the first argument).  The function
``bank(weight, stats, protected)`` of
private/snapshots/model-exact-addressed-projections-full-r5/earlier_gate_up_screen.py:17-33 is taken
from that file unmodified (its module imports serving-engine code that is not part of the reference
tree, so only that function's definition is compiled, with ``torch`` and ``SimpleNamespace`` in scope)
and run on the CPU on seeded synthetic weights and activation statistics.

Outputs ``tests/golden/bank_reference.npz``; the tests only read the ``.npz``.
"""
from __future__ import annotations

import ast
import sys
from pathlib import Path
from types import SimpleNamespace

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
SCREEN = "private/snapshots/model-exact-addressed-projections-full-r5/earlier_gate_up_screen.py"


def reference_bank(root: str):
    tree = ast.parse((Path(root) / SCREEN).read_text())
    fn = next(n for n in tree.body if isinstance(n, ast.FunctionDef) and n.name == "bank")
    scope = {"torch": torch, "SimpleNamespace": SimpleNamespace}
    exec(compile(ast.Module(body=[fn], type_ignores=[]), SCREEN, "exec"), scope)
    return scope["bank"]


def case(gen, N2, K, rows, protected, special):
    w = (torch.randn(N2, K, generator=gen) * 0.02)
    w[:, :4] *= 8.0                                   # a few heavy weight columns
    if special:
        w[:, 5] = 0.0                                 # an all-zero weight column
    x = torch.randn(rows, K, generator=gen)
    x[:, 7::97] *= 30.0                               # outlier activation channels
    x += torch.randn(K, generator=gen) * 0.3          # non-zero means: a real centring
    if special:
        x[:, 9] = 2.5                                 # a constant channel (variance floor)
    v = x.float()
    stats = {"count": rows, "sum": v.double().sum(0), "square": v.double().square().sum(0), "maximum": v.abs().amax(0)}
    return w.to(torch.bfloat16), stats


def main(root: str) -> None:
    bank = reference_bank(root)
    gen = torch.Generator().manual_seed(20261202)
    out = {}
    for name, (N2, K, rows, protected, special) in {"small": (128, 384, 200, 32, False),
                                                    "edges": (96, 256, 64, 16, True)}.items():
        w, stats = case(gen, N2, K, rows, protected, special)
        p = bank(w, stats, protected)
        pre = f"{name}_"
        out[pre + "weight"] = w.view(torch.int16).numpy().view(np.uint16)
        for k in ("sum", "square"):
            out[pre + k] = stats[k].numpy()
        out[pre + "count"] = np.array(stats["count"])
        out[pre + "maximum"] = stats["maximum"].numpy()
        out[pre + "protected"] = np.array(protected)
        for k in ("low_columns", "high_columns", "low_weight", "smoothing", "centers", "scales", "bias"):
            out[pre + k] = getattr(p, k).numpy()
        out[pre + "high_weight"] = p.high_weight.view(torch.int16).numpy().view(np.uint16)
    np.savez_compressed(HERE / "bank_reference.npz", **out)
    print("wrote", HERE / "bank_reference.npz", len(out), "arrays")


if __name__ == "__main__":
    if len(sys.argv) < 2:
        sys.exit("usage: python tests/golden/gen_bank_golden.py <reference root>")
    main(sys.argv[1])
