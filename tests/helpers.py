"""Shared test helpers: seeded synthetic inputs with the BASELINE shapes and dtype conversions."""
from __future__ import annotations

from types import SimpleNamespace

import numpy as np
import torch

from oracle import reax_oracle as ro


def gen(seed: int) -> torch.Generator:
    return torch.Generator().manual_seed(seed)


def bits(t: torch.Tensor) -> np.ndarray:
    """bf16 tensor (any device) -> numpy uint16 bit patterns."""
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16).copy()


def from_bits(b: np.ndarray, device="cpu") -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(b).view(np.int16)).view(torch.bfloat16).to(device)


def activations(g: torch.Generator, M: int, K: int, kind: str = "normal") -> torch.Tensor:
    """bf16 [M, K]: N(0,1) or Student-t(df=3) with 8 channels x50 (config 5)."""
    if kind == "normal":
        x = torch.randn(M, K, generator=g)
    else:
        normal = torch.randn(M, K, generator=g)
        chi2 = torch.randn(M, K, 3, generator=g).square().sum(-1)
        x = normal / torch.sqrt(chi2 / 3.0)
        idx = torch.arange(8) * (K // 8) + 3
        x[:, idx] *= 50.0
    return x.to(torch.bfloat16)


def int8_bank(g: torch.Generator, K: int, H: int, scale_lo=1e-3, scale_hi=1e-2, KH: int = 0, centered=False,
              pow2_smoothing=False, bias=True):
    """A gate/up bank in the reference's layout (earlier_gate_up_screen.py:30-33): W = [Wg; Wu] int8
    [2H, KL] uniform in [-127, 127], per-output-channel scales U(lo, hi).  KH > 0 adds BF16 outlier
    columns (high_columns) and their weights."""
    N2 = 2 * H
    perm = torch.randperm(K, generator=g)
    high = perm[:KH].sort().values
    keep = torch.ones(K, dtype=torch.bool)
    keep[high] = False
    low = keep.nonzero().flatten()
    KL = len(low)
    w = torch.randint(-127, 128, (N2, KL), generator=g, dtype=torch.int32).to(torch.int8)
    sw = (scale_lo + (scale_hi - scale_lo) * torch.rand(N2, generator=g)).float()
    # a non-zero bias makes the dequant's final add observable (bias = centers @ W_low^T in real banks)
    b = (torch.randn(N2, generator=g) * 0.5).float() if bias else torch.zeros(N2)
    wh = (torch.randn(N2, KH, generator=g) * 0.02).to(torch.bfloat16)
    smoothing = (2.0 ** torch.randint(-2, 3, (KL,), generator=g).float()) if pow2_smoothing else torch.ones(KL)
    centers = (torch.randn(KL, generator=g) * 0.05) if centered else torch.zeros(KL)
    return SimpleNamespace(width=K, centered=bool(centered), low_columns=low.to(torch.int32),
                           high_columns=high.to(torch.int32), low_weight=w.contiguous(), high_weight=wh.contiguous(),
                           smoothing=smoothing.contiguous(), centers=centers.contiguous(), scales=sw.contiguous(),
                           bias=b.contiguous())


def bank_to(bank, device):
    return SimpleNamespace(**{k: (v.to(device) if isinstance(v, torch.Tensor) else v) for k, v in vars(bank).items()})


def bank_numpy(bank):
    """The bank with numpy arrays (bf16 tensors as uint16 bits), for the oracle."""
    out = {}
    for k, v in vars(bank).items():
        if isinstance(v, torch.Tensor):
            out[k] = bits(v) if v.dtype == torch.bfloat16 else v.cpu().numpy()
        else:
            out[k] = v
    return SimpleNamespace(**out)


def ulp_report(got_bits: np.ndarray, want_bits: np.ndarray) -> dict:
    d = ro.ulp_distance_bf16(got_bits, want_bits)
    gf, wf = ro.bf16_to_f32(got_bits), ro.bf16_to_f32(want_bits)
    absdiff = np.abs(gf.astype(np.float64) - wf.astype(np.float64))
    rel = absdiff / np.maximum(np.abs(wf.astype(np.float64)), 1e-30)
    return dict(max_ulp=int(d.max()) if d.size else 0, n_diff=int((d > 0).sum()), n=int(d.size),
                max_abs=float(absdiff.max()) if d.size else 0.0, max_rel=float(rel[absdiff > 0].max()) if (absdiff > 0).any() else 0.0)
