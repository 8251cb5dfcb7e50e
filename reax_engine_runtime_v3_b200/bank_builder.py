"""Offline construction of a protected INT8 gate/up bank from a BF16 weight and activation statistics.

Restates the reference's calibration step ``bank(weight, stats, protected)``
(private/snapshots/model-exact-addressed-projections-full-r5/earlier_gate_up_screen.py:17-33), which
defines the layout every gate/up kernel here consumes:

1. Per input column, the activation mean and standard deviation from the running sums (float64 sums,
   the variance floored at 1e-12, the root taken in float32).
2. Importance = standard deviation x the column's L2 norm over all output rows.  The ``protected`` most
   important columns stay BF16 (``high_columns``, ascending); the rest are the INT8 columns
   (``low_columns``, ascending).
3. Smoothing per INT8 column: sqrt(activation range / weight range), snapped to a power of two with the
   exponent rounded and clamped to [-8, 8]; the activation range is the observed |max| plus |mean|.
4. Per output row: scale = max |W x smoothing| / 127 (floored at 1e-12), codes = round-half-even of
   W x smoothing / scale clamped to +-127.
5. Centring: the activations are quantized after subtracting the column means (``centered`` banks), so
   the bias restores ``means @ W_low^T`` (accumulated in float64, stored as float32).

The arithmetic is torch's (on whatever device the weight lives), in the same float32 / float64 steps as
the reference, so the same inputs give the same bank bit for bit on the same device.  This is the
offline bank builder, not a hot-path kernel: it runs once per weight.
"""
from __future__ import annotations

from types import SimpleNamespace

import torch

SMOOTHING_EXPONENT_LIMIT = 8     # smoothing in [2^-8, 2^8]
CODE_LIMIT = 127


def column_statistics(stats: dict) -> tuple[torch.Tensor, torch.Tensor]:
    """(mean float32 [K], standard deviation float32 [K]) from running sums ``sum``, ``square`` (float64)
    and ``count``."""
    count = stats["count"]
    mean = (stats["sum"] / count).float()
    variance = stats["square"] / count - mean.double().square()
    return mean, variance.clamp_min(1.0e-12).float().sqrt()


def protected_columns(weight: torch.Tensor, deviation: torch.Tensor, protected: int) -> tuple[torch.Tensor, torch.Tensor]:
    """(high, low) column indices, each ascending: the ``protected`` columns of largest activation
    deviation x weight-column norm, and the others."""
    norms = weight.float().square().sum(0).sqrt()
    high = (deviation * norms).topk(protected).indices.sort().values
    keep = torch.ones(weight.shape[1], device=weight.device, dtype=torch.bool)
    keep[high] = False
    return high, keep.nonzero().flatten()


def power_of_two_smoothing(activation_range: torch.Tensor, weight_range: torch.Tensor) -> torch.Tensor:
    ratio = (activation_range.clamp_min(1.0e-8) / weight_range.clamp_min(1.0e-8)).sqrt()
    exponent = ratio.log2().round().clamp(-SMOOTHING_EXPONENT_LIMIT, SMOOTHING_EXPONENT_LIMIT)
    return 2.0 ** exponent


def quantize_rows(values: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Per-output-row symmetric INT8: (codes int8 [N, KL], scales float32 [N])."""
    scales = values.abs().amax(1).clamp_min(1.0e-12) / float(CODE_LIMIT)
    codes = (values / scales[:, None]).round().clamp(-CODE_LIMIT, CODE_LIMIT).to(torch.int8)
    return codes, scales


def bank(weight: torch.Tensor, stats: dict, protected: int) -> SimpleNamespace:
    """A centred gate/up bank of ``weight`` (bf16 [N2, K], gate rows then up rows) with ``protected``
    BF16 columns.  ``stats``: ``count`` (rows seen), ``sum`` and ``square`` (float64 [K] running sums of
    the activations and their squares) and ``maximum`` (float32 [K] running max of |activation|).
    Returns the fields the kernels read: width, centered, low_columns, high_columns (int32),
    low_weight (int8 [N2, KL]), high_weight (bf16 [N2, KH]), smoothing, centers (float32 [KL]),
    scales, bias (float32 [N2])."""
    mean, deviation = column_statistics(stats)
    high, low = protected_columns(weight, deviation, protected)
    values = weight.float()[:, low]
    centers = mean[low].contiguous()
    activation_range = stats["maximum"][low] + centers.abs()
    smoothing = power_of_two_smoothing(activation_range, values.abs().amax(0))
    codes, scales = quantize_rows(values * smoothing)
    bias = (centers.double()[None, :] @ values.double().T).flatten().float()
    return SimpleNamespace(width=weight.shape[1], centered=True, low_columns=low.to(torch.int32),
                           high_columns=high.to(torch.int32), low_weight=codes.contiguous(),
                           high_weight=weight[:, high].contiguous(), smoothing=smoothing.contiguous(), centers=centers,
                           scales=scales.contiguous(), bias=bias.contiguous())


def statistics_of(x: torch.Tensor) -> dict:
    """Running statistics of activation rows ``x`` [rows, K] in the form ``bank`` takes (the calibration
    observer of earlier_gate_up_screen.py:50-53, over one batch)."""
    v = x.float()
    return {"count": len(v), "sum": v.double().sum(0), "square": v.double().square().sum(0),
            "maximum": v.abs().amax(0)}
