"""N-sharding of the gate/up operator over the GPUs of one node.

The intermediate dimension H splits into independent slices: rank r of W owns gate rows
[r*H/W, (r+1)*H/W) of the stacked [Wg; Wu] bank and the matching up rows [H + r*H/W, H + (r+1)*H/W),
with their per-channel scales and bias.  Every rank holds the (replicated) activations, quantizes them
itself (per-token quantization gives identical codes on every rank) and writes its own [M, H/W] slice
of the output.  Nothing is exchanged on the path.  Only when a caller asks for the concatenated
[M, H] output does one NCCL all-gather run (``gather=True``); it is separate from the GEMM.

The reference runs on one GPU (no NCCL anywhere in it); this layout follows the scope's multi-GPU rule:
shard the independent units, add a collective only where the caller needs the whole output.
"""
from __future__ import annotations

import copy

import torch


def shard_rows(H: int, rank: int, world: int):
    """Row indices of rank's gate and up slices inside the stacked [Wg; Wu] (2H rows)."""
    if H % world:
        raise ValueError(f"H={H} is not divisible by world size {world}")
    h = H // world
    gate = torch.arange(rank * h, (rank + 1) * h)
    return torch.cat([gate, gate + H]), h


def shard_bank(bank, rank: int, world: int, device=None):
    """This rank's slice of a gate/up bank (fields as in earlier_gate_up_screen.py:30-33)."""
    H = len(bank.low_weight) // 2
    rows, h = shard_rows(H, rank, world)
    b = copy.copy(bank)
    for name in ("low_weight", "high_weight", "scales", "bias"):
        t = getattr(bank, name)
        t = t[rows.to(t.device)].contiguous()
        setattr(b, name, t if device is None else t.to(device))
    if device is not None:
        for name in ("low_columns", "high_columns", "smoothing", "centers"):
            setattr(b, name, getattr(bank, name).to(device))
    return b


def shard_bf16_weight(w: torch.Tensor, rank: int, world: int, device=None):
    """This rank's [2H/W, K] slice of a stacked BF16 [Wg; Wu]."""
    rows, _ = shard_rows(w.shape[0] // 2, rank, world)
    s = w[rows.to(w.device)].contiguous()
    return s if device is None else s.to(device)


def gather_output(local: torch.Tensor, world: int, group=None, layout: str = "concat") -> torch.Tensor:
    """All-gather every rank's [M, h] slice.  ``layout="concat"`` returns [M, W*h] in global column
    order; ``layout="shard"`` returns the gathered [W, M, h] without the reorder copy."""
    M, h = local.shape
    flat = torch.empty((world * M, h), dtype=local.dtype, device=local.device)
    torch.distributed.all_gather_into_tensor(flat, local.contiguous(), group=group)
    stacked = flat.view(world, M, h)
    if layout == "shard":
        return stacked
    return stacked.permute(1, 0, 2).reshape(M, world * h)


class ShardedGateUp:
    """The INT8 gate/up operator over W ranks, one shard per rank.

    ``project(x, name, drop, gather)`` runs the rank's shard through the B200 kernel
    (``reaxv2.gate_up.Native.project``); ``product`` can be replaced only by tests that check the host
    logic on CPU ranks (gloo), where no kernel can run.
    """

    def __init__(self, bank, rank: int, world: int, device=None, group=None, product=None):
        self.rank, self.world, self.group = rank, world, group
        self.H = len(bank.low_weight) // 2
        self.bank = shard_bank(bank, rank, world, device)
        if product is None:
            from .reaxv2.gate_up import Native
            native = Native(None)
            product = lambda x, b, name, drop: native.project(x, b, name, drop)
        self._product = product

    def project(self, x, name="hybrid8_b128n256_s64n256", drop=0, gather=False, layout="concat"):
        local = self._product(x, self.bank, name, drop)
        if not gather or self.world == 1:
            return local
        return gather_output(local, self.world, self.group, layout)
