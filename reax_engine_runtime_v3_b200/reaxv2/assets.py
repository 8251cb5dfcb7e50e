"""Drop-in for ``reaxv2/assets.py``: the frozen, inference-only parameter banks and their routing.

``Assets(directory)`` reads ``manifest.json``, checks the sha256 of every file it names, loads the
parameter payload with ``torch.load(weights_only=True, mmap=True)`` (schema 1, checkpoint_start 12), moves
the gate/up banks and the projection banks to the GPU, and builds the operators that run them
(reaxv2/assets.py:14-43).  The kernel binaries the manifest names are still checksummed, as the
reference does, but not loaded: the B200 kernels live in ``libreax_b200.so``, so the operator classes
take the binary paths and ignore them.  ``Policy`` routes a layer's down / GDN projections to the
rotated or grouped INT8 projection (reaxv2/assets.py:46-82).  The manifest layout, the checks and
their messages, and the route choice (same family and cap; a route of the same length first, then the
nearest row count, first in table order on ties) are the reference's, so a bank that loads there
loads here and picks the same route.

``device`` (default ``"cuda"``) is an addition for hosts that only inspect a bank; the reference always
loads onto the GPU.
"""
from __future__ import annotations

import hashlib
import json
from pathlib import Path
from types import SimpleNamespace

import torch

from .driver import NativeInt8
from .gate_up import Native as GateUpNative
from .rotation import Native as RotationNative
from .sliced import Native as SlicedNative

SCHEMA, CHECKPOINT_START = 1, 12
ROUTED_LAYERS = range(12, 31)   # layers whose down / GDN projections the policy may route


def _checked(root: Path, entry: dict) -> Path:
    """The manifest entry's file, after its sha256 matched the manifest's."""
    path = root / entry["path"]
    with path.open("rb") as f:
        digest = hashlib.file_digest(f, "sha256").hexdigest()
    if digest != entry["sha256"]:
        raise ValueError("Inference asset checksum failed: " + entry["path"])
    return path


def _on_device(entries: dict, device) -> dict:
    """Each bank's fields as a namespace, tensors moved to `device`."""
    out = {}
    for key, fields in entries.items():
        out[key] = SimpleNamespace(**{name: (v.to(device=device) if isinstance(v, torch.Tensor) else v)
                                      for name, v in fields.items()})
    return out


def _route(table: dict, family: str, length, rows: int, cap):
    """The table entry for (family, cap) closest to (length, rows): same length first, then row count."""
    keys = [k for k in table if k[0] == family and k[3] == cap]
    return table[min(keys, key=lambda k: (k[1] != length, abs(k[2] - rows)))]


class Assets:
    def __init__(self, directory, device="cuda"):
        root = Path(directory)
        self.manifest = json.loads((root / "manifest.json").read_text())
        payload = torch.load(_checked(root, self.manifest["parameters"]), map_location="cpu",
                             weights_only=True, mmap=True)
        if payload["schema"] != SCHEMA or payload["checkpoint_start"] != CHECKPOINT_START:
            raise ValueError("Unsupported frozen projection schema")
        self.payload = payload
        self.gate_up_banks = _on_device(payload.pop("gate_up"), device)
        self.projections = _on_device(payload.pop("projections"), device)
        self.gate_up = GateUpNative(_checked(root, self.manifest["gate_up_kernels"]))
        self.sliced = SlicedNative(_checked(root, self.manifest["sliced_projection_kernels"]))
        self.rotated = {}
        for threads, files in self.manifest["rotated_projection_kernels"].items():
            _checked(root, files["matrix"])
            quantizer = NativeInt8(_checked(root, files["prepare"]))
            self.rotated[int(threads)] = RotationNative(self.sliced, quantizer, int(threads))

    def bind(self, core):
        self.policy = Policy(core, self)


class Policy:
    def __init__(self, core, assets):
        self.assets = assets
        layers = core.ff.layers
        self.indices = {id(layer): i for i, layer in enumerate(layers)}
        self.source = {"chunk_for": assets.payload["chunk_for"]}
        self.weights, self.by_pointer = {}, {}
        for index in ROUTED_LAYERS:
            if index >= len(layers):
                break
            layer = layers[index]
            down = layer["mlp"].down_proj.weight
            self.weights[index, "down"] = down
            self.by_pointer[down.data_ptr()] = index, "down"
            if layer["type"] == "linear_attention":
                out = layer["la"].out_proj.weight
                self.weights[index, "gdn_input"] = layer["fused"]["qkv_z"]
                self.weights[index, "gdn_output"] = out
                self.by_pointer[out.data_ptr()] = index, "gdn_output"

    def project(self, index, family, x, length):
        """The layer's projection of x through its routed INT8 operator, or None when no bank covers it."""
        payload, assets = self.assets.payload, self.assets
        chunk = payload["chunk_for"].get((index, family, length))
        if chunk is None:
            return None
        bank = assets.projections[index, family, chunk]
        if family == "gdn_input":
            route = _route(payload["projection_routes"], family, length, len(x), 128)
            return assets.sliced.project(x, bank, route["kernel"], route["drop"])
        route = _route(payload["rotation_routes"], family, length, len(x), payload["rotation_cap"])
        return assets.rotated[min(route["threads"], bank.block)].project(x, bank, route["kernel"], route["drop"])
