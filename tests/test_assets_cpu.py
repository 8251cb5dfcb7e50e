"""The frozen-bank loader (reaxv2/assets.py drop-in) on the CPU: manifest checksums, payload schema,
banks and the policy's route choice (reaxv2/assets.py:14-82)."""
import hashlib
import json
from types import SimpleNamespace

import pytest
import torch


def write_assets(root, payload, corrupt=None):
    """A manifest directory in the reference's layout: the payload and stand-in kernel binaries."""
    files = {"params.pt": None, "gate_up.cubin": b"gate-up kernels", "sliced.cubin": b"sliced kernels",
             "rot_matrix.bin": b"rotation matrix", "rot_prepare.cubin": b"rotation prepare"}
    torch.save(payload, root / "params.pt")
    for name, data in files.items():
        if data is not None:
            (root / name).write_bytes(data)

    def entry(name):
        digest = hashlib.sha256((root / name).read_bytes()).hexdigest()
        return {"path": name, "sha256": ("0" * 64 if name == corrupt else digest)}
    manifest = {"parameters": entry("params.pt"), "gate_up_kernels": entry("gate_up.cubin"),
                "sliced_projection_kernels": entry("sliced.cubin"),
                "rotated_projection_kernels": {"128": {"matrix": entry("rot_matrix.bin"),
                                                       "prepare": entry("rot_prepare.cubin")},
                                               "64": {"matrix": entry("rot_matrix.bin"),
                                                      "prepare": entry("rot_prepare.cubin")}}}
    (root / "manifest.json").write_text(json.dumps(manifest))


def payload(schema=1, start=12):
    g = torch.Generator().manual_seed(5)
    bank = dict(width=256, low_columns=torch.arange(256, dtype=torch.int32), scales=torch.rand(512, generator=g))
    proj = dict(width=1024, parts=2, group=512, block=256, chunk=512, hp=0, centers=torch.zeros(1024),
                low_weight=torch.zeros(256, 1024, dtype=torch.int8), scales=torch.ones(2, 256), bias=torch.zeros(2, 256))
    return {"schema": schema, "checkpoint_start": start, "gate_up": {12: bank},
            "projections": {(12, "down", 1024): proj, (13, "gdn_input", 1024): dict(proj, block=64)},
            "chunk_for": {(12, "down", 64): 1024, (13, "gdn_input", 64): 1024},
            "projection_routes": {("gdn_input", 64, 8, 128): dict(kernel="slice_m128n128", drop=0),
                                  ("gdn_input", 64, 32, 128): dict(kernel="slice_m64n128", drop=1)},
            "rotation_routes": {("down", 64, 16, 8): dict(kernel="slice_m128n256", drop=0, threads=128),
                                ("down", 64, 48, 8): dict(kernel="slice_m64n128", drop=0, threads=512),
                                ("down", 128, 20, 8): dict(kernel="slice_m128n128", drop=2, threads=64),
                                ("down", 64, 20, 4): dict(kernel="slice_m128n128k64", drop=0, threads=64)},
            "rotation_cap": 8}


def test_assets_load_banks_and_operators(tmp_path):
    from reax_engine_runtime_v3_b200.reaxv2.assets import Assets
    write_assets(tmp_path, payload())
    a = Assets(tmp_path, device="cpu")
    assert set(a.gate_up_banks) == {12} and a.gate_up_banks[12].width == 256
    assert a.projections[12, "down", 1024].low_weight.dtype == torch.int8
    assert sorted(a.rotated) == [64, 128] and a.rotated[128].threads == 128
    assert a.rotated[64].kernel_name(a.projections[12, "down", 1024]) == "rotation_g512_b256_t64"
    assert "gate_up" not in a.payload and "projections" not in a.payload


@pytest.mark.parametrize("bad", ["params.pt", "sliced.cubin", "rot_prepare.cubin"])
def test_assets_checksum_failure(tmp_path, bad):
    from reax_engine_runtime_v3_b200.reaxv2.assets import Assets
    write_assets(tmp_path, payload(), corrupt=bad)
    with pytest.raises(ValueError, match="Inference asset checksum failed: " + bad):
        Assets(tmp_path, device="cpu")


@pytest.mark.parametrize("schema,start", [(2, 12), (1, 11)])
def test_assets_schema_check(tmp_path, schema, start):
    from reax_engine_runtime_v3_b200.reaxv2.assets import Assets
    write_assets(tmp_path, payload(schema, start))
    with pytest.raises(ValueError, match="Unsupported frozen projection schema"):
        Assets(tmp_path, device="cpu")


class Recorder:
    def __init__(self, tag):
        self.tag, self.calls = tag, []

    def project(self, x, bank, kernel, drop):
        self.calls.append((len(x), kernel, drop))
        return self.tag


def core_with_layers(n):
    layers = []
    for i in range(n):
        layer = {"type": "linear_attention" if i % 2 else "full_attention",
                 "mlp": SimpleNamespace(down_proj=SimpleNamespace(weight=torch.zeros(2, 2)))}
        if i % 2:
            layer["fused"] = {"qkv_z": torch.zeros(2, 2)}
            layer["la"] = SimpleNamespace(out_proj=SimpleNamespace(weight=torch.zeros(2, 2)))
        layers.append(layer)
    return SimpleNamespace(ff=SimpleNamespace(layers=layers))


def test_policy_routes(tmp_path):
    from reax_engine_runtime_v3_b200.reaxv2.assets import Assets
    write_assets(tmp_path, payload())
    a = Assets(tmp_path, device="cpu")
    a.sliced = Recorder("sliced")
    a.rotated = {64: Recorder("r64"), 128: Recorder("r128"), 256: Recorder("r256")}
    a.bind(core_with_layers(32))
    p = a.policy
    assert sorted(k for k in p.weights if k[1] == "down")[0] == (12, "down") and (30, "down") in p.weights
    assert (11, "down") not in p.weights and (31, "down") not in p.weights
    assert (13, "gdn_output") in p.weights and (12, "gdn_output") not in p.weights
    # no bank for this (layer, family, length)
    assert p.project(12, "down", torch.zeros(5, 4), 128) is None
    # rotation routes: cap 8 only, same length first, then the nearest rows; threads capped at the bank's block
    assert p.project(12, "down", torch.zeros(17, 4), 64) == "r128"
    assert a.rotated[128].calls[-1] == (17, "slice_m128n256", 0)
    assert p.project(12, "down", torch.zeros(40, 4), 64) == "r256"      # route threads 512 -> block 256
    assert a.rotated[256].calls[-1] == (40, "slice_m64n128", 0)
    # grouped GDN input: rows 20 -> the 32-row route is nearer than the 8-row one? |20-8|=12 > |20-32|=12: tie,
    # the first in table order wins
    assert p.project(13, "gdn_input", torch.zeros(20, 4), 64) == "sliced"
    assert a.sliced.calls[-1] == (20, "slice_m128n128", 0)
    assert p.project(13, "gdn_input", torch.zeros(30, 4), 64) == "sliced"
    assert a.sliced.calls[-1] == (30, "slice_m64n128", 1)
