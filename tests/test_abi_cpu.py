"""CPU checks of the boundary: the C-ABI library builds, loads and exports every declared entry point,
and the Python drop-ins keep the reference's names and call signatures."""
import inspect
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "reax_b200.h"


def declared_symbols():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^REAX_API\s+[\w\s\*]+?\b(reax_\w+)\s*\(", text, flags=re.M)))


def test_header_declares_entry_points():
    names = declared_symbols()
    assert "reax_gate_up_i8" in names and "reax_quant_rows" in names and len(names) >= 15


def test_library_exports_every_declared_symbol():
    from reax_engine_runtime_v3_b200 import _native
    lib = _native.load()
    for name in declared_symbols():
        assert hasattr(lib, name), name
    assert set(_native.SIGNATURES) == set(declared_symbols())
    assert lib.reax_version() == 10000


def test_library_rejects_bad_shapes_without_touching_a_device():
    from reax_engine_runtime_v3_b200 import _native
    lib = _native.load()
    # N2 not a multiple of 256: rejected by host validation before any CUDA call
    rc = lib.reax_gate_up_i8(None, None, None, None, None, None, None, None, 16, 300, 128, 0, 150, None, 0, None)
    assert rc == 1 and b"N2" in lib.reax_last_error()
    rc = lib.reax_quant_rows(None, None, None, None, None, None, None, None, 4, 16, 32, 0, 0, None)
    assert rc == 1
    # empty batch: nothing to do
    assert lib.reax_quant_rows(None, None, None, None, None, None, None, None, 0, 16, 16, 0, 0, None) == 0
    # NULL maps (a dense bank) with centring, or with K not a multiple of 1024: rejected on the host
    rc = lib.reax_quant_rows(None, None, None, None, None, None, None, None, 4, 1024, 1024, 0, 1, None)
    assert rc == 1 and b"dense" in lib.reax_last_error()
    rc = lib.reax_quant_rows(None, None, None, None, None, None, None, None, 4, 1000, 1000, 0, 0, None)
    assert rc == 1 and b"dense" in lib.reax_last_error()
    with pytest.raises(RuntimeError, match="status 1"):
        _native.check(1)


def test_dropin_signatures_match_reference():
    from reax_engine_runtime_v3_b200.reaxv2 import gate_up, sliced, wide_warp_hybrid
    from reax_engine_runtime_v3_b200.runtime import mixed_origin_bf16, split_gated_projection
    params = lambda f: list(inspect.signature(f).parameters)
    assert params(gate_up.Native.product) == ["self", "x", "w", "xh", "wh", "sa", "sw", "bias", "name", "drop"]
    assert params(gate_up.Native.project) == ["self", "x", "p", "name", "drop"]
    assert params(sliced.Native.project) == ["self", "x", "p", "name", "drop", "reference"]
    assert params(sliced.Native.prepare) == ["self", "x", "p"]
    assert params(mixed_origin_bf16.Native.partials) == ["self", "x", "w", "split", "left", "right", "name"]
    assert params(mixed_origin_bf16.Native.project) == ["self", "x", "w", "split", "left", "right", "name"]
    assert params(split_gated_projection.Prepared.project_ready) == ["self", "x", "p", "ready", "name", "drop", "out"]
    assert params(wide_warp_hybrid.Native.product) == params(gate_up.Native.product)
    assert set(gate_up.CONFIGS) == {
        "hybrid8_b128n256_s64n256", "hybrid8_b64n256_s32n256", "hybrid8_b128n128_s32n128",
        "hybrid8_b128n256k32_s32n256k32", "hybrid8_b64n128k64_s32n128k64", "hybrid8_b64n128k32_s32n128k32",
        "hybrid8_b64n128k32_min2", "hybrid8_b32n128k32w4_min3"}
    assert set(mixed_origin_bf16.Native.shapes) == {"origin_m64n128", "origin_m128n128", "origin_m64n256",
                                                    "origin_m32n32"}


def test_install_registers_reference_module_names():
    import sys
    import reax_engine_runtime_v3_b200 as pkg
    saved = {k: sys.modules.get(k) for k in ("reaxv2", "reaxv2.gate_up", "runtime", "runtime.mixed_origin_bf16")}
    try:
        pkg.install()
        import reaxv2.gate_up as g
        import runtime.mixed_origin_bf16 as m
        assert g.__name__.startswith("reax_engine_runtime_v3_b200") and hasattr(m, "fold")
        assert hasattr(sys.modules["reaxv2.quantize"], "_prepare")
        assert hasattr(sys.modules["reaxv2.rotation"], "selected_kernel")
    finally:
        for k, v in saved.items():
            if v is None:
                sys.modules.pop(k, None)
            else:
                sys.modules[k] = v
        for k in list(sys.modules):
            if (k.startswith("reaxv2.") or k.startswith("runtime.")) and sys.modules[k].__name__.startswith(
                    "reax_engine_runtime_v3_b200"):
                sys.modules.pop(k, None)


def test_quantize_launchers_use_triton_call_syntax():
    from reax_engine_runtime_v3_b200.reaxv2 import quantize
    for k in (quantize._prepare, quantize.prepare_kernel, quantize.reduce_kernel):
        assert callable(k[(4,)])
