"""B200-native (sm_100a) implementation of REAX's quantized MLP gate/up path.

Drop-in modules mirror the reference's import names and call signatures:

  reax_engine_runtime_v3_b200.reaxv2.quantize   <- reaxv2/quantize.py   (_prepare, prepare_kernel, reduce_kernel)
  reax_engine_runtime_v3_b200.reaxv2.driver     <- reaxv2/driver.py     (NativeInt8)
  reax_engine_runtime_v3_b200.reaxv2.gate_up    <- reaxv2/gate_up.py    (CONFIGS, Native)
  reax_engine_runtime_v3_b200.reaxv2.sliced     <- reaxv2/sliced.py     (CONFIGS, Native)
  reax_engine_runtime_v3_b200.reaxv2.rotation   <- reaxv2/rotation.py   (Native, selected_kernel)
  reax_engine_runtime_v3_b200.reaxv2.assets     <- reaxv2/assets.py     (Assets, Policy)
  reax_engine_runtime_v3_b200.reaxv2.wide_warp_hybrid <- private/snapshots/*/wide_warp_hybrid.py (Native)
  reax_engine_runtime_v3_b200.runtime.mixed_origin_bf16      <- runtime/mixed_origin_bf16.py
  reax_engine_runtime_v3_b200.runtime.split_gated_projection <- runtime/split_gated_projection.py

``install()`` registers them under the reference's own module names (``reaxv2.gate_up`` ...) so
callers that import those names get this implementation.  Every kernel runs through the C ABI of
``libreax_b200.so``; there is no CPU or library fallback.
"""
from __future__ import annotations

__all__ = ["install", "__version__"]
__version__ = "1.0.0"


def install() -> None:
    """Make ``import reaxv2.gate_up`` (and the other reference module names) resolve to this package."""
    import importlib
    import sys

    from . import reaxv2 as pkg_reaxv2
    from . import runtime as pkg_runtime
    names = {
        "reaxv2": pkg_reaxv2,
        "runtime": pkg_runtime,
    }
    for sub in ("quantize", "driver", "gate_up", "sliced", "rotation", "assets", "wide_warp_hybrid"):
        names[f"reaxv2.{sub}"] = importlib.import_module(f"{__name__}.reaxv2.{sub}")
    for sub in ("mixed_origin_bf16", "split_gated_projection"):
        names[f"runtime.{sub}"] = importlib.import_module(f"{__name__}.runtime.{sub}")
    sys.modules.update(names)
