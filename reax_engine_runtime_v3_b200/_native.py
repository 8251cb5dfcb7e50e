"""ctypes binding of ``libreax_b200.so`` (the C ABI declared in ``include/reax_b200.h``).

The reference binds its kernels the same way: ``reaxv2/driver.py:3-13`` opens a shared library with
``ctypes.CDLL`` and turns every non-zero status into ``RuntimeError``.  There is no fallback: if the
library is missing or the device is not an sm_100 GPU, every entry point raises.
"""
from __future__ import annotations

import ctypes as C
import os
import threading
from pathlib import Path

import torch

LIB_PATH = Path(os.environ.get("REAX_B200_LIB", Path(__file__).resolve().parent / "libreax_b200.so"))

REAX_OK = 0
ERRORS = {1: "invalid argument", 2: "misaligned argument", 3: "CUDA failure", 4: "unsupported device",
          5: "workspace too small"}
STATUS_BITS = {0x1: "timeout waiting for a TMA stage", 0x2: "timeout waiting for a free stage",
               0x4: "timeout waiting for an accumulator", 0x8: "timeout waiting for a free accumulator",
               0x10: "timeout draining in-flight work", 0x20: "self-test wait expired",
               0x40: "a split tile had more contributors than the finisher gathers (plan limit)"}

_P = C.c_void_p
_I = C.c_int
_LL = C.c_longlong
_SZ = C.c_size_t
_ULL = C.c_ulonglong

SIGNATURES = {
    "reax_version": ([], _I),
    "reax_last_error": ([], C.c_char_p),
    "reax_workspace_bytes": ([_I], _SZ),
    "reax_set_wait_timeout_ns": ([_ULL], None),
    "reax_quant_rows": ([_P, _P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _P], _I),
    "reax_quant_rotated": ([_P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _P], _I),
    "reax_quant_groups": ([_P, _P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _P], _I),
    "reax_reduce_partials": ([_P, _P, _LL, _I, _P], _I),
    "reax_fold_partials": ([_P, _P, _P, _I, _I, _I, _I, _P], _I),
    "reax_silu_mul": ([_P, _P, _P, _I, _I, _LL, _LL, _P], _I),
    "reax_silu_table": ([_P, _P], _I),
    "reax_gate_up_i8": ([_P, _P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _P, _SZ, _P], _I),
    "reax_gate_up_i8_static": ([_P, _P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _P, _SZ, _P], _I),
    "reax_gate_up_i8_noalloc": ([_P, _P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _P], _I),
    "reax_project_i8": ([_P, _P, _P, _P, _P, _I, _P, _P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _P, _SZ, _P],
                        _I),
    "reax_gate_up_bf16": ([_P, _P, _P, _I, _I, _I, _I, _P, _SZ, _P], _I),
    "reax_bf16_partials": ([_P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _I, _P, _SZ, _P], _I),
    "reax_sliced_i8": ([_P, _P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _P, _SZ, _P], _I),
    "reax_sliced_i8_static": ([_P, _P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _P, _SZ, _P], _I),
    "reax_selftest_wait": ([_P, _ULL, _P], _I),
    "reax_noalloc_status": ([C.POINTER(C.c_uint), _I, _P], _I),
    "reax_set_stream_sms": ([_P, _I], _I),
}

_lib = None
_lib_lock = threading.Lock()


def load() -> C.CDLL:
    """Open the library once and declare every exported entry point; raises if it is missing."""
    global _lib
    if _lib is None:
        with _lib_lock:
            if _lib is None:
                if not LIB_PATH.exists():
                    raise RuntimeError(f"REAX B200 library not built: {LIB_PATH} is missing "
                                       "(run __graft_entry__.build() or reax_engine_runtime_v3_b200/build_lib.py)")
                lib = C.CDLL(str(LIB_PATH))
                for name, (args, res) in SIGNATURES.items():
                    fn = getattr(lib, name)
                    fn.argtypes = args
                    fn.restype = res
                _lib = lib
    return _lib


def check(status: int) -> None:
    """Raise ``RuntimeError`` for a non-zero C-ABI status, as ``NativeInt8.check`` does (reaxv2/driver.py:11-13)."""
    if status:
        message = load().reax_last_error().decode(errors="replace")
        raise RuntimeError(f"REAX B200 status {status} ({ERRORS.get(status, 'unknown')}): {message}")


def ptr(t: torch.Tensor | None) -> int | None:
    """Device address of a tensor (None for a missing or empty optional operand)."""
    if t is None or t.numel() == 0:
        return None
    return t.data_ptr()


def stream_handle(device: torch.device | None = None) -> int:
    """The current torch stream, as the reference passes it to cuLaunchKernel (reaxv2/gate_up.py:25-26)."""
    return torch.cuda.current_stream(device).cuda_stream


_sm_counts: dict[int, int] = {}


def sm_count(device: torch.device) -> int:
    """Multiprocessors of a CUDA device (cached)."""
    index = device.index if device.index is not None else torch.cuda.current_device()
    n = _sm_counts.get(index)
    if n is None:
        n = _sm_counts[index] = torch.cuda.get_device_properties(index).multi_processor_count
    return n


def require_cuda(*tensors: torch.Tensor) -> None:
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise RuntimeError("REAX B200 kernels take CUDA tensors only (no CPU path)")


# ------------------------------------------------------------------------------------------------------ workspace
_workspaces: dict[tuple[int, int], torch.Tensor] = {}
_ws_lock = threading.Lock()


def workspace(device: torch.device) -> torch.Tensor:
    """Zero-initialised GEMM workspace for (device, current stream), created once and reused.

    The kernels leave it zeroed, so it is never cleared again; one workspace per stream keeps two
    lanes replaying graphs concurrently apart (the reference keys its workspaces by stream too,
    runtime/native_core.py:102-115).
    """
    index = device.index if device.index is not None else torch.cuda.current_device()
    key = (index, stream_handle(device))
    ws = _workspaces.get(key)
    if ws is None:
        with _ws_lock:
            ws = _workspaces.get(key)
            if ws is None:
                size = load().reax_workspace_bytes(index)
                if size == 0:
                    raise RuntimeError("reax_workspace_bytes failed (no CUDA device?)")
                ws = torch.zeros(size, dtype=torch.uint8, device=torch.device("cuda", index))
                _workspaces[key] = ws
    return ws


def read_status(ws: torch.Tensor) -> int:
    """Device status word of a workspace (synchronizes); non-zero means a bounded wait expired."""
    return int(ws[:4].view(torch.int32).item())


def noalloc_status(clear: bool = False) -> int:
    """Status word of the allocation-free entry point's static scratch on the current device, after the
    current stream's work (synchronizes that stream)."""
    v = C.c_uint(0)
    check(load().reax_noalloc_status(C.byref(v), 1 if clear else 0, stream_handle()))
    return int(v.value)


def set_stream_sms(stream: torch.cuda.Stream, sms: int) -> None:
    """Give the GEMM launches on `stream` a share of `sms` SMs (0: the whole GPU); see reax_set_stream_sms."""
    check(load().reax_set_stream_sms(stream.cuda_stream, int(sms)))


def clear_status(ws: torch.Tensor) -> None:
    ws[:4].zero_()


def describe_status(status: int) -> str:
    return ", ".join(v for k, v in STATUS_BITS.items() if status & k) or "ok"
