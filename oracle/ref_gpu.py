"""Launch the reference's own kernels (compiled from source into ``oracle/_ref`` by ``build_ref.py``).

TEST INFRASTRUCTURE ONLY: the GPU tests and the bench's ``ref_kernel`` record use this to run the
reference's own kernels on the same B200 and inputs as ours (never as the product).  The launch
arithmetic restates the reference's launch contract:

* ``hybrid8_*`` (reaxv2/gate_up.py:11-27): kernel parameters (A, W, AH, WH, sa, sw, bias, out, M, N, K,
  KH, mb); mb = max(0, M // bm - drop) * bm; blocks = (mb / bm + ceil((M - mb) / small)) * (N / bn);
  128 threads for the ``w4`` variant, else 256; dynamic shared memory from the config table.
* ``slice_*`` (reaxv2/sliced.py:20-47): parameters (A, W, AH, WH, sa, sw, bias, partials, M, N, KL, KH,
  group, hp, mb), grid (blocks, 1, P), dynamic shared memory read from the ``<name>_required_smem``
  device global of the module.
* ``rotation_g{G}_b{B}_t{T}`` (reaxv2/rotation.py:14-30): parameters (x, centers, low, scales, M, K,
  chunk, parts), grid (M, parts, 1), T threads, 4 * G bytes of dynamic shared memory.
* ``addressed_*`` / ``band_*`` (private/snapshots/model-preaddressed-GUP-r1/wide_warp_hybrid.py:15-35 and
  its tail-bands-r2 copy): the ``hybrid8_*`` parameters at the fixed shape K=2432, KH=128, N=18432;
  (bm, small, bn, threads[, small bn]) from the snapshots' ``wide_warp_shapes.json``; blocks =
  (mb / bm + ceil((M - mb) / small)) * (N / bn), or (mb / bm) * (N / bn) + ceil((M - mb) / small) * (N / sn)
  for the bands; dynamic shared memory from ``<name>_required_smem``.  The activation-table build runs
  ``initialize_silu_table`` (256 x 256 threads) once before its first launch.
* the Triton quantizers ``_prepare`` (reaxv2/quantize.py:5-29, grid (M,)) and ``prepare_kernel``
  (:31-52, grid (M, P)), compiled ahead of time by ``build_ref.py``: 32 * num_warps threads, the
  kernel's own shared memory, and Triton's launcher convention of two trailing scratch pointers (null:
  these kernels use no scratch).
"""
from __future__ import annotations

import ctypes as C
import json
import math
from pathlib import Path

import torch

REF = Path(__file__).resolve().parent / "_ref"

# (big rows, small rows, N tile, dynamic shared memory) of the hybrid8_* kernels
HYBRID = {
    "hybrid8_b128n256_s64n256": (128, 64, 256, 98304),
    "hybrid8_b64n256_s32n256": (64, 32, 256, 81920),
    "hybrid8_b128n128_s32n128": (128, 32, 128, 98304),
    "hybrid8_b128n256k32_s32n256k32": (128, 32, 256, 73728),
    "hybrid8_b64n128k64_s32n128k64": (64, 32, 128, 49152),
    "hybrid8_b64n128k32_s32n128k32": (64, 32, 128, 36864),
    "hybrid8_b64n128k32_min2": (64, 32, 128, 36864),
    "hybrid8_b32n128k32w4_min3": (32, 16, 128, 30720),
}
# (big rows, small rows, N tile, threads) of the slice_* kernels
SLICE = {
    "slice_m128n128": (128, 32, 128, 256),
    "slice_m64n128": (64, 32, 128, 256),
    "slice_m64n128w4": (64, 32, 128, 128),
    "slice_m128n256": (128, 32, 256, 256),
    "slice_m128n128k64": (128, 32, 128, 256),
}
_ATTR_MAX_DYNAMIC_SMEM = 8

# v3 production gate/up variants: (bm, small, bn, threads) and, for the bands, the small tiles' bn
ADDRESSED = {
    "addressed_0_m128n256k32": (128, 32, 256, 256), "addressed_1_m128n256k32": (128, 32, 256, 256),
    "addressed_2_m128n256k64": (128, 32, 256, 256), "addressed_3_m128n256k64": (128, 32, 256, 256),
    "addressed_4_m64n256k32": (64, 32, 256, 256), "addressed_5_m64n256k64": (64, 32, 256, 256),
    "addressed_6_m128n128k32": (128, 32, 128, 256), "addressed_7_m128n128k64": (128, 32, 128, 256),
    "addressed_8_m128n192k32": (128, 32, 192, 384), "addressed_9_m64n192k32": (64, 32, 192, 192),
}
BANDS = {f"band_k{bk}_t{t}n{sn}k{sk}": (128, t, 256, 256, sn)
         for bk in (32, 64) for t, sn in ((64, 256), (96, 256), (160, 128), (192, 128), (224, 128)) for sk in (32, 64)}
PRODUCTION_SHAPE = (2432, 128, 18432)   # (KL, KH, N2) every addressed_* / band_* kernel is built for


def available(name: str) -> bool:
    return (REF / name).exists()


class Module:
    def __init__(self, cubin: str):
        self.cuda = C.CDLL("libcuda.so.1")
        torch.cuda.init()
        torch.zeros(1, device="cuda")              # make torch's primary context current
        self.image = C.create_string_buffer((REF / cubin).read_bytes())
        self.module = C.c_void_p()
        self._check(self.cuda.cuModuleLoadData(C.byref(self.module), self.image))
        self.functions = {}

    @staticmethod
    def _check(status):
        if status:
            raise RuntimeError(f"CUDA driver status {status}")

    def function(self, name: str, smem: int | None):
        if name not in self.functions:
            fn = C.c_void_p()
            self._check(self.cuda.cuModuleGetFunction(C.byref(fn), self.module, name.encode()))
            if smem is None:
                ptr, size, val = C.c_void_p(), C.c_size_t(), C.c_uint()
                self._check(self.cuda.cuModuleGetGlobal_v2(C.byref(ptr), C.byref(size), self.module,
                                                           (name + "_required_smem").encode()))
                self._check(self.cuda.cuMemcpyDtoH_v2(C.byref(val), ptr, 4))
                smem = val.value
            self._check(self.cuda.cuFuncSetAttribute(fn, _ATTR_MAX_DYNAMIC_SMEM, smem))
            self.functions[name] = (fn, smem)
        return self.functions[name]

    def launch(self, fn, grid, threads, smem, pointers, ints):
        args = [C.c_void_p(p) for p in pointers] + [C.c_int(v) for v in ints]
        params = (C.c_void_p * len(args))(*[C.cast(C.pointer(a), C.c_void_p) for a in args])
        stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
        self._check(self.cuda.cuLaunchKernel(fn, grid[0], grid[1], grid[2], threads, 1, 1, smem, stream, params, None))


class Hybrid8(Module):
    """The reference's gate/up kernel (kernel-source/legacy-v2/src/native_hybrid8.cu)."""

    def __init__(self):
        super().__init__("native_hybrid8.cubin")

    def product(self, x, w, xh, wh, sa, sw, bias, name="hybrid8_b128n256_s64n256", drop=0):
        m, k = x.shape
        n = w.shape[0]
        kh = xh.shape[1]
        bm, small, bn, shared = HYBRID[name]
        assert k % 128 == 0 and kh % 64 == 0 and n % bn == 0
        fn, smem = self.function(name, shared)
        mb = max(0, m // bm - drop) * bm
        blocks = (mb // bm + math.ceil((m - mb) / small)) * (n // bn)
        out = torch.empty((m, n // 2), device=x.device, dtype=torch.bfloat16)
        self.launch(fn, (blocks, 1, 1), 128 if "w4" in name else 256, smem,
                    [t.data_ptr() for t in (x, w, xh, wh, sa, sw, bias, out)], [m, n, k, kh, mb])
        return out


class Sliced8(Module):
    """The reference's grouped projection kernel (kernel-source/legacy-v2/src/sliced_linear8.cu)."""

    def __init__(self):
        super().__init__("sliced_linear8.cubin")

    def partials(self, low, w, high, wh, scales, sw, bias, group, hp, parts, name="slice_m128n256", drop=0):
        m, n = low.shape[0], w.shape[0]
        bm, sm, bn, threads = SLICE[name]
        assert n % bn == 0
        fn, smem = self.function(name, None)
        mb = max(0, m // bm - drop) * bm
        blocks = (mb // bm + math.ceil((m - mb) / sm)) * (n // bn)
        out = torch.empty((parts, m, n), device=low.device, dtype=torch.bfloat16)
        self.launch(fn, (blocks, 1, parts), threads, smem,
                    [t.data_ptr() for t in (low, w, high, wh, scales, sw, bias, out)],
                    [m, n, parts * group, parts * hp, group, hp, mb])
        return out


class Rotation(Module):
    """The reference's rotated quantizer (kernel-source/legacy-v2/src/block_rotation.cu)."""

    def __init__(self):
        super().__init__("block_rotation.cubin")

    def prepare(self, x, centers, chunk, parts, group, block, threads):
        m, k = x.shape
        fn, _ = self.function(f"rotation_g{group}_b{block}_t{threads}", 4 * group)
        low = torch.empty((m, parts * group), device=x.device, dtype=torch.int8)
        scales = torch.empty((parts, m), device=x.device, dtype=torch.float32)
        self.launch(fn, (m, parts, 1), threads, 4 * group, [t.data_ptr() for t in (x, centers, low, scales)],
                    [m, k, chunk, parts])
        return low, scales


class Addressed(Module):
    """The reference's v3 production gate/up kernels (kernel-source/src/model-preaddressed-GUP-r1/
    addressed_gate_up.cu, model-preaddressed-GUP-tail-bands-r2/band_gate_up.cu, and the activation-table
    build model-addressed-bulk-activation-table-r1/addressed_gate_up.cu)."""

    def __init__(self, cubin: str = "addressed_gate_up.cubin"):
        super().__init__(cubin)
        if cubin == "addressed_table_gate_up.cubin":
            fn = C.c_void_p()
            self._check(self.cuda.cuModuleGetFunction(C.byref(fn), self.module, b"initialize_silu_table"))
            stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
            self._check(self.cuda.cuLaunchKernel(fn, 256, 1, 1, 256, 1, 1, 0, stream, None, None))
            torch.cuda.synchronize()

    def product(self, x, w, xh, wh, sa, sw, bias, name, drop=0):
        m, k = x.shape
        n = w.shape[0]
        kh = xh.shape[1]
        assert (k, kh, n) == PRODUCTION_SHAPE
        fn, smem = self.function(name, None)
        if name in BANDS:
            bm, small, bn, threads, sn = BANDS[name]
            mb = max(0, m // bm - drop) * bm
            blocks = (mb // bm) * (n // bn) + math.ceil((m - mb) / small) * (n // sn)
        else:
            bm, small, bn, threads = ADDRESSED[name]
            mb = max(0, m // bm - drop) * bm
            blocks = (mb // bm + math.ceil((m - mb) / small)) * (n // bn)
        out = torch.empty((m, n // 2), device=x.device, dtype=torch.bfloat16)
        self.launch(fn, (blocks, 1, 1), threads, smem, [t.data_ptr() for t in (x, w, xh, wh, sa, sw, bias, out)],
                    [m, n, k, kh, mb])
        return out


TRITON = REF / "triton"


def _pow2(n: int) -> int:
    return 1 if n <= 1 else 1 << (n - 1).bit_length()


class TritonQuantizer:
    """The reference's Triton quantizers, run from the cubins ``build_ref.py`` compiled for sm_100."""

    def __init__(self):
        self.cuda = C.CDLL("libcuda.so.1")
        torch.cuda.init()
        torch.zeros(1, device="cuda")
        self.loaded = {}

    @staticmethod
    def available(name: str) -> bool:
        return (TRITON / f"{name}.cubin").exists()

    def _kernel(self, name):
        if name not in self.loaded:
            meta = json.loads((TRITON / f"{name}.json").read_text())
            assert meta["global_scratch_size"] == 0 and meta["profile_scratch_size"] == 0
            image = C.create_string_buffer((TRITON / f"{name}.cubin").read_bytes())
            mod, fn = C.c_void_p(), C.c_void_p()
            Module._check(self.cuda.cuModuleLoadData(C.byref(mod), image))
            Module._check(self.cuda.cuModuleGetFunction(C.byref(fn), mod, meta["kernel"].encode()))
            if meta["shared"] > 48 * 1024:
                Module._check(self.cuda.cuFuncSetAttribute(fn, _ATTR_MAX_DYNAMIC_SMEM, meta["shared"]))
            self.loaded[name] = (image, mod, fn, meta)
        return self.loaded[name]

    def _launch(self, name, grid, pointers):
        _, _, fn, meta = self._kernel(name)
        args = [C.c_void_p(p) for p in pointers] + [C.c_void_p(0), C.c_void_p(0)]   # global / profile scratch
        params = (C.c_void_p * len(args))(*[C.cast(C.pointer(a), C.c_void_p) for a in args])
        stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
        Module._check(self.cuda.cuLaunchKernel(fn, grid[0], grid[1], 1, 32 * meta["num_warps"], 1, 1, meta["shared"],
                                               stream, params, None))

    @staticmethod
    def prepare_name(K, KL, KH, center):
        return f"prepare_K{K}_KL{KL}_KH{KH}_C{int(bool(center))}"

    def prepare(self, x, low_columns, high_columns, smoothing, centers, center):
        """reaxv2.gate_up.Native.project's quantizer call (reaxv2/gate_up.py:31-36)."""
        m, k = x.shape
        kl, kh = len(low_columns), len(high_columns)
        name = self.prepare_name(k, kl, kh, center)
        low = torch.empty((m, kl), device=x.device, dtype=torch.int8)
        high = torch.empty((m, kh), device=x.device, dtype=torch.bfloat16)
        scales = torch.empty(m, device=x.device)
        if m:
            self._launch(name, (m, 1), [t.data_ptr() for t in (x, low_columns, high_columns, smoothing, centers, low,
                                                               high, scales)])
        return low, high, scales

    @staticmethod
    def groups_name(M, K, G, HP, P):
        return f"groups_M{M}_K{K}_G{G}_HP{HP}_P{P}"

    def prepare_groups(self, x, low_columns, high_columns, centers, smoothing, G, HP, P):
        """reaxv2.sliced.Native.project's quantizer call (reaxv2/sliced.py:14-17)."""
        m, k = x.shape
        name = self.groups_name(m, k, G, HP, P)
        low = torch.empty((m, P * G), device=x.device, dtype=torch.int8)
        high = torch.empty((m, P * HP), device=x.device, dtype=torch.bfloat16)
        scales = torch.empty((P, m), device=x.device)
        self._launch(name, (m, P), [t.data_ptr() for t in (x, low_columns, high_columns, centers, smoothing, low, high,
                                                           scales)])
        return low, high, scales
