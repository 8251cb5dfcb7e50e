"""CPU restatement of REAX's quantized MLP gate/up path.

TEST INFRASTRUCTURE ONLY.  Nothing in the product imports this module: only
``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline leg of
``bench.py`` use it, and only as the checker (or, for the CPU baseline, as the
timed port of the reference's arithmetic).

Every function restates one piece of the reference and cites the file:line it
follows (paths relative to the reference project root).  Arithmetic is numpy
float32 (IEEE-754 single, round-to-nearest-even, no fused multiply-add), int8
GEMMs are computed exactly in float64 (every partial sum is an integer below
2**53), and bfloat16 values travel as their uint16 bit patterns.

Pinning:
  * ``prepare_rows``/``prepare_groups``/``reduce_partials``/``fold`` are checked
    against golden vectors produced by running the reference's own Triton
    kernels (``reaxv2/quantize.py``, ``runtime/mixed_origin_bf16.py``) under
    Triton's CPU interpreter (``tests/golden/gen_golden.py``).
  * The SiLU formula is checked against the reference's all-65536-input domain
    check idea (``model-addressed-bulk-activation-table-r1/wide_warp_hybrid.py:41-49``)
    on the GPU, where the reference's own CUDA ``silu_f32`` runs.
  * The INT8 GEMM + dequant + SwiGLU chain is checked on the GPU against the
    reference's own kernel (``kernel-source/legacy-v2/src/native_hybrid8.cu``)
    compiled from source for sm_100a (``oracle/build_ref.py``).
"""
from __future__ import annotations

import numpy as np

F32 = np.float32

# ----------------------------------------------------------------------------------------------- bfloat16 bit helpers


def bf16_to_f32(bits: np.ndarray) -> np.ndarray:
    """bfloat16 bit patterns (uint16) -> float32 values (exact)."""
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16(values: np.ndarray) -> np.ndarray:
    """float32 -> bfloat16 bit patterns, round-to-nearest-even (``__float2bfloat16_rn``).

    NaN inputs map to a quiet NaN with the input's sign and upper payload bits.
    """
    v = np.ascontiguousarray(values, dtype=np.float32)
    u = v.view(np.uint32).astype(np.uint64)
    rounded = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    nan = np.isnan(v)
    if nan.any():
        rounded[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)
    return rounded


def round_bf16(values: np.ndarray) -> np.ndarray:
    """float32 -> nearest bfloat16 value, returned as float32."""
    return bf16_to_f32(f32_to_bf16(values))


# ------------------------------------------------------------------------------------ a1: per-token INT8 quantization


def quant_scale(amax: np.ndarray) -> np.ndarray:
    """``scale = max(absmax, 1e-12) / 127.`` (reaxv2/quantize.py:19), IEEE float32 division."""
    return (np.maximum(np.asarray(amax, dtype=F32), F32(1.0e-12)) / F32(127.0)).astype(F32)


def quant_codes(values: np.ndarray, scale: np.ndarray, clamp: bool = True) -> np.ndarray:
    """``nearbyint(div_rn(value, scale))`` then clamp to [-127, 127] (reaxv2/quantize.py:20-21).

    ``values`` is [M, C] float32, ``scale`` is [M] float32; division is IEEE round-to-nearest
    and ``np.rint`` rounds half to even, as libdevice ``nearbyint`` does.
    """
    q = np.rint(np.asarray(values, dtype=F32) / np.asarray(scale, dtype=F32)[:, None])
    if clamp:
        q = np.clip(q, -127.0, 127.0)
    return q.astype(np.int8)


def prepare_rows(x_bits, low_columns, high_columns, smoothing, centers, center):
    """Restates ``reaxv2.quantize._prepare`` (reaxv2/quantize.py:5-29), one row per program.

    x_bits [M, K] uint16 (bf16), low_columns [KL] int, high_columns [KH] int,
    smoothing/centers [KL] float32, center: bool.
    Returns (low int8 [M, KL], high uint16 [M, KH], scales float32 [M]).
    """
    x_bits = np.asarray(x_bits, dtype=np.uint16)
    M = x_bits.shape[0]
    low_columns = np.asarray(low_columns, dtype=np.int64)
    high_columns = np.asarray(high_columns, dtype=np.int64)
    KL, KH = len(low_columns), len(high_columns)
    if KL:
        value = bf16_to_f32(x_bits[:, low_columns])                      # :12-13
        if center:
            value = value - np.asarray(centers, dtype=F32)[None, :]       # :14-16
        value = value / np.asarray(smoothing, dtype=F32)[None, :]        # :17-18
        scales = quant_scale(np.abs(value).max(axis=1))                  # :19
        low = quant_codes(value, scales)                                  # :20-22
    else:
        scales = np.ones(M, dtype=F32)                                    # :24-25
        low = np.zeros((M, 0), dtype=np.int8)
    high = x_bits[:, high_columns] if KH else np.zeros((M, 0), dtype=np.uint16)   # :26-29
    return low, np.ascontiguousarray(high), scales.astype(F32)


# ---------------------------------------------------------------------------------- a2: grouped (sliced) quantization


def prepare_groups(x_bits, low_columns, high_columns, centers, smoothing, G, HP, P):
    """Restates ``reaxv2.quantize.prepare_kernel`` (reaxv2/quantize.py:31-52), grid (M, P).

    low_columns [P*G] (``-1`` pads a group), high_columns [P*HP] (``-1`` pads), centers and
    smoothing [P*G].  The centre is always subtracted, padded columns quantize as 0, and codes
    are not clamped (:44-45).
    Returns (low int8 [M, P*G], high uint16 [M, P*HP], scales float32 [P, M]).
    """
    x_bits = np.asarray(x_bits, dtype=np.uint16)
    M = x_bits.shape[0]
    src = np.asarray(low_columns, dtype=np.int64).reshape(P, G)
    mean = np.asarray(centers, dtype=F32).reshape(P, G)
    smooth = np.asarray(smoothing, dtype=F32).reshape(P, G)
    low = np.zeros((M, P * G), dtype=np.int8)
    scales = np.zeros((P, M), dtype=F32)
    for part in range(P):
        valid = src[part] >= 0
        raw = bf16_to_f32(x_bits[:, np.maximum(src[part], 0)])            # :38-39
        value = np.where(valid[None, :], (raw - mean[part][None, :]) / smooth[part][None, :], F32(0.0)).astype(F32)  # :40-42
        scale = quant_scale(np.abs(value).max(axis=1))                    # :43
        low[:, part * G:(part + 1) * G] = quant_codes(value, scale, clamp=False)   # :44-45
        scales[part] = scale                                              # :46
    if HP:
        hsrc = np.asarray(high_columns, dtype=np.int64)
        high = np.where(hsrc[None, :] >= 0, x_bits[:, np.maximum(hsrc, 0)], np.uint16(0)).astype(np.uint16)  # :47-52
    else:
        high = np.zeros((M, 0), dtype=np.uint16)
    return low, high, scales


def reduce_partials(partial_bits):
    """Restates ``reaxv2.quantize.reduce_kernel`` (reaxv2/quantize.py:55-61): ordered fp32 sum of bf16 partials."""
    parts = np.asarray(partial_bits, dtype=np.uint16)
    value = bf16_to_f32(parts[0])
    for p in range(1, parts.shape[0]):
        value = (value + bf16_to_f32(parts[p])).astype(F32)
    return f32_to_bf16(value)


# ------------------------------------------------------------------------------------------------ integer GEMM + dequant


def int_gemm(a: np.ndarray, w: np.ndarray) -> np.ndarray:
    """int32 ``acc[m, n] = sum_k a[m, k] * w[n, k]`` (the s8 x s8 -> s32 MMA of hybrid8_tiles.cuh:35-44).

    Computed by torch's CPU integer GEMM (int8 x int8 -> int32, exact: |acc| <= K * 127 * 128 < 2**31 for
    K below 2**17).
    """
    import torch
    a = np.ascontiguousarray(a, dtype=np.int8)
    w = np.ascontiguousarray(w, dtype=np.int8)
    if a.shape[1] == 0 or a.shape[0] == 0 or w.shape[0] == 0:
        return np.zeros((a.shape[0], w.shape[0]), dtype=np.int32)
    assert a.shape[1] < (1 << 17)
    return torch._int_mm(torch.from_numpy(a), torch.from_numpy(w).t()).numpy()


def dequant(acc: np.ndarray, sa: np.ndarray, sw: np.ndarray, bias: np.ndarray) -> np.ndarray:
    """``__fadd_rn(__fmul_rn(__fmul_rn(__int2float_rn(acc), sa[row]), sw[col]), bias[col])``
    (kernel-source/legacy-v2/src/native_hybrid8.cu:23-24): three separately rounded float32 ops."""
    raw = np.asarray(acc, dtype=np.int32).astype(F32)
    v = (raw * np.asarray(sa, dtype=F32)[:, None]).astype(F32)
    v = (v * np.asarray(sw, dtype=F32)[None, :]).astype(F32)
    return (v + np.asarray(bias, dtype=F32)[None, :]).astype(F32)


def bf16_gemm_f32(a_bits: np.ndarray, w_bits: np.ndarray) -> np.ndarray:
    """float32 ``sum_k a[m,k] * w[n,k]`` of bf16 operands: computed in float64 then rounded once.

    The reference accumulates in float32 through ``mma.sync.m16n8k16`` in ascending k
    (hybrid8_tiles.cuh:392-397); that hardware order is not restated, so BF16 results are compared
    with a tolerance.
    """
    if a_bits.shape[1] == 0:
        return np.zeros((a_bits.shape[0], w_bits.shape[0]), dtype=F32)
    a = bf16_to_f32(a_bits).astype(np.float64)
    w = bf16_to_f32(w_bits).astype(np.float64)
    return (a @ w.T).astype(F32)


# ------------------------------------------------------------------------------------------------------- SiLU / SwiGLU


def silu_f32(g: np.ndarray) -> np.ndarray:
    """``silu_f32(x) = __fdiv_rn(x, 1.0f + expf(-x))`` (hybrid8_tiles.cuh:675), every step in float32.

    ``exp`` here is the correctly rounded float32 exponential (float64 ``exp`` rounded once), not
    CUDA's ``expf``; the two can differ by a few float32 ulps, which can move a bfloat16 rounding
    in rare cases.  GPU parity tests therefore also run the oracle with the GPU's own SiLU table.
    """
    g = np.asarray(g, dtype=F32)
    with np.errstate(over="ignore", invalid="ignore"):
        e = np.exp(-g.astype(np.float64)).astype(F32)          # overflows to +inf below about -88.7
    t = (F32(1.0) + e).astype(F32)
    with np.errstate(invalid="ignore", divide="ignore"):
        return (g / t).astype(F32)


_SILU_TABLE = None


def silu_table() -> np.ndarray:
    """``bf16(silu_f32(x))`` for every bfloat16 bit pattern x (uint16[65536] -> uint16[65536]).

    The reference builds the same table on the device (model-addressed-bulk-activation-table-r1/
    addressed_gate_up.cu:115-127) and checks it against the direct formula over the whole domain
    (model-addressed-bulk-activation-table-r1/wide_warp_hybrid.py:41-49).
    """
    global _SILU_TABLE
    if _SILU_TABLE is None:
        allbits = np.arange(65536, dtype=np.uint32).astype(np.uint16)
        _SILU_TABLE = f32_to_bf16(silu_f32(bf16_to_f32(allbits)))
    return _SILU_TABLE


def swiglu_bits(g_bits: np.ndarray, u_bits: np.ndarray, table: np.ndarray | None = None) -> np.ndarray:
    """``swiglu1``: s = bf16(silu_f32(g)); out = bf16(float(s) * float(u)) (hybrid8_tiles.cuh:676-679).

    The same contract as the engine's ``silu_mul`` (vendor/s1eng/s1eng/fused.py:131-164).
    ``table`` (uint16[65536]) replaces the SiLU step when given, e.g. a table read back from the GPU.
    """
    table = silu_table() if table is None else np.asarray(table, dtype=np.uint16)
    s = bf16_to_f32(table[np.asarray(g_bits, dtype=np.uint16)])
    return f32_to_bf16((s * bf16_to_f32(u_bits)).astype(F32))


# ------------------------------------------------------------------------------------------- a4-a9: INT8 gate/up + SwiGLU


def gate_up_values(a, w, ah_bits, wh_bits, sa, sw, bias):
    """float32 [M, N2] gate|up values before bf16 rounding (native_hybrid8.cu:9-26).

    INT8 part exact (dequant as :23-24).  The BF16 outlier part (:26) is accumulated by mma.sync
    m16n8k16 into the registers that hold the dequantized values, 16 columns per instruction in
    ascending order (hybrid8_tiles.cuh:454-550): restated as one float32 add per 16-column block of
    that block's dot product (computed in float64, exact for these products and sums).  The tensor
    cores' own rounding inside a block is not restated, so this models the association, not the bits.
    """
    v = dequant(int_gemm(a, w), sa, sw, bias)
    if ah_bits is not None and np.asarray(ah_bits).shape[1] > 0:
        v = add_bf16_blocks(v, np.asarray(ah_bits), np.asarray(wh_bits))
    return v


def gate_up_ill_conditioned(a, w, ah_bits, wh_bits, sa, sw, bias, slack: float = 2.0 ** -19) -> np.ndarray:
    """bool [M, N2 // 2]: outputs whose gate or up value is small against the magnitudes summed into it
    (|dequant| + sum |ah * wh| over the BF16 columns), so that float32 accumulation errors of ``slack``
    times that magnitude exceed half a bf16 ulp of the value.  Such values can round differently when
    the order or the rounding of the accumulation differs (tensor cores vs exact block sums)."""
    v = gate_up_values(a, w, ah_bits, wh_bits, sa, sw, bias).astype(np.float64)
    mag = np.abs(dequant(int_gemm(a, w), sa, sw, bias).astype(np.float64))
    if ah_bits is not None and np.asarray(ah_bits).shape[1] > 0:
        mag = mag + np.abs(bf16_to_f32(np.asarray(ah_bits)).astype(np.float64)) @ \
            np.abs(bf16_to_f32(np.asarray(wh_bits)).astype(np.float64)).T
    half_ulp = np.maximum(np.abs(v), 2.0 ** -126) * 2.0 ** -9        # half a bf16 ulp (8 significand bits)
    bad = slack * mag > half_ulp
    H = v.shape[1] // 2
    return bad[:, :H] | bad[:, H:]


def add_bf16_blocks(v: np.ndarray, ah_bits: np.ndarray, wh_bits: np.ndarray, block: int = 16) -> np.ndarray:
    """v (float32 [M, N]) + the BF16 columns' products, one float32 rounding per ``block`` columns in
    ascending order (the k-chain of the reference's mma.sync.m16n8k16 accumulation)."""
    a = bf16_to_f32(ah_bits).astype(np.float64)
    w = bf16_to_f32(wh_bits).astype(np.float64)
    v = np.asarray(v, F32).copy()
    for k0 in range(0, a.shape[1], block):
        v = (v.astype(np.float64) + a[:, k0:k0 + block] @ w[:, k0:k0 + block].T).astype(F32)
    return v


def gate_up_pre_bits(a, w, ah_bits, wh_bits, sa, sw, bias):
    """(g, u) uint16 bf16 [M, N2 // 2]: the gate and up values as the SwiGLU receives them
    (hybrid8_tiles.cuh:694-710 rounds each to bf16 first)."""
    v = gate_up_values(a, w, ah_bits, wh_bits, sa, sw, bias)
    H = v.shape[1] // 2
    return f32_to_bf16(v[:, :H]), f32_to_bf16(v[:, H:])


def gate_up_product(a, w, ah_bits, wh_bits, sa, sw, bias, table=None):
    """Restates ``reaxv2.gate_up.Native.product`` (reaxv2/gate_up.py:11-27) and its kernel
    ``hybrid_tile`` (native_hybrid8.cu:4-28) with ``store_tile_swiglu`` (hybrid8_tiles.cuh:681-713).

    a int8 [M, KL]; w int8 [N2, KL] = [Wg; Wu] (gate rows first, hybrid8_tiles.cuh:93-94);
    ah_bits uint16 [M, KH]; wh_bits uint16 [N2, KH]; sa [M]; sw, bias [N2].
    Returns uint16 (bf16) [M, N2 // 2].
    """
    v = gate_up_values(a, w, ah_bits, wh_bits, sa, sw, bias)
    H = v.shape[1] // 2
    g = f32_to_bf16(v[:, :H])
    u = f32_to_bf16(v[:, H:])
    return swiglu_bits(g, u, table)


def gate_up_project(x_bits, bank, table=None):
    """Restates ``reaxv2.gate_up.Native.project`` (reaxv2/gate_up.py:29-37): quantize then product.

    ``bank`` has the fields of the reference's bank namespace (earlier_gate_up_screen.py:30-33):
    width, centered, low_columns, high_columns, low_weight, high_weight, smoothing, centers,
    scales, bias (numpy arrays; high_weight as uint16 bf16 bits).
    """
    low, high, scales = prepare_rows(x_bits, bank.low_columns, bank.high_columns, bank.smoothing,
                                     bank.centers, bank.centered)
    return gate_up_product(low, bank.low_weight, high, bank.high_weight, scales, bank.scales, bank.bias, table)


# ------------------------------------------------------------------------------------------ a11: grouped (sliced) INT8


def sliced_partials(low, w, high_bits, wh_bits, scales, sw, bias, group, hp, parts):
    """Restates ``sliced_tile`` (kernel-source/legacy-v2/src/sliced_linear8.cu:4-32): one bf16 partial per K group.

    low int8 [M, P*G]; w int8 [N, P*G]; high_bits [M, P*HP]; wh_bits [N, P*HP]; scales [P, M];
    sw, bias [P, N].  Returns uint16 [P, M, N].
    """
    M, N = low.shape[0], w.shape[0]
    out = np.zeros((parts, M, N), dtype=np.uint16)
    for z in range(parts):
        k0, k1 = z * group, (z + 1) * group
        v = dequant(int_gemm(low[:, k0:k1], w[:, k0:k1]), scales[z], sw[z], bias[z])      # :11-27
        if hp > 0:
            h0, h1 = z * hp, (z + 1) * hp
            v = add_bf16_blocks(v, high_bits[:, h0:h1], wh_bits[:, h0:h1])  # :28-30
        out[z] = f32_to_bf16(v)                                                          # :31
    return out


def sliced_project(x_bits, bank):
    """Restates ``reaxv2.sliced.Native.project`` (reaxv2/sliced.py:20-47): grouped quant, partials, ordered fold."""
    low, high, scales = prepare_groups(x_bits, bank.low_columns, bank.high_columns, bank.centers, bank.smoothing,
                                       bank.group, bank.hp, bank.parts)
    partials = sliced_partials(low, bank.low_weight, high, bank.high_weight, scales, bank.scales, bank.bias,
                               bank.group, bank.hp, bank.parts)
    if bank.parts == 1:
        return partials[0]
    return reduce_partials(partials)


# ---------------------------------------------------------------------- (f) rotated quantizer of the down projection


def rotation_negated(columns: np.ndarray) -> np.ndarray:
    """Columns whose value the rotation negates: bit 16 of ``column * 1103515245 + 12345`` in uint32
    arithmetic (kernel-source/legacy-v2/src/block_rotation.cu:17-18)."""
    h = (np.asarray(columns, dtype=np.uint64) * np.uint64(1103515245) + np.uint64(12345)) & np.uint64(0xFFFFFFFF)
    return (h & np.uint64(65536)) != 0


def prepare_rotated(x_bits, centers, chunk, parts, group, block):
    """Restates ``prepare_row<G,T,B>`` (kernel-source/legacy-v2/src/block_rotation.cu:5-65), launched by
    ``reaxv2.rotation.Native.prepare`` (reaxv2/rotation.py:14-30) with grid (M, parts).

    For row r and part p, value o in [0, group) is ``x[r, c] - centers[c]`` at column c = p*chunk + o when
    o < chunk and c < K, else 0 (:13-16); it is negated when the column's hash bit is set, even when it is
    a zero pad (:17-18).  Walsh-Hadamard butterflies (lo, hi) -> (lo + hi, lo - hi) then run on aligned
    blocks of ``block`` values, index bit 0 first (:20-45); the scale is ``max(1e-12, absmax) * fl(1/127)``
    (:46-58) and the codes ``float2int_rn(div_rn(v, scale))`` without a clamp (:60-62).
    Returns (low int8 [M, parts*group], scales float32 [parts, M]).
    """
    x = bf16_to_f32(x_bits)
    M, K = x.shape
    centers = np.asarray(centers, dtype=F32)
    low = np.zeros((M, parts * group), dtype=np.int8)
    scales = np.zeros((parts, M), dtype=F32)
    o = np.arange(group)
    for part in range(parts):
        col = part * chunk + o
        valid = (o < chunk) & (col < K)
        v = np.zeros((M, group), dtype=F32)
        v[:, valid] = (x[:, col[valid]] - centers[col[valid]][None, :]).astype(F32)
        v = np.where(rotation_negated(col)[None, :], -v, v).astype(F32)
        d = 1
        while d < block:
            lo = o[(o & d) == 0]
            a, b = v[:, lo].copy(), v[:, lo + d].copy()
            v[:, lo] = (a + b).astype(F32)
            v[:, lo + d] = (a - b).astype(F32)
            d *= 2
        amax = np.fmax.reduce(np.abs(v), axis=1, initial=F32(0.0)).astype(F32)
        scale = (np.fmax(amax, F32(1.0e-12)) * (F32(1.0) / F32(127.0))).astype(F32)
        q = np.rint((v / scale[:, None]).astype(F32))
        q = np.nan_to_num(q, nan=0.0)
        low[:, part * group:(part + 1) * group] = q.astype(np.int32).astype(np.int8)
        scales[part] = scale
    return low, scales


def rotated_project(x_bits, bank):
    """Restates ``reaxv2.rotation.Native.project`` (reaxv2/rotation.py:12-13 -> reaxv2/sliced.py:20-47):
    the rotated quantizer, the grouped INT8 partials (no BF16 columns) and the ordered fold."""
    low, scales = prepare_rotated(x_bits, bank.centers, bank.chunk, bank.parts, bank.group, bank.block)
    partials = sliced_partials(low, bank.low_weight, np.zeros((low.shape[0], 0), np.uint16),
                               np.zeros((bank.low_weight.shape[0], 0), np.uint16), scales, bank.scales, bank.bias,
                               bank.group, 0, bank.parts)
    if bank.parts == 1:
        return partials[0]
    return reduce_partials(partials)


# ------------------------------------------------------------------------------------------- a12: BF16 mixed-origin path


def slice_bounds(K: int, parts: int, chunk: int):
    """K ranges of the split plan: slice s covers [s*chunk, min(K, (s+1)*chunk)) (hybrid8_tiles.cuh:5-7 comment).

    With ``parts == 1`` the single slice is the whole of K (runtime/mixed_origin_bf16.py:28).
    """
    if parts <= 1:
        return [(0, K)]
    return [(min(K, s * chunk), min(K, (s + 1) * chunk)) for s in range(parts)]


def bf16_partials(x_bits, w_bits, split, left, right):
    """Restates ``mixed_origin_bf16.Native.partials`` (runtime/mixed_origin_bf16.py:34-44).

    Rows ``< split`` follow the ``left`` plan, the rest the ``right`` plan (each ``{parts, chunk}``).
    Slice s of a row is bf16(float32 sum over the slice); slices past a row's plan, and empty slices,
    are written as zeros (as the reference's slice kernel does for empty slices, n64_parts.cu:11-16).
    Returns uint16 [max(P0, P1), M, N].
    """
    x_bits = np.asarray(x_bits, dtype=np.uint16)
    w_bits = np.asarray(w_bits, dtype=np.uint16)
    M, K = x_bits.shape
    N = w_bits.shape[0]
    P = max(left["parts"], right["parts"])
    out = np.zeros((P, M, N), dtype=np.uint16)
    for rows, plan in ((slice(0, min(split, M)), left), (slice(min(split, M), M), right)):
        if rows.start >= rows.stop:
            continue
        for s, (k0, k1) in enumerate(slice_bounds(K, plan["parts"], plan["chunk"])):
            if k1 > k0:
                out[s, rows] = f32_to_bf16(bf16_gemm_f32(x_bits[rows, k0:k1], w_bits[:, k0:k1]))
    return out


def fold(parts_bits, split, P0, P1):
    """Restates the ``fold`` kernel (runtime/mixed_origin_bf16.py:8-17): rows < split sum P0 partials,
    the rest P1, in slice order, in float32; one bf16 rounding."""
    parts = np.asarray(parts_bits, dtype=np.uint16)
    M = parts.shape[1]
    count = np.where(np.arange(M) < split, P0, P1)
    value = bf16_to_f32(parts[0])
    for p in range(1, max(P0, P1)):
        active = (p < count)[:, None]
        value = np.where(active, (value + bf16_to_f32(parts[p])).astype(F32), value).astype(F32)
    return f32_to_bf16(value)


def bf16_project(x_bits, w_bits, split, left, right):
    """``mixed_origin_bf16.Native.project`` (runtime/mixed_origin_bf16.py:45-48): partials then fold -> [M, N2] bf16."""
    parts = bf16_partials(x_bits, w_bits, split, left, right)
    return fold(parts, split, left["parts"], right["parts"])


def gate_up_bf16(x_bits, w_bits, split, left, right, table=None):
    """BF16-weight gate/up + SwiGLU: the mixed-origin projection of [Wg; Wu] followed by ``silu_mul``
    (vendor/s1eng/s1eng/fused.py:145-164).  Returns uint16 [M, N2 // 2]."""
    gu = bf16_project(x_bits, w_bits, split, left, right)
    H = gu.shape[1] // 2
    return swiglu_bits(gu[:, :H], gu[:, H:], table)


# --------------------------------------------------------------------------------------------------------- comparison


def ulp_distance_bf16(a_bits: np.ndarray, b_bits: np.ndarray) -> np.ndarray:
    """Distance in bfloat16 ulps between two arrays of finite bf16 bit patterns (signed-magnitude ordering)."""
    def key(bits):
        b = np.asarray(bits, dtype=np.uint16).astype(np.int32)
        mag = b & 0x7FFF
        return np.where(b & 0x8000, -mag, mag)
    return np.abs(key(a_bits) - key(b_bits))


# ----------------------------------------------------------------------------- a13: offline bank construction


def build_bank(weight_bits, count, col_sum, col_square, col_max, protected):
    """Restates ``bank(weight, stats, protected)``
    (private/snapshots/model-exact-addressed-projections-full-r5/earlier_gate_up_screen.py:17-33) in numpy.

    weight_bits uint16 (bf16) [N2, K]; count rows; col_sum, col_square float64 [K] running sums of the
    activations and their squares; col_max float32 [K] running max |activation|.  Returns a namespace
    with the bank fields (low/high columns int32, low_weight int8, high_weight uint16 bits, smoothing,
    centers, scales, bias float32).
    """
    from types import SimpleNamespace
    w = bf16_to_f32(np.asarray(weight_bits, np.uint16))                                # :19 weight.float()
    mean = (np.asarray(col_sum, np.float64) / count).astype(F32)                       # :18
    var = np.asarray(col_square, np.float64) / count - mean.astype(np.float64) ** 2    # :19
    energy = np.sqrt(np.maximum(var, 1e-12).astype(F32))
    norms = np.sqrt((w.astype(np.float64) ** 2).sum(0).astype(F32))                    # float32 column norms
    importance = (energy * norms).astype(F32)
    order = np.argsort(-importance, kind="stable")
    high = np.sort(order[:protected])                                                  # :20
    keep = np.ones(w.shape[1], bool)
    keep[high] = False
    low = np.nonzero(keep)[0]                                                          # :21-22
    values = w[:, low]
    centers = mean[low]                                                                # :23
    amax = (np.asarray(col_max, F32)[low] + np.abs(centers)).astype(F32)
    ratio = np.sqrt((np.maximum(amax, F32(1e-8)) / np.maximum(np.abs(values).max(0), F32(1e-8))).astype(F32))  # :24
    smoothing = np.exp2(np.clip(np.round(np.log2(ratio)), -8, 8)).astype(F32)          # :25
    scaled = (values * smoothing[None, :]).astype(F32)                                 # :26
    scales = (np.maximum(np.abs(scaled).max(1), F32(1e-12)) / F32(127.0)).astype(F32)
    codes = np.clip(np.round((scaled / scales[:, None]).astype(F32)), -127, 127).astype(np.int8)   # :27
    bias = (values.astype(np.float64) @ centers.astype(np.float64)).astype(F32)        # :28
    return SimpleNamespace(width=w.shape[1], centered=True, low_columns=low.astype(np.int32),
                           high_columns=high.astype(np.int32), low_weight=codes,
                           high_weight=np.asarray(weight_bits, np.uint16)[:, high], smoothing=smoothing,
                           centers=centers, scales=scales, bias=bias)
