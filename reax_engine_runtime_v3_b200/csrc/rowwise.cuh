// HBM-bound kernels of the gate/up path: per-token INT8 quantization (row and grouped variants),
// the ordered bf16 partial reductions, the SwiGLU of a computed gate|up pair, the SiLU domain table
// and the bounded-wait self test.
#pragma once

#include "common.cuh"

namespace reax {

// Division used by the quantizer where the reference writes a plain '/' in Triton
// (reaxv2/quantize.py:18-19,42): kDivIeee = IEEE round-to-nearest, kDivFull = PTX div.full.f32.
enum QuantDivision : int { kDivIeee = 0, kDivFull = 1 };
// The division the library's quantizers use: Triton lowers the reference's fp32 '/' to div.full.f32.
constexpr int kQuantDiv = kDivFull;

template <int DIV>
REAX_DEVI float quant_div(float a, float b) {
    if constexpr (DIV == kDivIeee) {
        return __fdiv_rn(a, b);
    } else {
        float r;
        asm("div.full.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
        return r;
    }
}

// Max over `nthreads` threads (tid in [0, nthreads), whole warps) of non-negative, non-NaN floats (each
// thread's fmaxf-accumulated absmax).  For such floats the order of the bit patterns as unsigned
// integers is the order of the values, so one redux.sync per warp finds the warp's max; every thread
// then reads the warps' maxima.  bar() synchronizes the nthreads threads.
template <class Bar>
REAX_DEVI float group_max_nonneg(float v, float* red, int tid, int nthreads, Bar bar) {
    const unsigned m = __reduce_max_sync(0xffffffffu, __float_as_uint(v));
    bar();   // red may still be read by a previous call
    if ((tid & 31) == 0) red[tid / 32] = __uint_as_float(m);
    bar();
    float r = red[0];
    for (int i = 1; i < nthreads / 32; ++i) r = fmaxf(r, red[i]);
    return r;
}

REAX_DEVI float block_max_nonneg(float v, float* red) {
    return group_max_nonneg(v, red, threadIdx.x, blockDim.x, [] { __syncthreads(); });
}

// Eight consecutive quantizer inputs of one row: x[row, src[c]] for c in [c0, c0 + 8), as float.
// With aligned_x the eight columns c0.. of x are requested together with the source indices (the usual
// bank maps low column c to column c); when the indices confirm it, no further load is needed, else the
// sources are loaded as one 16-byte run when consecutive and aligned, or gathered.
REAX_DEVI void load8_columns(const __nv_bfloat16* xr, const int* src, int c0, bool aligned_x, float (&v)[8],
                             int (&idx)[8]) {
    const int4 i0 = __ldg(reinterpret_cast<const int4*>(src + c0));
    const int4 i1 = __ldg(reinterpret_cast<const int4*>(src + c0) + 1);
    uint4 guess = make_uint4(0u, 0u, 0u, 0u);
    if (aligned_x) guess = __ldg(reinterpret_cast<const uint4*>(xr + c0));
    idx[0] = i0.x; idx[1] = i0.y; idx[2] = i0.z; idx[3] = i0.w;
    idx[4] = i1.x; idx[5] = i1.y; idx[6] = i1.z; idx[7] = i1.w;
    bool run = aligned_x && (idx[0] & 7) == 0;
#pragma unroll
    for (int i = 1; i < 8; ++i) run = run && idx[i] == idx[0] + i;
    if (run) {
        const uint4 raw = idx[0] == c0 ? guess : __ldg(reinterpret_cast<const uint4*>(xr + idx[0]));
        const __nv_bfloat16* b = reinterpret_cast<const __nv_bfloat16*>(&raw);
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = __bfloat162float(b[i]);
    } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = __bfloat162float(xr[idx[i]]);
    }
}

// ------------------------------------------------------------------------------ a1: per-token quantization
// One CTA per row (reaxv2/quantize.py:5-29).  Pass 1: v = (x - centre) / smoothing, absmax over the
// row; scale = max(absmax, 1e-12) / 127.  Pass 2 stores nearbyint(div_rn(v, scale)) clamped to
// [-127, 127].  The first kQuantHeld chunks of 8 columns of each thread (rows up to 32 x THREADS
// columns) keep v in registers between the passes; columns past them are recomputed from a re-read of
// the row (same float ops, same result).  Few rows take kQuantThreads threads per row, so that each
// row's work is spread wide; many rows take kQuantThreadsMany, so that more rows are in flight per SM.
constexpr int kQuantHeld = 4;
constexpr int kQuantThreads = 512;
constexpr int kQuantThreadsMany = 128;

// v for 8 consecutive low columns starting at c0.
template <int DIV, bool FAST = false>
REAX_DEVI void quant_prep8(const __nv_bfloat16* xr, const int* low_columns, const float* smoothing,
                           const float* centers, int c0, int center, bool aligned_x, float (&t)[8]) {
    int idx[8];
    load8_columns(xr, low_columns, c0, aligned_x, t, idx);
    const float4 s0 = __ldg(reinterpret_cast<const float4*>(smoothing + c0));
    const float4 s1 = __ldg(reinterpret_cast<const float4*>(smoothing + c0) + 1);
    const float sm[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
    float ce[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if (center) {
        const float4 c0v = __ldg(reinterpret_cast<const float4*>(centers + c0));
        const float4 c1v = __ldg(reinterpret_cast<const float4*>(centers + c0) + 1);
        ce[0] = c0v.x; ce[1] = c0v.y; ce[2] = c0v.z; ce[3] = c0v.w;
        ce[4] = c1v.x; ce[5] = c1v.y; ce[6] = c1v.z; ce[7] = c1v.w;
    }
    // x / 1 is x under both divisions, so chunks whose smoothing is all ones (every BASELINE bank) skip it
    bool ones = FAST;
#pragma unroll
    for (int i = 0; i < 8; ++i) ones = ones && sm[i] == 1.0f;
    if (ones) {
#pragma unroll
        for (int i = 0; i < 8; ++i) t[i] = center ? __fsub_rn(t[i], ce[i]) : t[i];
    } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) t[i] = quant_div<DIV>(center ? __fsub_rn(t[i], ce[i]) : t[i], sm[i]);
    }
}

// nearbyint(div_rn(t, scale)) with a multiply for almost every value.  q = t * inv, inv = fl(1 / scale),
// is within 3 * 2^-24 * |t / scale| of the exact quotient, and the correctly rounded quotient within
// 2^-24 * |t / scale|; the quantizer's |t / scale| stays below 128 (|t| <= absmax, scale ~ absmax / 127),
// so both lie within 2^-15 of each other and round to the same integer unless q is within 2^-14 of a
// half-integer.  Those values, and NaN, take the IEEE division.
template <bool FAST>
REAX_DEVI float quant_rint_div(float t, float scale, float inv) {
    if constexpr (!FAST) return rintf(__fdiv_rn(t, scale));
    const float q = __fmul_rn(t, inv);
    const float n = rintf(q);
    if (fabsf(__fsub_rn(q, n)) < 0.5f - 6.103515625e-05f) return n;
    return rintf(__fdiv_rn(t, scale));
}

// Codes of 8 values, stored at lr[c0..c0+8); inv = fl(1 / scale).
template <bool FAST>
REAX_DEVI void quant_store8(int8_t* lr, int c0, const float (&t)[8], float scale, float inv, bool vec_store) {
    uint32_t packed[2] = {0u, 0u};
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const float r = fminf(fmaxf(quant_rint_div<FAST>(t[i], scale, inv), -127.f), 127.f);
        packed[i / 4] |= (static_cast<uint32_t>(static_cast<int>(r)) & 0xFFu) << (8 * (i % 4));
    }
    if (vec_store) {
        *reinterpret_cast<uint2*>(lr + c0) = make_uint2(packed[0], packed[1]);
    } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) lr[c0 + i] = static_cast<int8_t>((packed[i / 4] >> (8 * (i % 4))) & 0xFFu);
    }
}

// The low columns of one row, quantized by nthreads threads (tid in [0, nthreads)): codes into lr and
// the scale into *scale_out; bar() synchronizes the nthreads threads, red holds nthreads / 32 floats.
// FAST (the many-rows kernels): codes by quant_rint_div's multiply and unit smoothing skipped, for
// throughput; decode rows keep the plain division, whose latency is shorter.  Same codes either way.
template <int DIV, bool FAST, class Bar>
REAX_DEVI void quant_row(const __nv_bfloat16* xr, const int* low_columns, const float* smoothing,
                         const float* centers, int center, bool aligned_x, int KL, int tid, int nthreads, float* red,
                         Bar bar, int8_t* lr, float* scale_out) {
    const int KL8 = KL & ~7;
    const int step = nthreads * 8;
    float held[kQuantHeld][8];
    float amax = 0.f;
#pragma unroll
    for (int j = 0; j < kQuantHeld; ++j) {
        const int c0 = tid * 8 + j * step;
        if (c0 < KL8) {
            quant_prep8<DIV, FAST>(xr, low_columns, smoothing, centers, c0, center, aligned_x, held[j]);
#pragma unroll
            for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(held[j][i]));
        }
    }
    for (int c0 = tid * 8 + kQuantHeld * step; c0 < KL8; c0 += step) {
        float t[8];
        quant_prep8<DIV, FAST>(xr, low_columns, smoothing, centers, c0, center, aligned_x, t);
#pragma unroll
        for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(t[i]));
    }
    for (int c = KL8 + tid; c < KL; c += nthreads) {
        float t = __bfloat162float(xr[__ldg(low_columns + c)]);
        if (center) t = __fsub_rn(t, __ldg(centers + c));
        t = quant_div<DIV>(t, __ldg(smoothing + c));
        amax = fmaxf(amax, fabsf(t));
    }
    amax = group_max_nonneg(amax, red, tid, nthreads, bar);
    const float scale = quant_div<DIV>(fmaxf(amax, 1.0e-12f), 127.0f);
    const float inv = FAST ? __frcp_rn(scale) : 0.f;
    if (tid == 0) *scale_out = scale;
    const bool vec_store = (KL & 7) == 0;
#pragma unroll
    for (int j = 0; j < kQuantHeld; ++j) {
        const int c0 = tid * 8 + j * step;
        if (c0 < KL8) quant_store8<FAST>(lr, c0, held[j], scale, inv, vec_store);
    }
    for (int c0 = tid * 8 + kQuantHeld * step; c0 < KL8; c0 += step) {
        float t[8];
        quant_prep8<DIV, FAST>(xr, low_columns, smoothing, centers, c0, center, aligned_x, t);
        quant_store8<FAST>(lr, c0, t, scale, inv, vec_store);
    }
    for (int c = KL8 + tid; c < KL; c += nthreads) {
        float t = __bfloat162float(xr[__ldg(low_columns + c)]);
        if (center) t = __fsub_rn(t, __ldg(centers + c));
        t = quant_div<DIV>(t, __ldg(smoothing + c));
        const float r = fminf(fmaxf(quant_rint_div<FAST>(t, scale, inv), -127.f), 127.f);
        lr[c] = static_cast<int8_t>(static_cast<int>(r));
    }
}

template <int DIV, int THREADS>
__global__ void __launch_bounds__(THREADS) quant_rows_kernel(const __nv_bfloat16* __restrict__ x,
                                                         const int* __restrict__ low_columns,
                                                         const int* __restrict__ high_columns,
                                                         const float* __restrict__ smoothing,
                                                         const float* __restrict__ centers, int8_t* __restrict__ low,
                                                         __nv_bfloat16* __restrict__ high, float* __restrict__ scales,
                                                         int K, int KL, int KH, int center, int aligned_x) {
    __shared__ float red[32];
    grid_dependency_wait();
    grid_dependents_launch();
    const int row = blockIdx.x;
    const __nv_bfloat16* xr = x + static_cast<size_t>(row) * K;
    if (KL > 0) {
        quant_row<DIV, THREADS != kQuantThreads>(xr, low_columns, smoothing, centers, center, aligned_x != 0, KL,
                                                 threadIdx.x, blockDim.x, red, [] { __syncthreads(); },
                                                 low + static_cast<size_t>(row) * KL, scales + row);
    } else if (threadIdx.x == 0) {
        scales[row] = 1.0f;
    }
    __nv_bfloat16* hr = high + static_cast<size_t>(row) * KH;
    for (int c = threadIdx.x; c < KH; c += blockDim.x) hr[c] = xr[__ldg(high_columns + c)];
}

// Stages the bank's maps in shared memory (lc_s, sm_s, ce_s when center, hc_s) and says whether this
// thread's share of the low columns is the identity map (*ident) and of the smoothing all ones (*unit).
// The low-column map, smoothing and centres (16-byte aligned, checked by the host) are read as 16-byte
// runs, B runs per thread in flight at once, so a CTA pays about one L2 round trip per B runs a thread
// stages instead of one per column it stages.
// issued() runs once, right after the first batch of loads has gone out (the streaming kernel then
// requests its first rows, so that the maps' loads are not queued behind them).
template <int B, class Issued>
REAX_DEVI void stage_maps(const int* __restrict__ low_columns, const float* __restrict__ smoothing,
                          const float* __restrict__ centers, const int* __restrict__ high_columns, int KL, int KH,
                          int center, int* lc_s, float* sm_s, float* ce_s, int* hc_s, bool* ident, bool* unit,
                          Issued issued) {
    bool id = true, un = true;
    const int T = static_cast<int>(blockDim.x), t = static_cast<int>(threadIdx.x);
    const int KL4 = KL / 4;
    bool first = true;
    for (int base = 0; base < KL4; base += B * T) {   // whole batches, so that every thread calls issued()
        int4 a[B];
        float4 sv[B], cv[B];
#pragma unroll
        for (int b = 0; b < B; ++b) {
            const int i = base + t + b * T;
            if (i < KL4) {
                a[b] = __ldg(reinterpret_cast<const int4*>(low_columns) + i);
                sv[b] = __ldg(reinterpret_cast<const float4*>(smoothing) + i);
                if (center) cv[b] = __ldg(reinterpret_cast<const float4*>(centers) + i);
            }
        }
        if (first) issued();
        first = false;
#pragma unroll
        for (int b = 0; b < B; ++b) {
            const int i = base + t + b * T;
            if (i >= KL4) break;
            const int c = 4 * i;
            lc_s[c] = a[b].x; lc_s[c + 1] = a[b].y; lc_s[c + 2] = a[b].z; lc_s[c + 3] = a[b].w;
            sm_s[c] = sv[b].x; sm_s[c + 1] = sv[b].y; sm_s[c + 2] = sv[b].z; sm_s[c + 3] = sv[b].w;
            if (center) { ce_s[c] = cv[b].x; ce_s[c + 1] = cv[b].y; ce_s[c + 2] = cv[b].z; ce_s[c + 3] = cv[b].w; }
            id = id && a[b].x == c && a[b].y == c + 1 && a[b].z == c + 2 && a[b].w == c + 3;
            un = un && sv[b].x == 1.0f && sv[b].y == 1.0f && sv[b].z == 1.0f && sv[b].w == 1.0f;
        }
    }
    if (first) issued();
    for (int c = 4 * KL4 + t; c < KL; c += T) {   // the last KL % 4 columns
        const int src = __ldg(low_columns + c);
        const float s = __ldg(smoothing + c);
        lc_s[c] = src;
        sm_s[c] = s;
        if (center) ce_s[c] = __ldg(centers + c);
        id = id && src == c;
        un = un && s == 1.0f;
    }
    for (int base = t; base < KH; base += B * T) {
        int h[B];
#pragma unroll
        for (int b = 0; b < B; ++b)
            if (base + b * T < KH) h[b] = __ldg(high_columns + base + b * T);
#pragma unroll
        for (int b = 0; b < B; ++b)
            if (base + b * T < KH) hc_s[base + b * T] = h[b];
    }
    *ident = id;
    *unit = un;
}

// Many rows (prefill): persistent CTAs of `groups` groups of kStreamGroupWarps warps, each group with its
// own `depth` row buffers in shared memory.  Group g quantizes the CTA's rows g, g + groups, ... (row j of
// the group is blockIdx.x + (g + groups j) gridDim.x), each loaded whole by a bulk copy (TMA) into the
// group's buffer j % depth; once every thread of the group has read row j, the group requests row
// j + depth into the same buffer.  Only the group that owns a buffer waits on it and refills it, so its
// k-th wait on a buffer always follows its own consumption of phase k - 1 (a parity wait never runs ahead
// of the buffer).  groups x depth rows are in flight per SM with no per-element load instructions, and
// the warps of a group split each row's columns (the absmax is combined through shared memory at a named
// barrier of the group), so enough warps run per SM to hide the arithmetic's latency.  The CTA stages the
// bank's column maps, smoothing and centres in shared memory once.  When the low columns are the identity
// map, the smoothing all ones and there is no centring (every BASELINE bank), a row is read as 16-byte
// runs: the absmax is a bf16x2 max, and the codes come two at a time from packed float32 pairs (below);
// otherwise each value is gathered and divided as in quant_row.  The float32 operations that decide the
// scale and the codes are quant_row's, so both are the same.  A row whose copy does not land within
// timeout_ns gets a NaN scale and ends its group's work (a failed copy; no other path leaves a row
// unwritten).
constexpr int kStreamGroupWarps = 4;
constexpr int kStreamMaxGroups = 8;
constexpr int kStreamMaxBufs = 32;
constexpr int kStreamBarBytes = kStreamMaxBufs * 8 + kStreamMaxGroups * 2 * kStreamGroupWarps * 4;

// Four codes (the low bytes of a, b, c, d) as one little-endian word.
REAX_DEVI uint32_t pack4_low_bytes(uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
    return __byte_perm(__byte_perm(a, b, 0x0040), __byte_perm(c, d, 0x0040), 0x5410);
}

// NaN-propagating maximum of three float32 values (sm_100 three-input max.NaN).
REAX_DEVI float max3_nan(float a, float b, float c) {
    float d;
    asm("max.NaN.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
    return d;
}
// A bf16x2 word whose two magnitudes are max(|a|, |b|) lane-wise (the signs are the XOR of the inputs');
// a NaN input yields the other input, as fmaxf drops a NaN.
REAX_DEVI uint32_t bf16x2_max_abs(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("max.xorsign.abs.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}
// Float32 absmax of the bf16 values of a row's 16-byte runs, folded into the bf16x2 word m (its
// magnitudes): exact, NaN dropped as fmaxf does.  amax_of(m) reads it out.
REAX_DEVI uint32_t absmax_run(uint32_t m, const uint4 v) {
    return bf16x2_max_abs(m, bf16x2_max_abs(bf16x2_max_abs(v.x, v.y), bf16x2_max_abs(v.z, v.w)));
}
REAX_DEVI float amax_of(uint32_t m) {
    return fmaxf(__uint_as_float((m & 0x7FFFu) << 16), __uint_as_float(m & 0x7FFF0000u));
}

// Codes of four bf16 pairs (the words of a 16-byte run) for scale / inv = rcp_rn(scale), as 8 bytes, when
// every value x of the run has |x| <= the row's absmax (the scale's source).
// Per pair: s = fma(x, inv, 1.5 * 2^23) holds n = rint(x * inv) (exact product) in its low bits, and
// e = fma(x, inv, 1.5 * 2^23 - s) = x * inv - n with one rounding.  inv = (1 / scale)(1 + d), |d| <= 2^-24,
// and |x / scale| <= 127.0001, so x * inv lies within 2^-16 of x / scale, and div_rn(x, scale) within 2^-18
// of x / scale: unless x * inv is within 2^-15 of a half-integer, rint(div_rn(x, scale)) = n, the
// reference's code.  The packed check e^2 - (1/4 - 2^-14) < 0 (|e| < 1/2 - 2^-14, give or take far less
// than the margin) certifies that, and |n| <= 127 (so the clamp at +-127 is a no-op and s's low byte is
// the code) follows from |x| <= absmax: scale = div_full(max(absmax, 1e-12), 127) within 2 ulp, so
// |x * inv| <= 127 (1 + 2^-21).  The eight checks meet in one NaN-propagating max: a run with a value at
// a half-integer, a NaN or an infinite x * inv (a NaN margin) is coded by quant_rint_div and the clamp,
// value by value.
REAX_DEVI uint2 quant_codes8_packed(const uint4 v, float scale, float inv) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
    const uint64_t inv2 = f2(inv, inv), magic2 = f2(12582912.0f, 12582912.0f);
    const uint64_t lim2 = f2(-(0.25f - 6.103515625e-05f), -(0.25f - 6.103515625e-05f));
    uint32_t r[8];
    float t[8];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const uint64_t x = bf16x2_to_f2(w[i]);
        const uint64_t s2 = fma2_rn(x, inv2, magic2);
        const uint64_t e = fma2_rn(x, inv2, sub2_rn(magic2, s2));
        const uint64_t m = fma2_rn(e, e, lim2);
        t[2 * i] = f2_lo(m);
        t[2 * i + 1] = f2_hi(m);
        r[2 * i] = __float_as_uint(f2_lo(s2));
        r[2 * i + 1] = __float_as_uint(f2_hi(s2));
    }
    const float worst = max3_nan(max3_nan(t[0], t[1], t[2]), max3_nan(t[3], t[4], t[5]), max3_nan(t[6], t[7], t[7]));
    if (!(worst < 0.f)) {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const float x = __uint_as_float(i % 2 == 0 ? w[i / 2] << 16 : w[i / 2] & 0xFFFF0000u);
            r[i] = static_cast<uint32_t>(static_cast<int>(fminf(fmaxf(quant_rint_div<true>(x, scale, inv), -127.f), 127.f)));
        }
    }
    return make_uint2(pack4_low_bytes(r[0], r[1], r[2], r[3]), pack4_low_bytes(r[4], r[5], r[6], r[7]));
}

template <int DIV>
__global__ void __launch_bounds__(32 * kStreamGroupWarps * kStreamMaxGroups, 1) quant_rows_stream_kernel(
    const __nv_bfloat16* __restrict__ x, const int* __restrict__ low_columns, const int* __restrict__ high_columns,
    const float* __restrict__ smoothing, const float* __restrict__ centers, int8_t* __restrict__ low,
    __nv_bfloat16* __restrict__ high, float* __restrict__ scales, int M, int K, int KL, int KH, int center, int depth,
    unsigned long long timeout_ns) {
    extern __shared__ __align__(128) uint8_t qs[];
    constexpr int GT = 32 * kStreamGroupWarps;                   // threads of a group
    const int group = threadIdx.x / GT, gt = threadIdx.x % GT;   // group, thread within it
    const int gw = gt / 32, lane = threadIdx.x % 32;
    const int groups = static_cast<int>(blockDim.x) / GT;
    const int nbuf = groups * depth;                             // the host keeps it <= kStreamMaxBufs
    const uint32_t row_bytes = static_cast<uint32_t>(K) * 2u;   // the host keeps K % 8 == 0
    uint64_t* bars = reinterpret_cast<uint64_t*>(qs);           // [group][depth]
    // the warps' maxima of a row, two slots so that row j + 1 can write while row j's are still read
    float* red = reinterpret_cast<float*>(qs + kStreamMaxBufs * 8) + group * 2 * kStreamGroupWarps;   // [2][warp]
    uint8_t* rows = qs + kStreamBarBytes;                        // [group][depth][K] bf16
    int* lc_s = reinterpret_cast<int*>(rows + static_cast<size_t>(nbuf) * row_bytes);
    float* sm_s = reinterpret_cast<float*>(lc_s + KL);
    float* ce_s = sm_s + KL;                                     // KL floats when center
    int* hc_s = reinterpret_cast<int*>(ce_s + (center ? KL : 0));
    if (threadIdx.x == 0) {
        for (int i = 0; i < nbuf; ++i) mbar_init(&bars[i], 1);
        fence_mbar_init();
    }
    __syncthreads();
    grid_dependency_wait();
    grid_dependents_launch();
    // row j of this group, its buffer and that buffer's barrier
    auto row_of = [&](int j) { return static_cast<int>(blockIdx.x) + (group + groups * j) * static_cast<int>(gridDim.x); };
    auto slot_of = [&](int j) { return group * depth + j % depth; };
    auto buf_of = [&](int j) { return reinterpret_cast<__nv_bfloat16*>(rows + static_cast<size_t>(slot_of(j)) * row_bytes); };
    auto fetch = [&](int j) {
        const int r = row_of(j);
        if (r >= M) return;
        mbar_arrive_expect_tx(&bars[slot_of(j)], row_bytes);
        bulk_load(buf_of(j), x + static_cast<size_t>(r) * K, row_bytes, &bars[slot_of(j)]);
    };
    auto group_sync = [&] { named_bar_sync(1 + group, GT); };
    // the bank's maps: their loads go out first and the first rows are requested right after them (queued
    // behind the rows' copies, the maps' loads took microseconds to return)
    bool ident, unit;
    stage_maps<2>(low_columns, smoothing, centers, high_columns, KL, KH, center, lc_s, sm_s, ce_s, hc_s, &ident, &unit,
                  [&] {
                      if (gt == 0)
                          for (int j = 0; j < depth; ++j) fetch(j);
                  });
    const bool aligned_low = (reinterpret_cast<uintptr_t>(low) & 7u) == 0;   // 8-byte code stores
    const bool fast = __syncthreads_and(ident && unit && !center && (KL & 7) == 0 && aligned_low) != 0;
    unit = __syncthreads_and(unit) != 0;

    // One group barrier per row: after it every thread has finished row j - 1 (so its buffer is refilled
    // with row j - 1 + depth) and every warp's maximum of row j (or its failed copy, as -1) is visible.
    for (int j = 0;; ++j) {
        const int r = row_of(j);
        if (r >= M) break;
        const __nv_bfloat16* xb = buf_of(j);
        float* red_j = red + (j & 1) * kStreamGroupWarps;
        // every thread waits (its own view of the copy); a warp in which any thread gave up reports -1
        const bool landed = mbar_wait_bounded_suspend(&bars[slot_of(j)], static_cast<uint32_t>(j / depth) & 1u,
                                                      timeout_ns);
        const bool warp_landed = __all_sync(0xffffffffu, landed);
        // x / 1 is x under both divisions (unit smoothing skips them)
        auto value = [&](int c) {
            float t = __bfloat162float(xb[lc_s[c]]);
            if (center) t = __fsub_rn(t, ce_s[c]);
            return unit ? t : quant_div<DIV>(t, sm_s[c]);
        };
        float amax = 0.f;
        if (KL > 0 && warp_landed) {
            if (fast) {
                // |x| of bf16 pairs by masking the sign bits; a bf16x2 max keeps the larger (NaN dropped, as
                // fmaxf does), which is exactly the float32 absmax of the same values
                uint32_t m = 0u;
#pragma unroll 4
                for (int c8 = gt; c8 < KL / 8; c8 += GT) m = absmax_run(m, reinterpret_cast<const uint4*>(xb)[c8]);
                amax = amax_of(m);
            } else {
                for (int c = gt; c < KL; c += GT) amax = fmaxf(amax, fabsf(value(c)));
            }
            // one redux per warp; the warps' maxima meet through shared memory at the group barrier
            amax = __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(amax)));
        }
        if (lane == 0) red_j[gw] = warp_landed ? amax : -1.0f;
        fence_proxy_async_smem();   // this thread's reads of row j - 1's buffer come before its refill
        group_sync();
        if (gt == 0 && j > 0) fetch(j - 1 + depth);
        bool failed = false;
#pragma unroll
        for (int w = 0; w < kStreamGroupWarps; ++w) {
            failed = failed || red_j[w] < 0.f;
            amax = fmaxf(amax, red_j[w]);
        }
        if (failed) {
            if (gt == 0) scales[r] = __int_as_float(0x7fffffff);
            break;
        }
        if (KL > 0) {
            const float scale = quant_div<DIV>(fmaxf(amax, 1.0e-12f), 127.0f);
            const float inv = __frcp_rn(scale);
            if (gt == 0) scales[r] = scale;
            int8_t* lr = low + static_cast<size_t>(r) * KL;
            if (fast) {
#pragma unroll 2
                for (int c8 = gt; c8 < KL / 8; c8 += GT)
                    *reinterpret_cast<uint2*>(lr + 8 * c8) = quant_codes8_packed(reinterpret_cast<const uint4*>(xb)[c8], scale, inv);
            } else {
                for (int c = gt; c < KL; c += GT)
                    lr[c] = static_cast<int8_t>(static_cast<int>(fminf(fmaxf(quant_rint_div<true>(value(c), scale, inv), -127.f), 127.f)));
            }
        } else if (gt == 0) {
            scales[r] = 1.0f;
        }
        __nv_bfloat16* hr = high + static_cast<size_t>(r) * KH;
        for (int c = gt; c < KH; c += GT) hr[c] = xb[hc_s[c]];
    }
}

// Shared memory of quant_rows_stream_kernel with nbuf (= warps x depth) row buffers of K columns.
inline size_t quant_stream_smem(int K, int KL, int KH, int center, int nbuf) {
    return static_cast<size_t>(kStreamBarBytes) + static_cast<size_t>(nbuf) * K * 2 +
           static_cast<size_t>(KL) * 4 * (center ? 3 : 2) + static_cast<size_t>(KH) * 4;
}

// Dense banks (the low columns are every column in order, unit smoothing, no centring, no high columns:
// every BASELINE bank), many rows: persistent CTAs of kDenseThreads threads, one row at a time each, several
// CTAs per SM.  Each thread holds V 16-byte runs of the row in registers (K = 1024 V columns): the absmax of
// the bf16 values (bf16x2 magnitudes, NaN dropped as fmaxf does), one redux per warp and the warps' maxima
// through shared memory, then the codes from the held runs by quant_codes8_packed -- the float32 operations
// of quant_row, so the same scales and codes.  No shared-memory staging and no bulk copies: the rows' loads
// are plain 16-byte loads, V per thread in flight at once, and the many resident CTAs keep enough rows in
// flight to stream HBM.  The host passes NULL maps for such a bank (reax_quant_rows).
constexpr int kDenseThreads = 128;
// CTAs per SM the compiler budgets registers for (more rows in flight per SM), as many as fit without
// spilling the held runs: 16 for up to two runs per thread, 12 for up to four, 8 beyond
template <int V>
constexpr int dense_min_blocks() { return V <= 2 ? 16 : (V <= 4 ? 12 : 8); }

template <int DIV, int V>
__global__ void __launch_bounds__(kDenseThreads, dense_min_blocks<V>()) quant_rows_dense_kernel(const __nv_bfloat16* __restrict__ x,
                                                                        int8_t* __restrict__ low,
                                                                        float* __restrict__ scales, int M, int K) {
    __shared__ float red[2][kDenseThreads / 32];
    grid_dependency_wait();
    grid_dependents_launch();
    const int t = static_cast<int>(threadIdx.x), w = t / 32;
    int j = 0;
    for (int r = blockIdx.x; r < M; r += gridDim.x, ++j) {
        const uint4* xr = reinterpret_cast<const uint4*>(x + static_cast<size_t>(r) * K);
        uint4 v[V];
#pragma unroll
        for (int i = 0; i < V; ++i) v[i] = __ldcs(xr + t + i * kDenseThreads);   // read once: streaming
        uint32_t m = 0u;
#pragma unroll
        for (int i = 0; i < V; ++i) m = absmax_run(m, v[i]);
        const float wmax = __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(amax_of(m))));
        // two slots: row j + 1 writes the other slot while slow threads may still read row j's
        if ((t & 31) == 0) red[j & 1][w] = wmax;
        __syncthreads();
        float amax = red[j & 1][0];
#pragma unroll
        for (int i = 1; i < kDenseThreads / 32; ++i) amax = fmaxf(amax, red[j & 1][i]);
        const float scale = quant_div<DIV>(fmaxf(amax, 1.0e-12f), 127.0f);
        const float inv = __frcp_rn(scale);
        if (t == 0) scales[r] = scale;
        uint2* lr = reinterpret_cast<uint2*>(low + static_cast<size_t>(r) * K);
#pragma unroll
        for (int i = 0; i < V; ++i) lr[t + i * kDenseThreads] = quant_codes8_packed(v[i], scale, inv);
    }
}

// ---------------------------------------------------------------------------- a2: grouped quantization
// grid (M, P): row `blockIdx.x`, group `blockIdx.y` (reaxv2/quantize.py:31-52).  Sources of -1 pad a
// group and quantize as 0; the centre is always subtracted; the codes are not clamped.
template <int DIV>
__global__ void __launch_bounds__(256) quant_groups_kernel(const __nv_bfloat16* __restrict__ x,
                                                           const int* __restrict__ low_columns,
                                                           const int* __restrict__ high_columns,
                                                           const float* __restrict__ centers,
                                                           const float* __restrict__ smoothing,
                                                           int8_t* __restrict__ low, __nv_bfloat16* __restrict__ high,
                                                           float* __restrict__ scales, int M, int K, int G, int HP,
                                                           int P) {
    __shared__ float red[33];
    grid_dependency_wait();
    grid_dependents_launch();
    const int row = blockIdx.x, part = blockIdx.y;
    const __nv_bfloat16* xr = x + static_cast<size_t>(row) * K;
    float amax = 0.f;
    for (int o = threadIdx.x; o < G; o += blockDim.x) {
        const int pos = part * G + o;
        const int src = __ldg(low_columns + pos);
        float t = 0.f;
        if (src >= 0) t = quant_div<DIV>(__fsub_rn(__bfloat162float(xr[src]), __ldg(centers + pos)), __ldg(smoothing + pos));
        amax = fmaxf(amax, fabsf(t));
    }
    amax = block_max_nonneg(amax, red);
    const float scale = quant_div<DIV>(fmaxf(amax, 1.0e-12f), 127.0f);
    if (threadIdx.x == 0) scales[static_cast<size_t>(part) * M + row] = scale;
    int8_t* lr = low + static_cast<size_t>(row) * P * G;
    for (int o = threadIdx.x; o < G; o += blockDim.x) {
        const int pos = part * G + o;
        const int src = __ldg(low_columns + pos);
        float t = 0.f;
        if (src >= 0) t = quant_div<DIV>(__fsub_rn(__bfloat162float(xr[src]), __ldg(centers + pos)), __ldg(smoothing + pos));
        lr[pos] = static_cast<int8_t>(__float2int_rn(rintf(__fdiv_rn(t, scale))));
    }
    __nv_bfloat16* hr = high + static_cast<size_t>(row) * P * HP;
    for (int o = threadIdx.x; o < HP; o += blockDim.x) {
        const int idx = part * HP + o;
        const int src = __ldg(high_columns + idx);
        hr[idx] = src >= 0 ? xr[src] : __float2bfloat16_rn(0.f);
    }
}

// -------------------------------------------------------------- rotated quantizer of the down projection
// One CTA per (row, part) (block_rotation.cu:5-65, launched by reaxv2/rotation.py:14-30).  The part's
// group values sit in shared memory: the centred input columns, negated by the column's hash bit, zero
// past the part's chunk or past K.  Walsh-Hadamard butterflies (lo, hi) -> (lo + hi, lo - hi) then run
// on aligned blocks of `block` values, one stage per index bit, bit 0 first, each stage's pairs shared
// out over the threads.  Every value goes through the same additions in the same order as in the
// reference (whose thread layout spreads the same stages over lanes, warps and registers), so the
// transform, the scale max(1e-12, absmax) * fl(1/127) and the codes float2int_rn(div_rn(v, scale)) (no
// clamp) are bit-identical.  The kernel is a few short loops, so a CTA starts without fetching a long
// unrolled body.
constexpr int kRotThreads = 256;
constexpr int kRotMaxGroup = 8192;

__global__ void __launch_bounds__(kRotThreads) quant_rotated_kernel(
    const __nv_bfloat16* __restrict__ x, const float* __restrict__ centers, int8_t* __restrict__ low,
    float* __restrict__ scales, int M, int K, int chunk, int parts, int group, int block) {
    extern __shared__ float rot_s[];   // group values, then 32 floats for the maximum
    grid_dependency_wait();
    grid_dependents_launch();
    const int t = threadIdx.x, T = blockDim.x;
    const int row = blockIdx.x, part = blockIdx.y;
    const __nv_bfloat16* xr = x + static_cast<size_t>(row) * K;
    for (int o = t; o < group; o += T) {
        const int c = part * chunk + o;
        float a = 0.f;
        if (o < chunk && c < K) a = __fsub_rn(__bfloat162float(xr[c]), __ldg(centers + c));
        const uint32_t h = static_cast<uint32_t>(c) * 1103515245u + 12345u;
        rot_s[o] = (h & 65536u) ? -a : a;
    }
    for (int d = 1; d < block; d *= 2) {
        __syncthreads();
        for (int q = t; q < group / 2; q += T) {
            const int lo = ((q & ~(d - 1)) << 1) | (q & (d - 1));
            const float a = rot_s[lo], b = rot_s[lo + d];
            rot_s[lo] = __fadd_rn(a, b);
            rot_s[lo + d] = __fsub_rn(a, b);
        }
    }
    __syncthreads();
    float m = 0.f;
    for (int o = t; o < group; o += T) m = fmaxf(m, fabsf(rot_s[o]));
    m = group_max_nonneg(m, rot_s + group, t, T, [] { __syncthreads(); });
    const float scale = __fmul_rn(fmaxf(m, 1.0e-12f), 1.0f / 127.0f);
    if (t == 0) scales[static_cast<size_t>(part) * M + row] = scale;
    int8_t* lr = low + static_cast<size_t>(row) * parts * group + static_cast<size_t>(part) * group;
    for (int o = t; o < group; o += T) lr[o] = static_cast<int8_t>(__float2int_rn(__fdiv_rn(rot_s[o], scale)));
}

// ----------------------------------------------- register-resident rotated quantization (two kernels)
// A thread holds R runs of V consecutive columns, run k at group index o = k T V + t V (T threads, a
// multiple of 32).  Index bits below log2(V) are register bits and the next five lane bits; a block
// wider than 32 V columns has its higher stages exchanged through shared memory by index, two barriers
// each.  Column pairs travel as packed float32 pairs (add, sub and fma .rn.f32x2 round each lane as
// the scalar op does).  The stages run bit 0 first with the reference's roundings.  A lane or exchange
// stage is one fused multiply-add per pair: fma(+1, lo, hi) = lo + hi on the low side and
// fma(-1, hi, lo) = lo - hi on the high side (the product by +-1 is exact, so the one rounding is the
// sum's).  ex holds the group for the exchanges; every thread of the CTA calls together.
template <int V, int R>
REAX_DEVI void rot_stages(uint64_t (&p)[R][V / 2], int t, int T, int block, float* ex) {
    constexpr int W = V / 2;
    const int lane = t & 31;
    // index bit 0, inside a pair (block >= 2), then the register bits between pairs
#pragma unroll
    for (int k = 0; k < R; ++k)
#pragma unroll
        for (int i = 0; i < W; ++i) {
            const float a = f2_lo(p[k][i]), b = f2_hi(p[k][i]);
            p[k][i] = f2(__fadd_rn(a, b), __fsub_rn(a, b));
        }
#pragma unroll
    for (int dp = 1; dp < W; dp *= 2) {
        if (2 * dp >= block) break;
#pragma unroll
        for (int k = 0; k < R; ++k)
#pragma unroll
            for (int i = 0; i < W; ++i) {
                if (i & dp) continue;
                const uint64_t a = p[k][i], b = p[k][i + dp];
                p[k][i] = add2_rn(a, b);
                p[k][i + dp] = sub2_rn(a, b);
            }
    }
    // lane bits (index distance V dl)
#pragma unroll
    for (int dl = 1; dl < 32; dl *= 2) {
        if (V * dl >= block) break;   // the same for the whole CTA
        const float s = (lane & dl) ? -1.f : 1.f;
        const uint64_t sg = f2(s, s);
#pragma unroll
        for (int k = 0; k < R; ++k)
#pragma unroll
            for (int i = 0; i < W; ++i) {
                const float a = __shfl_xor_sync(0xffffffffu, f2_lo(p[k][i]), dl);
                const float b = __shfl_xor_sync(0xffffffffu, f2_hi(p[k][i]), dl);
                p[k][i] = fma2_rn(sg, p[k][i], f2(a, b));
            }
    }
    // wider stages (index distance D >= 32 V) through shared memory
    for (int D = 32 * V; D < block; D *= 2) {
#pragma unroll
        for (int k = 0; k < R; ++k)
#pragma unroll
            for (int i = 0; i < W; ++i) *reinterpret_cast<uint64_t*>(ex + (k * T + t) * V + 2 * i) = p[k][i];
        __syncthreads();
#pragma unroll
        for (int k = 0; k < R; ++k) {
            const int o0 = (k * T + t) * V;
            const float s = (o0 & D) ? -1.f : 1.f;
            const uint64_t sg = f2(s, s);
#pragma unroll
            for (int i = 0; i < W; ++i)
                p[k][i] = fma2_rn(sg, p[k][i], *reinterpret_cast<const uint64_t*>(ex + (o0 ^ D) + 2 * i));
        }
        __syncthreads();
    }
}

// The thread's absmax (fmaxf passes over NaN, as the reference's maximum does).
template <int V, int R>
REAX_DEVI float rot_absmax(const uint64_t (&p)[R][V / 2]) {
    float m = 0.f;
#pragma unroll
    for (int k = 0; k < R; ++k)
#pragma unroll
        for (int i = 0; i < V / 2; ++i) m = fmaxf(m, fmaxf(fabsf(f2_lo(p[k][i])), fabsf(f2_hi(p[k][i]))));
    return m;
}

// The codes float2int_rn(div_rn(v, scale)) of the thread's values, as bytes in the flat order k V + j.
// The code of v is rint(q), q = v * inv with inv = rcp_rn(scale), rounded by adding and removing
// 1.5 * 2^23 (exact for |q| < 2^22; the sum's low byte is the code mod 256).  q is within 2^-16 of
// v / scale and fl(v / scale) within 2^-17, because |v / scale| <= 127 (1 + 2^-22): so when q is more
// than 2^-14 away from a half-integer, rint of either is the same integer.  The check, in packed form:
// t = e e - (1/4 - 2^-14), with e = q - rint(q), is negative when |e| < 0.5 - 2^-14, give or take far
// less than the margin.  If ptxas fuses the packed product into the packed sums after it, the sum and e
// come from the exact product v inv, which is within 2^-17 of v / scale too, and the argument holds
// unchanged.  A thread with any other quotient (or a NaN, which fails the check) divides all its values.
template <int V, int R>
REAX_DEVI void rot_codes(const uint64_t (&p)[R][V / 2], float scale, uint32_t (&w)[(R * V + 3) / 4]) {
    const float inv = __frcp_rn(scale);
    const uint64_t inv2 = f2(inv, inv), magic2 = f2(12582912.0f, 12582912.0f);
    const uint64_t lim2 = f2(-(0.25f - 6.103515625e-05f), -(0.25f - 6.103515625e-05f));
    uint32_t pend0 = 0u, pend1 = 0u;      // the first two codes of a word still to be completed
    bool ok = true;
#pragma unroll
    for (int k = 0; k < R; ++k)
#pragma unroll
        for (int i = 0; i < V / 2; ++i) {
            const uint64_t q = mul2_rn(p[k][i], inv2);
            const uint64_t r = add2_rn(q, magic2);
            const uint64_t e = sub2_rn(q, sub2_rn(r, magic2));
            const uint64_t tt = fma2_rn(e, e, lim2);
            ok = ok && f2_lo(tt) < 0.f && f2_hi(tt) < 0.f;
            const uint32_t c0 = __float_as_uint(f2_lo(r)), c1 = __float_as_uint(f2_hi(r));
            const int f = k * V + 2 * i;   // flat index of c0 among the thread's codes
            if (f % 4 == 0) pend0 = c0, pend1 = c1;
            else w[f / 4] = pack4_low_bytes(pend0, pend1, c0, c1);
        }
    if (!ok) {
#pragma unroll
        for (int k = 0; k < R; ++k)
#pragma unroll
            for (int i = 0; i < V / 2; ++i) {
                const uint32_t c0 = static_cast<uint32_t>(__float2int_rn(__fdiv_rn(f2_lo(p[k][i]), scale)));
                const uint32_t c1 = static_cast<uint32_t>(__float2int_rn(__fdiv_rn(f2_hi(p[k][i]), scale)));
                const int f = k * V + 2 * i;
                if (f % 4 == 0) pend0 = c0, pend1 = c1;
                else w[f / 4] = pack4_low_bytes(pend0, pend1, c0, c1);
            }
    }
    if constexpr ((R * V) % 4 != 0) w[(R * V + 3) / 4 - 1] = pack4_low_bytes(pend0, pend1, 0u, 0u);
}

// The thread's codes at lr[(k T + t) V ...], one vector store per run (V-byte aligned codes).
template <int V, int R>
REAX_DEVI void rot_store(int8_t* lr, int t, int T, const uint32_t (&w)[(R * V + 3) / 4]) {
#pragma unroll
    for (int k = 0; k < R; ++k) {
        int8_t* dst = lr + (k * T + t) * V;
        if constexpr (V == 8) *reinterpret_cast<uint2*>(dst) = make_uint2(w[2 * k], w[2 * k + 1]);
        else if constexpr (V == 4) *reinterpret_cast<uint32_t*>(dst) = w[k];
        else *reinterpret_cast<uint16_t*>(dst) = static_cast<uint16_t>(w[k / 2] >> (16 * (k % 2)));
    }
}

// One CTA of group / V threads per (row, part), V consecutive columns per thread (one run).  The
// column sign is bit 16 of the hash, carried at bit 31 of the hash shifted left by 15 ((h << 15) is
// linear in the column mod 2^32) and xor-ed into the float.  The group's maximum is one redux per warp,
// one barrier and one redux over the warps' maxima.  vec (host-checked: 16-byte aligned x and centers,
// K and chunk multiples of V, V-byte aligned codes) lets a thread load and store its run as vectors.
template <int V>
__global__ void __launch_bounds__(1024) quant_rotated_lanes_kernel(
    const __nv_bfloat16* __restrict__ x, const float* __restrict__ centers, int8_t* __restrict__ low,
    float* __restrict__ scales, int M, int K, int chunk, int parts, int group, int block, int vec) {
    static_assert(V == 2 || V == 4 || V == 8, "two, four or eight columns per thread");
    constexpr int W = V / 2;
    constexpr uint32_t kHashStep = 1103515245u << 15;
    extern __shared__ float rot_s[];   // 32 warp maxima, then the group when it has wider stages
    grid_dependency_wait();
    grid_dependents_launch();
    const int t = threadIdx.x, lane = t & 31, T = blockDim.x;
    const int row = blockIdx.x, part = blockIdx.y;
    const int o0 = t * V, c0 = part * chunk + o0;
    const __nv_bfloat16* xr = x + static_cast<size_t>(row) * K;
    uint64_t p[1][W];
    if (vec && o0 < chunk && c0 < K) {
        uint32_t xw[W];
        float cv[V];
        if constexpr (V == 8) {
            *reinterpret_cast<uint4*>(xw) = __ldg(reinterpret_cast<const uint4*>(xr + c0));
            *reinterpret_cast<float4*>(cv) = __ldg(reinterpret_cast<const float4*>(centers + c0));
            *reinterpret_cast<float4*>(cv + 4) = __ldg(reinterpret_cast<const float4*>(centers + c0) + 1);
        } else if constexpr (V == 4) {
            *reinterpret_cast<uint2*>(xw) = __ldg(reinterpret_cast<const uint2*>(xr + c0));
            *reinterpret_cast<float4*>(cv) = __ldg(reinterpret_cast<const float4*>(centers + c0));
        } else {
            xw[0] = __ldg(reinterpret_cast<const uint32_t*>(xr + c0));
            *reinterpret_cast<float2*>(cv) = __ldg(reinterpret_cast<const float2*>(centers + c0));
        }
#pragma unroll
        for (int i = 0; i < W; ++i) p[0][i] = sub2_rn(bf16x2_to_f2(xw[i]), f2(cv[2 * i], cv[2 * i + 1]));
    } else {
        float a[V];
#pragma unroll
        for (int j = 0; j < V; ++j) {
            const int c = c0 + j;
            a[j] = (o0 + j < chunk && c < K) ? __fsub_rn(__bfloat162float(xr[c]), __ldg(centers + c)) : 0.f;
        }
#pragma unroll
        for (int i = 0; i < W; ++i) p[0][i] = f2(a[2 * i], a[2 * i + 1]);
    }
    const uint32_t hs0 = (static_cast<uint32_t>(c0) * 1103515245u + 12345u) << 15;
#pragma unroll
    for (int i = 0; i < W; ++i) {
        const uint32_t h0 = hs0 + static_cast<uint32_t>(2 * i) * kHashStep;
        const uint32_t h1 = hs0 + static_cast<uint32_t>(2 * i + 1) * kHashStep;
        p[0][i] ^= (static_cast<uint64_t>(h1 & 0x80000000u) << 32) | (h0 & 0x80000000u);
    }
    rot_stages<V, 1>(p, t, T, block, rot_s + 32);
    const unsigned wm = __reduce_max_sync(0xffffffffu, __float_as_uint(rot_absmax<V, 1>(p)));
    if (lane == 0) rot_s[t >> 5] = __uint_as_float(wm);
    __syncthreads();
    const float m = __uint_as_float(__reduce_max_sync(0xffffffffu, lane < (T >> 5) ? __float_as_uint(rot_s[lane]) : 0u));
    const float scale = __fmul_rn(fmaxf(m, 1.0e-12f), 1.0f / 127.0f);
    if (t == 0) scales[static_cast<size_t>(part) * M + row] = scale;
    uint32_t w[(V + 3) / 4];
    rot_codes<V, 1>(p, scale, w);
    int8_t* lr = low + static_cast<size_t>(row) * parts * group + static_cast<size_t>(part) * group;
    if (vec) {
        rot_store<V, 1>(lr, t, T, w);
    } else {
#pragma unroll
        for (int j = 0; j < V; ++j) lr[o0 + j] = static_cast<int8_t>(w[j / 4] >> (8 * (j % 4)));
    }
}

// The same quantizer for launches of many rows: a CTA of T = group / (V R) threads keeps one part's
// column constants in registers and walks the rows blockIdx.x, blockIdx.x + gridDim.x, ..., with the
// inputs of the next kRotAhead - 1 rows requested while it transforms the current one.  The centred,
// sign-flipped input of a valid column is fma(s, x, -s c) with s = +-1: s x - s c is s (x - c) exactly,
// so its one rounding gives s fl(x - c), the reference's value.  A column past the chunk or past K is
// +0; the reference negates some of those zeros, which changes no code and no scale (a zero's sign only
// reaches the sign of a zero sum, and |v| and rint(v / scale) are the same for both zeros).  Needs the
// vector conditions of quant_rotated_lanes_kernel.
constexpr int kRotAhead = 3;   // rows of input a thread of quant_rotated_rows_kernel has requested

template <int V, int R>
__global__ void __launch_bounds__(1024) quant_rotated_rows_kernel(
    const __nv_bfloat16* __restrict__ x, const float* __restrict__ centers, int8_t* __restrict__ low,
    float* __restrict__ scales, int M, int K, int chunk, int parts, int group, int block) {
    static_assert(V == 2 || V == 4 || V == 8, "two, four or eight columns per run");
    constexpr int W = V / 2;                  // packed pairs per run
    constexpr uint32_t kHashStep = 1103515245u << 15;
    extern __shared__ float rot_s[];          // two sets of 32 warp maxima, then the group for exchanges
    float* red = rot_s;
    const int t = threadIdx.x, lane = t & 31, T = blockDim.x, nw = T >> 5;
    const int part = blockIdx.y;
    // the column constants: s = +-1 (bit 16 of the hash, at bit 31 of the hash shifted left by 15) and -s c
    uint64_t s2[R][W], nc2[R][W];
    bool valid[R];
#pragma unroll
    for (int k = 0; k < R; ++k) {
        const int o0 = (k * T + t) * V, c0 = part * chunk + o0;
        valid[k] = o0 < chunk && c0 < K;
        float cv[V];
#pragma unroll
        for (int j = 0; j < V; ++j) cv[j] = 0.f;
        if (valid[k]) {
            if constexpr (V == 8) {
                *reinterpret_cast<float4*>(cv) = __ldg(reinterpret_cast<const float4*>(centers + c0));
                *reinterpret_cast<float4*>(cv + 4) = __ldg(reinterpret_cast<const float4*>(centers + c0) + 1);
            } else if constexpr (V == 4) {
                *reinterpret_cast<float4*>(cv) = __ldg(reinterpret_cast<const float4*>(centers + c0));
            } else {
                *reinterpret_cast<float2*>(cv) = __ldg(reinterpret_cast<const float2*>(centers + c0));
            }
        }
        const uint32_t hs0 = (static_cast<uint32_t>(c0) * 1103515245u + 12345u) << 15;
#pragma unroll
        for (int i = 0; i < W; ++i) {
            const float sa = ((hs0 + static_cast<uint32_t>(2 * i) * kHashStep) & 0x80000000u) ? -1.f : 1.f;
            const float sb = ((hs0 + static_cast<uint32_t>(2 * i + 1) * kHashStep) & 0x80000000u) ? -1.f : 1.f;
            s2[k][i] = f2(sa, sb);
            nc2[k][i] = f2(-sa * cv[2 * i], -sb * cv[2 * i + 1]);   // exact
        }
    }
    grid_dependency_wait();
    grid_dependents_launch();
    const int stride = gridDim.x;
    int row = blockIdx.x;
    // the inputs of rows row, row + stride, ..., kRotAhead rows in flight
    uint32_t in[kRotAhead][R][W];
#pragma unroll
    for (int a = 0; a < kRotAhead; ++a)
#pragma unroll
        for (int k = 0; k < R; ++k)
#pragma unroll
            for (int i = 0; i < W; ++i) in[a][k][i] = 0u;   // invalid runs stay zero
    const auto load_row = [&](int r, uint32_t (&dst)[R][W]) {
        if (r >= M) return;
        const __nv_bfloat16* xr = x + static_cast<size_t>(r) * K + static_cast<size_t>(part) * chunk;
#pragma unroll
        for (int k = 0; k < R; ++k) {
            if (!valid[k]) continue;
            const __nv_bfloat16* src = xr + (k * T + t) * V;
            if constexpr (V == 8) {
                const uint4 u = __ldg(reinterpret_cast<const uint4*>(src));
                dst[k][0] = u.x; dst[k][1] = u.y; dst[k][2] = u.z; dst[k][3] = u.w;
            } else if constexpr (V == 4) {
                const uint2 u = __ldg(reinterpret_cast<const uint2*>(src));
                dst[k][0] = u.x; dst[k][1] = u.y;
            } else {
                dst[k][0] = __ldg(reinterpret_cast<const uint32_t*>(src));
            }
        }
    };
#pragma unroll
    for (int a = 0; a < kRotAhead; ++a) load_row(row + a * stride, in[a]);
    int buf = 0;
    for (; row < M; row += stride) {
        uint64_t p[R][W];
#pragma unroll
        for (int k = 0; k < R; ++k)
#pragma unroll
            for (int i = 0; i < W; ++i) p[k][i] = fma2_rn(s2[k][i], bf16x2_to_f2(in[0][k][i]), nc2[k][i]);
#pragma unroll
        for (int a = 0; a + 1 < kRotAhead; ++a)
#pragma unroll
            for (int k = 0; k < R; ++k)
#pragma unroll
                for (int i = 0; i < W; ++i) in[a][k][i] = in[a + 1][k][i];
        load_row(row + kRotAhead * stride, in[kRotAhead - 1]);
        rot_stages<V, R>(p, t, T, block, rot_s + 64);
        // the group's maximum: one redux per warp, one barrier (the two sets of maxima alternate by row)
        const unsigned wm = __reduce_max_sync(0xffffffffu, __float_as_uint(rot_absmax<V, R>(p)));
        if (lane == 0) red[buf * 32 + (t >> 5)] = __uint_as_float(wm);
        __syncthreads();
        const float m =
            __uint_as_float(__reduce_max_sync(0xffffffffu, lane < nw ? __float_as_uint(red[buf * 32 + lane]) : 0u));
        buf ^= 1;
        const float scale = __fmul_rn(fmaxf(m, 1.0e-12f), 1.0f / 127.0f);
        if (t == 0) scales[static_cast<size_t>(part) * M + row] = scale;
        uint32_t w[(R * V + 3) / 4];
        rot_codes<V, R>(p, scale, w);
        rot_store<V, R>(low + static_cast<size_t>(row) * parts * group + static_cast<size_t>(part) * group, t, T, w);
    }
}

// ------------------------------------------------------------------ a3 / a12: ordered partial reductions
// out[i] = bf16(((float(p0[i]) + float(p1[i])) + ...) over `count(row)` partials, float32 adds in
// partial order (reaxv2/quantize.py:55-61; runtime/mixed_origin_bf16.py:8-17).  With `split` null
// every row sums P0 partials; otherwise rows < split[0] sum P0 and the others P1.  With `vec` set
// (16-byte aligned planes of a multiple of 8 elements, and N % 8 == 0 when split is given) eight
// elements move per 16-byte access.
__global__ void __launch_bounds__(256) fold_partials_kernel(const __nv_bfloat16* __restrict__ parts,
                                                            const int* __restrict__ split,
                                                            __nv_bfloat16* __restrict__ out, long long total,
                                                            int N, int P0, int P1, int vec) {
    grid_dependency_wait();
    const int border = split ? __ldg(split) : 0x7fffffff;
    const int Pm = max(P0, P1);
    const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
    for (long long v = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; v * 8 < total; v += stride) {
        const long long i0 = v * 8;
        // vec: 16-byte aligned planes and, with a split, rows of a multiple of 8 elements
        if (vec && i0 + 8 <= total) {
            const int row = static_cast<int>(i0 / N);
            const int count = row < border ? P0 : P1;
            uint4 raw = __ldg(reinterpret_cast<const uint4*>(parts + i0));
            float acc[8];
            const __nv_bfloat16* b = reinterpret_cast<const __nv_bfloat16*>(&raw);
#pragma unroll
            for (int j = 0; j < 8; ++j) acc[j] = __bfloat162float(b[j]);
            for (int p = 1; p < Pm; ++p) {
                if (p >= count) break;
                raw = __ldg(reinterpret_cast<const uint4*>(parts + p * total + i0));
#pragma unroll
                for (int j = 0; j < 8; ++j) acc[j] = __fadd_rn(acc[j], __bfloat162float(b[j]));
            }
            uint4 o;
            uint32_t* ow = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
            for (int j = 0; j < 4; ++j) ow[j] = pack_bf16x2(__float2bfloat16_rn(acc[2 * j]), __float2bfloat16_rn(acc[2 * j + 1]));
            *reinterpret_cast<uint4*>(out + i0) = o;
        } else {
            for (long long i = i0; i < total && i < i0 + 8; ++i) {
                const int row = static_cast<int>(i / N);
                const int count = row < border ? P0 : P1;
                float acc = __bfloat162float(parts[i]);
                for (int p = 1; p < count; ++p) acc = __fadd_rn(acc, __bfloat162float(parts[p * total + i]));
                out[i] = __float2bfloat16_rn(acc);
            }
        }
    }
}

// ----------------------------------------------------------------------------------------- SwiGLU pair
// out[r, c] = bf16(bf16(silu_f32(g[r, c])) * u[r, c]) for row-strided gate and up views
// (vendor/s1eng/s1eng/fused.py:145-164, the same rounding points as hybrid8_tiles.cuh:676-679).
__global__ void __launch_bounds__(256) silu_mul_kernel(const __nv_bfloat16* __restrict__ g,
                                                       const __nv_bfloat16* __restrict__ u,
                                                       __nv_bfloat16* __restrict__ out, int rows, int cols,
                                                       long long gs, long long us) {
    __shared__ uint16_t tab[kSiluTabBytes / 2];
    silu_table_fill(tab, threadIdx.x, blockDim.x);
    __syncthreads();
    grid_dependency_wait();
    const long long total = static_cast<long long>(rows) * cols;
    const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
    for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < total; i += stride) {
        const long long r = i / cols, c = i % cols;
        const float gv = __bfloat162float(g[r * gs + c]);
        const float uv = __bfloat162float(u[r * us + c]);
        out[i] = swiglu_bf16(gv, uv, tab);
    }
}

// table[i] = bf16(silu_f32(bf16 value with bit pattern i)) for all 65536 patterns.
__global__ void silu_table_kernel(__nv_bfloat16* __restrict__ table) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < 65536) {
        const float x = __bfloat162float(__ushort_as_bfloat16(static_cast<unsigned short>(i)));
        table[i] = __float2bfloat16_rn(silu_f32(x));
    }
}

// ----------------------------------------------------------------------------------- bounded-wait test
// Waits on an mbarrier that nothing ever arrives on, with the same bounded wait the GEMM uses; when
// the limit expires it ORs kStatusSelfTest into *status and returns, leaving the context usable.
__global__ void selftest_wait_kernel(unsigned* status, unsigned long long timeout_ns) {
    __shared__ uint64_t bar;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        fence_mbar_init();
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        if (!mbar_wait_bounded(&bar, 0, timeout_ns, nullptr)) atomicOr(status, kStatusSelfTest);
    }
    __syncthreads();
}

}  // namespace reax
