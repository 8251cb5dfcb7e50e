// tcgen05 GEMM kernels of the gate/up path (sm_100a).
//
// One warp-specialised persistent kernel computes C = A[M, K] x B[N, K]^T tile by tile with the
// 5th-generation tensor cores and hands each accumulator tile to an epilogue.  Twelve warps:
//   warps 0, 2, 3  TMA producers, one box each per K block (B first half / gate rows, B second half /
//                  up rows, A / activation rows), into a smem ring of stages (128B swizzle)
//   warp 1         TMEM allocator + MMA issuer: one thread issues tcgen05.mma (M = 128, K = 32 bytes)
//   warps 4..11    epilogue: tcgen05.ld of its TMEM lane quarter, dequant / SwiGLU / bf16 store
// The control warps (0-3) give registers to the epilogue warps with setmaxnreg.
//
// Token-major tiles: 128 rows of A (tokens) x 256 rows of B.  For the gate/up SwiGLU epilogue the B
// rows are R gate rows W[n0 .. n0+R) followed by the matching up rows W[H+n0 ..) (the interleave of
// the reference's loader, hybrid8_tiles.cuh:93-94; R = 128 unless the plan balances rows per tile),
// so TMEM columns j and R8+j of one lane hold the gate and up accumulators of one output element.
// Weight-major tiles (few tokens): the R gate rows and the R up rows are the A operands of two MMAs
// whose B operand is the activation tile; TMEM lanes are weight rows and columns are tokens.
//
// Work distribution ("stream-K hybrid"): the tile list (grouped GROUP_M x n_tiles order, for L2
// reuse) is cut into data-parallel tiles, dealt round-robin to the CTAs, and a remainder (< 2 waves)
// whose K blocks are split evenly between all CTAs.  A CTA that computes only part of a tile writes
// its int32 partial to its own workspace slot and adds its K-block count to the tile's counter; the
// CTA that completes the tile sums every partial (integer addition: exact, order-free) with its own
// TMEM accumulator and runs the epilogue, then clears the counter.
//
// Every mbarrier wait is bounded (timeout_ns of global time); on expiry the kernel ORs a bit into
// the caller's status word, raises a shared abort flag so the other roles stop, drains its own
// in-flight TMA copies and MMAs (again bounded), frees its TMEM and returns.
#pragma once

#include "common.cuh"

namespace reax {

constexpr int kBM = 128;                        // A rows per tile (MMA M)
constexpr int kBN = 256;                        // B rows per tile (MMA N)
constexpr int kRowBytes = 128;                  // K bytes per stage row: one 128-byte swizzle row
constexpr int kAStage = kBM * kRowBytes;        // 16 KiB
constexpr int kBStage = kBN * kRowBytes;        // 32 KiB
constexpr int kStageBytes = kAStage + kBStage;  // 48 KiB
// Weight-major plans carve the same pool (STAGES x kStageBytes) into up to kMaxStages smaller stages:
// [gate box | up box | activation box], sized by the plan, so more K blocks are in flight when tiles
// have few rows.
constexpr int kMaxStages = 16;
// Stages a weight producer requests before its dependency wait (early_b).  A deeper early request
// only lengthens the TMA queue that the activation's first box waits behind once the wait returns
// (measured on B200: 4 stages beat the whole ring by 1-2 % per decode step).
constexpr int kEarlyStages = 4;
constexpr int kTmemCols = 512;
constexpr int kSlotInts = kBM * kBN;            // one split-tile partial: 128 x 256 int32 (128 KiB)
constexpr int kSwapMaxTok = 64;                 // weight-major tiles: at most 64 token columns per accumulator
// Weight-major output block staged for the stores: per token, the tile's (<= 128) columns placed at
// their 16-byte phase in the output row, so rows of 136 halfwords.
constexpr int kOutStagePitch = kBN / 2 + 8;
constexpr int kOutStageBytes = kSwapMaxTok * kOutStagePitch * 2;
// Token-major tiles with TMA stores use the same region: one 32 x 32 bf16 box per epilogue warp.
constexpr int kOutTmaWarpBytes = 32 * 32 * 2;
// How long the contributor holding a split tile's last K blocks waits for the others to publish
// before it publishes itself (a performance choice; both paths give the same result).
constexpr unsigned long long kFinisherWaitNs = 10000;

// Thread layout: warp 0 issues the TMA copies, warp 1 the MMAs (it also owns TMEM), warps 2-3 only hand
// their registers over, and warps kCtlWarps.. run the epilogue.  Warp w runs on SM sub-partition w % 4,
// so every sub-partition holds one control warp and EPI_WARPS / 4 epilogue warps.
constexpr int kCtlWarps = 4;
constexpr int kCtlThreads = 32 * kCtlWarps;
// Registers per thread after the split (setmaxnreg): the control warps shrink to kCtlRegs and the
// epilogue warps grow to kEpiRegs.  The host launches a variant only when its compiled register count
// R satisfies R * (kCtlWarps + EPI_WARPS) >= kCtlRegs * kCtlWarps + kEpiRegs * EPI_WARPS (with
// 8 epilogue warps R = 168 gives exactly 56 + 2 * 224 per sub-partition), so the growth never waits.
constexpr int kCtlRegs = 64;
constexpr int kEpiRegs = 216;

enum EpilogueKind : int { kEpiSwiglu = 0, kEpiPlain = 1 };

struct TcParams {
    CUtensorMap tm_a;    // INT8 A [M, KL] (K blocks [0, kb_int))
    CUtensorMap tm_b;    // INT8 B [rows, KL]
    CUtensorMap tm_ah;   // BF16 A [M, KH or K] (K blocks [kb_int, kb_int + kb_f16))
    CUtensorMap tm_bh;   // BF16 B [rows, KH or K]
    const float* sa;     // per-row scale of A (INT8 path), indexed part * sa_part_stride + row
    const float* sw;     // per-column scale of B (INT8 path), indexed part * n_part_stride + column
    const float* bias;   // per-column bias (INT8 path)
    __nv_bfloat16* out;  // bf16 output: SwiGLU [M, ldo] or plain [parts][M, ldo]
    long long out_part_stride;  // elements between output parts (plain epilogue)
    int M;               // valid A rows
    int H;               // SwiGLU: row offset of the up half inside B; plain: unused
    int ldo;             // output row stride (elements)
    int kb_int;          // K blocks through kind::i8 (128 int8 each)
    int kb_f16;          // K blocks through kind::f16 (64 bf16 each)
    int kb_int_part;     // K-block offset between consecutive parts (INT8 part of a grouped projection)
    int kb_f16_part;     // same for the BF16 columns
    int sa_part_stride;  // = M for grouped projections, 0 otherwise
    int n_part_stride;   // = N for grouped projections, 0 otherwise
    int m_tiles, n_tiles, parts, group_m;
    int tiles;           // parts * m_tiles * n_tiles
    int dp_tiles;        // tiles dealt whole; tiles [dp_tiles, tiles) are split by K blocks
    long long sk_iters;  // (tiles - dp_tiles) * (kb_int + kb_f16)
    int acc_bufs;        // 2 = double-buffered accumulators; 1 = INT8 region + float32 region of one tile
    int mode;            // 0 = INT8 dequant (+ BF16 columns added), 1 = BF16 only (float32 accumulators)
    int* ws_partials;    // [gridDim.x][2][kSlotInts] int32
    int* ws_counters;    // [2 * gridDim.x] int32, zero between launches
    unsigned* status;    // OR-ed error bits (kStatus*)
    unsigned long long timeout_ns;
    int evict_first_b;   // stream B with an evict-first L2 policy (weights read once)
    int n_tok;           // weight-major (swap) kernels: token columns per accumulator, a multiple of 16 >= M
    int out_vec16;       // out is 16-byte aligned and ldo a multiple of 8: rows can be stored in 16-byte pieces
    // SwiGLU tiles: gate rows (and as many up rows) per tile, <= 128 (128 unless the plan balances
    // R = ceil(H / SMs) rows per tile).  The up rows follow the gate rows tile_rows8 rows further on
    // in the B stage (and in TMEM for token-major tiles).
    int tile_rows;
    int tile_rows8;      // tile_rows rounded up to whole 8-row swizzle atoms
    int a_rows;          // token-major: activation rows per A box (128, or n_tok rounded to 16 for few tokens)
    int stages;          // weight-major pipeline stages (<= kMaxStages)
    int stage_bytes;     // weight-major stage size (a multiple of 1024)
    // The kernel before this one on the stream is this library's quantizer, which signals its dependents
    // only after its own dependency wait: the first weight tiles may be requested before this kernel's
    // wait, since nothing in flight then can still be writing them (not with slice_mode).
    int early_b;
    // Mixed-origin slicing (BF16 partials): parts = P0 + P1 and part z < P0 is slice z of plan 0 (rows
    // < *split), part z >= P0 is slice z - P0 of plan 1 (rows >= *split).  Slice s of a plan covers K
    // blocks [s * chunk_kb, (s + 1) * chunk_kb) clipped to the K extent; its output part is s.
    int slice_mode;
    int plan_parts0;
    int plan_chunk_kb0, plan_chunk_kb1;
    const int* split;
    // CTA pairs (PAIR kernels): tiles are dealt to pairs of CTAs (clusters of two), cta_shift = 1; 0 otherwise
    int cta_shift;
    // Token-major SwiGLU tiles: store the output through shared memory with TMA (tm_out: the output [M, H]
    // bf16, boxes of 32 rows x 32 columns, 64-byte swizzle) instead of per-thread global stores.
    int out_tma;
    CUtensorMap tm_out;
    // INT8 weight-major tiles: K blocks per pipeline stage.  1: one 2-D box per producer and K block (gate
    // rows, up rows, activation rows).  kk > 1 (tiles of at most 64 rows): tm_b is a 4-D map of W viewed as
    // [K blocks][2 halves][H rows][128 bytes] and tm_a a 3-D map of A as [K blocks][M rows][128 bytes], so
    // one copy brings the gate and up rows of kk K blocks and another their activation rows.  Small decode
    // tiles are bound by the number of copies a CTA's TMA unit completes (a few hundred ns each, whatever
    // their size), so fewer, larger copies stream the same rows several times faster.
    int kk;
    // SwiGLU tiles with K-block stages whose [gate | up] slab has at most 64 rows: M = 64 MMAs.  Their
    // accumulator rows 16 q .. 16 q + 15 sit in TMEM lanes 32 q .. 32 q + 15 (lane quarter q).
    int m64;
};

// The unit that tiles are dealt to (a CTA, or a CTA pair) and how many there are.
REAX_DEVI int unit_id(const TcParams& p) { return static_cast<int>(blockIdx.x) >> p.cta_shift; }
REAX_DEVI int unit_count(const TcParams& p) { return static_cast<int>(gridDim.x) >> p.cta_shift; }

struct Segment {
    int tile;    // linear tile index (grouped order)
    int k0;      // first K block
    int k1;      // one past the last K block
    bool whole;  // this CTA computes every K block of the tile
};

struct Cursor {
    int dp_i;
    long long sk;
    long long sk_end;
};

// First stream-K iteration of CTA c: floor(c * S / G).  The host keeps S * (G + 1) below 2^31, so 32-bit
// arithmetic is exact here and in sk_owner.
REAX_DEVI long long sk_begin(const TcParams& p, int c) {
    return static_cast<long long>(static_cast<unsigned>(p.sk_iters) * static_cast<unsigned>(c) / gridDim.x);
}

REAX_DEVI Cursor cursor_init(const TcParams& p) {
    Cursor c;
    c.dp_i = 0;
    c.sk = sk_begin(p, blockIdx.x);
    c.sk_end = sk_begin(p, blockIdx.x + 1);
    return c;
}

// linear tile -> (part, m tile, n tile); inside a part, groups of group_m m-tiles sweep all n-tiles
REAX_DEVI void tile_coords(const TcParams& p, int t, int& part, int& mt, int& nt) {
    const int per_part = p.m_tiles * p.n_tiles;
    part = t / per_part;
    const int r0 = t % per_part;
    const int per_group = p.group_m * p.n_tiles;
    const int g = r0 / per_group, r = r0 % per_group;
    const int first_m = g * p.group_m;
    const int gm = min(p.group_m, p.m_tiles - first_m);
    mt = first_m + r % gm;
    nt = r / gm;
}

// Row range and output part of a tile's plan (slice mode); the whole of [0, M) and `part` otherwise.
REAX_DEVI void tile_plan(const TcParams& p, int part, int split, int& row_lo, int& row_hi, int& out_part) {
    if (!p.slice_mode) {
        row_lo = 0;
        row_hi = p.M;
        out_part = part;
        return;
    }
    const bool second = part >= p.plan_parts0;
    row_lo = second ? split : 0;
    row_hi = second ? p.M : split;
    out_part = second ? part - p.plan_parts0 : part;
}

// K-block range of a data-parallel tile; false when the tile has nothing to compute (slice mode:
// an empty slice, or a tile without rows of its plan).
REAX_DEVI bool tile_active(const TcParams& p, int t, int split, int& k0, int& k1) {
    const int KB = p.kb_int + p.kb_f16;
    if (!p.slice_mode) {
        k0 = 0;
        k1 = KB;
        return true;
    }
    int part, mt, nt;
    tile_coords(p, t, part, mt, nt);
    int row_lo, row_hi, s;
    tile_plan(p, part, split, row_lo, row_hi, s);
    const int chunk = part >= p.plan_parts0 ? p.plan_chunk_kb1 : p.plan_chunk_kb0;
    k0 = min(KB, s * chunk);
    k1 = min(KB, (s + 1) * chunk);
    if (k1 <= k0) return false;
    const int r0 = mt * kBM, r1 = min(p.M, r0 + kBM);
    return max(r0, row_lo) < min(r1, row_hi);
}

REAX_DEVI bool cursor_next(const TcParams& p, int split, Cursor& c, Segment& s) {
    const int KB = p.kb_int + p.kb_f16;
    while (true) {
        const int t = unit_id(p) + c.dp_i * unit_count(p);
        if (t >= p.dp_tiles) break;
        ++c.dp_i;
        if (tile_active(p, t, split, s.k0, s.k1)) {
            s.tile = t;
            s.whole = true;
            return true;
        }
    }
    if (c.sk < c.sk_end) {
        // The range is walked from its last tile back to its first.  A split tile's first K blocks lie
        // at the end of some CTA's range and are computed (and published) first there; its last K
        // blocks lie at the start of the next CTA's range and are computed last there, by the CTA that
        // completes the tile, long after the others have published.
        const long long last = c.sk_end - 1;
        const int st = static_cast<int>(last / KB);
        const long long tb = static_cast<long long>(st) * KB;
        const long long lo = c.sk > tb ? c.sk : tb;
        s.tile = p.dp_tiles + st;
        s.k0 = static_cast<int>(lo - tb);
        s.k1 = static_cast<int>(c.sk_end - tb);
        s.whole = (s.k0 == 0 && s.k1 == KB);
        c.sk_end = lo;
        return true;
    }
    return false;
}

// CTA whose stream-K range holds iteration i (ranges are floor(c * S / G) .. floor((c+1) * S / G)).
REAX_DEVI int sk_owner(const TcParams& p, long long i) {
    return static_cast<int>((static_cast<unsigned>(i + 1) * gridDim.x - 1u) / static_cast<unsigned>(p.sk_iters));
}

REAX_DEVI int sk_slot(const TcParams& p, int c, int st) {
    const int KB = p.kb_int + p.kb_f16;
    return static_cast<int>(sk_begin(p, c) / KB) == st ? 0 : 1;
}

REAX_DEVI void raise_error(const TcParams& p, int* abort_flag, unsigned bit) {
    atomicOr(p.status, bit);
    *reinterpret_cast<volatile int*>(abort_flag) = 1;
}

// ------------------------------------------------------------------------------------------------ epilogue math

// INT8 dequant of one accumulator element (native_hybrid8.cu:23-24): three separately rounded ops.
REAX_DEVI float dequant1(uint32_t acc_bits, float sa_row, float sw_col, float bias_col) {
    return __fadd_rn(__fmul_rn(__fmul_rn(__int2float_rn(static_cast<int>(acc_bits)), sa_row), sw_col), bias_col);
}

// Split-tile helper shared by both epilogues: publish this CTA's int32 partial of accumulator columns
// [c_lo, c_hi) (and [c_lo + pair_off, c_hi + pair_off) when pair_off > 0: the up half of a SwiGLU
// tile), valid lanes only, then learn whether this CTA completes the tile.  W = columns per TMEM load.
//
// Before publishing, the counter is read: when every other contributor has already published (their
// K-block counts add up to KB minus ours) this CTA is the one that completes the tile and skips its
// own publication; it then resets the counter after its epilogue like any finishing CTA.  Nobody
// else can reach KB afterwards because all other contributors have already counted.
REAX_DEVI int ld_acquire_gpu(const int* ptr) {
    int v;
    asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(ptr) : "memory");
    return v;
}

template <int EPI_WARPS, int W>
REAX_DEVI bool publish_partial(const TcParams& p, const Segment& seg, int st, uint32_t t_acc, int c_lo, int c_hi,
                               int pair_off, int lane_row, bool lane_ok, int* last_flag) {
    const int KB = p.kb_int + p.kb_f16;
    if (threadIdx.x == kCtlThreads) *last_flag = (ld_acquire_gpu(p.ws_counters + st) + (seg.k1 - seg.k0) == KB) ? 1 : 0;
    named_bar_sync(1, EPI_WARPS * 32);
    if (*reinterpret_cast<volatile int*>(last_flag) != 0) {
        __threadfence();
        named_bar_sync(1, EPI_WARPS * 32);   // every thread has read the flag before it is reused
        return true;
    }
    named_bar_sync(1, EPI_WARPS * 32);
    int4* slot = reinterpret_cast<int4*>(p.ws_partials +
                                         (static_cast<size_t>(blockIdx.x) * 2 + sk_slot(p, blockIdx.x, st)) * kSlotInts);
    for (int h = 0; h < (pair_off > 0 ? 2 : 1); ++h) {
        const int off = h * pair_off;
        for (int cc = c_lo + off; cc < c_hi + off; cc += W) {
            uint32_t a[W];
            if constexpr (W == 32) tmem_ld_x32_sync(t_acc + cc, a);
            else tmem_ld_x8_sync(t_acc + cc, a);
            if (lane_ok) {
#pragma unroll
                for (int i = 0; i < W; i += 4)
                    __stcg(slot + ((cc + i) / 4) * kBM + lane_row, make_int4(a[i], a[i + 1], a[i + 2], a[i + 3]));
            }
        }
    }
    __threadfence();
    named_bar_sync(1, EPI_WARPS * 32);
    if (threadIdx.x == kCtlThreads) {
        const int n = seg.k1 - seg.k0;
        const int old = atomicAdd(p.ws_counters + st, n);
        *last_flag = (old + n == KB) ? 1 : 0;
    }
    named_bar_sync(1, EPI_WARPS * 32);
    const bool finish = *reinterpret_cast<volatile int*>(last_flag) != 0;
    if (finish) __threadfence();
    return finish;
}

// Wait, for at most limit_ns, until every other contributor of split tile st has counted its K blocks;
// then this CTA completes the tile without publishing (nobody else can reach KB any more) and the
// contributors' partials are visible to all its epilogue threads.  Only the contributor holding the
// tile's last K blocks calls it: those start its range, which it walks backwards, so it reaches them
// last, while every other contributor reaches this tile first in its own range and publishes without
// waiting; no two CTAs ever wait on each other.  When the limit passes (a contributor not resident
// yet, say) the caller publishes like any other contributor.  All epilogue threads call it.
template <int EPI_WARPS>
REAX_DEVI bool wait_others_counted(const TcParams& p, const Segment& seg, int st, int* last_flag, uint64_t limit_ns) {
    const int KB = p.kb_int + p.kb_f16;
    if (threadIdx.x == kCtlThreads) {
        const int need = KB - (seg.k1 - seg.k0);
        const uint64_t t0 = global_timer_ns();
        int done = 0;
        while (true) {
            if (ld_acquire_gpu(p.ws_counters + st) == need) {
                done = 1;
                break;
            }
            if (global_timer_ns() - t0 > limit_ns) break;
            __nanosleep(100);
        }
        *last_flag = done;
    }
    named_bar_sync(1, EPI_WARPS * 32);
    const bool complete = *reinterpret_cast<volatile int*>(last_flag) != 0;
    named_bar_sync(1, EPI_WARPS * 32);   // every thread has read the flag before it is reused
    if (complete) __threadfence();
    return complete;
}

// After every epilogue thread has stored its share of this CTA's partial of split tile st: count the
// CTA's K blocks (one thread, after a release fence that covers the whole CTA's stores) and learn
// whether that count completed the tile.  All epilogue threads call it.
template <int EPI_WARPS>
REAX_DEVI bool count_published(const TcParams& p, const Segment& seg, int st, int* last_flag) {
    const int KB = p.kb_int + p.kb_f16;
    named_bar_sync(1, EPI_WARPS * 32);
    if (threadIdx.x == kCtlThreads) {
        __threadfence();
        const int n = seg.k1 - seg.k0;
        *last_flag = (atomicAdd(p.ws_counters + st, n) + n == KB) ? 1 : 0;
    }
    named_bar_sync(1, EPI_WARPS * 32);
    const bool finish = *reinterpret_cast<volatile int*>(last_flag) != 0;
    named_bar_sync(1, EPI_WARPS * 32);   // every thread has read the flag before it is reused
    if (finish) __threadfence();
    return finish;
}

// Weight-major tile of segment s: (sw, sw, bias, bias) of this thread's gate and up rows (weight row
// `row` of the tile).
REAX_DEVI float4 swap_column_scales(const TcParams& p, const Segment& s, int row) {
    int part, mt, nt;
    tile_coords(p, s.tile, part, mt, nt);
    const int j = min(nt * p.tile_rows + row, p.H - 1);   // lanes past the tile's rows load a valid column
    return make_float4(__ldg(p.sw + j), __ldg(p.sw + p.H + j), __ldg(p.bias + j), __ldg(p.bias + p.H + j));
}

// Slots of a split tile's other contributors (CTA order), resolved once per tile.
constexpr int kMaxContrib = 8;
REAX_DEVI int contributors(const TcParams& p, int st, const int4* (&contrib)[kMaxContrib]) {
    const int KB = p.kb_int + p.kb_f16;
    const int c_first = sk_owner(p, static_cast<long long>(st) * KB);
    const int c_last = sk_owner(p, static_cast<long long>(st + 1) * KB - 1);
    int n = 0;
    for (int c = c_first; c <= c_last; ++c) {
        if (c == static_cast<int>(blockIdx.x)) continue;
        if (sk_begin(p, c + 1) <= sk_begin(p, c)) continue;
        if (n == kMaxContrib) {   // the host plans at most kMaxContrib others; report rather than drop one
            atomicOr(p.status, kStatusPlanLimit);
            break;
        }
        contrib[n++] = reinterpret_cast<const int4*>(p.ws_partials +
                                                      (static_cast<size_t>(c) * 2 + sk_slot(p, c, st)) * kSlotInts);
    }
    return n;
}

// Add the other contributors' partials of accumulator columns [col, col + W) to a[].
template <int W>
REAX_DEVI void add_partials(const int4* const (&contrib)[kMaxContrib], int n, int col, int lane_row, uint32_t (&a)[W]) {
    for (int ci = 0; ci < n; ++ci) {
#pragma unroll
        for (int i = 0; i < W; i += 4) {
            const int4 v = __ldcg(contrib[ci] + ((col + i) / 4) * kBM + lane_row);
            a[i] += v.x;
            a[i + 1] += v.y;
            a[i + 2] += v.z;
            a[i + 3] += v.w;
        }
    }
}

// MODE 0: INT8 accumulators with dequant (ADD_F: plus a float32 region of BF16 columns);
// MODE 1: float32 accumulators of BF16 operands.  p.mode / p.kb_f16 must agree with the template.
// SWAP: weight-major tiles for small M (SwiGLU only, no BF16 column region): the 128 gate rows and the
// 128 up rows of the tile are the A operands of two MMAs (M=128, N=n_tok) whose B operand is the
// activation tile (n_tok token rows); TMEM lanes are weight rows, columns [0, n_tok) gate and
// [n_tok, 2 n_tok) up, one column per token.  Every TMEM lane quarter then holds real rows even when
// only a few tokens exist, so all four SM sub-partitions share the epilogue.
// PAIR: token-major INT8 SwiGLU tiles of 256 token rows computed by a CTA pair (a cluster of two) with
// tcgen05.mma.cta_group::2 (M = 256): each CTA loads its own 128 token rows and half of the tile's B rows
// (rank 0 the gate rows, rank 1 the matching up rows) into its own shared memory, rank 0 issues the MMAs
// (N = 256: gate then up columns) on both CTAs' operands, and each CTA's TMEM receives its 128 token rows,
// gate in columns [0, 128) and up in [128, 256) as for a single-CTA tile, so the epilogue is the same.
// Per SM this moves two thirds of the operand bytes of a single-CTA 128 x 256 tile for the same MMA work.
template <int EPI_WARPS, int STAGES, int EPI, int MODE, bool ADD_F, bool SWAP, bool PAIR = false>
__global__ void __launch_bounds__(kCtlThreads + 32 * EPI_WARPS, 1) tc_gemm_kernel(const __grid_constant__ TcParams p) {
    static_assert(!SWAP || !ADD_F, "weight-major tiles: no BF16 column region");
    static_assert(!PAIR || (EPI == kEpiSwiglu && !ADD_F && !SWAP), "CTA pairs: INT8 or BF16 SwiGLU tiles");
    static_assert(EPI_WARPS * kOutTmaWarpBytes <= kOutStageBytes, "TMA store boxes fit the staging region");
    // the CTA's rank in its pair (0 issues the MMAs) and the pair's per-stage box bytes
    const uint32_t rank = PAIR ? cluster_ctarank() : 0u;
    constexpr int kPairBox = kBM * kRowBytes;   // 128 rows x 128 bytes: a CTA's A box and its half of B
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* stage_a = smem;
    uint8_t* stage_b = smem + STAGES * kAStage;
    // per accumulator buffer: the tile's per-column scale and bias (token-major) or per-token scale
    // (weight-major), staged before the accumulator is ready
    uint8_t* out_stage = stage_b + STAGES * kBStage;                           // [kSwapMaxTok][kBN / 2] bf16
    uint16_t* silu_tab_s = reinterpret_cast<uint16_t*>(out_stage + kOutStageBytes);   // SiLU table
    float* stage_sw = reinterpret_cast<float*>(out_stage + kOutStageBytes + kSiluTabBytes);   // [2][kBN]
    float* stage_bias = stage_sw + 2 * kBN;                                    // [2][kBN]
    uint64_t* full = reinterpret_cast<uint64_t*>(stage_bias + 2 * kBN);
    uint64_t* empty = full + kMaxStages;
    uint64_t* acc_full = empty + kMaxStages;
    uint64_t* acc_empty = acc_full + 2;
    uint64_t* drain = acc_empty + 2;
    // ADD_F: the epilogue has written a tile's dequantized values into the float32 region (one arrival
    // per epilogue warp), so the MMA issuer may add the BF16 columns' products on top of them
    uint64_t* deq_ready = drain + 1;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(deq_ready + 1);
    int* abort_flag = reinterpret_cast<int*>(tmem_slot + 1);
    int* last_flag = abort_flag + 1;
    // pipeline stages and the boxes inside them
    // pair stages: [this CTA's half of B | its A box], 32 KiB each
    const int ns = (SWAP || PAIR) ? p.stages : STAGES;
    auto box_a = [&](int st) -> uint8_t* {   // activation box (weight-major) or A tile
        if constexpr (PAIR) return smem + st * (2 * kPairBox) + kPairBox;
        return SWAP ? smem + st * p.stage_bytes + 2 * p.tile_rows8 * kRowBytes : stage_a + st * kAStage;
    };
    auto box_b = [&](int st) -> uint8_t* {   // gate rows (weight-major) or the first half of B
        if constexpr (PAIR) return smem + st * (2 * kPairBox);
        return SWAP ? smem + st * p.stage_bytes : stage_b + st * kBStage;
    };
    auto box_bu = [&](int st) -> uint8_t* {  // up rows (weight-major) or the second half of B
        return SWAP ? smem + st * p.stage_bytes + p.tile_rows8 * kRowBytes
                    : stage_b + st * kBStage + (EPI == kEpiSwiglu ? p.tile_rows8 * kRowBytes : kBStage / 2);
    };

    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;

    // INT8 weight-major tiles with stages of kk > 1 K blocks (p.kk): two producers, one copy each per stage.
    // A slab is one K block of the tile's weight rows: the gate rows then the up rows (SwiGLU), or the rows
    // of one output-column range (plain, grouped projections).
    const bool multi = SWAP && MODE == 0 && p.kk > 1;
    const int slab_rows = (EPI == kEpiSwiglu ? 2 : 1) * p.tile_rows8;
    if (threadIdx.x == 0) {
        for (int s = 0; s < ns; ++s) {
            // one arrival per producer: gate, up and activation boxes (multi: weight slabs and activation
            // boxes); for a pair, rank 0's barrier counts both CTAs' B-half and A boxes
            mbar_init(&full[s], PAIR ? 4 : (multi ? 2 : 3));
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&acc_full[b], 1);
            mbar_init(&acc_empty[b], PAIR ? 2 * EPI_WARPS : EPI_WARPS);   // a pair: both CTAs' epilogue warps
        }
        mbar_init(drain, 1);
        mbar_init(deq_ready, EPI_WARPS);
        *abort_flag = 0;
        *last_flag = 0;
        fence_mbar_init();
    }
    if (warp == 0 && lane == 0) {
        tma_prefetch_desc(&p.tm_a);
        tma_prefetch_desc(&p.tm_b);
        tma_prefetch_desc(&p.tm_ah);
        tma_prefetch_desc(&p.tm_bh);
        if (p.out_tma) tma_prefetch_desc(&p.tm_out);
    }
    if (warp == 1) {
        if constexpr (PAIR) {
            tmem_alloc_pair(tmem_slot, kTmemCols);
            tmem_relinquish_pair();
        } else {
            tmem_alloc(tmem_slot, kTmemCols);
            tmem_relinquish();
        }
    }
    tc_fence_before();
    __syncthreads();
    // a pair: the other CTA's barriers are initialised before anything arrives on them remotely
    if constexpr (PAIR) cluster_sync_all();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    volatile int* vabort = abort_flag;

    // Inputs of this kernel may be written by the kernel launched just before it on the stream
    // (programmatic dependent launch): everything above overlapped that kernel's tail, and each role
    // waits for that kernel before its first global access (the producer may first load weight tiles,
    // see early_b).  From then on the next kernel may be scheduled: every kernel this library launches
    // with programmatic serialization waits for this grid's completion before it touches memory, and
    // other launches on the stream keep full serialization.
    auto dependency_wait = [&]() -> int {
        grid_dependency_wait();
        grid_dependents_launch();
        return p.slice_mode ? min(max(__ldg(p.split), 0), p.M) : 0;
    };

    if (warp < kCtlWarps) {
    regs_shrink<kCtlRegs>();
    if ((warp == 0 || warp >= 2) && multi) {
        // ------------------------------------------------------- TMA producers, stages of kk K blocks
        // Stage layout: kk slabs of slab_rows weight rows (one copy by warp 0: a 4-D box of the gate and up
        // rows, or a 3-D box of a grouped projection's rows), then kk activation boxes of n_tok rows (one 3-D
        // copy by warp 3); warp 2 has nothing to load.  A segment is loaded in stages of kk K blocks from its
        // first; the K blocks of its last stage past the segment's end are loaded (the next group's, or zeros
        // past K) but never multiplied.
        if (lane == 0 && warp != 2) {
            const bool act = warp == 3;
            const int kk = p.kk;
            const uint64_t policy = act ? l2_policy_evict_last()
                                        : (p.evict_first_b ? l2_policy_evict_first() : l2_policy_evict_normal());
            const uint32_t tx = static_cast<uint32_t>(kk * (act ? p.n_tok : slab_rows) * kRowBytes);
            int stage = 0;
            uint32_t phase = 0, armed = 0, armed_parity = 0;
            // K block kb of group `part` (grouped projections) sits at K block part * kb_int_part + kb
            auto load = [&](int st, int kb, int part, int nt) {
                mbar_arrive_expect_tx(&full[st], tx);
                uint8_t* base = smem + st * p.stage_bytes;
                const int z = part * p.kb_int_part + kb;
                if (act) tma_load_3d(base + kk * slab_rows * kRowBytes, &p.tm_a, &full[st], 0, 0, z, policy);
                else if constexpr (EPI == kEpiSwiglu) tma_load_4d(base, &p.tm_b, &full[st], 0, nt * p.tile_rows, 0, z, policy);
                else tma_load_3d(base, &p.tm_b, &full[st], 0, nt * p.tile_rows, z, policy);
            };
            // early_b: the first segment's first weight stages before the dependency wait (as below)
            int pre = 0;
            if (!act && p.early_b && !p.slice_mode) {
                Cursor c0 = cursor_init(p);
                Segment s0;
                if (cursor_next(p, 0, c0, s0)) {
                    int part, mt, nt;
                    tile_coords(p, s0.tile, part, mt, nt);
                    pre = min(min(ns, (kEarlyStages + kk - 1) / kk), (s0.k1 - s0.k0 + kk - 1) / kk);
                    for (int i = 0; i < pre; ++i) load(i, s0.k0 + i * kk, part, nt);
                }
            }
            const int split = dependency_wait();
            bool ok = true, first = true;
            Cursor cur = cursor_init(p);
            Segment seg;
            while (ok && cursor_next(p, split, cur, seg)) {
                int part, mt, nt;
                tile_coords(p, seg.tile, part, mt, nt);
                for (int kb = seg.k0, i = 0; kb < seg.k1; kb += kk, ++i) {
                    if (!(first && i < pre)) {   // a stage requested early owns its fresh slot (see below)
                        if (!mbar_wait_bounded(&empty[stage], phase ^ 1, p.timeout_ns, vabort)) {
                            if (!*vabort) raise_error(p, abort_flag, kStatusTimeoutEmpty);
                            ok = false;
                            break;
                        }
                        load(stage, kb, part, nt);
                    }
                    armed |= 1u << stage;
                    armed_parity = (armed_parity & ~(1u << stage)) | (phase << stage);
                    if (++stage == ns) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
                first = false;
            }
            for (int s = 0; s < ns; ++s) {   // drain: every copy started has landed before the CTA exits
                if (armed & (1u << s)) {
                    if (!mbar_wait_bounded(&full[s], (armed_parity >> s) & 1, p.timeout_ns, nullptr))
                        atomicOr(p.status, kStatusTimeoutDrain);
                }
            }
        }
    } else if (warp == 0 || warp >= 2) {
        // ----------------------------------------------------------------------------- TMA producers
        // One box per producer and K block: warp 0 the gate rows (first half of B), warp 2 the up rows
        // (second half of B), warp 3 the activation rows (A).  Each arms the stage's full barrier with
        // its own bytes (three arrivals per phase), so the three copies are issued in parallel.
        // A pair has two boxes per CTA and K block: warp 0 loads this CTA's half of B (rank 0 the gate rows,
        // rank 1 the up rows), warp 3 its 128 activation rows; warp 2 has nothing to load.
        if (lane == 0 && !(PAIR && warp == 2)) {
            const int role = warp == 0 ? 0 : warp - 1;   // 0 gate, 1 up, 2 activation
            const uint64_t policy = role == 2 ? l2_policy_evict_last()
                                              : (p.evict_first_b ? l2_policy_evict_first() : l2_policy_evict_normal());
            const int b_rows = (EPI == kEpiSwiglu) ? p.tile_rows : kBN / 2;
            const int a_rows = SWAP ? p.n_tok : p.a_rows;
            const uint32_t box_tx = static_cast<uint32_t>((role == 2 ? a_rows : b_rows) * kRowBytes);
            int stage = 0;
            uint32_t phase = 0;
            uint32_t armed = 0;        // bit s: stage s has been armed at least once
            uint32_t armed_parity = 0; // bit s: parity of the last arming of stage s
            // this producer's box of K block kb of the tile (part, m0, b0, b1) into stage st
            // arm the stage's full barrier with this box's bytes (a pair: rank 0's barrier counts both CTAs')
            auto arm = [&](int st) {
                if constexpr (PAIR) mbar_arrive_expect_tx_cluster(cluster_map(&full[st], 0), box_tx);
                else mbar_arrive_expect_tx(&full[st], box_tx);
            };
            auto load_box = [&](int st, int kb, int part, int m0, int b0, int b1) {
                uint8_t* dst = role == 0 ? box_b(st) : (role == 1 ? box_bu(st) : box_a(st));
                const int y = role == 0 ? ((PAIR && rank == 1) ? b1 : b0) : (role == 1 ? b1 : m0);
                if constexpr (PAIR) {   // INT8 (128 codes) or BF16 (64 values) per K block
                    const bool i8 = kb < p.kb_int;
                    const int x = i8 ? kb * kRowBytes : (kb - p.kb_int) * (kRowBytes / 2);
                    const CUtensorMap* map = role == 2 ? (i8 ? &p.tm_a : &p.tm_ah) : (i8 ? &p.tm_b : &p.tm_bh);
                    tma_load_2d_pair(dst, map, cluster_map(&full[st], 0), x, y, policy);
                } else if (kb < p.kb_int) {
                    const int x = (part * p.kb_int_part + kb) * kRowBytes;
                    tma_load_2d(dst, role == 2 ? &p.tm_a : &p.tm_b, &full[st], x, y, policy);
                } else {
                    const int x = (part * p.kb_f16_part + kb - p.kb_int) * (kRowBytes / 2);
                    tma_load_2d(dst, role == 2 ? &p.tm_ah : &p.tm_bh, &full[st], x, y, policy);
                }
            };
            auto tile_rows = [&](const Segment& sg, int& part, int& m0, int& b0, int& b1) {
                int mt, nt;
                tile_coords(p, sg.tile, part, mt, nt);
                m0 = PAIR ? mt * 2 * kBM + kBM * static_cast<int>(rank) : mt * kBM;
                b0 = (EPI == kEpiSwiglu) ? nt * p.tile_rows : nt * kBN;
                b1 = (EPI == kEpiSwiglu) ? p.H + nt * p.tile_rows : nt * kBN + kBN / 2;
            };
            // early_b: the weight producers request the first segment's first kEarlyStages K blocks
            // before the dependency wait (the weights are not produced by the kernel this one waits for).
            int pre = 0;
            if (role != 2 && p.early_b && !p.slice_mode) {
                Cursor c0 = cursor_init(p);
                Segment s0;
                if (cursor_next(p, 0, c0, s0)) {
                    int part, m0, b0, b1;
                    tile_rows(s0, part, m0, b0, b1);
                    pre = min(min(ns, kEarlyStages), s0.k1 - s0.k0);
                    for (int i = 0; i < pre; ++i) {
                        arm(i);
                        load_box(i, s0.k0 + i, part, m0, b0, b1);
                        armed |= 1u << i;
                    }
                }
            }
            const int split = dependency_wait();
            bool ok = true;
            Cursor cur = cursor_init(p);
            Segment seg;
            bool first = true;
            while (ok && cursor_next(p, split, cur, seg)) {
                int part, m0, b0, b1;
                tile_rows(seg, part, m0, b0, b1);
                for (int kb = seg.k0; kb < seg.k1; ++kb) {
                    // A K block requested early already owns its (then fresh) stage: it must not wait on
                    // the stage's empty barrier, whose first phase the other producers and the MMAs may
                    // have completed by now.
                    if (!(first && kb - seg.k0 < pre)) {
                        if (!mbar_wait_bounded(&empty[stage], phase ^ 1, p.timeout_ns, vabort)) {
                            if (!*vabort) raise_error(p, abort_flag, kStatusTimeoutEmpty);
                            ok = false;
                            break;
                        }
                        arm(stage);
                        load_box(stage, kb, part, m0, b0, b1);
                    }
                    armed |= 1u << stage;
                    armed_parity = (armed_parity & ~(1u << stage)) | (phase << stage);
                    if (++stage == ns) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
                first = false;
            }
            // Drain: every copy this thread started must have landed before the CTA can exit.  A pair's copies
            // complete on rank 0's barriers, which only rank 0 can wait on: there the MMA issuer consumes every
            // K block that was loaded and drains its MMAs before the pair's final cluster barrier, which
            // neither CTA passes before the other has arrived.
            for (int s = 0; s < (PAIR ? 0 : ns); ++s) {
                if (armed & (1u << s)) {
                    if (!mbar_wait_bounded(&full[s], (armed_parity >> s) & 1, p.timeout_ns, nullptr)) {
                        atomicOr(p.status, kStatusTimeoutDrain);
                    }
                }
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------------------------- MMA issuer
        // (a pair: rank 0 issues the MMAs of both CTAs; rank 1's warp 1 only holds its TMEM allocation)
        if (lane == 0 && (!PAIR || rank == 0)) {
            const int split = dependency_wait();
            // token-major SwiGLU tiles: N = the gate rows and the up rows of the tile (2 x tile_rows8)
            const int n_mma = SWAP ? p.n_tok : (EPI == kEpiSwiglu ? 2 * p.tile_rows8 : kBN);
            const uint32_t idesc_i8 = idesc_i8_s32(PAIR ? 2 * kBM : kBM, n_mma);
            const uint32_t idesc_f16 = idesc_bf16_f32(PAIR ? 2 * kBM : kBM, n_mma);
            int stage = 0;
            uint32_t phase = 0;
            int buf = 0;
            uint32_t acc_phase = 0;
            uint32_t deq_phase = 0;
            Cursor cur = cursor_init(p);
            Segment seg;
            bool ok = true;
            while (ok && cursor_next(p, split, cur, seg)) {
                // ADD_F: the INT8 region is free once the epilogue has dequantized the previous tile out of
                // it (the deq_ready wait before that tile's BF16 MMAs), so the next tile's INT8 MMAs run
                // under the previous tile's BF16 MMAs and epilogue; the float32 region is reused only after
                // the next deq_ready, which the epilogue signals after it has read that region.
                if constexpr (!ADD_F) {
                    if (!mbar_wait_bounded(&acc_empty[buf], acc_phase ^ 1, p.timeout_ns, vabort)) {
                        if (!*vabort) raise_error(p, abort_flag, kStatusTimeoutAccEmpty);
                        break;
                    }
                    tc_fence_after();
                }
                const uint32_t d_int = tmem_base + buf * kBN;
                const uint32_t d_f32 = (MODE == 1) ? tmem_base + buf * kBN : tmem_base + kBN;
                const int first_f = max(seg.k0, p.kb_int);
                if (multi) {
                    const uint32_t idesc_s = p.m64 ? idesc_i8_s32(64, n_mma) : idesc_i8;
                    // stages of kk K blocks: per K block j of a stage, its [gate | up] slab against its
                    // activation box (TMEM lanes [0, tile_rows8) gate rows, [tile_rows8, 2 tile_rows8) up
                    // rows, columns the tokens); K blocks past the segment's end are skipped
                    const uint32_t slab = static_cast<uint32_t>(slab_rows) * kRowBytes;
                    for (int kb = seg.k0; kb < seg.k1; kb += p.kk) {
                        if (!mbar_wait_bounded(&full[stage], phase, p.timeout_ns, vabort)) {
                            if (!*vabort) raise_error(p, abort_flag, kStatusTimeoutFull);
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        const uint32_t base = smem_u32(smem + stage * p.stage_bytes);
                        const int nb = min(p.kk, seg.k1 - kb);
                        for (int j = 0; j < nb; ++j) {
                            // one M = 128 MMA covers the slab's rows (slab_rows <= 128)
                            const uint64_t wd = sw128_kmajor_desc(base + j * slab);
                            const uint64_t ad = sw128_kmajor_desc(base + p.kk * slab + j * p.n_tok * kRowBytes);
#pragma unroll
                            for (int k = 0; k < 4; ++k) {
                                const uint32_t acc = (kb + j > seg.k0 || k > 0) ? 1u : 0u;
                                umma_i8(d_int, wd + 2 * k, ad + 2 * k, idesc_s, acc);
                            }
                        }
                        umma_commit(&empty[stage]);
                        if (++stage == ns) {
                            stage = 0;
                            phase ^= 1;
                        }
                    }
                }
                for (int kb = seg.k0; kb < (multi ? seg.k0 : seg.k1); ++kb) {
                    if (!mbar_wait_bounded(&full[stage], phase, p.timeout_ns, vabort)) {
                        if (!*vabort) raise_error(p, abort_flag, kStatusTimeoutFull);
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint64_t ad = sw128_kmajor_desc(smem_u32(box_a(stage)));
                    const uint64_t bd = sw128_kmajor_desc(smem_u32(box_b(stage)));
                    const uint64_t bd_up = sw128_kmajor_desc(smem_u32(box_bu(stage)));
                    if (kb < p.kb_int) {
#pragma unroll
                        for (int k = 0; k < 4; ++k) {
                            const uint32_t acc = (kb > seg.k0 || k > 0) ? 1u : 0u;
                            if constexpr (SWAP) {
                                umma_i8(d_int, bd + 2 * k, ad + 2 * k, idesc_i8, acc);
                                umma_i8(d_int + p.n_tok, bd_up + 2 * k, ad + 2 * k, idesc_i8, acc);
                            } else if constexpr (PAIR) {
                                umma_i8_pair(d_int, ad + 2 * k, bd + 2 * k, idesc_i8, acc);
                            } else {
                                umma_i8(d_int, ad + 2 * k, bd + 2 * k, idesc_i8, acc);
                            }
                        }
                    } else {
                        if constexpr (ADD_F) {
                            // The BF16 columns add into the dequantized values, 16 columns per MMA in
                            // ascending order, as the reference's mma.sync chain adds them into its
                            // dequantized registers (native_hybrid8.cu:26, hybrid8_tiles.cuh:454-550):
                            // wait until the epilogue has stored those values in the float32 region.
                            if (kb == p.kb_int) {
                                if (!mbar_wait_bounded(deq_ready, deq_phase, p.timeout_ns, vabort)) {
                                    if (!*vabort) raise_error(p, abort_flag, kStatusTimeoutAccEmpty);
                                    ok = false;
                                    break;
                                }
                                deq_phase ^= 1;
                                tc_fence_after();
                            }
                        }
#pragma unroll
                        for (int k = 0; k < 4; ++k) {
                            const uint32_t acc = (ADD_F || kb > first_f || k > 0) ? 1u : 0u;
                            if constexpr (SWAP) {
                                umma_f16(d_f32, bd + 2 * k, ad + 2 * k, idesc_f16, acc);
                                umma_f16(d_f32 + p.n_tok, bd_up + 2 * k, ad + 2 * k, idesc_f16, acc);
                            } else {
                                if constexpr (PAIR) umma_f16_pair(d_f32, ad + 2 * k, bd + 2 * k, idesc_f16, acc);
                                else umma_f16(d_f32, ad + 2 * k, bd + 2 * k, idesc_f16, acc);
                            }
                        }
                    }
                    if constexpr (PAIR) umma_commit_pair(&empty[stage]);   // frees the stage in both CTAs
                    else umma_commit(&empty[stage]);
                    // ADD_F: the INT8 accumulators of the tile are complete
                    if (ADD_F && kb == p.kb_int - 1) umma_commit(&acc_full[0]);
                    if (++stage == ns) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
                if (!ok) break;
                if constexpr (PAIR) umma_commit_pair(&acc_full[buf]);   // both CTAs' accumulators are ready
                else umma_commit(&acc_full[ADD_F ? 1 : buf]);
                if (p.acc_bufs == 2) {
                    buf ^= 1;
                    if (buf == 0) acc_phase ^= 1;
                } else {
                    acc_phase ^= 1;
                }
            }
            // Drain: all MMAs issued by this thread complete before TMEM is freed.
            if constexpr (PAIR) umma_commit_pair_local(drain);
            else umma_commit(drain);
            if (!mbar_wait_bounded(drain, 0, p.timeout_ns, nullptr)) atomicOr(p.status, kStatusTimeoutDrain);
        }
        __syncwarp();
    }
    // Teardown of the control warps; every role ends in its own copy, so no code runs under both
    // register counts.  A pair meets at a cluster barrier first: neither CTA frees its TMEM or exits while
    // rank 0's MMAs may still read the other's shared memory or its epilogue still arrives remotely.
    tc_fence_before();
    __syncthreads();
    if constexpr (PAIR) cluster_sync_all();
    if (warp == 1) {
        tc_fence_after();
        if constexpr (PAIR) tmem_dealloc_pair(tmem_base, kTmemCols);
        else tmem_dealloc(tmem_base, kTmemCols);
    }
    return;
    }

    regs_grow<kEpiRegs>();
    if constexpr (EPI == kEpiSwiglu) {
        // the SiLU table, built while the first accumulator is still being computed
        silu_table_fill(silu_tab_s, threadIdx.x - kCtlThreads, EPI_WARPS * 32);
        named_bar_sync(1, EPI_WARPS * 32);
    }
    const int split = dependency_wait();
    {
        // --------------------------------------------------------------------------------- epilogue
        // Epilogue warps only ever stop at the accumulator wait, and only on its own timeout (no abort
        // flag), so either all of them pass a segment or none does: the named barriers stay matched.
        const int e = warp - kCtlWarps;
        const int q = warp & 3;                      // TMEM lane quarter this warp may access
        const int r_tile = q * 32 + lane;            // accumulator row (= TMEM lane) of this thread
        constexpr int kSplit = EPI_WARPS / 4;        // warps sharing one lane quarter split the columns
        const uint32_t lane_off = static_cast<uint32_t>(q * 32) << 16;
        int buf = 0;
        uint32_t acc_phase = 0;
        Cursor cur = cursor_init(p);
        Segment seg;
        // Weight-major tiles: every tile covers all tokens, so the token scales are staged once, and each
        // segment's column scales and biases are loaded one segment ahead (a cursor kept one step in
        // front), so that they have landed when the segment starts.
        Cursor ahead = cur;
        Segment aseg;
        float4 next_cs = make_float4(0.f, 0.f, 0.f, 0.f);   // (sw gate, sw up, bias gate, bias up)
        if constexpr (SWAP && MODE == 0 && EPI == kEpiSwiglu) {
            for (int t = threadIdx.x - kCtlThreads; t < p.n_tok; t += EPI_WARPS * 32)
                stage_sw[t] = t < p.M ? __ldg(p.sa + t) : 0.f;
            named_bar_sync(1, EPI_WARPS * 32);
            if (cursor_next(p, split, ahead, aseg)) next_cs = swap_column_scales(p, aseg, q * 32 + lane);
        }
        while (cursor_next(p, split, cur, seg)) {
            int part, mt, nt;
            tile_coords(p, seg.tile, part, mt, nt);
            const int m0 = PAIR ? mt * 2 * kBM + kBM * static_cast<int>(rank) : mt * kBM;
            int row_lo, row_hi, out_part;
            tile_plan(p, part, split, row_lo, row_hi, out_part);
            float* s_sw = stage_sw + buf * kBN;
            float* s_bias = stage_bias + buf * kBN;
            const bool whole = seg.whole;
            const int st = seg.tile - p.dp_tiles;
            const uint32_t t_int = tmem_base + buf * kBN + lane_off;
            const uint32_t t_f32 = ((MODE == 1) ? tmem_base + buf * kBN : tmem_base + kBN) + lane_off;
            const uint32_t t_acc = (MODE == 0) ? t_int : t_f32;

            if (SWAP && multi && EPI == kEpiPlain) {
                // ------------- weight-major grouped-projection tile of kk-block stages: lanes are output columns
                // TMEM lane L < tile_rows holds output column n0 + L of group `part`, columns the tokens; each
                // thread dequantizes its column's values, ((acc * sa) * sw) + bias as for token-major tiles,
                // and stores them (a warp writes 32 consecutive columns of a token row).
                const int n0 = nt * p.tile_rows;
                const int j = n0 + r_tile;
                const bool col_ok = r_tile < p.tile_rows && j < p.H;   // plain weight-major plans: H = N
                const int jc = part * p.n_part_stride + min(j, p.H - 1);
                const uint64_t sw2 = col_ok ? f2(__ldg(p.sw + jc), __ldg(p.sw + jc)) : 0ull;
                const uint64_t b2 = col_ok ? f2(__ldg(p.bias + jc), __ldg(p.bias + jc)) : 0ull;
                const float* sa_p = p.sa + part * p.sa_part_stride;
                __nv_bfloat16* out_p = p.out + out_part * p.out_part_stride;
                const int per_warp = p.n_tok / kSplit;
                const int tok_lo = (e / 4) * per_warp;
                if (!mbar_wait_bounded(&acc_full[buf], acc_phase, p.timeout_ns, nullptr)) {
                    raise_error(p, abort_flag, kStatusTimeoutAccFull);
                    break;
                }
                tc_fence_after();
                if (q * 32 < p.tile_rows) {   // warp-uniform: this lane quarter holds output columns
                    for (int t0 = tok_lo; t0 < tok_lo + per_warp && t0 < p.M; t0 += 8) {
                        uint32_t a[8];
                        tmem_ld_x8_sync(t_acc + t0, a);
                        if (col_ok) {
#pragma unroll
                            for (int i = 0; i < 8; i += 2) {
                                const int t = t0 + i;
                                const float s0 = t < p.M ? __ldg(sa_p + t) : 0.f;
                                const float s1 = t + 1 < p.M ? __ldg(sa_p + t + 1) : 0.f;
                                const uint32_t w = bf16x2_rn(dequant2(a[i], a[i + 1], f2(s0, s1), sw2, b2));
                                if (t < p.M) out_p[static_cast<size_t>(t) * p.ldo + j] = __ushort_as_bfloat16(w & 0xFFFFu);
                                if (t + 1 < p.M)
                                    out_p[static_cast<size_t>(t + 1) * p.ldo + j] = __ushort_as_bfloat16(w >> 16);
                            }
                        }
                    }
                }
            } else if (SWAP && multi) {
                // ------------------------ weight-major tile of kk-block stages: one accumulator per lane row
                // TMEM lane L < tile_rows8 holds gate row n0 + L, lane tile_rows8 + L its up row, columns the
                // tokens.  Every lane dequantizes its rows' values into a [token][lane] bf16 block in shared
                // memory; then the threads pair each gate value with its up value, consecutive threads on
                // consecutive output columns.  The plan never splits these tiles.
                const int r8 = p.tile_rows8;
                const int n0 = nt * p.tile_rows;
                // this lane's slab row (M = 64 MMAs: 16 rows per lane quarter, in its first 16 lanes)
                const int sr = p.m64 ? (lane < 16 ? q * 16 + lane : 2 * r8) : r_tile;
                const bool is_up = sr >= r8;
                const int r = is_up ? sr - r8 : sr;
                const bool row_ok = sr < 2 * r8 && r < p.tile_rows && n0 + r < p.H;
                const int wrow = (is_up ? p.H : 0) + min(n0 + r, p.H - 1);
                const uint64_t sw2 = row_ok ? f2(__ldg(p.sw + wrow), __ldg(p.sw + wrow)) : 0ull;
                const uint64_t b2 = row_ok ? f2(__ldg(p.bias + wrow), __ldg(p.bias + wrow)) : 0ull;
                const int per_warp = p.n_tok / kSplit;                  // the warps of a lane quarter split the tokens
                const int tok_lo = (e / 4) * per_warp;
                uint16_t* xs = reinterpret_cast<uint16_t*>(out_stage);  // [n_tok][kOutStagePitch] bf16 values
                if (!mbar_wait_bounded(&acc_full[buf], acc_phase, p.timeout_ns, nullptr)) {
                    raise_error(p, abort_flag, kStatusTimeoutAccFull);
                    break;
                }
                tc_fence_after();
                if (q * (p.m64 ? 16 : 32) < 2 * r8) {   // warp-uniform: this lane quarter holds gate or up rows
                    for (int t0 = tok_lo; t0 < tok_lo + per_warp && t0 < p.M; t0 += 8) {
                        uint32_t a[8];
                        tmem_ld_x8_sync(t_acc + t0, a);
                        if (row_ok) {
#pragma unroll
                            for (int i = 0; i < 8; i += 2) {
                                const uint64_t sa2 = *reinterpret_cast<const uint64_t*>(stage_sw + t0 + i);
                                const uint32_t w = bf16x2_rn(dequant2(a[i], a[i + 1], sa2, sw2, b2));
                                xs[(t0 + i) * kOutStagePitch + sr] = static_cast<uint16_t>(w & 0xFFFFu);
                                xs[(t0 + i + 1) * kOutStagePitch + sr] = static_cast<uint16_t>(w >> 16);
                            }
                        }
                    }
                }
                named_bar_sync(1, EPI_WARPS * 32);
                const int nv = min(p.tile_rows, p.H - n0);   // output columns of the tile
                const int total = p.M * nv;
                for (int idx = static_cast<int>(threadIdx.x) - kCtlThreads; idx < total; idx += EPI_WARPS * 32) {
                    const int t = idx / nv, c = idx - t * nv;
                    const float gv = __uint_as_float(static_cast<uint32_t>(xs[t * kOutStagePitch + c]) << 16);
                    const float uv = __uint_as_float(static_cast<uint32_t>(xs[t * kOutStagePitch + r8 + c]) << 16);
                    p.out[static_cast<size_t>(t) * p.ldo + n0 + c] = swiglu_bf16(gv, uv, silu_tab_s);
                }
                named_bar_sync(1, EPI_WARPS * 32);   // the staging block is free again
            } else if constexpr (SWAP && EPI == kEpiSwiglu) {
                // ---------------------------------------------- weight-major tile: lanes are weight rows
                const int n_tok = p.n_tok;
                const int n0 = nt * p.tile_rows;               // gate row (= output column) of lane 0
                const int j = n0 + r_tile;                     // this thread's output column
                // lanes past the tile's rows (or past H in the last tile) hold rows of no output column
                const bool col_ok = r_tile < p.tile_rows && j < p.H;
                const int per_warp = n_tok / kSplit;           // token columns each warp finishes
                const int tok_lo = (e / 4) * per_warp;
                const int n_w = min(per_warp, p.M - tok_lo);   // real tokens among them (<= 0: none)
                const float swg = next_cs.x, swu = next_cs.y, bg = next_cs.z, bu = next_cs.w;
                if constexpr (MODE == 0) {
                    if (cursor_next(p, split, ahead, aseg)) next_cs = swap_column_scales(p, aseg, r_tile);
                }
                const float* s_sa = stage_sw;   // token scales, staged once
                // split tile: the other contributors' partial slots, resolved while the MMAs still run
                const int4* contrib[kMaxContrib];
                const int n_contrib = whole ? 0 : contributors(p, st, contrib);

                // The segment, specialised on the pairs of token columns a warp finishes (per_warp
                // rounded up to 8, 16 or 32) and taken in chunks of at most 8 pairs, so that a chunk's
                // accumulators, partials and results stay in registers.  Within a chunk no branch
                // separates the pairs (one warp vote for the chunk's SiLU), so their chains overlap;
                // columns past the warp's real tokens compute on padding and are never stored.
                auto segment = [&](auto pairs_c) -> bool {
                    constexpr int PAIRS = decltype(pairs_c)::value;
                    constexpr int CH = PAIRS < 8 ? PAIRS : 8;
                    constexpr int NCH = PAIRS / CH;
                    // this warp's gate and up accumulators of chunk c of its token columns
                    auto load_acc = [&](int c, uint32_t (&g)[2 * CH], uint32_t (&u)[2 * CH]) {
                        const int t0 = tok_lo + 2 * CH * c;
                        tmem_ld_pairs_sync<CH>(t_acc + t0, t_acc + n_tok + t0, g, u);
                    };
                    // one contributor's int32 partial of chunk c: gate and up columns, four tokens per int4
                    // (lanes of no output column neither publish nor gather: their sums are never stored)
                    auto fetch = [&](const int4* src, int c, int4 (&pg)[CH / 2], int4 (&pu)[CH / 2]) {
#pragma unroll
                        for (int i = 0; i < CH / 2; ++i) {
                            const int t = tok_lo + 2 * CH * c + 4 * i;
                            pg[i] = col_ok ? __ldcg(src + (t / 4) * kBM + r_tile) : make_int4(0, 0, 0, 0);
                            pu[i] = col_ok ? __ldcg(src + ((n_tok + t) / 4) * kBM + r_tile) : make_int4(0, 0, 0, 0);
                        }
                    };
                    auto add = [&](uint32_t (&g)[2 * CH], uint32_t (&u)[2 * CH], const int4 (&pg)[CH / 2],
                                   const int4 (&pu)[CH / 2]) {
#pragma unroll
                        for (int i = 0; i < CH / 2; ++i) {
                            g[4 * i] += pg[i].x; g[4 * i + 1] += pg[i].y; g[4 * i + 2] += pg[i].z; g[4 * i + 3] += pg[i].w;
                            u[4 * i] += pu[i].x; u[4 * i + 1] += pu[i].y; u[4 * i + 2] += pu[i].z; u[4 * i + 3] += pu[i].w;
                        }
                    };
                    int4 qg[CH / 2], qu[CH / 2];   // the first contributor's partial of chunk 0
                    // The contributor holding the tile's last K blocks waits (bounded) for the others
                    // instead of publishing, and fetches the first one's partial while its own last MMAs
                    // still run.
                    // A finisher whose split segment is the CTA's last gathers the other partials through the
                    // pipeline ring, idle once this segment's accumulators are complete: every thread copies
                    // its share of every contributor's chunks at once (cp.async, no registers held), instead
                    // of one contributor's chunk per L2 round trip.
                    Cursor peek = cur;
                    Segment after;
                    const bool ring_free = !cursor_next(p, split, peek, after);
                    const bool ring_gather = ring_free && n_contrib > 0 &&
                                             NCH * n_contrib * (CH / 2) * 2 * (EPI_WARPS * 32) * 16 <= STAGES * (kAStage + kBStage);
                    bool early = false;
                    if (!whole && seg.k1 == p.kb_int + p.kb_f16) {
                        early = wait_others_counted<EPI_WARPS>(p, seg, st, last_flag, kFinisherWaitNs);
                        if (early && n_contrib > 0 && !ring_gather) fetch(contrib[0], 0, qg, qu);
                    }
                    if (!mbar_wait_bounded(&acc_full[buf], acc_phase, p.timeout_ns, nullptr)) {
                        raise_error(p, abort_flag, kStatusTimeoutAccFull);
                        return false;
                    }
                    tc_fence_after();
                    bool finish = whole || early;
                    if (!finish) {
                        // Publish this warp's gate columns and the matching up columns (one TMEM round trip
                        // per chunk), then count this CTA's K blocks; the contributor whose count completes
                        // the tile finishes it.  One thread fences for the CTA after the barrier.
                        int4* slot = reinterpret_cast<int4*>(
                            p.ws_partials + (static_cast<size_t>(blockIdx.x) * 2 + sk_slot(p, blockIdx.x, st)) * kSlotInts);
#pragma unroll
                        for (int c = 0; c < NCH; ++c) {
                            uint32_t g[2 * CH], u[2 * CH];
                            load_acc(c, g, u);
#pragma unroll
                            for (int i = 0; i < CH / 2; ++i) {
                                const int tw = 2 * CH * c + 4 * i;   // token offset within the warp's columns
                                if (col_ok && tw < per_warp) {
                                    __stcg(slot + ((tok_lo + tw) / 4) * kBM + r_tile,
                                           make_int4(g[4 * i], g[4 * i + 1], g[4 * i + 2], g[4 * i + 3]));
                                    __stcg(slot + ((n_tok + tok_lo + tw) / 4) * kBM + r_tile,
                                           make_int4(u[4 * i], u[4 * i + 1], u[4 * i + 2], u[4 * i + 3]));
                                }
                            }
                        }
                        finish = count_published<EPI_WARPS>(p, seg, st, last_flag);
                        if (finish && n_contrib > 0 && !ring_gather) fetch(contrib[0], 0, qg, qu);
                    }
                    if (!finish) return true;
                    // ring slot of this thread's int4 i (gate h = 0, up h = 1) of contributor ci, chunk c
                    const int etid = static_cast<int>(threadIdx.x) - kCtlThreads;
                    auto ring_slot = [&](int c, int ci, int i, int h) -> int4* {
                        return reinterpret_cast<int4*>(smem) +
                               ((((c * n_contrib + ci) * (CH / 2) + i) * 2 + h) * (EPI_WARPS * 32) + etid);
                    };
                    if (ring_gather) {
                        fence_proxy_async_smem();   // the ring's last writes were TMA copies
                        if (col_ok) {
#pragma unroll
                            for (int c = 0; c < NCH; ++c) {
                                if (2 * CH * c >= n_w) break;   // warp-uniform, as in the chunk loop below
                                for (int ci = 0; ci < n_contrib; ++ci)
#pragma unroll
                                    for (int i = 0; i < CH / 2; ++i) {
                                        const int t = tok_lo + 2 * CH * c + 4 * i;
                                        cp_async16_cg(ring_slot(c, ci, i, 0), contrib[ci] + (t / 4) * kBM + r_tile);
                                        cp_async16_cg(ring_slot(c, ci, i, 1), contrib[ci] + ((n_tok + t) / 4) * kBM + r_tile);
                                    }
                            }
                        }
                        cp_async_wait_all();
                    }
                    const uint64_t swg2 = f2(swg, swg), swu2 = f2(swu, swu), bg2 = f2(bg, bg), bu2 = f2(bu, bu);
                    uint16_t* ot = reinterpret_cast<uint16_t*>(out_stage);
                    const int ph = n0 & 7;
#pragma unroll
                    for (int c = 0; c < NCH; ++c) {
                        const int tc = 2 * CH * c;   // the chunk's first token within the warp's columns
                        if (tc >= n_w) break;        // no real token left for this warp (warp-uniform)
                        uint32_t g[2 * CH], u[2 * CH];
                        load_acc(c, g, u);
                        if (ring_gather) {
                            if (col_ok) {
                                for (int ci = 0; ci < n_contrib; ++ci) {
                                    int4 pg[CH / 2], pu[CH / 2];
#pragma unroll
                                    for (int i = 0; i < CH / 2; ++i) {
                                        pg[i] = *ring_slot(c, ci, i, 0);
                                        pu[i] = *ring_slot(c, ci, i, 1);
                                    }
                                    add(g, u, pg, pu);
                                }
                            }
                        } else if (n_contrib > 0) {
                            if (c > 0) fetch(contrib[0], c, qg, qu);
                            add(g, u, qg, qu);
                            for (int ci = 1; ci < n_contrib; ++ci) {
                                int4 pg[CH / 2], pu[CH / 2];
                                fetch(contrib[ci], c, pg, pu);
                                add(g, u, pg, pu);
                            }
                        }
                        // dequant, bf16, then SwiGLU of every token pair of the chunk through the SiLU table
                        uint32_t gw[CH], uw[CH], o[CH];
#pragma unroll
                        for (int i = 0; i < CH; ++i) {
                            uint64_t vg, vu;
                            if constexpr (MODE == 0) {
                                const uint64_t sa2 = *reinterpret_cast<const uint64_t*>(s_sa + tok_lo + tc + 2 * i);
                                vg = dequant2(g[2 * i], g[2 * i + 1], sa2, swg2, bg2);
                                vu = dequant2(u[2 * i], u[2 * i + 1], sa2, swu2, bu2);
                            } else {
                                vg = f2(__uint_as_float(g[2 * i]), __uint_as_float(g[2 * i + 1]));
                                vu = f2(__uint_as_float(u[2 * i]), __uint_as_float(u[2 * i + 1]));
                            }
                            gw[i] = bf16x2_rn(vg);
                            uw[i] = bf16x2_rn(vu);
                        }
                        swiglu2_bits_n<CH>(gw, uw, o, silu_tab_s);
                        if (p.out_vec16) {
                            // The tile's [tokens x columns] block goes through shared memory, each token row
                            // placed at the 16-byte phase of its destination (ph = n0 % 8 halfwords; out is
                            // 16-byte aligned and ldo a multiple of 8), so the copy writes whole aligned
                            // 16-byte pieces and 2-byte stores only where a piece sticks out of [n0, n_end).
                            if (col_ok) {
#pragma unroll
                                for (int i = 0; i < CH; ++i)
                                    if (tc + 2 * i < per_warp) {
                                        const int t = tok_lo + tc + 2 * i;
                                        ot[t * kOutStagePitch + ph + r_tile] = static_cast<uint16_t>(o[i] & 0xFFFFu);
                                        ot[(t + 1) * kOutStagePitch + ph + r_tile] = static_cast<uint16_t>(o[i] >> 16);
                                    }
                            }
                        } else {
#pragma unroll
                            for (int i = 0; i < CH; ++i) {
                                const int t = tok_lo + tc + 2 * i;
                                if (col_ok && tc + 2 * i < n_w)
                                    p.out[static_cast<size_t>(t) * p.ldo + j] = __ushort_as_bfloat16(o[i] & 0xFFFFu);
                                if (col_ok && tc + 2 * i + 1 < n_w)
                                    p.out[static_cast<size_t>(t + 1) * p.ldo + j] = __ushort_as_bfloat16(o[i] >> 16);
                            }
                        }
                    }
                    if (p.out_vec16) {
                        named_bar_sync(1, EPI_WARPS * 32);
                        if (!whole && threadIdx.x == kCtlThreads) p.ws_counters[st] = 0;
                        // one token row per warp and iteration, one 16-byte piece per lane (at most 17 pieces)
                        const int n_end = min(n0 + p.tile_rows, p.H);       // one past the tile's last column
                        const int pieces = (ph + (n_end - n0) + 7) >> 3;
                        const int c0 = n0 - ph + 8 * lane;                 // first column of this lane's piece
                        const bool full = c0 >= n0 && c0 + 8 <= n_end;
                        for (int t = e; t < p.M; t += EPI_WARPS) {
                            if (lane >= pieces) continue;
                            const uint4 v = *reinterpret_cast<const uint4*>(ot + t * kOutStagePitch + 8 * lane);
                            __nv_bfloat16* dst = p.out + static_cast<size_t>(t) * p.ldo + c0;
                            if (full) {
                                *reinterpret_cast<uint4*>(dst) = v;
                            } else {
                                const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                                for (int h = 0; h < 8; ++h)
                                    if (c0 + h >= n0 && c0 + h < n_end)
                                        dst[h] = __ushort_as_bfloat16(static_cast<uint16_t>(w[h >> 1] >> (16 * (h & 1))));
                            }
                        }
                        named_bar_sync(1, EPI_WARPS * 32);   // the staging block is free again
                    } else if (!whole) {
                        named_bar_sync(1, EPI_WARPS * 32);
                        if (threadIdx.x == kCtlThreads) p.ws_counters[st] = 0;
                    }
                    return true;
                };
                bool ok;
                if (per_warp <= 8) ok = segment(IntC<4>{});
                else if (per_warp <= 16) ok = segment(IntC<8>{});
                else ok = segment(IntC<16>{});
                if (!ok) break;
            } else {
                // ------------------------------------------------ token-major tile: lanes are token rows
                constexpr int kCols = (EPI == kEpiSwiglu) ? kBN / 2 : kBN;   // output columns of a tile, at most
                const int c_lo = (e / 4) * (kCols / kSplit);
                const int c_hi = c_lo + kCols / kSplit;
                // SwiGLU tiles hold tile_rows gate columns (the last tile of a row may hold fewer: c_end) and
                // their up columns up_off TMEM columns further on
                const int rows = (EPI == kEpiSwiglu) ? p.tile_rows : kBN;
                const int up_off = (EPI == kEpiSwiglu) ? p.tile_rows8 : 0;
                const int c_end = (EPI == kEpiSwiglu) ? min(rows, p.H - nt * rows) : kBN;
                const int grow = m0 + r_tile;
                const bool row_ok = grow >= row_lo && grow < row_hi;
                // Stage this tile's column scales / biases and this row's scale while the MMAs still run.
                float sa_row = 0.f;
                if constexpr (MODE == 0) {
                    for (int t = threadIdx.x - kCtlThreads; t < kBN; t += EPI_WARPS * 32) {
                        int col;
                        if constexpr (EPI == kEpiSwiglu)   // columns past c_end repeat a valid one (never stored)
                            col = part * p.n_part_stride + nt * rows +
                                  (t < kBN / 2 ? min(t, c_end - 1) : p.H + min(t - kBN / 2, c_end - 1));
                        else
                            col = part * p.n_part_stride + nt * kBN + t;
                        s_sw[t] = __ldg(p.sw + col);
                        s_bias[t] = __ldg(p.bias + col);
                    }
                    if (row_ok) sa_row = __ldg(p.sa + part * p.sa_part_stride + grow);
                    named_bar_sync(1, EPI_WARPS * 32);
                }
                if (!mbar_wait_bounded(&acc_full[buf], acc_phase, p.timeout_ns, nullptr)) {
                    raise_error(p, abort_flag, kStatusTimeoutAccFull);
                    break;
                }
                tc_fence_after();
                bool finish = whole;
                if (!whole) {
                    // SwiGLU tiles publish the gate columns [c_lo, c_hi) and the up columns up_off + [c_lo, c_hi)
                    finish = publish_partial<EPI_WARPS, 32>(p, seg, st, t_int, c_lo, c_hi, up_off, r_tile, row_ok,
                                                            last_flag);
                }
                constexpr bool add_f = (MODE == 0 && ADD_F);
                const uint64_t sa2 = f2(sa_row, sa_row);
                if constexpr (add_f) {
                    // Dequantize the INT8 accumulators into the float32 region, where the MMA issuer then
                    // adds the BF16 columns' products on top (tiles with BF16 columns are never split).
                    // Rows past the tile's rows and columns past c_end get values that are never stored.
                    for (int cc = c_lo; cc < c_hi; cc += 32) {
                        if (cc >= c_end) break;   // the same for the whole CTA
                        for (int h = 0; h < (EPI == kEpiSwiglu ? 2 : 1); ++h) {
                            const int col = cc + h * up_off;   // TMEM column; its scales sit at s_sw[cc + h * kBN / 2]
                            const int sc = cc + h * (kBN / 2);
                            uint32_t a[32];
                            tmem_ld_x32_sync(t_int + col, a);
#pragma unroll
                            for (int i = 0; i < 32; i += 2) {
                                const int si = (EPI == kEpiSwiglu ? sc : col) + i;
                                const uint64_t v = dequant2(a[i], a[i + 1], sa2, *reinterpret_cast<const uint64_t*>(s_sw + si),
                                                            *reinterpret_cast<const uint64_t*>(s_bias + si));
                                a[i] = static_cast<uint32_t>(v);
                                a[i + 1] = static_cast<uint32_t>(v >> 32);
                            }
                            tmem_st_x32(t_f32 + col, a);
                        }
                    }
                    tmem_wait_st();
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(deq_ready);
                    if (!mbar_wait_bounded(&acc_full[1], acc_phase, p.timeout_ns, nullptr)) {
                        raise_error(p, abort_flag, kStatusTimeoutAccFull);
                        break;
                    }
                    tc_fence_after();
                }
                if (finish) {
                    const int4* contrib[kMaxContrib];
                    const int n_contrib = whole ? 0 : contributors(p, st, contrib);
                    // float32 values to round: BF16-only accumulators, or the dequantized values with the
                    // BF16 columns added (ADD_F)
                    constexpr bool f32_vals = (MODE == 1 || add_f);
                    const uint32_t t_rd = add_f ? t_f32 : t_acc;
                    for (int cc = c_lo; cc < c_hi; cc += 32) {
                        if (cc >= c_end) break;   // the same for the whole CTA
                        uint32_t g[32];
                        uint32_t u[32];
                        if constexpr (EPI == kEpiSwiglu) {
                            tmem_ld2_x32_sync(t_rd + cc, t_rd + up_off + cc, g, u);
                        } else {
                            tmem_ld_x32_sync(t_rd + cc, g);
                        }
                        // whole warps outside the tile's rows skip; the others stay converged for the SiLU's
                        // warp vote, and only their stores and partial sums are per row
                        if (__all_sync(0xFFFFFFFFu, !row_ok)) continue;
                        if (row_ok && !whole) {
                            add_partials<32>(contrib, n_contrib, cc, r_tile, g);
                            if constexpr (EPI == kEpiSwiglu) add_partials<32>(contrib, n_contrib, up_off + cc, r_tile, u);
                        }
                        uint32_t packed[16];
                        __nv_bfloat16* dst;
                        if constexpr (EPI == kEpiSwiglu) {
                            // bf16 gate/up values of the 16 pairs, then their SiLU through the table (one vote)
                            uint32_t gw[16], uw[16];
#pragma unroll
                            for (int i = 0; i < 32; i += 2) {
                                uint64_t vg, vu;
                                if constexpr (!f32_vals) {
                                    const uint64_t swg = *reinterpret_cast<const uint64_t*>(s_sw + cc + i);
                                    const uint64_t swu = *reinterpret_cast<const uint64_t*>(s_sw + kBN / 2 + cc + i);
                                    const uint64_t bgv = *reinterpret_cast<const uint64_t*>(s_bias + cc + i);
                                    const uint64_t buv = *reinterpret_cast<const uint64_t*>(s_bias + kBN / 2 + cc + i);
                                    vg = dequant2(g[i], g[i + 1], sa2, swg, bgv);
                                    vu = dequant2(u[i], u[i + 1], sa2, swu, buv);
                                } else {
                                    vg = f2(__uint_as_float(g[i]), __uint_as_float(g[i + 1]));
                                    vu = f2(__uint_as_float(u[i]), __uint_as_float(u[i + 1]));
                                }
                                gw[i / 2] = bf16x2_rn(vg);
                                uw[i / 2] = bf16x2_rn(vu);
                            }
                            swiglu2_bits_n<16>(gw, uw, packed, silu_tab_s);
                            dst = p.out + static_cast<size_t>(grow) * p.ldo + nt * rows + cc;
                        } else {
#pragma unroll
                            for (int i = 0; i < 32; i += 2) {
                                uint64_t v;
                                if constexpr (!f32_vals) {
                                    const uint64_t s2 = *reinterpret_cast<const uint64_t*>(s_sw + cc + i);
                                    const uint64_t b2 = *reinterpret_cast<const uint64_t*>(s_bias + cc + i);
                                    v = dequant2(g[i], g[i + 1], sa2, s2, b2);
                                } else {
                                    v = f2(__uint_as_float(g[i]), __uint_as_float(g[i + 1]));
                                }
                                packed[i / 2] = bf16x2_rn(v);
                            }
                            dst = p.out + out_part * p.out_part_stride + static_cast<size_t>(grow) * p.ldo + nt * kBN + cc;
                        }
                        if (EPI == kEpiSwiglu && p.out_tma) {
                            // The warp's 32 rows x 32 columns through shared memory (64-byte rows, 16-byte chunk
                            // c of row r at c ^ ((r >> 1) & 3), the tensor map's 64-byte swizzle, so the four
                            // 16-byte writes of the 32 lanes are free of bank conflicts), then one TMA store;
                            // rows past M and columns past H are clipped by the tensor map.  The buffer is
                            // reused once the previous store has read it.
                            uint8_t* wbuf = out_stage + e * kOutTmaWarpBytes;
                            if (lane == 0) bulk_wait_read_all();
                            __syncwarp();
#pragma unroll
                            for (int i = 0; i < 4; ++i)
                                *reinterpret_cast<uint4*>(wbuf + lane * 64 + ((i ^ ((lane >> 1) & 3)) * 16)) =
                                    make_uint4(packed[4 * i], packed[4 * i + 1], packed[4 * i + 2], packed[4 * i + 3]);
                            fence_proxy_async_smem();
                            __syncwarp();
                            if (lane == 0) {
                                tma_store_2d(&p.tm_out, wbuf, nt * rows + cc, m0 + q * 32);
                                bulk_commit_group();
                            }
                        } else if (row_ok) {
                            if (EPI != kEpiSwiglu || (rows & 7) == 0) {
                                // 16-byte pieces: c_end is a multiple of 8, so a piece is wholly in or out
#pragma unroll
                                for (int i = 0; i < 4; ++i)
                                    if (cc + 8 * i < c_end)
                                        reinterpret_cast<uint4*>(dst)[i] =
                                            make_uint4(packed[4 * i], packed[4 * i + 1], packed[4 * i + 2], packed[4 * i + 3]);
                            } else {
#pragma unroll
                                for (int i = 0; i < 32; ++i)
                                    if (cc + i < c_end) dst[i] = __ushort_as_bfloat16(static_cast<uint16_t>(packed[i / 2] >> (16 * (i & 1))));
                            }
                        }
                    }
                    if (!whole) {
                        named_bar_sync(1, EPI_WARPS * 32);
                        if (threadIdx.x == kCtlThreads) p.ws_counters[st] = 0;
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                if constexpr (PAIR) mbar_arrive_cluster(cluster_map(&acc_empty[buf], 0));   // rank 0 issues the MMAs
                else mbar_arrive(&acc_empty[buf]);
            }
            if (p.acc_bufs == 2) {
                buf ^= 1;
                if (buf == 0) acc_phase ^= 1;
            } else {
                acc_phase ^= 1;
            }
        }
    }

    // the epilogue's TMA stores have completed before the grid does
    if (warp >= kCtlWarps && lane == 0 && p.out_tma) bulk_wait_all();
    tc_fence_before();
    __syncthreads();
    if constexpr (PAIR) cluster_sync_all();
}

}  // namespace reax
