// Shared device helpers for the REAX gate/up kernels on sm_100a (B200).
//
// Thin inline-PTX wrappers for the Blackwell pieces the kernels are built from: mbarriers (with
// bounded waits), TMA tiled loads, tcgen05 MMA / commit / TMEM alloc / TMEM loads, plus the
// bf16 arithmetic of the reference's epilogue (SiLU and SwiGLU rounding points).
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#define REAX_DEVI __device__ __forceinline__

namespace reax {

// ------------------------------------------------------------------------------------------------ status words
// Bits OR-ed into the device status word (word 0 of the caller's workspace, or of the allocation-free
// entry's static scratch) when a bounded wait gives up.  The host reads the workspace word directly and
// the scratch word with reax_noalloc_status(); a kernel that sets one of these has returned early and
// its output is invalid.
enum : uint32_t {
    kStatusTimeoutFull = 1u << 0,      // MMA issuer waited too long for a TMA stage
    kStatusTimeoutEmpty = 1u << 1,     // producer waited too long for a free stage
    kStatusTimeoutAccFull = 1u << 2,   // epilogue waited too long for an accumulator
    kStatusTimeoutAccEmpty = 1u << 3,  // MMA issuer waited too long for a free accumulator
    kStatusTimeoutDrain = 1u << 4,     // teardown waited too long for in-flight copies / MMAs
    kStatusSelfTest = 1u << 5,         // reax_selftest_wait(): the wait on a never-arriving barrier expired
    kStatusPlanLimit = 1u << 6,        // a split tile had more contributors than a finisher can gather
};

REAX_DEVI uint32_t smem_u32(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }

REAX_DEVI uint64_t global_timer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// ---------------------------------------------------------------------------------------------------- mbarrier
REAX_DEVI void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
REAX_DEVI void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }

REAX_DEVI void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
REAX_DEVI void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
REAX_DEVI bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// Wait until the phase with the given parity has completed, for at most `limit_ns` nanoseconds of
// global time.  Also gives up early when `*abort` (a shared flag another role sets after its own
// timeout) becomes non-zero.  Returns false when it gave up.
REAX_DEVI bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, uint64_t limit_ns, volatile int* abort) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_timer_ns();
    while (true) {
        if (mbar_try_wait(bar, parity)) return true;
        if (abort != nullptr && *abort) return false;
        if (global_timer_ns() - t0 > limit_ns) return false;
    }
}

// mbar_wait_bounded for waits that are expected to last (a copy in flight): each try asks the hardware to
// suspend the thread for up to suspend_ns while the phase is incomplete, so a waiting warp does not take
// issue slots from the warps that work.
REAX_DEVI bool mbar_try_wait_suspend(uint64_t* bar, uint32_t parity, uint32_t suspend_ns) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(suspend_ns)
        : "memory");
    return ok != 0;
}
REAX_DEVI bool mbar_wait_bounded_suspend(uint64_t* bar, uint32_t parity, uint64_t limit_ns) {
    if (mbar_try_wait_suspend(bar, parity, 1000u)) return true;
    const uint64_t t0 = global_timer_ns();
    while (true) {
        if (mbar_try_wait_suspend(bar, parity, 1000u)) return true;
        if (global_timer_ns() - t0 > limit_ns) return false;
    }
}

// ---------------------------------------------------------------------------------------------------------- TMA
REAX_DEVI void tma_prefetch_desc(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}
// 2-D tiled load of one box into shared memory, completing `bytes` on `bar`.  x is the innermost
// (contiguous) coordinate in elements; callers keep x * element size a multiple of 16 bytes.
REAX_DEVI void tma_load_2d(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int x, int y, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%3, %4}], [%2], %5;" ::"r"(smem_u32(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "l"(policy)
        : "memory");
}
// 3-D and 4-D tiled loads (x innermost, x = 0 here: the box covers the whole 128-byte innermost extent).
REAX_DEVI void tma_load_3d(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int x, int y, int z, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%3, %4, %5}], [%2], %6;" ::"r"(smem_u32(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z), "l"(policy)
        : "memory");
}
REAX_DEVI void tma_load_4d(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int x, int y, int z, int w,
                           uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%3, %4, %5, %6}], [%2], %7;" ::"r"(smem_u32(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z), "r"(w), "l"(policy)
        : "memory");
}
// 2-D tiled store of one box from this CTA's shared memory to global memory (coordinates x, y >= 0; the
// tensor map clips the box at the tensor's bounds), in the thread's bulk async-group.
REAX_DEVI void tma_store_2d(const CUtensorMap* map, const void* smem_src, int x, int y) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                     reinterpret_cast<uint64_t>(map)),
                 "r"(smem_u32(smem_src)), "r"(x), "r"(y)
                 : "memory");
}
REAX_DEVI void bulk_commit_group() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// Wait until the thread's committed bulk stores have read their shared-memory source (the buffer is free).
REAX_DEVI void bulk_wait_read_all() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
// Wait until the thread's committed bulk stores have completed.
REAX_DEVI void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// 1-D bulk copy of `bytes` (a multiple of 16; both addresses 16-byte aligned) from global memory into
// this CTA's shared memory, completing on `bar`.
REAX_DEVI void bulk_load(void* smem_dst, const void* gsrc, uint32_t bytes, uint64_t* bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_u32(smem_dst)),
                 "l"(gsrc), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}
// Order this thread's earlier generic-proxy accesses of shared memory before later async-proxy ones
// (e.g. a bulk copy into a buffer the thread has just read).
REAX_DEVI void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
// 16 bytes from global memory (through L2) into this thread's shared memory, asynchronously; the
// thread's own copies are complete, and visible to it, after cp_async_wait_all().
REAX_DEVI void cp_async16_cg(void* smem_dst, const void* gsrc) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem_dst)), "l"(gsrc) : "memory");
}
REAX_DEVI void cp_async_wait_all() { asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory"); }

REAX_DEVI uint64_t l2_policy_evict_first() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}
REAX_DEVI uint64_t l2_policy_evict_last() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
    return p;
}
REAX_DEVI uint64_t l2_policy_evict_normal() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_normal.b64 %0, 1.0;" : "=l"(p));
    return p;
}

// ------------------------------------------------------------------------------------------------------ tcgen05
// Shared-memory matrix descriptor for a K-major operand tile stored with the 128-byte swizzle:
// rows of 128 bytes, 8-row core groups 1024 bytes apart (SBO), version 1 (sm_100), layout 2 (SW128).
REAX_DEVI uint64_t sw128_kmajor_desc(uint32_t smem_addr) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((smem_addr >> 4) & 0x3FFF);        // start address, bits [0,14)
    d |= static_cast<uint64_t>(1) << 16;                           // leading byte offset (unused for SW128 K-major)
    d |= static_cast<uint64_t>(1024 >> 4) << 32;                   // stride byte offset, bits [32,46)
    d |= static_cast<uint64_t>(1) << 46;                           // descriptor version for sm_100
    d |= static_cast<uint64_t>(2) << 61;                           // swizzle mode: 128B
    return d;
}

// Instruction descriptors (dense, K-major A and B, no negation).  c_format bits [4,6), a/b format
// bits [7,10)/[10,13), N>>3 bits [17,23), M>>4 bits [24,29).
__host__ __device__ constexpr uint32_t idesc_i8_s32(int M, int N) {
    return (2u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(N >> 3) << 17) |
           (static_cast<uint32_t>(M >> 4) << 24);
}
__host__ __device__ constexpr uint32_t idesc_bf16_f32(int M, int N) {
    return (1u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(N >> 3) << 17) |
           (static_cast<uint32_t>(M >> 4) << 24);
}

REAX_DEVI void umma_i8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}
REAX_DEVI void umma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// Arrive once on `bar` when every tcgen05 operation this thread issued before it has completed.
REAX_DEVI void umma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}
REAX_DEVI void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
REAX_DEVI void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// TMEM allocation: whole-warp instructions.
REAX_DEVI void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
                 "r"(ncols)
                 : "memory");
}
REAX_DEVI void tmem_relinquish() { asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory"); }
REAX_DEVI void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// ------------------------------------------------------------------- CTA pairs (tcgen05 .cta_group::2)
// Two CTAs of a cluster (ranks 0 and 1) share one MMA of M = 256: each holds 128 rows of A and half of the
// N rows of B in its own shared memory at the same offsets, rank 0 issues the MMAs, and each CTA's TMEM
// receives its 128 accumulator rows.  Every tcgen05 instruction of such a kernel uses .cta_group::2.
REAX_DEVI uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
// Address in the shared-memory window of CTA `rank` of this cluster of the object at `p` in this CTA.
REAX_DEVI uint32_t cluster_map(const void* p, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
    return r;
}
// Every thread of both CTAs: release this CTA's prior shared-memory writes (mbarrier inits) to the
// cluster and wait for the other CTA to do the same.
REAX_DEVI void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Arrivals on an mbarrier of either CTA of the pair, with the default (CTA-scope release) semantics: a
// cluster-scope release puts a cluster-wide memory barrier in front of every arrival, which waits for the
// thread's earlier copies and so serialises a producer's boxes.  The data these arrivals publish is TMA
// bytes (counted by complete_tx) or TMEM reads (ordered by tcgen05.fence::before_thread_sync), neither
// of which needs it.
REAX_DEVI void mbar_arrive_expect_tx_cluster(uint32_t bar_cluster_addr, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cluster.b64 _, [%0], %1;" ::"r"(bar_cluster_addr), "r"(bytes)
                 : "memory");
}
REAX_DEVI void mbar_arrive_cluster(uint32_t bar_cluster_addr) {
    asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(bar_cluster_addr) : "memory");
}
// Tiled load of one box into this CTA's shared memory whose completion is counted on an mbarrier of either
// CTA of the pair (bar_cluster_addr: a shared::cluster address).  No multicast: each CTA loads its own boxes.
REAX_DEVI void tma_load_2d_pair(void* smem_dst, const CUtensorMap* map, uint32_t bar_cluster_addr, int x, int y,
                                uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%3, %4}], [%2], %5;" ::"r"(smem_u32(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster_addr), "r"(x), "r"(y), "l"(policy)
        : "memory");
}
REAX_DEVI void umma_i8_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}
REAX_DEVI void umma_f16_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// Arrive once on the mbarrier at the offset of `bar` in both CTAs of the pair when every tcgen05
// operation this thread issued before it has completed.
REAX_DEVI void umma_commit_pair(uint64_t* bar) {
    asm volatile(
        "{\n\t.reg .b16 m;\n\tmov.b16 m, 3;\n\t"
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], m;\n\t}" ::"r"(
            smem_u32(bar))
        : "memory");
}
// Arrive on the mbarrier at `bar` of this CTA only (the drain barrier before TMEM is freed).
REAX_DEVI void umma_commit_pair_local(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}
REAX_DEVI void tmem_alloc_pair(uint32_t* dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
                 "r"(ncols)
                 : "memory");
}
REAX_DEVI void tmem_relinquish_pair() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
REAX_DEVI void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// 32 lanes x 32 consecutive 32-bit columns: register i of lane t <- TMEM[lane base + t][column + i].
REAX_DEVI void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
}
REAX_DEVI void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Load 32 columns and wait for them in one asm block, so no use of `r` can be scheduled before the
// wait::ld (the registers are only defined once the whole block has executed).
REAX_DEVI void tmem_ld_x32_sync(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n\t"
        "tcgen05.wait::ld.sync.aligned;"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr)
        : "memory");
}

// 32 lanes x 8 columns, with the wait in the same asm block.
REAX_DEVI void tmem_ld_x8_sync(uint32_t taddr, uint32_t (&r)[8]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];\n\t"
        "tcgen05.wait::ld.sync.aligned;"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
        : "r"(taddr)
        : "memory");
}

// Two 8-column loads and one wait.
REAX_DEVI void tmem_ld_x8_pair_sync(uint32_t ta, uint32_t tb, uint32_t (&a)[8], uint32_t (&b)[8]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%16];\n\t"
        "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%8,%9,%10,%11,%12,%13,%14,%15}, [%17];\n\t"
        "tcgen05.wait::ld.sync.aligned;"
        : "=r"(a[0]), "=r"(a[1]), "=r"(a[2]), "=r"(a[3]), "=r"(a[4]), "=r"(a[5]), "=r"(a[6]), "=r"(a[7]),
          "=r"(b[0]), "=r"(b[1]), "=r"(b[2]), "=r"(b[3]), "=r"(b[4]), "=r"(b[5]), "=r"(b[6]), "=r"(b[7])
        : "r"(ta), "r"(tb)
        : "memory");
}

// The same into the first 8 entries of 32-entry arrays.
REAX_DEVI void tmem_ld_x8_pair_sync(uint32_t ta, uint32_t tb, uint32_t (&a)[32], uint32_t (&b)[32]) {
    tmem_ld_x8_pair_sync(ta, tb, *reinterpret_cast<uint32_t(*)[8]>(a), *reinterpret_cast<uint32_t(*)[8]>(b));
}

// Two 32-column loads (e.g. the gate and the up half of one output chunk) and one wait.
REAX_DEVI void tmem_ld2_x32_sync(uint32_t ta, uint32_t tb, uint32_t (&a)[32], uint32_t (&b)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%64];\n\t"
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%32,%33,%34,%35,%36,%37,%38,%39,%40,%41,%42,%43,%44,%45,%46,%47,"
        "%48,%49,%50,%51,%52,%53,%54,%55,%56,%57,%58,%59,%60,%61,%62,%63}, [%65];\n\t"
        "tcgen05.wait::ld.sync.aligned;"
        : "=r"(a[0]), "=r"(a[1]), "=r"(a[2]), "=r"(a[3]), "=r"(a[4]), "=r"(a[5]), "=r"(a[6]), "=r"(a[7]),
          "=r"(a[8]), "=r"(a[9]), "=r"(a[10]), "=r"(a[11]), "=r"(a[12]), "=r"(a[13]), "=r"(a[14]), "=r"(a[15]),
          "=r"(a[16]), "=r"(a[17]), "=r"(a[18]), "=r"(a[19]), "=r"(a[20]), "=r"(a[21]), "=r"(a[22]), "=r"(a[23]),
          "=r"(a[24]), "=r"(a[25]), "=r"(a[26]), "=r"(a[27]), "=r"(a[28]), "=r"(a[29]), "=r"(a[30]), "=r"(a[31]),
          "=r"(b[0]), "=r"(b[1]), "=r"(b[2]), "=r"(b[3]), "=r"(b[4]), "=r"(b[5]), "=r"(b[6]), "=r"(b[7]),
          "=r"(b[8]), "=r"(b[9]), "=r"(b[10]), "=r"(b[11]), "=r"(b[12]), "=r"(b[13]), "=r"(b[14]), "=r"(b[15]),
          "=r"(b[16]), "=r"(b[17]), "=r"(b[18]), "=r"(b[19]), "=r"(b[20]), "=r"(b[21]), "=r"(b[22]), "=r"(b[23]),
          "=r"(b[24]), "=r"(b[25]), "=r"(b[26]), "=r"(b[27]), "=r"(b[28]), "=r"(b[29]), "=r"(b[30]), "=r"(b[31])
        : "r"(ta), "r"(tb)
        : "memory");
}

// Two 16-column loads and one wait.
REAX_DEVI void tmem_ld2_x16_sync(uint32_t ta, uint32_t tb, uint32_t (&a)[16], uint32_t (&b)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%32];\n\t"
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%33];\n\t"
        "tcgen05.wait::ld.sync.aligned;"
        : "=r"(a[0]), "=r"(a[1]), "=r"(a[2]), "=r"(a[3]), "=r"(a[4]), "=r"(a[5]), "=r"(a[6]), "=r"(a[7]),
          "=r"(a[8]), "=r"(a[9]), "=r"(a[10]), "=r"(a[11]), "=r"(a[12]), "=r"(a[13]), "=r"(a[14]), "=r"(a[15]),
          "=r"(b[0]), "=r"(b[1]), "=r"(b[2]), "=r"(b[3]), "=r"(b[4]), "=r"(b[5]), "=r"(b[6]), "=r"(b[7]),
          "=r"(b[8]), "=r"(b[9]), "=r"(b[10]), "=r"(b[11]), "=r"(b[12]), "=r"(b[13]), "=r"(b[14]), "=r"(b[15])
        : "r"(ta), "r"(tb)
        : "memory");
}

// Store 32 consecutive 32-bit columns of this warp's 32 lanes: TMEM[lane base + t][column + i] <- register
// i of lane t.  tmem_wait_st() makes them complete before the thread goes on (e.g. to signal the MMA
// issuer, after tc_fence_before()).
REAX_DEVI void tmem_st_x32(uint32_t taddr, const uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
        "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};"
        ::"r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
          "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]),
          "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]),
          "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
}
REAX_DEVI void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Gate and up accumulators of 2 * PAIRS token columns (8, 16 or 32) with one wait.
template <int PAIRS>
REAX_DEVI void tmem_ld_pairs_sync(uint32_t ta, uint32_t tb, uint32_t (&a)[2 * PAIRS], uint32_t (&b)[2 * PAIRS]) {
    static_assert(PAIRS == 4 || PAIRS == 8 || PAIRS == 16, "8, 16 or 32 columns");
    if constexpr (PAIRS == 4) tmem_ld_x8_pair_sync(ta, tb, a, b);
    else if constexpr (PAIRS == 8) tmem_ld2_x16_sync(ta, tb, a, b);
    else tmem_ld2_x32_sync(ta, tb, a, b);
}

// Compile-time integer for generic lambdas.
template <int N>
struct IntC {
    static constexpr int value = N;
};

// Named barrier over `count` threads (a multiple of 32).
REAX_DEVI void named_bar_sync(int id, int count) { asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory"); }

// Per-warpgroup register split (setmaxnreg; every thread of the warpgroup executes it).  A grow waits
// until other warps of the CTA have released enough registers, so callers pair it with shrinks whose
// total covers it.
template <int N> REAX_DEVI void regs_shrink() { asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N)); }
template <int N> REAX_DEVI void regs_grow() { asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N)); }

// Programmatic dependent launch: wait for the preceding grid's memory to be visible.
REAX_DEVI void grid_dependency_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
REAX_DEVI void grid_dependents_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ------------------------------------------------------------------------------------------- bf16 arithmetic
REAX_DEVI float bf16_round(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }

// silu(x) = x / (1 + expf(-x)) with CUDA's expf and an IEEE round-to-nearest division, all in
// float32: the arithmetic of the reference's silu_f32 (hybrid8_tiles.cuh:675).
REAX_DEVI float silu_f32(float x) { return __fdiv_rn(x, 1.0f + expf(-x)); }

// ------------------------------------------------------------------------------------------ SiLU table
// For a bf16-valued x, bf16(silu_f32(x)) depends only on the 16-bit pattern of x, and outside the
// exponent fields [kSiluTabElo, kSiluTabEhi] (|x| in [2^-10, 128)) it needs no table:
//   |x| < 2^-10   -> bf16(x * 0.5): 1 + expf(-x) lies within 2^-10 of 2 - x, so the quotient is within
//                    a relative 2^-11 of x / 2, which is a bf16 value (or rounds to the same bf16
//                    subnormal as x * 0.5 does);
//   x >= 128      -> x: expf(-x) < 2^-24, so 1 + expf(-x) rounds to 1;
//   x <= -128     -> -0: expf(-x) overflows to +inf and x / inf = -0;
//   +inf          -> +inf (+inf / (1 + 0));
//   -inf, NaN     -> NaN (-inf / +inf, or a NaN operand).  Every NaN the reference can produce here is
//                    multiplied by u next, which gives the canonical NaN whatever the payload, so
//                    one NaN serves for all of them.
// The 2 x 17 x 128 patterns in between are tabulated by the exact formula (8.5 KiB of shared memory).
// The test over all 65536 bf16 patterns compares this path with bf16(silu_f32(x)), the value the
// reference's SwiGLU multiplies by (hybrid8_tiles.cuh:676-678).
constexpr uint32_t kSiluTabElo = 117;                                   // 2^-10
constexpr uint32_t kSiluTabEhi = 133;                                   // [64, 128)
constexpr uint32_t kSiluTabHalf = (kSiluTabEhi - kSiluTabElo + 1) * 128;  // patterns of one sign
constexpr int kSiluTabBytes = static_cast<int>(2 * kSiluTabHalf * 2);

// Fill the table: entry i < kSiluTabHalf is the positive pattern (kSiluTabElo << 7) + i, the rest the
// negative ones in the same order.
REAX_DEVI void silu_table_fill(uint16_t* tab, int tid, int nthreads) {
    for (int i = tid; i < static_cast<int>(2 * kSiluTabHalf); i += nthreads) {
        const uint32_t sign = static_cast<uint32_t>(i) >= kSiluTabHalf ? 0x8000u : 0u;
        const uint32_t mag = static_cast<uint32_t>(i) % kSiluTabHalf + (kSiluTabElo << 7);
        tab[i] = __bfloat16_as_ushort(__float2bfloat16_rn(silu_f32(__uint_as_float((sign | mag) << 16))));
    }
}

// bf16(silu_f32(x)) for a bf16-valued x through the table.
REAX_DEVI float silu_tab(float x, const uint16_t* tab) {
    const uint32_t b = __float_as_uint(x) >> 16;
    const uint32_t mag = b & 0x7FFFu;
    const uint32_t rel = mag - (kSiluTabElo << 7);        // wraps for |x| < 2^-10
    const bool in_tab = rel < kSiluTabHalf;
    const uint32_t idx = (in_tab ? rel : 0u) + ((b & 0x8000u) ? kSiluTabHalf : 0u);
    const float t = __uint_as_float(static_cast<uint32_t>(tab[idx]) << 16);
    const bool tiny = mag < (kSiluTabElo << 7);
    const float small = bf16_round(__fmul_rn(x, 0.5f));
    const bool special = (mag & 0x7F80u) == 0x7F80u;      // +-inf, NaN
    const float big = special ? (x > 0.0f ? x : __uint_as_float(0x7FFFFFFFu)) : ((b & 0x8000u) ? -0.0f : x);
    return in_tab ? t : (tiny ? small : big);
}

// out = bf16(float(bf16(silu_f32(g))) * u) for bf16-valued g and u (hybrid8_tiles.cuh:676-679).
REAX_DEVI __nv_bfloat16 swiglu_bf16(float g_bf16_value, float u_bf16_value, const uint16_t* tab) {
    return __float2bfloat16_rn(__fmul_rn(silu_tab(g_bf16_value, tab), u_bf16_value));
}

// ------------------------------------------------------------------------------------- packed float32 pairs
// sm_100 executes two float32 lanes per instruction (add/mul/fma .rn.f32x2); each lane is rounded
// exactly like the scalar IEEE op, so packed arithmetic keeps every result bit-identical.
REAX_DEVI uint64_t f2(float lo, float hi) {
    return (static_cast<uint64_t>(__float_as_uint(hi)) << 32) | __float_as_uint(lo);
}
REAX_DEVI float f2_lo(uint64_t v) { return __uint_as_float(static_cast<uint32_t>(v)); }
REAX_DEVI float f2_hi(uint64_t v) { return __uint_as_float(static_cast<uint32_t>(v >> 32)); }
REAX_DEVI uint64_t mul2_rn(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
REAX_DEVI uint64_t add2_rn(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
REAX_DEVI uint64_t sub2_rn(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
REAX_DEVI uint64_t fma2_rn(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}
// two float32 -> packed bf16x2 (round to nearest even), low lane first
REAX_DEVI uint32_t bf16x2_rn(uint64_t v) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(f2_lo(v), f2_hi(v));
    return *reinterpret_cast<const uint32_t*>(&h);
}
// packed bf16x2 -> the two values as a float32 pair (exact)
REAX_DEVI uint64_t bf16x2_to_f2(uint32_t w) { return f2(__uint_as_float(w << 16), __uint_as_float(w & 0xFFFF0000u)); }

// INT8 dequant of two accumulators, lane-wise ((acc * sa) * sw) + bias with three IEEE roundings.
// Only the first product is packed: ptxas contracts a packed mul.rn.f32x2 feeding a packed
// add.rn.f32x2 into one fused multiply-add (measured on sm_100a with CUDA 12.9), which would round
// (t * sw + bias) once instead of twice; the scalar mul.rn / add.rn pair is never contracted.
REAX_DEVI uint64_t dequant2(uint32_t a0, uint32_t a1, uint64_t sa2, uint64_t sw2, uint64_t b2) {
    const uint64_t raw = f2(__int2float_rn(static_cast<int>(a0)), __int2float_rn(static_cast<int>(a1)));
    const uint64_t t = mul2_rn(raw, sa2);
    const float v0 = __fadd_rn(__fmul_rn(f2_lo(t), f2_lo(sw2)), f2_lo(b2));
    const float v1 = __fadd_rn(__fmul_rn(f2_hi(t), f2_hi(sw2)), f2_hi(b2));
    return f2(v0, v1);
}

// SwiGLU of N (gate, up) pairs given as packed bf16x2 words: o[i] = bf16x2 of bf16(silu(g) * u), lane-wise,
// from (gw[i], uw[i]).  When every lane of the warp has all its gate values inside the table's range (the
// usual case) each SiLU is one shared-memory load, and one warp vote covers all N pairs, so their table
// loads do not wait on one another; otherwise the warp takes silu_tab's full case analysis.  All 32 lanes
// of the warp must call it together.
template <int N>
REAX_DEVI void swiglu2_bits_n(const uint32_t (&gw)[N], const uint32_t (&uw)[N], uint32_t (&o)[N],
                              const uint16_t* tab) {
    constexpr uint32_t lo = kSiluTabElo << 7;
    bool in = true;
#pragma unroll
    for (int i = 0; i < N; ++i)
        in = in && ((gw[i] & 0x7FFFu) - lo) < kSiluTabHalf && (((gw[i] >> 16) & 0x7FFFu) - lo) < kSiluTabHalf;
    uint32_t s0[N], s1[N];   // bf16(silu) of both gates as float32 bit patterns
    if (__all_sync(0xFFFFFFFFu, in)) {
#pragma unroll
        for (int i = 0; i < N; ++i) {
            const uint32_t b0 = gw[i] & 0xFFFFu, b1 = gw[i] >> 16;
            s0[i] = static_cast<uint32_t>(tab[(b0 & 0x7FFFu) - lo + (b0 >> 15) * kSiluTabHalf]) << 16;
            s1[i] = static_cast<uint32_t>(tab[(b1 & 0x7FFFu) - lo + (b1 >> 15) * kSiluTabHalf]) << 16;
        }
    } else {
#pragma unroll
        for (int i = 0; i < N; ++i) {
            s0[i] = __float_as_uint(silu_tab(__uint_as_float(gw[i] << 16), tab));
            s1[i] = __float_as_uint(silu_tab(__uint_as_float(gw[i] & 0xFFFF0000u), tab));
        }
    }
#pragma unroll
    for (int i = 0; i < N; ++i)
        o[i] = bf16x2_rn(mul2_rn((static_cast<uint64_t>(s1[i]) << 32) | s0[i], bf16x2_to_f2(uw[i])));
}

REAX_DEVI uint32_t pack_bf16x2(__nv_bfloat16 lo, __nv_bfloat16 hi) {
    return static_cast<uint32_t>(__bfloat16_as_ushort(lo)) | (static_cast<uint32_t>(__bfloat16_as_ushort(hi)) << 16);
}

}  // namespace reax
