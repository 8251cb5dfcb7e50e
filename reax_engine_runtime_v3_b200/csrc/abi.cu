// C ABI of the B200 gate/up path (declarations and contracts: include/reax_b200.h).
//
// Host side of every entry point: argument validation (the preconditions the reference asserts in
// reaxv2/gate_up.py:14 and reaxv2/sliced.py:26, plus the alignment the kernels need), TMA tensor-map
// encoding, the tile / stream-K plan of the tcgen05 kernels, and the launches.  Nothing here
// allocates device memory or synchronizes, so every entry point is usable inside graph capture.
#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <utility>

#include <cudaTypedefs.h>

#include "gate_up_tc.cuh"
#include "reax_b200.h"
#include "rowwise.cuh"

namespace {

constexpr int kVersion = 10000;           // 1.0.0
constexpr int kEpiWarps = 8;
constexpr int kStages = 4;
constexpr int kMaxDevices = 64;
constexpr size_t kStatusBytes = 256;
constexpr unsigned long long kDefaultTimeoutNs = 2000000000ull;   // 2 s

// Quantizer division for the plain '/' of reaxv2/quantize.py:18-19,42 (see rowwise.cuh).
constexpr int kQuantDivision = reax::kQuantDiv;

thread_local std::string g_last_error;
unsigned long long g_timeout_ns = kDefaultTimeoutNs;

int fail(int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return code;
}

int cuda_fail(cudaError_t e, const char* what) {
    return fail(REAX_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

struct DeviceInfo {
    bool ready = false;
    int sms = 0;
    int major = 0, minor = 0;
    bool smem_set = false;
    bool stream_smem_set = false;
    int pair_clusters = 0;   // CTA pairs of the pair GEMM that can be resident at once (GPC layout permitting)
};
// Shared memory the many-rows quantizer may use per CTA (one CTA per SM), and the rows from which it runs.
constexpr size_t kQuantStreamSmemMax = 227 * 1024;
constexpr int kQuantStreamMinRowsPerSm = 4;
DeviceInfo g_dev[kMaxDevices];
std::mutex g_dev_mutex;

// The kernel variants: (epilogue, mode, BF16 columns added to INT8 accumulators).
enum Variant : int {
    kSwigluI8 = 0, kSwigluI8F, kSwigluBf16, kPlainI8, kPlainI8F, kPlainBf16, kSwapI8, kSwapBf16, kPairI8, kPairBf16,
    kPlainSwapI8, kVariants
};

// Token rows from which an INT8 gate/up launch without BF16 columns takes CTA-pair tiles (256 token rows x
// 128 gate + 128 up columns per pair, tcgen05 cta_group::2).
constexpr int kPairMinRows = 512;
// Grouped INT8 projections with fewer tiles than SMs may split their tiles by K (parity-green, but the
// down projection's 40-tile decode launches measured 16-17.6 us split against 10.3-11 us whole, so off).
constexpr bool kSplitPlainTiles = false;   // measured slower at every decode shape
// Stages of a pair's ring: [half of B | A box] of 32 KiB each in the same pool as four 48 KiB stages.
constexpr int kPairStages = 6;

// Activation rows up to which the gate/up kernels use weight-major (swap) tiles.
constexpr int kSwapMaxRows = reax::kSwapMaxTok;

void* tc_kernel_ptr(int v) {
    using namespace reax;
    switch (v) {
        case kSwigluI8: return reinterpret_cast<void*>(&tc_gemm_kernel<kEpiWarps, kStages, kEpiSwiglu, 0, false, false>);
        case kSwigluI8F: return reinterpret_cast<void*>(&tc_gemm_kernel<kEpiWarps, kStages, kEpiSwiglu, 0, true, false>);
        case kSwigluBf16: return reinterpret_cast<void*>(&tc_gemm_kernel<kEpiWarps, kStages, kEpiSwiglu, 1, false, false>);
        case kPlainI8: return reinterpret_cast<void*>(&tc_gemm_kernel<kEpiWarps, kStages, kEpiPlain, 0, false, false>);
        case kPlainI8F: return reinterpret_cast<void*>(&tc_gemm_kernel<kEpiWarps, kStages, kEpiPlain, 0, true, false>);
        case kPlainBf16: return reinterpret_cast<void*>(&tc_gemm_kernel<kEpiWarps, kStages, kEpiPlain, 1, false, false>);
        case kSwapI8: return reinterpret_cast<void*>(&tc_gemm_kernel<kEpiWarps, kStages, kEpiSwiglu, 0, false, true>);
        case kPairI8:
            return reinterpret_cast<void*>(&tc_gemm_kernel<kEpiWarps, kStages, kEpiSwiglu, 0, false, false, true>);
        case kPairBf16:
            return reinterpret_cast<void*>(&tc_gemm_kernel<kEpiWarps, kStages, kEpiSwiglu, 1, false, false, true>);
        case kPlainSwapI8: return reinterpret_cast<void*>(&tc_gemm_kernel<kEpiWarps, kStages, kEpiPlain, 0, false, true>);
        default: return reinterpret_cast<void*>(&tc_gemm_kernel<kEpiWarps, kStages, kEpiSwiglu, 1, false, true>);
    }
}

int variant_of(int epi, const reax::TcParams& p) {
    if (p.cta_shift == 1) return p.mode == 1 ? kPairBf16 : kPairI8;
    if (p.n_tok > 0) return p.mode == 1 ? kSwapBf16 : (epi == reax::kEpiPlain ? kPlainSwapI8 : kSwapI8);
    if (epi == reax::kEpiSwiglu) return p.mode == 1 ? kSwigluBf16 : (p.kb_f16 > 0 ? kSwigluI8F : kSwigluI8);
    return p.mode == 1 ? kPlainBf16 : (p.kb_f16 > 0 ? kPlainI8F : kPlainI8);
}

// pipeline stages + weight-major output staging + SiLU table + 1 KiB alignment slack + staged column
// scales/biases (2 x 2 x 256 floats) + barriers
constexpr size_t tc_smem_bytes() {
    return static_cast<size_t>(kStages) * reax::kStageBytes + reax::kOutStageBytes + reax::kSiluTabBytes + 1024 +
           4096 + 512;
}

// Current device, its SM count, and a check that it is sm_100; sets kernel attributes once.
int current_device(int* dev_out, DeviceInfo** info_out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
    if (dev < 0 || dev >= kMaxDevices) return fail(REAX_ERR_DEVICE, "device ordinal %d out of range", dev);
    std::lock_guard<std::mutex> lock(g_dev_mutex);
    DeviceInfo& d = g_dev[dev];
    if (!d.ready) {
        if ((e = cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess)
            return cuda_fail(e, "cudaDeviceGetAttribute(SM count)");
        if ((e = cudaDeviceGetAttribute(&d.major, cudaDevAttrComputeCapabilityMajor, dev)) != cudaSuccess)
            return cuda_fail(e, "cudaDeviceGetAttribute(major)");
        if ((e = cudaDeviceGetAttribute(&d.minor, cudaDevAttrComputeCapabilityMinor, dev)) != cudaSuccess)
            return cuda_fail(e, "cudaDeviceGetAttribute(minor)");
        d.ready = true;
    }
    if (d.major != 10 || d.minor != 0)
        return fail(REAX_ERR_DEVICE, "device %d is sm_%d%d; this library is built for sm_100a (B200)", dev, d.major,
                    d.minor);
    if (!d.smem_set) {
        const int bytes = static_cast<int>(tc_smem_bytes());
        for (int v = 0; v < kVariants; ++v)
            if ((e = cudaFuncSetAttribute(tc_kernel_ptr(v), cudaFuncAttributeMaxDynamicSharedMemorySize, bytes)) !=
                cudaSuccess)
                return cuda_fail(e, "cudaFuncSetAttribute(tcgen05 kernel smem)");
        // The kernels move registers from the control warps to the epilogue warps (setmaxnreg): refuse
        // to launch a build whose register count cannot cover the split, since the grow would never return.
        for (int v = 0; v < kVariants; ++v) {
            cudaFuncAttributes fa{};
            if ((e = cudaFuncGetAttributes(&fa, tc_kernel_ptr(v))) != cudaSuccess)
                return cuda_fail(e, "cudaFuncGetAttributes(tcgen05 kernel)");
            const int warps = reax::kCtlWarps + kEpiWarps;
            if (fa.numRegs < reax::kCtlRegs || fa.numRegs > reax::kEpiRegs ||
                fa.numRegs * warps < reax::kCtlRegs * reax::kCtlWarps + reax::kEpiRegs * kEpiWarps)
                return fail(REAX_ERR_DEVICE, "tcgen05 kernel variant %d compiled to %d registers per thread, which "
                            "cannot cover the %d/%d register split", v, fa.numRegs, reax::kCtlRegs, reax::kEpiRegs);
        }
        // A persistent grid of CTA pairs must fit in one wave: not every GPC may host clusters of two on all
        // its SMs, so ask how many pairs can be resident rather than assuming SMs / 2.
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(2 * (d.sms / 2), 1, 1);
        cfg.blockDim = dim3(reax::kCtlThreads + 32 * kEpiWarps, 1, 1);
        cfg.dynamicSmemBytes = tc_smem_bytes();
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = 2;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        int clusters = 0;
        if ((e = cudaOccupancyMaxActiveClusters(&clusters, tc_kernel_ptr(kPairI8), &cfg)) != cudaSuccess)
            return cuda_fail(e, "cudaOccupancyMaxActiveClusters(pair GEMM)");
        d.pair_clusters = clusters;
        d.smem_set = true;
    }
    *dev_out = dev;
    *info_out = &d;
    return REAX_OK;
}

// ------------------------------------------------------------------------------------------ per-stream SM share
// A caller that runs several lanes at once (streams whose launches overlap) can give each lane's GEMMs a
// share of the SMs (reax_set_stream_sms): the planner then sizes tiles and grids for that many SMs, so the
// lanes' persistent grids sit side by side instead of queueing for the whole GPU.
constexpr int kMaxStreamShares = 64;
struct StreamShare {
    void* stream;
    int sms;
};
StreamShare g_shares[kMaxStreamShares];
int g_n_shares = 0;
std::mutex g_share_mutex;

// SMs the GEMM plans of `stream` may use on a device of `sms` SMs, for a launch of M token rows.  The share
// applies to weight-streaming (decode) launches of at most kSwapMaxRows rows, which are HBM- and latency-
// bound and gain from running beside the other lane; larger launches are compute-bound and plan for the
// whole GPU.
int stream_sms(void* stream, int sms, int M) {
    if (M > reax::kSwapMaxTok) return sms;
    std::lock_guard<std::mutex> lock(g_share_mutex);
    for (int i = 0; i < g_n_shares; ++i)
        if (g_shares[i].stream == stream) return std::min(sms, g_shares[i].sms);
    return sms;
}

// ------------------------------------------------------------------------------------------------ tensor maps
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;
cudaError_t g_encode_status = cudaSuccess;

int get_encoder(PFN_cuTensorMapEncodeTiled_v12000* fn) {
    std::call_once(g_encode_once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        g_encode_status = cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q);
        if (g_encode_status == cudaSuccess && q == cudaDriverEntryPointSuccess)
            g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    if (g_encode == nullptr) {
        if (g_encode_status != cudaSuccess) return cuda_fail(g_encode_status, "cudaGetDriverEntryPointByVersion");
        return fail(REAX_ERR_CUDA, "cuTensorMapEncodeTiled not available from the driver");
    }
    *fn = g_encode;
    return REAX_OK;
}

// 2-D map of a row-major [rows, inner] tensor, box = 128 bytes of the inner dimension x box_rows rows,
// 128-byte swizzle, zero fill out of bounds.
int make_map(CUtensorMap* map, CUtensorMapDataType dt, size_t elem, const void* base, uint64_t inner, uint64_t rows,
             uint64_t row_stride_elems, uint32_t box_rows = 128) {
    PFN_cuTensorMapEncodeTiled_v12000 enc;
    int rc = get_encoder(&enc);
    if (rc != REAX_OK) return rc;
    cuuint64_t dims[2] = {inner, rows};
    cuuint64_t strides[1] = {row_stride_elems * elem};
    cuuint32_t box[2] = {static_cast<cuuint32_t>(reax::kRowBytes / elem), box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                     CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
        return fail(REAX_ERR_INVALID, "cuTensorMapEncodeTiled failed (%d) for a [%llu, %llu] tensor", static_cast<int>(r),
                    static_cast<unsigned long long>(rows), static_cast<unsigned long long>(inner));
    return REAX_OK;
}

// Maps of weight-major INT8 tiles with stages of kk K blocks (TcParams::kk): the weights [2H, KL] as
// [KL / 128 K blocks][2 halves][H rows][128 bytes], box kk x 2 x box_rows x 128 bytes, so that one copy
// lands, per K block, the tile's box_rows gate rows and then the matching up rows; the activation codes
// [M, KL] as [K blocks][M rows][128 bytes], box kk x n_tok x 128 bytes.  Rows past H or M read as zeros.
int make_multi_maps(CUtensorMap* a_map, CUtensorMap* w_map, const void* A, const void* W, uint64_t KL, uint64_t M,
                    uint64_t H, uint32_t n_tok, uint32_t box_rows, uint32_t kk) {
    PFN_cuTensorMapEncodeTiled_v12000 enc;
    int rc = get_encoder(&enc);
    if (rc != REAX_OK) return rc;
    const cuuint32_t estr[4] = {1, 1, 1, 1};
    {
        cuuint64_t dims[4] = {static_cast<cuuint64_t>(reax::kRowBytes), H, 2, KL / reax::kRowBytes};
        cuuint64_t strides[3] = {KL, H * KL, static_cast<cuuint64_t>(reax::kRowBytes)};
        cuuint32_t box[4] = {static_cast<cuuint32_t>(reax::kRowBytes), box_rows, 2, kk};
        CUresult r = enc(w_map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, const_cast<void*>(W), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (r != CUDA_SUCCESS)
            return fail(REAX_ERR_INVALID, "cuTensorMapEncodeTiled failed (%d) for the [%llu, %llu] weight stages",
                        static_cast<int>(r), static_cast<unsigned long long>(2 * H), static_cast<unsigned long long>(KL));
    }
    {
        cuuint64_t dims[3] = {static_cast<cuuint64_t>(reax::kRowBytes), M, KL / reax::kRowBytes};
        cuuint64_t strides[2] = {KL, static_cast<cuuint64_t>(reax::kRowBytes)};
        cuuint32_t box[3] = {static_cast<cuuint32_t>(reax::kRowBytes), n_tok, kk};
        CUresult r = enc(a_map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(A), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (r != CUDA_SUCCESS)
            return fail(REAX_ERR_INVALID, "cuTensorMapEncodeTiled failed (%d) for the [%llu, %llu] activation stages",
                        static_cast<int>(r), static_cast<unsigned long long>(M), static_cast<unsigned long long>(KL));
    }
    return REAX_OK;
}

// Maps of weight-major grouped-projection tiles with stages of kk K blocks: the weights [N, KT] (KT = P * G
// codes per row) as [KT / 128 K blocks][N rows][128 bytes], box kk x box_rows x 128 bytes, and the activation
// codes [M, KT] as [K blocks][M rows][128 bytes], box kk x n_tok x 128 bytes.
int make_plain_multi_maps(CUtensorMap* a_map, CUtensorMap* w_map, const void* A, const void* W, uint64_t KT, uint64_t M,
                          uint64_t N, uint32_t n_tok, uint32_t box_rows, uint32_t kk) {
    PFN_cuTensorMapEncodeTiled_v12000 enc;
    int rc = get_encoder(&enc);
    if (rc != REAX_OK) return rc;
    const cuuint32_t estr[3] = {1, 1, 1};
    const void* bases[2] = {W, A};
    const uint64_t rows[2] = {N, M};
    const uint32_t boxes[2] = {box_rows, n_tok};
    CUtensorMap* maps[2] = {w_map, a_map};
    for (int i = 0; i < 2; ++i) {
        cuuint64_t dims[3] = {static_cast<cuuint64_t>(reax::kRowBytes), rows[i], KT / reax::kRowBytes};
        cuuint64_t strides[2] = {KT, static_cast<cuuint64_t>(reax::kRowBytes)};
        cuuint32_t box[3] = {static_cast<cuuint32_t>(reax::kRowBytes), boxes[i], kk};
        CUresult r = enc(maps[i], CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(bases[i]), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (r != CUDA_SUCCESS)
            return fail(REAX_ERR_INVALID, "cuTensorMapEncodeTiled failed (%d) for the [%llu, %llu] grouped stages",
                        static_cast<int>(r), static_cast<unsigned long long>(rows[i]), static_cast<unsigned long long>(KT));
    }
    return REAX_OK;
}

// Map of a bf16 output [rows, cols] with row stride ld (elements) for TMA stores of 32 x 32 boxes with the
// 64-byte swizzle (the epilogue's shared-memory layout).
int make_out_map(CUtensorMap* map, const void* base, uint64_t cols, uint64_t rows, uint64_t ld) {
    PFN_cuTensorMapEncodeTiled_v12000 enc;
    int rc = get_encoder(&enc);
    if (rc != REAX_OK) return rc;
    cuuint64_t dims[2] = {cols, rows};
    cuuint64_t strides[1] = {ld * 2};
    cuuint32_t box[2] = {32, 32};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
        return fail(REAX_ERR_INVALID, "cuTensorMapEncodeTiled failed (%d) for the [%llu, %llu] output", static_cast<int>(r),
                    static_cast<unsigned long long>(rows), static_cast<unsigned long long>(cols));
    return REAX_OK;
}

// ------------------------------------------------------------------------------------------------- workspace
struct Workspace {
    unsigned* status;
    int* counters;
    int* partials;
};

size_t workspace_bytes_for(int sms) {
    const size_t counters = ((static_cast<size_t>(2 * sms) * sizeof(int)) + 255) / 256 * 256;
    return kStatusBytes + counters + static_cast<size_t>(sms) * 2 * reax::kSlotInts * sizeof(int);
}

int carve_workspace(void* ws, size_t bytes, int sms, Workspace* w) {
    if (ws == nullptr) return fail(REAX_ERR_WORKSPACE, "workspace is NULL");
    if (!aligned(ws, 256)) return fail(REAX_ERR_ALIGN, "workspace must be 256-byte aligned");
    const size_t need = workspace_bytes_for(sms);
    if (bytes < need) return fail(REAX_ERR_WORKSPACE, "workspace has %zu bytes, %zu needed", bytes, need);
    uint8_t* b = static_cast<uint8_t*>(ws);
    w->status = reinterpret_cast<unsigned*>(b);
    w->counters = reinterpret_cast<int*>(b + kStatusBytes);
    const size_t counters = ((static_cast<size_t>(2 * sms) * sizeof(int)) + 255) / 256 * 256;
    w->partials = reinterpret_cast<int*>(b + kStatusBytes + counters);
    return REAX_OK;
}

// ----------------------------------------------------------------------------------------------- tcgen05 plan
// Tiles are dealt whole while at least one full wave remains beyond them; the rest (between one and
// two waves of tiles, or every tile when there are fewer tiles than SMs) is split by K blocks.
void plan_schedule(reax::TcParams& p, int sms, bool allow_split, int* grid) {
    const int KB = p.kb_int + p.kb_f16;
    const int T = p.tiles;
    if (!allow_split || T % sms == 0 || KB < 2) {
        p.dp_tiles = T;
        p.sk_iters = 0;
        *grid = T < sms ? T : sms;
        return;
    }
    p.dp_tiles = T > sms ? (T / sms - 1) * sms : 0;
    p.sk_iters = static_cast<long long>(T - p.dp_tiles) * KB;
    if (p.sk_iters * (sms + 1) >= (1LL << 31)) {
        // the kernel's stream-K range arithmetic is 32-bit: deal every tile whole instead
        p.dp_tiles = T;
        p.sk_iters = 0;
        *grid = T < sms ? T : sms;
        return;
    }
    // Every CTA's K range covers at least two K blocks and at least ceil(KB / kMaxContrib) of them, so a
    // split tile has at most kMaxContrib + 1 contributors (the finisher gathers kMaxContrib partials).
    long long g = sms;
    const long long min_len = std::max<long long>(2, (KB + reax::kMaxContrib - 1) / reax::kMaxContrib);
    if (p.sk_iters / min_len < g) g = std::max<long long>(1, p.sk_iters / min_len);
    *grid = static_cast<int>(g);
}

// Weight-major pipeline: stages of [gate box | up box | activation box] (each 128 bytes wide, the weight
// boxes rounded up to whole 8-row swizzle atoms), as many as fit the kStages x kStageBytes pool (at most
// kMaxStages).  The M = 128 MMAs read 128 rows from each weight box, so the last stage's up box keeps
// 16 KiB of the pool behind it.
// Whole INT8 weight-major tiles whose K-block slab (the gate then the up rows of a SwiGLU tile, or a grouped
// projection tile's rows) has at most 128 rows stream kk > 1 K blocks per stage (TcParams::kk) and multiply
// each slab with one M = 128 MMA: the largest kk in {8, 4, 2} whose stage of kk x [slab | activation] rows
// leaves at least two stages in the pool; 1 otherwise.
constexpr int kFusedMinRows = 24;
int multi_kk(int slab_rows, int n_tok, int* stage_bytes, int* stages) {
    const int pool = kStages * reax::kStageBytes;
    if (slab_rows > reax::kBM) return 1;
    for (int kk = 8; kk >= 2; kk /= 2) {
        const int bytes = ((kk * (slab_rows + n_tok) * reax::kRowBytes) + 1023) & ~1023;
        // the M = 128 MMAs read 128 rows from each slab: past the last stage's last slab they read at most
        // 16 KiB beyond the pool, inside the output staging region that follows it
        const int n = std::min(reax::kMaxStages, pool / bytes);
        if (n >= 2) {
            if (stage_bytes) *stage_bytes = bytes;
            if (stages) *stages = n;
            return kk;
        }
    }
    return 1;
}

void set_swap_pipeline(reax::TcParams& p, bool multi_ok) {
    const int r8 = (p.tile_rows + 7) & ~7;
    p.kk = multi_ok ? multi_kk(2 * r8, p.n_tok, &p.stage_bytes, &p.stages) : 1;
    if (p.kk > 1) {
        p.tile_rows8 = r8;
        p.m64 = 2 * r8 <= 64 ? 1 : 0;
        return;
    }
    const int bytes = (((2 * r8 + p.n_tok) * reax::kRowBytes) + 1023) & ~1023;
    const int pool = kStages * reax::kStageBytes;
    int stages = (pool - r8 * reax::kRowBytes - reax::kBM * reax::kRowBytes) / bytes + 1;
    if (stages > reax::kMaxStages) stages = reax::kMaxStages;
    p.tile_rows8 = r8;
    p.stage_bytes = bytes;
    p.stages = stages;
}

// Gate rows per few-token tile (R <= 128) and whether the plan splits tiles by K.
// - Large H: whole tiles.  128-row tiles unless they leave a partial wave of at least half the SMs;
//   then an even share R = ceil(H / (waves * SMs)) fills whole waves.  The TMA box covers R weight rows,
//   the MMA still computes 128 (rows past R are never stored), and the weight bytes read stay the same.
// - Small H (fewer than half a wave of 128-row tiles): R = ceil(H * s / SMs) rows, so about SMs / s
//   tiles, each split by K over about s CTAs.  s in {1, 2, 4, 8} minimises the estimated launch time:
//   a CTA spends about kKBlockNs per K block whatever its rows, the weights stream at about
//   kHbmBytesPerNs, and a split adds the exchange of int32 partials, kSplitNs[s] + kSplitTokNs[s] per
//   token column of the tile (the finisher gathers s - 1 partials of 2 x 128 x n_tok words).  The
//   constants are fitted to launches timed on B200 at K = 4096, H = 1792 and 3584, n_tok = 16 .. 64.
int tile_rows_for(int H, int K_blocks, int n_tok, int sms, bool can_split, bool multi, bool* split) {
    *split = false;
    const int t128 = (H + 127) / 128;
    if (t128 % sms == 0) return 128;
    if (2 * t128 >= sms) {
        const int waves = (t128 + sms - 1) / sms;
        return (H + waves * sms - 1) / (waves * sms);
    }
    // A CTA's time per K block, measured on B200: about 470 ns with one-K-block stages, whose eight M = 128
    // MMAs take about 340 ns and whose three copies as long; whole tiles of up to 64 gate rows with stages of
    // kk K blocks (multi_kk: two copies per stage, four MMAs per K block) about 230 ns.
    constexpr double kKBlockNs = 470.0, kHbmBytesPerNs = 6400.0;
    auto kblock_ns = [&](int r, int s) {
        const bool fused = multi && s == 1 && multi_kk(2 * ((r + 7) & ~7), n_tok, nullptr, nullptr) > 1;
        return fused ? 230.0 : kKBlockNs;
    };
    constexpr double kSplitNs[4] = {0.0, 2860.0, 2930.0, 5920.0};
    constexpr double kSplitTokNs[4] = {0.0, 40.0, 57.0, 136.0};
    const double hbm_ns = 2.0 * H * K_blocks * 128.0 / kHbmBytesPerNs;
    int best_r = 128;
    double best = 1e30;
    for (int i = 0, s = 1; s <= 8; ++i, s *= 2) {
        if (s > 1 && !can_split) break;
        int r = (H * s + sms - 1) / sms;
        if (r > 128) break;
        // whole tiles with kk-block stages cost about the same per CTA from 1 to 64 gate rows, and
        // launches of tiles below kFusedMinRows rows measured slower on B200 (more, smaller copies): at
        // least that many rows per tile, on fewer CTAs
        if (s == 1 && multi && r < kFusedMinRows && multi_kk(2 * kFusedMinRows, n_tok, nullptr, nullptr) > 1)
            r = std::min(H, kFusedMinRows);
        const int tiles = (H + r - 1) / r;
        const double per_cta = static_cast<double>(tiles) * K_blocks / std::min(sms, tiles * s);
        const double t = std::max(per_cta * kblock_ns(r, s), hbm_ns) + kSplitNs[i] + kSplitTokNs[i] * n_tok;
        if (t < best) {
            best = t;
            best_r = r;
            *split = s > 1;
        }
    }
    return best_r;
}

// Tile plan of a SwiGLU gate/up launch: orientation, gate rows per tile, activation box rows.  Few
// tokens take weight-major tiles (the weights as the MMA's A operand; measured faster on B200 than
// token-major tiles of the same rows) unless BF16 outlier columns need token-major tiles; either way
// with balanced gate rows and an activation box of round16(M) rows.  Returns whether the tiles are
// weight-major; *split says whether the plan may split tiles by K.
bool plan_gate_up_tiles(reax::TcParams& p, int M, int H, int K_blocks, bool weight_major_ok, bool can_split, int sms,
                        bool multi_ok, bool* split) {
    const bool few = M <= kSwapMaxRows;
    const bool swap = weight_major_ok && few;
    p.n_tok = swap ? ((M + 15) / 16) * 16 : 0;
    *split = can_split;
    p.tile_rows = 128;
    if (few) p.tile_rows = tile_rows_for(H, K_blocks, ((M + 15) / 16) * 16, sms, can_split, swap && multi_ok, split);
    p.tile_rows8 = (p.tile_rows + 7) & ~7;
    p.a_rows = M < reax::kBM ? ((M + 15) / 16) * 16 : reax::kBM;
    if (swap) set_swap_pipeline(p, multi_ok && !*split);   // kk-block stages only for whole tiles
    // out 16-byte aligned and ldo % 8 == 0 (checked by the callers): 128-row weight-major tiles store
    // through shared memory in 16-byte pieces; balanced weight-major tiles store their columns directly
    p.out_vec16 = p.tile_rows == 128 ? 1 : 0;
    return swap;
}

int launch_tc(int epi, const reax::TcParams& p, int grid, cudaStream_t stream) {
    // Plain-epilogue plans split tiles by K only for INT8 grouped tiles without BF16 columns (the float32
    // mixed-origin partials and the BF16-column association are never split).
    if (epi == reax::kEpiPlain && p.sk_iters > 0 && (p.mode != 0 || p.kb_f16 > 0))
        return fail(REAX_ERR_INVALID, "internal: this plain-epilogue plan must not split tiles by K");
    if (p.kk > 1 && (p.sk_iters > 0 || (epi == reax::kEpiSwiglu ? 2 : 1) * p.tile_rows8 > reax::kBM || p.n_tok == 0))
        return fail(REAX_ERR_INVALID, "internal: K-block stages need whole weight-major tiles of at most %d weight rows",
                    reax::kBM);
    if (p.n_tok > 0 && epi == reax::kEpiPlain && p.kk < 2)
        return fail(REAX_ERR_INVALID, "internal: weight-major grouped tiles need K-block stages");
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid, 1, 1);
    cfg.blockDim = dim3(reax::kCtlThreads + 32 * kEpiWarps, 1, 1);
    cfg.dynamicSmemBytes = tc_smem_bytes();
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (p.cta_shift == 1) {   // CTA pairs: clusters of two
        attr[1].id = cudaLaunchAttributeClusterDimension;
        attr[1].val.clusterDim.x = 2;
        attr[1].val.clusterDim.y = 1;
        attr[1].val.clusterDim.z = 1;
        cfg.numAttrs = 2;
    }
    void* args[1] = {const_cast<reax::TcParams*>(&p)};
    cudaError_t e = cudaLaunchKernelExC(&cfg, tc_kernel_ptr(variant_of(epi, p)), args);
    if (e != cudaSuccess) return cuda_fail(e, "tcgen05 GEMM launch");
    return REAX_OK;
}

void init_params(reax::TcParams& p) {
    std::memset(&p, 0, sizeof(p));
    p.group_m = 16;
    p.acc_bufs = 2;
    p.timeout_ns = g_timeout_ns;
    p.parts = 1;
    p.tile_rows = 128;
    p.tile_rows8 = 128;
    p.a_rows = 128;
    p.kk = 1;
}

// Plain launch (no attributes) whose error comes from the launch call itself, so no sticky error
// state of unrelated work is read or reset.
template <typename... KArgs, typename... Args>
int launch_plain(const char* what, void (*kernel)(KArgs...), dim3 grid, dim3 block, cudaStream_t stream,
                 Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = 0;
    cfg.stream = stream;
    cfg.attrs = nullptr;
    cfg.numAttrs = 0;
    cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
    if (e != cudaSuccess) return cuda_fail(e, what);
    return REAX_OK;
}

// Launch with programmatic stream serialization: the kernel may be scheduled while its predecessor on
// the stream still runs, once that predecessor signals griddepcontrol.launch_dependents.  Only for
// kernels that execute griddepcontrol.wait before their first memory access.
template <typename... KArgs, typename... Args>
int launch_dependent(const char* what, void (*kernel)(KArgs...), dim3 grid, dim3 block, cudaStream_t stream,
                     Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = 0;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
    if (e != cudaSuccess) return cuda_fail(e, what);
    return REAX_OK;
}

int elementwise_grid(long long work, int sms) {
    long long g = (work + 255) / 256;
    const long long cap = static_cast<long long>(sms) * 16;
    if (g > cap) g = cap;
    if (g < 1) g = 1;
    return static_cast<int>(g);
}

// ------------------------------------------------------------------------ allocation-free variant
// Scratch of reax_gate_up_i8_noalloc: one array per GPU that loads this library, held until exit.
// It keeps the layout of a caller workspace (status word, split counters, split partials) sized for
// kNoAllocMaxCtas CTAs; larger grids are planned down to that count.
constexpr size_t kNoAllocScratchBytes = 16u << 20;   // 16 MiB
constexpr int kNoAllocMaxCtas = 63;                  // split partials of 63 CTAs (2 x 128 KiB each) fit
static_assert(kStatusBytes + 512 + static_cast<size_t>(kNoAllocMaxCtas) * 2 * reax::kSlotInts * sizeof(int) <=
                  kNoAllocScratchBytes,
              "no-alloc scratch too small for its CTA cap");
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

void* g_noalloc_addr[kMaxDevices] = {};
std::mutex g_noalloc_mutex;

// Device address of the scratch array on `dev` (the current device); resolved once per device.
// In host code g_noalloc_scratch only names a host-side stand-in, so the address must come from
// cudaGetSymbolAddress with that device current.
int noalloc_scratch(int dev, void** out) {
    std::lock_guard<std::mutex> lock(g_noalloc_mutex);
    if (g_noalloc_addr[dev] == nullptr) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(no-alloc scratch)");
        g_noalloc_addr[dev] = p;
    }
    *out = g_noalloc_addr[dev];
    return REAX_OK;
}

// Argument checks shared by the INT8 gate/up entry points (the reference's asserts, reaxv2/gate_up.py:14,
// plus the kernels' alignment needs).  *empty: M == 0, nothing to launch.
int check_gate_up_args(const char* who, const int8_t* A, const int8_t* W, const void* AH, const void* WH,
                       const float* sa, const float* sw, const float* bias, const void* out, int M, int N2, int KL,
                       int KH, int ldo, bool* empty) {
    *empty = false;
    if (M < 0 || N2 <= 0 || KL < 0 || KH < 0 || KL + KH == 0)
        return fail(REAX_ERR_INVALID, "%s: bad sizes M=%d N2=%d KL=%d KH=%d", who, M, N2, KL, KH);
    if (KL % 128 != 0 || KH % 64 != 0 || N2 % 256 != 0)
        return fail(REAX_ERR_INVALID, "%s: needs KL %% 128 == 0, KH %% 64 == 0, N2 %% 256 == 0 (KL=%d KH=%d N2=%d)",
                    who, KL, KH, N2);
    if (ldo < N2 / 2 || ldo % 8 != 0) return fail(REAX_ERR_INVALID, "%s: ldo=%d (needs >= N2/2, %% 8 == 0)", who, ldo);
    if (KL == 0) return fail(REAX_ERR_INVALID, "%s: KL must be > 0 (the INT8 part of the bank is empty)", who);
    if (M == 0) {
        *empty = true;
        return REAX_OK;
    }
    if (!out || !sw || !bias || !A || !W || !sa || (KH && (!AH || !WH)))
        return fail(REAX_ERR_INVALID, "%s: NULL pointer argument", who);
    if (!aligned(A, 16) || !aligned(W, 16) || !aligned(AH, 16) || !aligned(WH, 16) || !aligned(sw, 16) ||
        !aligned(bias, 16) || !aligned(out, 16))
        return fail(REAX_ERR_ALIGN, "%s: operands, sw, bias and out must be 16-byte aligned", who);
    return REAX_OK;
}

// CTA-pair tiles: 256 token rows per pair (128 per CTA), 128 gate + 128 up rows, a six-stage ring of
// [half of B | A box] stages of 32 KiB.
void set_pair_tiles(reax::TcParams& p) {
    p.cta_shift = 1;
    p.tile_rows = 128;
    p.tile_rows8 = 128;
    p.a_rows = reax::kBM;
    p.stages = kPairStages;
    p.stage_bytes = 2 * reax::kBM * reax::kRowBytes;
    p.out_vec16 = 0;
}

// Tile plan, tensor maps and operands of an INT8 gate/up launch (everything but the scratch pointers,
// early_b and the schedule), shared by the workspace and the allocation-free entry points so that both
// run the same kernel on the same plan.  *split_ok: whether the plan may split tiles by K.
int fill_gate_up_params(reax::TcParams& p, int sms, bool pair_ok, const int8_t* A, const int8_t* W, const void* AH,
                        const void* WH, const float* sa, const float* sw, const float* bias, void* out, int M, int N2,
                        int KL, int KH, int ldo, bool* split_ok) {
    init_params(p);
    // many tokens and no BF16 columns: CTA-pair tiles of 256 token rows (whole tiles, dealt to pairs)
    const bool pair = KH == 0 && M >= kPairMinRows && sms >= 2 && pair_ok;
    // few tokens and no BF16 columns: weight-major tiles, the activation box covers n_tok token rows
    const bool swap = !pair && plan_gate_up_tiles(p, M, N2 / 2, KL / 128 + KH / 64, KH == 0, KH == 0, sms, true, split_ok);
    if (pair) {
        set_pair_tiles(p);
        *split_ok = false;
    }
    int rc;
    if (swap && p.kk > 1) {
        if ((rc = make_multi_maps(&p.tm_a, &p.tm_b, A, W, KL, M, N2 / 2, p.n_tok, p.tile_rows8, p.kk)) != REAX_OK) return rc;
    } else {
        if ((rc = make_map(&p.tm_a, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, A, KL, M, KL, swap ? p.n_tok : p.a_rows)) != REAX_OK)
            return rc;
        if ((rc = make_map(&p.tm_b, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, W, KL, N2, KL, p.tile_rows)) != REAX_OK) return rc;
    }
    if (KH) {
        if ((rc = make_map(&p.tm_ah, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, AH, KH, M, KH, p.a_rows)) != REAX_OK) return rc;
        if ((rc = make_map(&p.tm_bh, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, WH, KH, N2, KH, p.tile_rows)) != REAX_OK)
            return rc;
    } else {
        p.tm_ah = p.tm_a;
        p.tm_bh = p.tm_b;
    }
    // token-major tiles of 128 gate rows store their output through shared memory with TMA, one box of 32
    // rows x 32 columns per warp and chunk (16-byte aligned; a box never reaches the next tile's columns).
    // Balanced tiles of few tokens with BF16 columns keep the per-thread stores.
    if (!swap && p.tile_rows == 128) {
        if ((rc = make_out_map(&p.tm_out, out, N2 / 2, M, ldo)) != REAX_OK) return rc;
        p.out_tma = 1;
    }
    p.sa = sa;
    p.sw = sw;
    p.bias = bias;
    p.out = static_cast<__nv_bfloat16*>(out);
    p.M = M;
    p.H = N2 / 2;
    p.ldo = ldo;
    p.kb_int = KL / 128;
    p.kb_f16 = KH / 64;
    const int unit_rows = reax::kBM << p.cta_shift;   // token rows per tile: 128, or 256 for a pair
    p.m_tiles = (M + unit_rows - 1) / unit_rows;
    p.n_tiles = (N2 / 2 + p.tile_rows - 1) / p.tile_rows;
    p.tiles = p.m_tiles * p.n_tiles;
    p.mode = 0;
    p.acc_bufs = KH ? 1 : 2;
    p.evict_first_b = p.m_tiles == 1 ? 1 : 0;
    return REAX_OK;
}

// Whole tiles dealt to CTA pairs: grid = two CTAs per pair, at most one pair per two SMs of the share and
// no more pairs than can be resident at once (`resident`).
void plan_pairs(reax::TcParams& p, int sms, int resident, int* grid) {
    p.dp_tiles = p.tiles;
    p.sk_iters = 0;
    *grid = 2 * std::max(1, std::min(p.tiles, std::min(sms / 2, resident)));
}

// reax_gate_up_i8 with the option of requesting the first weight tiles before the dependency wait.
int gate_up_i8_launch(const int8_t* A, const int8_t* W, const void* AH, const void* WH, const float* sa, const float* sw,
                      const float* bias, void* out, int M, int N2, int KL, int KH, int ldo, void* workspace,
                      size_t workspace_bytes, void* stream, int early_b) {
    bool empty = false;
    int rc = check_gate_up_args("gate_up_i8", A, W, AH, WH, sa, sw, bias, out, M, N2, KL, KH, ldo, &empty);
    if (rc != REAX_OK || empty) return rc;
    int dev;
    DeviceInfo* info;
    if ((rc = current_device(&dev, &info)) != REAX_OK) return rc;
    Workspace ws;
    if ((rc = carve_workspace(workspace, workspace_bytes, info->sms, &ws)) != REAX_OK) return rc;
    reax::TcParams p;
    bool split_ok = false;
    const int sms = stream_sms(stream, info->sms, M);
    if ((rc = fill_gate_up_params(p, sms, info->pair_clusters > 0, A, W, AH, WH, sa, sw, bias, out, M, N2, KL, KH, ldo, &split_ok)) != REAX_OK)
        return rc;
    p.ws_partials = ws.partials;
    p.ws_counters = ws.counters;
    p.status = ws.status;
    p.early_b = early_b;
    int grid = 0;
    if (p.cta_shift) plan_pairs(p, sms, info->pair_clusters, &grid);
    else plan_schedule(p, sms, split_ok, &grid);
    return launch_tc(reax::kEpiSwiglu, p, grid, static_cast<cudaStream_t>(stream));
}

template <int V>
int launch_dense(const void* x, int8_t* low, float* scales, int M, int K, int sms, cudaStream_t s) {
    static int per_sm[kMaxDevices] = {};   // resident CTAs per SM, from the occupancy calculator, per device
    int dev = 0;
    cudaGetDevice(&dev);
    if (per_sm[dev] == 0) {
        int n = 0;
        cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, reax::quant_rows_dense_kernel<kQuantDivision, V>,
                                                                       reax::kDenseThreads, 0);
        if (e != cudaSuccess) return cuda_fail(e, "cudaOccupancyMaxActiveBlocksPerMultiprocessor (dense quantizer)");
        per_sm[dev] = std::max(1, n);
    }
    const int grid = std::min(M, sms * per_sm[dev]);
    return launch_dependent("quant_rows (dense) launch", reax::quant_rows_dense_kernel<kQuantDivision, V>, dim3(grid),
                            dim3(reax::kDenseThreads), s, static_cast<const __nv_bfloat16*>(x), low, scales, M, K);
}

// reax_quant_rows for a dense bank (NULL low_columns and smoothing): every column in order, unit smoothing,
// no centring, no high columns, K a multiple of 1024 up to 8192.
int quant_rows_dense(const void* x, int8_t* low, float* scales, int M, int K, int KL, int KH, int center,
                     void* stream) {
    if (KL != K || KH != 0 || center != 0 || K % 1024 != 0 || K > 8192)
        return fail(REAX_ERR_INVALID,
                    "quant_rows: NULL low_columns and smoothing (a dense bank) need KL == K, KH == 0, no centring and "
                    "K a multiple of 1024 up to 8192 (K=%d KL=%d KH=%d center=%d)", K, KL, KH, center);
    if (!x || !low || !scales) return fail(REAX_ERR_INVALID, "quant_rows: NULL pointer argument");
    if (!aligned(x, 16) || !aligned(low, 8))
        return fail(REAX_ERR_ALIGN, "quant_rows: a dense bank needs x 16-byte and low 8-byte aligned");
    int dev;
    DeviceInfo* info;
    int rc = current_device(&dev, &info);
    if (rc != REAX_OK) return rc;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    switch (K / 1024) {
        case 1: return launch_dense<1>(x, low, scales, M, K, info->sms, s);
        case 2: return launch_dense<2>(x, low, scales, M, K, info->sms, s);
        case 3: return launch_dense<3>(x, low, scales, M, K, info->sms, s);
        case 4: return launch_dense<4>(x, low, scales, M, K, info->sms, s);
        case 5: return launch_dense<5>(x, low, scales, M, K, info->sms, s);
        case 6: return launch_dense<6>(x, low, scales, M, K, info->sms, s);
        case 7: return launch_dense<7>(x, low, scales, M, K, info->sms, s);
        default: return launch_dense<8>(x, low, scales, M, K, info->sms, s);
    }
}
}  // namespace

extern "C" {

int reax_version(void) { return kVersion; }

const char* reax_last_error(void) { return g_last_error.c_str(); }

void reax_set_wait_timeout_ns(unsigned long long ns) { g_timeout_ns = ns == 0 ? kDefaultTimeoutNs : ns; }

size_t reax_workspace_bytes(int device) {
    int dev = device;
    if (dev < 0 && cudaGetDevice(&dev) != cudaSuccess) return 0;
    int sms = 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 0;
    return workspace_bytes_for(sms);
}

int reax_quant_rows(const void* x, const int32_t* low_columns, const int32_t* high_columns, const float* smoothing,
                    const float* centers, int8_t* low, void* high, float* scales, int M, int K, int KL, int KH,
                    int center, void* stream) {
    if (M < 0 || K < 0 || KL < 0 || KH < 0 || KL + KH > K)
        return fail(REAX_ERR_INVALID, "quant_rows: bad sizes M=%d K=%d KL=%d KH=%d", M, K, KL, KH);
    if (M == 0) return REAX_OK;
    // NULL low_columns and smoothing with low columns to quantize: a dense bank (low column c is column c,
    // unit smoothing); with KL == 0 the maps are never read and may be NULL
    const bool dense = KL > 0 && low_columns == nullptr && smoothing == nullptr;
    if (dense) return quant_rows_dense(x, low, scales, M, K, KL, KH, center, stream);
    if (!x || !scales || (KL && (!low_columns || !smoothing || !low || (center && !centers))) ||
        (KH && (!high_columns || !high)))
        return fail(REAX_ERR_INVALID, "quant_rows: NULL pointer argument");
    if (!aligned(low_columns, 16) || !aligned(smoothing, 16) || (center && !aligned(centers, 16)))
        return fail(REAX_ERR_ALIGN, "quant_rows: low_columns, smoothing and centers must be 16-byte aligned");
    int dev;
    DeviceInfo* info;
    int rc = current_device(&dev, &info);
    if (rc != REAX_OK) return rc;
    const int aligned_x = (aligned(x, 16) && K % 8 == 0) ? 1 : 0;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    // many rows: persistent CTAs streaming whole rows into a ring of shared-memory buffers by bulk copies,
    // as many rows in flight per SM as the shared memory holds (at most kStreamMaxBufs)
    if (M > kQuantStreamMinRowsPerSm * info->sms && aligned_x) {
        // row buffers that fit, shared out as groups x depth: the most rows in flight, then the most groups
        // (of kStreamGroupWarps warps, at most kStreamMaxGroups)
        int nbuf = reax::kStreamMaxBufs;
        while (nbuf > 0 && reax::quant_stream_smem(K, KL, KH, center, nbuf) > kQuantStreamSmemMax) --nbuf;
        int groups = 0, depth = 0;
        for (int g = 2; g <= reax::kStreamMaxGroups; ++g)
            if (g * (nbuf / g) >= groups * depth) groups = g, depth = nbuf / g;
        if (groups >= 2 && depth >= 1) {
            const size_t smem = reax::quant_stream_smem(K, KL, KH, center, groups * depth);
            if (!info->stream_smem_set) {
                cudaError_t e = cudaFuncSetAttribute(reax::quant_rows_stream_kernel<kQuantDivision>,
                                                     cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                     static_cast<int>(kQuantStreamSmemMax));
                if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(quant_rows_stream_kernel smem)");
                info->stream_smem_set = true;
            }
            cudaLaunchConfig_t cfg = {};
            cfg.gridDim = dim3(static_cast<unsigned>(std::min(M, info->sms)), 1, 1);
            cfg.blockDim = dim3(32 * reax::kStreamGroupWarps * groups, 1, 1);
            cfg.dynamicSmemBytes = smem;
            cfg.stream = s;
            cudaLaunchAttribute attr[1];
            attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
            attr[0].val.programmaticStreamSerializationAllowed = 1;
            cfg.attrs = attr;
            cfg.numAttrs = 1;
            const cudaError_t e = cudaLaunchKernelEx(
                &cfg, reax::quant_rows_stream_kernel<kQuantDivision>, static_cast<const __nv_bfloat16*>(x),
                static_cast<const int*>(low_columns), static_cast<const int*>(high_columns), smoothing, centers, low,
                static_cast<__nv_bfloat16*>(high), scales, M, K, KL, KH, center ? 1 : 0, depth, g_timeout_ns);
            return e == cudaSuccess ? REAX_OK : cuda_fail(e, "quant_rows launch");
        }
    }
    // more rows than four per SM: narrower CTAs (wide enough to hold a row's values up to 8192 columns),
    // more rows in flight on each SM
    if (M > 4 * info->sms && KL <= 32 * reax::kQuantThreadsMany)
        return launch_dependent("quant_rows launch", reax::quant_rows_kernel<kQuantDivision, reax::kQuantThreadsMany>,
                                dim3(M), dim3(reax::kQuantThreadsMany), s, static_cast<const __nv_bfloat16*>(x),
                                static_cast<const int*>(low_columns), static_cast<const int*>(high_columns), smoothing,
                                centers, low, static_cast<__nv_bfloat16*>(high), scales, K, KL, KH, center ? 1 : 0,
                                aligned_x);
    if (M > 4 * info->sms && KL <= 64 * reax::kQuantThreadsMany)
        return launch_dependent("quant_rows launch",
                                reax::quant_rows_kernel<kQuantDivision, 2 * reax::kQuantThreadsMany>, dim3(M),
                                dim3(2 * reax::kQuantThreadsMany), s, static_cast<const __nv_bfloat16*>(x),
                                static_cast<const int*>(low_columns), static_cast<const int*>(high_columns), smoothing,
                                centers, low, static_cast<__nv_bfloat16*>(high), scales, K, KL, KH, center ? 1 : 0,
                                aligned_x);
    return launch_dependent("quant_rows launch", reax::quant_rows_kernel<kQuantDivision, reax::kQuantThreads>, dim3(M),
                            dim3(reax::kQuantThreads), s, static_cast<const __nv_bfloat16*>(x),
                            static_cast<const int*>(low_columns), static_cast<const int*>(high_columns), smoothing,
                            centers, low, static_cast<__nv_bfloat16*>(high), scales, K, KL, KH, center ? 1 : 0,
                            aligned_x);
}

int reax_quant_rotated(const void* x, const float* centers, int8_t* low, float* scales, int M, int K, int chunk,
                       int parts, int group, int block, void* stream) {
    if (M < 0 || K <= 0 || chunk <= 0 || parts < 1 || group <= 0 || block < 2)
        return fail(REAX_ERR_INVALID, "quant_rotated: bad sizes M=%d K=%d chunk=%d parts=%d group=%d block=%d", M, K,
                    chunk, parts, group, block);
    if ((block & (block - 1)) != 0 || group % block != 0 || group > reax::kRotMaxGroup || chunk > group)
        return fail(REAX_ERR_INVALID,
                    "quant_rotated: needs block a power of two dividing group, group <= %d and chunk <= group "
                    "(group=%d block=%d chunk=%d)", reax::kRotMaxGroup, group, block, chunk);
    if (M == 0) return REAX_OK;
    if (!x || !centers || !low || !scales) return fail(REAX_ERR_INVALID, "quant_rotated: NULL pointer argument");
    int dev;
    DeviceInfo* info;
    int rc = current_device(&dev, &info);
    if (rc != REAX_OK) return rc;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(M, parts, 1);
    cfg.stream = static_cast<cudaStream_t>(stream);
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const __nv_bfloat16* xb = static_cast<const __nv_bfloat16*>(x);
    cudaError_t e;
    // Groups of a multiple of 64 columns (every reference shape) keep their values in registers, V
    // consecutive columns per thread.
    int V = 0;
    for (int c : {8, 4, 2})
        if (!V && group % (32 * c) == 0 && group / c <= 1024) V = c;
    if (!V) {
        cfg.blockDim = dim3(reax::kRotThreads, 1, 1);
        cfg.dynamicSmemBytes = static_cast<size_t>(group + 32) * sizeof(float);
        e = cudaLaunchKernelEx(&cfg, reax::quant_rotated_kernel, xb, centers, low, scales, M, K, chunk, parts, group,
                               block);
        return e == cudaSuccess ? REAX_OK : cuda_fail(e, "quant_rotated launch");
    }
    const bool vec = K % V == 0 && chunk % V == 0 && aligned(x, 16) && aligned(centers, 16) &&
                     aligned(low, static_cast<size_t>(V));
    // Many rows of two-column runs (groups of an odd multiple of 64 columns): persistent CTAs of
    // group / (2 R) threads, each walking rows of one part, three runs per thread when the group is a
    // multiple of 192 columns, so that a thread has six values.  Wider runs measured faster with one CTA
    // per (row, part) at every row count.
    if (vec && V == 2) {
        using RowsKernel = void (*)(const __nv_bfloat16*, const float*, int8_t*, float*, int, int, int, int, int, int);
        const int R = (group / 64) % 3 == 0 ? 3 : 1;
        const RowsKernel rk = R == 3 ? reax::quant_rotated_rows_kernel<2, 3> : reax::quant_rotated_rows_kernel<2, 1>;
        const int threads = group / (V * R);
        const size_t smem = static_cast<size_t>(64 + (block > 32 * V ? group : 0)) * sizeof(float);
        int per_sm = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, rk, threads, smem) != cudaSuccess || per_sm < 1)
            per_sm = 1;
        const long long resident = static_cast<long long>(per_sm) * info->sms;
        if (static_cast<long long>(M) * parts >= 2 * resident) {
            cfg.gridDim = dim3(static_cast<unsigned>(std::max<long long>(1, std::min<long long>(M, resident / parts))),
                               parts, 1);
            cfg.blockDim = dim3(threads, 1, 1);
            cfg.dynamicSmemBytes = smem;
            e = cudaLaunchKernelEx(&cfg, rk, xb, centers, low, scales, M, K, chunk, parts, group, block);
            return e == cudaSuccess ? REAX_OK : cuda_fail(e, "quant_rotated launch");
        }
    }
    // Otherwise one CTA of group / V threads per (row, part).
    using LaneKernel = void (*)(const __nv_bfloat16*, const float*, int8_t*, float*, int, int, int, int, int, int,
                                int);
    const LaneKernel lk = V == 8 ? reax::quant_rotated_lanes_kernel<8>
                          : V == 4 ? reax::quant_rotated_lanes_kernel<4>
                                   : reax::quant_rotated_lanes_kernel<2>;
    cfg.blockDim = dim3(group / V, 1, 1);
    cfg.dynamicSmemBytes = static_cast<size_t>(32 + (block > 32 * V ? group : 0)) * sizeof(float);
    e = cudaLaunchKernelEx(&cfg, lk, xb, centers, low, scales, M, K, chunk, parts, group, block, vec ? 1 : 0);
    return e == cudaSuccess ? REAX_OK : cuda_fail(e, "quant_rotated launch");
}

int reax_quant_groups(const void* x, const int32_t* low_columns, const int32_t* high_columns, const float* centers,
                      const float* smoothing, int8_t* low, void* high, float* scales, int M, int K, int G, int HP,
                      int P, void* stream) {
    if (M < 0 || K <= 0 || G < 0 || HP < 0 || P < 1)
        return fail(REAX_ERR_INVALID, "quant_groups: bad sizes M=%d K=%d G=%d HP=%d P=%d", M, K, G, HP, P);
    if (M == 0) return REAX_OK;
    if (!x || !scales || !low_columns || !centers || !smoothing || (G && !low) || (HP && (!high_columns || !high)))
        return fail(REAX_ERR_INVALID, "quant_groups: NULL pointer argument");
    int dev;
    DeviceInfo* info;
    int rc = current_device(&dev, &info);
    if (rc != REAX_OK) return rc;
    return launch_dependent("quant_groups launch", reax::quant_groups_kernel<kQuantDivision>, dim3(M, P), dim3(256),
                        static_cast<cudaStream_t>(stream), static_cast<const __nv_bfloat16*>(x),
                        static_cast<const int*>(low_columns), static_cast<const int*>(high_columns), centers,
                        smoothing, low, static_cast<__nv_bfloat16*>(high), scales, M, K, G, HP, P);
}

int reax_reduce_partials(const void* partials, void* out, long long total, int P, void* stream) {
    if (total < 0 || P < 1) return fail(REAX_ERR_INVALID, "reduce_partials: bad sizes total=%lld P=%d", total, P);
    if (total == 0) return REAX_OK;
    if (!partials || !out) return fail(REAX_ERR_INVALID, "reduce_partials: NULL pointer argument");
    int dev;
    DeviceInfo* info;
    int rc = current_device(&dev, &info);
    if (rc != REAX_OK) return rc;
    const int vec = (aligned(partials, 16) && aligned(out, 16) && total % 8 == 0) ? 1 : 0;
    return launch_plain("reduce_partials launch", reax::fold_partials_kernel,
                        dim3(elementwise_grid((total + 7) / 8, info->sms)), dim3(256), static_cast<cudaStream_t>(stream),
                        static_cast<const __nv_bfloat16*>(partials), static_cast<const int*>(nullptr),
                        static_cast<__nv_bfloat16*>(out), total, 1, P, P, vec);
}

int reax_fold_partials(const void* parts, const int32_t* split, void* out, int M, int N, int P0, int P1,
                       void* stream) {
    if (M < 0 || N <= 0 || P0 < 1 || P1 < 1)
        return fail(REAX_ERR_INVALID, "fold_partials: bad sizes M=%d N=%d P0=%d P1=%d", M, N, P0, P1);
    if (M == 0) return REAX_OK;
    if (!parts || !split || !out) return fail(REAX_ERR_INVALID, "fold_partials: NULL pointer argument");
    int dev;
    DeviceInfo* info;
    int rc = current_device(&dev, &info);
    if (rc != REAX_OK) return rc;
    const long long total = static_cast<long long>(M) * N;
    return launch_plain("fold_partials launch", reax::fold_partials_kernel,
                        dim3(elementwise_grid((total + 7) / 8, info->sms)), dim3(256), static_cast<cudaStream_t>(stream),
                        static_cast<const __nv_bfloat16*>(parts), static_cast<const int*>(split),
                        static_cast<__nv_bfloat16*>(out), total, N, P0, P1,
                        (aligned(parts, 16) && aligned(out, 16) && N % 8 == 0) ? 1 : 0);
}

int reax_silu_mul(const void* g, const void* u, void* out, int rows, int cols, long long g_stride, long long u_stride,
                  void* stream) {
    if (rows < 0 || cols < 0 || g_stride < cols || u_stride < cols)
        return fail(REAX_ERR_INVALID, "silu_mul: bad sizes rows=%d cols=%d", rows, cols);
    if (rows == 0 || cols == 0) return REAX_OK;
    if (!g || !u || !out) return fail(REAX_ERR_INVALID, "silu_mul: NULL pointer argument");
    int dev;
    DeviceInfo* info;
    int rc = current_device(&dev, &info);
    if (rc != REAX_OK) return rc;
    return launch_plain("silu_mul launch", reax::silu_mul_kernel,
                        dim3(elementwise_grid(static_cast<long long>(rows) * cols, info->sms)), dim3(256),
                        static_cast<cudaStream_t>(stream), static_cast<const __nv_bfloat16*>(g),
                        static_cast<const __nv_bfloat16*>(u), static_cast<__nv_bfloat16*>(out), rows, cols, g_stride,
                        u_stride);
}

int reax_silu_table(void* table, void* stream) {
    if (!table) return fail(REAX_ERR_INVALID, "silu_table: NULL table");
    int dev;
    DeviceInfo* info;
    int rc = current_device(&dev, &info);
    if (rc != REAX_OK) return rc;
    return launch_plain("silu_table launch", reax::silu_table_kernel, dim3(256), dim3(256),
                        static_cast<cudaStream_t>(stream), static_cast<__nv_bfloat16*>(table));
}

int reax_gate_up_i8(const int8_t* A, const int8_t* W, const void* AH, const void* WH, const float* sa, const float* sw,
                    const float* bias, void* out, int M, int N2, int KL, int KH, int ldo, void* workspace,
                    size_t workspace_bytes, void* stream) {
    return gate_up_i8_launch(A, W, AH, WH, sa, sw, bias, out, M, N2, KL, KH, ldo, workspace, workspace_bytes, stream, 0);
}

int reax_gate_up_i8_static(const int8_t* A, const int8_t* W, const void* AH, const void* WH, const float* sa,
                           const float* sw, const float* bias, void* out, int M, int N2, int KL, int KH, int ldo,
                           void* workspace, size_t workspace_bytes, void* stream) {
    return gate_up_i8_launch(A, W, AH, WH, sa, sw, bias, out, M, N2, KL, KH, ldo, workspace, workspace_bytes, stream, 1);
}

int reax_project_i8(const void* x, const int32_t* low_columns, const int32_t* high_columns, const float* smoothing,
                    const float* centers, int center, const int8_t* W, const void* WH, const float* sw,
                    const float* bias, int8_t* low, void* high, float* scales, void* out, int M, int K, int KL, int KH,
                    int N2, int ldo, void* workspace, size_t workspace_bytes, void* stream) {
    int rc = reax_quant_rows(x, low_columns, high_columns, smoothing, centers, low, high, scales, M, K, KL, KH, center,
                             stream);
    if (rc != REAX_OK) return rc;
    // The GEMM follows the quantizer on the stream, so it may request its first weight tiles before its
    // dependency wait (early_b).
    return gate_up_i8_launch(low, W, KH ? high : nullptr, KH ? WH : nullptr, scales, sw, bias, out, M, N2, KL, KH, ldo,
                             workspace, workspace_bytes, stream, 1);
}

int reax_gate_up_bf16(const void* x, const void* w, void* out, int M, int N2, int K, int ldo, void* workspace,
                      size_t workspace_bytes, void* stream) {
    if (M < 0 || N2 <= 0 || K <= 0) return fail(REAX_ERR_INVALID, "gate_up_bf16: bad sizes M=%d N2=%d K=%d", M, N2, K);
    if (K % 64 != 0 || N2 % 256 != 0)
        return fail(REAX_ERR_INVALID, "gate_up_bf16: needs K %% 64 == 0 and N2 %% 256 == 0 (K=%d N2=%d)", K, N2);
    if (ldo < N2 / 2 || ldo % 8 != 0) return fail(REAX_ERR_INVALID, "gate_up_bf16: ldo=%d (needs >= N2/2, %% 8 == 0)", ldo);
    if (M == 0) return REAX_OK;
    if (!x || !w || !out) return fail(REAX_ERR_INVALID, "gate_up_bf16: NULL pointer argument");
    if (!aligned(x, 16) || !aligned(w, 16) || !aligned(out, 16))
        return fail(REAX_ERR_ALIGN, "gate_up_bf16: x, w and out must be 16-byte aligned");
    int dev;
    DeviceInfo* info;
    int rc = current_device(&dev, &info);
    if (rc != REAX_OK) return rc;
    Workspace ws;
    if ((rc = carve_workspace(workspace, workspace_bytes, info->sms, &ws)) != REAX_OK) return rc;
    reax::TcParams p;
    init_params(p);
    bool split_ok = false;   // BF16 tiles are never split
    const int sms = stream_sms(stream, info->sms, M);
    // many tokens: CTA-pair tiles of 256 token rows (as the INT8 gate/up), else the single-CTA plans
    const bool pair = M >= kPairMinRows && sms >= 2 && info->pair_clusters > 0;
    const bool swap = !pair && plan_gate_up_tiles(p, M, N2 / 2, K / 64, true, false, sms, false, &split_ok);
    if (pair) set_pair_tiles(p);
    if ((rc = make_map(&p.tm_ah, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, x, K, M, K, swap ? p.n_tok : p.a_rows)) != REAX_OK)
        return rc;
    if ((rc = make_map(&p.tm_bh, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, w, K, N2, K, p.tile_rows)) !=
        REAX_OK)
        return rc;
    p.tm_a = p.tm_ah;
    p.tm_b = p.tm_bh;
    if (!swap && p.tile_rows == 128) {   // token-major tiles of 128 gate rows: output through TMA stores
        if ((rc = make_out_map(&p.tm_out, out, N2 / 2, M, ldo)) != REAX_OK) return rc;
        p.out_tma = 1;
    }
    p.out = static_cast<__nv_bfloat16*>(out);
    p.M = M;
    p.H = N2 / 2;
    p.ldo = ldo;
    p.kb_int = 0;
    p.kb_f16 = K / 64;
    p.m_tiles = (M + (reax::kBM << p.cta_shift) - 1) / (reax::kBM << p.cta_shift);
    p.n_tiles = (N2 / 2 + p.tile_rows - 1) / p.tile_rows;
    p.tiles = p.m_tiles * p.n_tiles;
    p.mode = 1;
    p.acc_bufs = 2;
    p.ws_partials = ws.partials;
    p.ws_counters = ws.counters;
    p.status = ws.status;
    p.evict_first_b = p.m_tiles == 1 ? 1 : 0;
    int grid = 0;
    // float32 partial sums of one tile would round differently from one unsplit accumulation, which
    // would make a row's result depend on the batch it came in: BF16 tiles are never split.
    if (p.cta_shift) plan_pairs(p, sms, info->pair_clusters, &grid);
    else plan_schedule(p, sms, false, &grid);
    return launch_tc(reax::kEpiSwiglu, p, grid, static_cast<cudaStream_t>(stream));
}

int reax_bf16_partials(const void* x, const void* w, const int32_t* split, void* parts, int M, int N, int K, int chunk0,
                       int chunk1, int P0, int P1, void* workspace, size_t workspace_bytes, void* stream) {
    if (M < 0 || N <= 0 || K <= 0 || P0 < 1 || P1 < 1)
        return fail(REAX_ERR_INVALID, "bf16_partials: bad sizes M=%d N=%d K=%d P0=%d P1=%d", M, N, K, P0, P1);
    if (K % 64 != 0 || N % 256 != 0 || (P0 > 1 && (chunk0 <= 0 || chunk0 % 64 != 0)) ||
        (P1 > 1 && (chunk1 <= 0 || chunk1 % 64 != 0)))
        return fail(REAX_ERR_INVALID, "bf16_partials: needs K %% 64 == 0, N %% 256 == 0, chunks multiples of 64");
    if (M == 0) return REAX_OK;
    if (!x || !w || !split || !parts) return fail(REAX_ERR_INVALID, "bf16_partials: NULL pointer argument");
    if (!aligned(x, 16) || !aligned(w, 16) || !aligned(parts, 16))
        return fail(REAX_ERR_ALIGN, "bf16_partials: x, w and parts must be 16-byte aligned");
    int dev;
    DeviceInfo* info;
    int rc = current_device(&dev, &info);
    if (rc != REAX_OK) return rc;
    Workspace ws;
    if ((rc = carve_workspace(workspace, workspace_bytes, info->sms, &ws)) != REAX_OK) return rc;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int KB = K / 64;
    const int ck0 = P0 > 1 ? chunk0 / 64 : KB;
    const int ck1 = P1 > 1 ? chunk1 / 64 : KB;
    const size_t plane = static_cast<size_t>(M) * N * 2;
    // slices whose K range is empty for a plan are zero planes (the kernel skips them)
    for (int sidx = 0; sidx < (P0 > P1 ? P0 : P1); ++sidx) {
        const bool empty0 = sidx < P0 && sidx * ck0 >= KB;
        const bool empty1 = sidx < P1 && sidx * ck1 >= KB;
        if (empty0 || empty1) {
            cudaError_t e = cudaMemsetAsync(static_cast<uint8_t*>(parts) + sidx * plane, 0, plane, s);
            if (e != cudaSuccess) return cuda_fail(e, "bf16_partials zero fill");
        }
    }
    reax::TcParams p;
    init_params(p);
    if ((rc = make_map(&p.tm_ah, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, x, K, M, K)) != REAX_OK) return rc;
    if ((rc = make_map(&p.tm_bh, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, w, K, N, K)) != REAX_OK) return rc;
    p.tm_a = p.tm_ah;
    p.tm_b = p.tm_bh;
    p.out = static_cast<__nv_bfloat16*>(parts);
    p.out_part_stride = static_cast<long long>(M) * N;
    p.M = M;
    p.ldo = N;
    p.kb_int = 0;
    p.kb_f16 = KB;
    p.m_tiles = (M + reax::kBM - 1) / reax::kBM;
    p.n_tiles = N / reax::kBN;
    p.parts = P0 + P1;
    p.tiles = p.parts * p.m_tiles * p.n_tiles;
    p.mode = 1;
    p.acc_bufs = 2;
    p.slice_mode = 1;
    p.plan_parts0 = P0;
    p.plan_chunk_kb0 = ck0;
    p.plan_chunk_kb1 = ck1;
    p.split = split;
    p.ws_partials = ws.partials;
    p.ws_counters = ws.counters;
    p.status = ws.status;
    int grid = 0;
    plan_schedule(p, stream_sms(stream, info->sms, M), false, &grid);
    return launch_tc(reax::kEpiPlain, p, grid, s);
}

namespace {

int sliced_i8_launch(const int8_t* A, const int8_t* W, const void* AH, const void* WH, const float* sa, const float* sw,
                     const float* bias, void* partials, int M, int N, int G, int HP, int P, void* workspace,
                     size_t workspace_bytes, void* stream, int early_b) {
    if (M < 0 || N <= 0 || G <= 0 || HP < 0 || P < 1)
        return fail(REAX_ERR_INVALID, "sliced_i8: bad sizes M=%d N=%d G=%d HP=%d P=%d", M, N, G, HP, P);
    if (G % 128 != 0 || HP % 64 != 0 || N % 256 != 0)
        return fail(REAX_ERR_INVALID, "sliced_i8: needs G %% 128 == 0, HP %% 64 == 0, N %% 256 == 0 (G=%d HP=%d N=%d)", G,
                    HP, N);
    if (M == 0) return REAX_OK;
    if (!A || !W || !sa || !sw || !bias || !partials || (HP && (!AH || !WH)))
        return fail(REAX_ERR_INVALID, "sliced_i8: NULL pointer argument");
    if (!aligned(A, 16) || !aligned(W, 16) || !aligned(AH, 16) || !aligned(WH, 16) || !aligned(sw, 16) ||
        !aligned(bias, 16) || !aligned(partials, 16))
        return fail(REAX_ERR_ALIGN, "sliced_i8: operands, sw, bias and partials must be 16-byte aligned");
    int dev;
    DeviceInfo* info;
    int rc = current_device(&dev, &info);
    if (rc != REAX_OK) return rc;
    Workspace ws;
    if ((rc = carve_workspace(workspace, workspace_bytes, info->sms, &ws)) != REAX_OK) return rc;
    reax::TcParams p;
    init_params(p);
    if ((rc = make_map(&p.tm_a, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, A, static_cast<uint64_t>(P) * G, M,
                       static_cast<uint64_t>(P) * G)) != REAX_OK)
        return rc;
    if ((rc = make_map(&p.tm_b, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, W, static_cast<uint64_t>(P) * G, N,
                       static_cast<uint64_t>(P) * G)) != REAX_OK)
        return rc;
    if (HP) {
        if ((rc = make_map(&p.tm_ah, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, AH, static_cast<uint64_t>(P) * HP, M,
                           static_cast<uint64_t>(P) * HP)) != REAX_OK)
            return rc;
        if ((rc = make_map(&p.tm_bh, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, WH, static_cast<uint64_t>(P) * HP, N,
                           static_cast<uint64_t>(P) * HP)) != REAX_OK)
            return rc;
    } else {
        p.tm_ah = p.tm_a;
        p.tm_bh = p.tm_b;
    }
    p.sa = sa;
    p.sw = sw;
    p.bias = bias;
    p.out = static_cast<__nv_bfloat16*>(partials);
    p.out_part_stride = static_cast<long long>(M) * N;
    p.M = M;
    p.ldo = N;
    p.kb_int = G / 128;
    p.kb_f16 = HP / 64;
    p.kb_int_part = G / 128;
    p.kb_f16_part = HP / 64;
    p.sa_part_stride = M;
    p.n_part_stride = N;
    p.m_tiles = (M + reax::kBM - 1) / reax::kBM;
    p.n_tiles = N / reax::kBN;
    p.parts = P;
    p.tiles = P * p.m_tiles * p.n_tiles;
    p.mode = 0;
    p.acc_bufs = HP ? 1 : 2;
    p.ws_partials = ws.partials;
    p.ws_counters = ws.counters;
    p.status = ws.status;
    p.early_b = early_b;
    int grid = 0;
    const int sms = stream_sms(stream, info->sms, M);
    if (HP == 0 && M <= kSwapMaxRows && P * N <= reax::kBM * sms) {
        // Few tokens, and every group's columns fit one wave of tiles of at most 128 columns: weight-major
        // tiles of R = P * N / SMs (rounded up) output columns of one group, K-block stages, whole tiles.
        // (With a smaller SM share, two waves of these tiles measured no faster than the token-major tiles,
        // which leave the other SMs to a concurrent lane.)
        reax::TcParams q = p;
        q.n_tok = ((M + 15) / 16) * 16;
        q.tile_rows = std::min(reax::kBM, std::max(16, (P * N + sms - 1) / sms));
        q.tile_rows8 = (q.tile_rows + 7) & ~7;
        q.kk = multi_kk(q.tile_rows8, q.n_tok, &q.stage_bytes, &q.stages);
        if (q.kk > 1) {
            if ((rc = make_plain_multi_maps(&q.tm_a, &q.tm_b, A, W, static_cast<uint64_t>(P) * G, M, N, q.n_tok,
                                            q.tile_rows8, q.kk)) != REAX_OK)
                return rc;
            q.H = N;   // output columns per group
            q.n_tiles = (N + q.tile_rows - 1) / q.tile_rows;
            q.tiles = P * q.m_tiles * q.n_tiles;
            plan_schedule(q, sms, false, &grid);
            return launch_tc(reax::kEpiPlain, q, grid, static_cast<cudaStream_t>(stream));
        }
    }
    // Token-major tiles.  Fewer tiles than SMs (decode) may split them by K over the SMs (int32 partials,
    // exact); tiles with BF16 columns are never split: their float32 association must stay the reference's.
    plan_schedule(p, sms, HP == 0 && kSplitPlainTiles, &grid);
    return launch_tc(reax::kEpiPlain, p, grid, static_cast<cudaStream_t>(stream));
}

}  // namespace

int reax_sliced_i8(const int8_t* A, const int8_t* W, const void* AH, const void* WH, const float* sa, const float* sw,
                   const float* bias, void* partials, int M, int N, int G, int HP, int P, void* workspace,
                   size_t workspace_bytes, void* stream) {
    return sliced_i8_launch(A, W, AH, WH, sa, sw, bias, partials, M, N, G, HP, P, workspace, workspace_bytes, stream,
                            0);
}

int reax_sliced_i8_static(const int8_t* A, const int8_t* W, const void* AH, const void* WH, const float* sa,
                          const float* sw, const float* bias, void* partials, int M, int N, int G, int HP, int P,
                          void* workspace, size_t workspace_bytes, void* stream) {
    return sliced_i8_launch(A, W, AH, WH, sa, sw, bias, partials, M, N, G, HP, P, workspace, workspace_bytes, stream,
                            1);
}

int reax_selftest_wait(void* workspace, unsigned long long timeout_ns, void* stream) {
    if (workspace && !aligned(workspace, 256)) return fail(REAX_ERR_WORKSPACE, "selftest_wait: bad workspace");
    int dev;
    DeviceInfo* info;
    int rc = current_device(&dev, &info);
    if (rc != REAX_OK) return rc;
    // NULL: the allocation-free entry point's status word, so that its reporting path can be exercised
    if (!workspace && (rc = noalloc_scratch(dev, &workspace)) != REAX_OK) return rc;
    return launch_plain("selftest_wait launch", reax::selftest_wait_kernel, dim3(1), dim3(32),
                        static_cast<cudaStream_t>(stream), static_cast<unsigned*>(workspace), timeout_ns);
}

int reax_gate_up_i8_noalloc(const int8_t* A, const int8_t* W, const void* AH, const void* WH, const float* sa,
                            const float* sw, const float* bias, void* out, int M, int N2, int KL, int KH, int ldo,
                            void* stream) {
    bool empty = false;
    int rc = check_gate_up_args("gate_up_i8_noalloc", A, W, AH, WH, sa, sw, bias, out, M, N2, KL, KH, ldo, &empty);
    if (rc != REAX_OK || empty) return rc;
    int dev;
    DeviceInfo* info;
    if ((rc = current_device(&dev, &info)) != REAX_OK) return rc;
    void* scratch = nullptr;
    if ((rc = noalloc_scratch(dev, &scratch)) != REAX_OK) return rc;
    reax::TcParams p;
    bool split_ok = false;
    const int sms = stream_sms(stream, info->sms, M);
    if ((rc = fill_gate_up_params(p, sms, info->pair_clusters > 0, A, W, AH, WH, sa, sw, bias, out, M, N2, KL, KH, ldo, &split_ok)) != REAX_OK)
        return rc;
    // Whole-tile plans need no partials; a plan that splits tiles is re-planned for at most
    // kNoAllocMaxCtas CTAs, whose partials the static scratch holds.
    int grid = 0;
    if (p.cta_shift) plan_pairs(p, sms, info->pair_clusters, &grid);
    else plan_schedule(p, sms, split_ok, &grid);
    if (p.sk_iters > 0 && grid > kNoAllocMaxCtas) plan_schedule(p, kNoAllocMaxCtas, true, &grid);
    const int slots = p.sk_iters > 0 ? grid : 0;
    const size_t counter_bytes = ((static_cast<size_t>(2 * (slots > 0 ? slots : 1)) * sizeof(int)) + 255) / 256 * 256;
    const size_t need = kStatusBytes + counter_bytes + static_cast<size_t>(slots) * 2 * reax::kSlotInts * sizeof(int);
    if (need > kNoAllocScratchBytes)
        return fail(REAX_ERR_WORKSPACE, "gate_up_i8_noalloc: plan needs %zu bytes of scratch, the maximum is %zu", need,
                    kNoAllocScratchBytes);
    uint8_t* b = static_cast<uint8_t*>(scratch);
    p.status = reinterpret_cast<unsigned*>(b);
    p.ws_counters = reinterpret_cast<int*>(b + kStatusBytes);
    p.ws_partials = reinterpret_cast<int*>(b + kStatusBytes + counter_bytes);
    // The array keeps the previous call's contents: the status word and the split counters must start at zero.
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const cudaError_t e = cudaMemsetAsync(scratch, 0, kStatusBytes + counter_bytes, s);
    if (e != cudaSuccess) return cuda_fail(e, "gate_up_i8_noalloc: clearing the scratch");
    return launch_tc(reax::kEpiSwiglu, p, grid, s);
}

int reax_set_stream_sms(void* stream, int sms) {
    if (sms < 0) return fail(REAX_ERR_INVALID, "set_stream_sms: sms=%d", sms);
    std::lock_guard<std::mutex> lock(g_share_mutex);
    for (int i = 0; i < g_n_shares; ++i)
        if (g_shares[i].stream == stream) {
            if (sms == 0) g_shares[i] = g_shares[--g_n_shares];
            else g_shares[i].sms = sms;
            return REAX_OK;
        }
    if (sms == 0) return REAX_OK;
    if (g_n_shares == kMaxStreamShares)
        return fail(REAX_ERR_INVALID, "set_stream_sms: more than %d streams with an SM share", kMaxStreamShares);
    g_shares[g_n_shares++] = StreamShare{stream, sms};
    return REAX_OK;
}

int reax_noalloc_status(unsigned* status, int clear, void* stream) {
    if (!status) return fail(REAX_ERR_INVALID, "noalloc_status: NULL status pointer");
    int dev;
    DeviceInfo* info;
    int rc = current_device(&dev, &info);
    if (rc != REAX_OK) return rc;
    void* scratch = nullptr;
    if ((rc = noalloc_scratch(dev, &scratch)) != REAX_OK) return rc;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    cudaError_t e = cudaMemcpyAsync(status, scratch, sizeof(unsigned), cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess && clear) e = cudaMemsetAsync(scratch, 0, sizeof(unsigned), s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    return e == cudaSuccess ? REAX_OK : cuda_fail(e, "noalloc_status");
}

}  // extern "C"
