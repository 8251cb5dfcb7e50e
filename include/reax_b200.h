/*
 * reax_b200.h - C ABI of the B200 (sm_100a) gate/up path of the REAX engine.
 *
 * Drop-in boundary: every entry point replaces one launch the reference performs through the CUDA
 * driver (reaxv2/driver.py:4-13 loads a cubin; the wrappers cuLaunchKernel named kernels) or through
 * Triton.  Pointers are device pointers owned by the caller (torch tensors in the Python shim);
 * sizes are element counts; `stream` is a cudaStream_t.  No entry point allocates, synchronizes the
 * host, or resets CUDA error state, so all of them may be called inside CUDA-graph capture.
 *
 * Return value: REAX_OK (0) or one of the REAX_ERR_* codes below; reax_last_error() then returns a
 * message for the calling thread.  bf16 tensors are passed as void* (IEEE bfloat16, row-major).
 */
#ifndef REAX_B200_H
#define REAX_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define REAX_API __attribute__((visibility("default")))
#else
#define REAX_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define REAX_OK 0
#define REAX_ERR_INVALID 1   /* shape, size or pointer argument violates a precondition */
#define REAX_ERR_ALIGN 2     /* a pointer or stride is not aligned as the kernel requires */
#define REAX_ERR_CUDA 3      /* a CUDA runtime / driver call or kernel launch failed */
#define REAX_ERR_DEVICE 4    /* the current device is not an sm_100 (B200-class) GPU */
#define REAX_ERR_WORKSPACE 5 /* workspace missing or smaller than reax_workspace_bytes() */

/* Device status bits a kernel ORs into the workspace status word (offset 0) when a bounded wait
 * expired; the kernel then returned early and its output is invalid. */
#define REAX_STATUS_TIMEOUT_FULL 0x1u
#define REAX_STATUS_TIMEOUT_EMPTY 0x2u
#define REAX_STATUS_TIMEOUT_ACC_FULL 0x4u
#define REAX_STATUS_TIMEOUT_ACC_EMPTY 0x8u
#define REAX_STATUS_TIMEOUT_DRAIN 0x10u
#define REAX_STATUS_SELFTEST 0x20u
#define REAX_STATUS_PLAN_LIMIT 0x40u

/* Library version (major * 10000 + minor * 100 + patch). */
REAX_API int reax_version(void);

/* Message describing the last error returned on the calling thread ("" if none). */
REAX_API const char* reax_last_error(void);

/* Bytes of workspace the GEMM entry points need on `device` (-1 = current device).  The workspace
 * must be zero-filled once when allocated; the kernels leave it zeroed (status word aside).  One
 * workspace may not be used by two launches that can run at the same time (use one per stream). */
REAX_API size_t reax_workspace_bytes(int device);

/* SM share of the decode GEMM launches on `stream` (at most 64 token rows: weight-streaming launches):
 * their tile plans and grids use at most `sms` SMs (0 removes the share: the whole GPU).  Larger launches
 * are compute-bound and always plan for the whole GPU.  For callers that run several lanes at once (streams whose launches
 * overlap, as the reference's two serving lanes do: runtime/bootstrap.py:29, vendor/s1eng/s1eng/kprio.py):
 * each lane's persistent grid then fits beside the other's instead of queueing for the whole GPU.
 * At most 64 streams hold a share.  No counterpart in the reference, whose kernels take fixed grids. */
REAX_API int reax_set_stream_sms(void* stream, int sms);

/* Default bound (nanoseconds) of every device-side wait; reax_set_wait_timeout_ns() changes it for
 * later launches from any thread (0 restores the default of 2 s). */
REAX_API void reax_set_wait_timeout_ns(unsigned long long ns);

/* ---- a1: per-token dynamic INT8 quantization --------------------------------------------------
 * Replaces reaxv2.quantize._prepare[(M,)] (reaxv2/quantize.py:5-29, launched at reaxv2/gate_up.py:34-36).
 * x bf16 [M, K]; low_columns int32 [KL]; high_columns int32 [KH]; smoothing, centers float32 [KL];
 * center = CENTER flag.  Writes low int8 [M, KL], high bf16 [M, KH], scales float32 [M].
 * low_columns and smoothing both NULL describe a dense bank: low column c is column c of x and the
 * smoothing is all ones (KL == K, KH == 0, center == 0, K a multiple of 1024 up to 8192, x 16-byte and
 * low 8-byte aligned); the same codes and scales come from plain row loads, which suits many rows.  A
 * caller that knows its bank is dense passes NULL maps; anything else is REAX_ERR_INVALID. */
REAX_API int reax_quant_rows(const void* x, const int32_t* low_columns, const int32_t* high_columns,
                    const float* smoothing, const float* centers, int8_t* low, void* high, float* scales,
                    int M, int K, int KL, int KH, int center, void* stream);

/* ---- a2: grouped quantization ---------------------------------------------------------------------
 * Replaces reaxv2.quantize.prepare_kernel[(M, P)] (reaxv2/quantize.py:31-52, launched at
 * reaxv2/sliced.py:14-17).  low_columns int32 [P*G] (-1 pads), high_columns int32 [P*HP] (-1 pads),
 * centers, smoothing float32 [P*G].  Writes low int8 [M, P*G], high bf16 [M, P*HP], scales [P, M]. */
REAX_API int reax_quant_groups(const void* x, const int32_t* low_columns, const int32_t* high_columns,
                      const float* centers, const float* smoothing, int8_t* low, void* high, float* scales,
                      int M, int K, int G, int HP, int P, void* stream);

/* ---- rotated quantizer of the INT8 down projection -------------------------------------------------
 * Replaces reaxv2.rotation.Native.prepare (reaxv2/rotation.py:14-30), which launches
 * rotation_g{G}_b{B}_t{T} (kernel-source/legacy-v2/src/block_rotation.cu:5-65) with grid (M, parts).
 * For row r and part p, value o < group is x[r, p*chunk + o] - centers[p*chunk + o] when o < chunk and
 * the column is below K (0 otherwise), negated when bit 16 of column * 1103515245 + 12345 (uint32) is
 * set; Walsh-Hadamard butterflies (lo, hi) -> (lo + hi, lo - hi) on aligned blocks of `block` values,
 * index bit 0 first; scale = max(1e-12, absmax) * fl(1/127); codes float2int_rn(div_rn(v, scale)).
 * x bf16 [M, K], centers float32 [K] -> low int8 [M, parts*group], scales float32 [parts, M].
 * Requires block a power of two (>= 2) dividing group, group <= 8192 and chunk <= group (every
 * reference rotation_* shape). */
REAX_API int reax_quant_rotated(const void* x, const float* centers, int8_t* low, float* scales, int M, int K,
                                int chunk, int parts, int group, int block, void* stream);

/* ---- a3: ordered fp32 sum of bf16 partials -----------------------------------------------------
 * Replaces reaxv2.quantize.reduce_kernel (reaxv2/quantize.py:55-61, launched at reaxv2/sliced.py:45-46).
 * partials bf16 [P, total] -> out bf16 [total]. */
REAX_API int reax_reduce_partials(const void* partials, void* out, long long total, int P, void* stream);

/* ---- a12: mixed-origin fold ------------------------------------------------------------------------
 * Replaces runtime/mixed_origin_bf16.fold (runtime/mixed_origin_bf16.py:8-17, launched at :47).
 * parts bf16 [max(P0,P1), M, N]; split int32[1] on the device: rows < split[0] sum P0 partials,
 * the others P1.  out bf16 [M, N]. */
REAX_API int reax_fold_partials(const void* parts, const int32_t* split, void* out, int M, int N, int P0, int P1,
                       void* stream);

/* ---- SwiGLU of a computed gate/up pair ------------------------------------------------------------
 * The engine's silu_mul contract (vendor/s1eng/s1eng/fused.py:145-164): out[r, c] =
 * bf16(bf16(silu_f32(g[r, c])) * u[r, c]); g and u are row-strided views (strides in elements),
 * out is contiguous [rows, cols]. */
REAX_API int reax_silu_mul(const void* g, const void* u, void* out, int rows, int cols, long long g_stride,
                  long long u_stride, void* stream);

/* bf16(silu_f32(x)) for all 65536 bf16 bit patterns x, written to table bf16 [65536]; the device
 * formula the SwiGLU epilogues use (the reference's table builder and domain check:
 * model-addressed-bulk-activation-table-r1/addressed_gate_up.cu:115-127, wide_warp_hybrid.py:41-49). */
REAX_API int reax_silu_table(void* table, void* stream);

/* ---- a5-a9: fused INT8 gate/up GEMM + dequant + SwiGLU ---------------------------------------------
 * Replaces reaxv2.gate_up.Native.product (reaxv2/gate_up.py:11-27) launching the hybrid8_* kernels
 * (kernel-source/legacy-v2/src/native_hybrid8.cu:56-80), and the v3 addressed_* / band_* variants
 * (wide_warp_hybrid.py:15-35).
 * A int8 [M, KL] (codes), W int8 [N2, KL] = [Wg; Wu], AH bf16 [M, KH], WH bf16 [N2, KH] (may be
 * NULL when KH == 0), sa float32 [M], sw and bias float32 [N2]; out bf16 rows of ldo elements,
 * [M, N2/2] written.  Requires KL % 128 == 0, KH % 64 == 0, N2 % 256 == 0. */
REAX_API int reax_gate_up_i8(const int8_t* A, const int8_t* W, const void* AH, const void* WH, const float* sa,
                    const float* sw, const float* bias, void* out, int M, int N2, int KL, int KH, int ldo,
                    void* workspace, size_t workspace_bytes, void* stream);

/* ---- a5-a9 for weights that the preceding kernel does not write ----------------------------------------
 * No counterpart in the reference: reax_gate_up_i8 with the same arguments and requirements, for a
 * caller that guarantees that the kernel launched just before this one on the stream does not write W
 * or WH (the usual case: banks are written once and then only read).  The GEMM then requests its
 * first weight tiles before it waits for that kernel, so the weight stream starts under the tail of
 * the previous launch.  A, AH, sa, sw and bias are still read only after the wait. */
REAX_API int reax_gate_up_i8_static(const int8_t* A, const int8_t* W, const void* AH, const void* WH, const float* sa,
                                    const float* sw, const float* bias, void* out, int M, int N2, int KL, int KH,
                                    int ldo, void* workspace, size_t workspace_bytes, void* stream);

/* ---- a1 + a4-a9: quantize, then the fused INT8 gate/up --------------------------------------------
 * Replaces reaxv2.gate_up.Native.project (reaxv2/gate_up.py:29-37): reax_quant_rows on x bf16 [M, K]
 * into low int8 [M, KL], high bf16 [M, KH] and scales float32 [M], then reax_gate_up_i8 on them with W,
 * WH, sw and bias (the bank) into out.  Because the GEMM follows this library's quantizer on the
 * stream, it requests its first weight tiles while the quantizer still runs.  Same requirements as the
 * two calls it makes (NULL low_columns and smoothing: a dense bank, as for reax_quant_rows). */
REAX_API int reax_project_i8(const void* x, const int32_t* low_columns, const int32_t* high_columns,
                             const float* smoothing, const float* centers, int center, const int8_t* W,
                             const void* WH, const float* sw, const float* bias, int8_t* low, void* high,
                             float* scales, void* out, int M, int K, int KL, int KH, int N2, int ldo, void* workspace,
                             size_t workspace_bytes, void* stream);

/* ---- a5-a9 without a caller workspace ----------------------------------------------------------------
 * No counterpart in the reference: the same INT8 gate/up + dequant + SwiGLU as reax_gate_up_i8, for
 * callers that cannot allocate device memory for a workspace - e.g. a serving process that has handed
 * all GPU memory to its own pool at start-up, or a plugin host that passes only input and output
 * buffers.  It allocates nothing: its split-tile scratch is a fixed 16 MiB static device array that
 * every GPU loading this library holds until exit; plans that split tiles are limited to 63 CTAs so
 * their partials fit, and a plan needing more scratch is rejected with REAX_ERR_WORKSPACE.
 * The first call on a device resolves the array's device address (cudaGetSymbolAddress) and should
 * come before any stream capture.  All calls share the array and each call clears its status word
 * and counters, so calls that overlap on the GPU (other streams, other threads) race: serialize them.
 * A bounded wait that expires inside the kernel is recorded in the array's status word (the
 * REAX_STATUS_* bits below; the output of that call is then invalid): read it with
 * reax_noalloc_status() before the next call clears it.
 * Arguments and requirements as reax_gate_up_i8, without workspace / workspace_bytes. */
REAX_API int reax_gate_up_i8_noalloc(const int8_t* A, const int8_t* W, const void* AH, const void* WH,
                                     const float* sa, const float* sw, const float* bias, void* out, int M, int N2,
                                     int KL, int KH, int ldo, void* stream);

/* Status word of reax_gate_up_i8_noalloc's static scratch on the current device, after the work queued
 * on `stream` so far (this call synchronizes `stream`, so it is not for use inside stream capture):
 * 0, or the REAX_STATUS_* bits of the last allocation-free call whose bounded wait expired.  The word
 * is shared by every allocation-free call on the device; each such call clears it when it starts, and
 * `clear` != 0 clears it here after reading.  No counterpart in the reference (the allocation-free
 * entry point has none). */
REAX_API int reax_noalloc_status(unsigned* status, int clear, void* stream);

/* ---- a12 (fused): BF16-weight gate/up GEMM + SwiGLU, unsplit plan ------------------------------------
 * The mixed-origin BF16 projection with parts = 1 on both origins (runtime/mixed_origin_bf16.py:19-48:
 * one float32 accumulation over K, one bf16 rounding) of [Wg; Wu], followed by the silu_mul SwiGLU.
 * x bf16 [M, K], w bf16 [N2, K] -> out bf16 rows of ldo elements, [M, N2/2] written.
 * Requires K % 64 == 0, N2 % 256 == 0. */
REAX_API int reax_gate_up_bf16(const void* x, const void* w, void* out, int M, int N2, int K, int ldo, void* workspace,
                      size_t workspace_bytes, void* stream);

/* ---- a12: mixed-origin BF16 partials -----------------------------------------------------------------
 * Replaces runtime/mixed_origin_bf16.Native.partials (runtime/mixed_origin_bf16.py:34-44).
 * x bf16 [M, K], w bf16 [N, K]; split int32[1] on the device; rows < split[0] use (P0, chunk0),
 * the others (P1, chunk1); slice s covers K columns [s*chunk, min(K, (s+1)*chunk)).
 * parts bf16 [max(P0,P1), M, N]: slice s of a row = bf16(float32 sum over the slice); empty slices
 * are written as zeros; slices at or past a row's own plan count are left untouched.
 * Requires K % 64 == 0, chunk0 and chunk1 multiples of 64, N % 256 == 0. */
REAX_API int reax_bf16_partials(const void* x, const void* w, const int32_t* split, void* parts, int M, int N, int K,
                       int chunk0, int chunk1, int P0, int P1, void* workspace, size_t workspace_bytes,
                       void* stream);

/* ---- a11: grouped (sliced) INT8 projection ----------------------------------------------------------
 * Replaces the slice_* kernels launched by reaxv2.sliced.Native.project (reaxv2/sliced.py:20-47) and
 * runtime/split_gated_projection.Prepared.project_ready (:22-43).
 * A int8 [M, P*G], W int8 [N, P*G], AH bf16 [M, P*HP], WH bf16 [N, P*HP], sa float32 [P, M],
 * sw and bias float32 [P, N]; partials bf16 [P, M, N] (part z = bf16 of the dequantized group-z sum
 * plus its BF16 columns).  Requires G % 128 == 0, HP % 64 == 0, N % 256 == 0. */
REAX_API int reax_sliced_i8(const int8_t* A, const int8_t* W, const void* AH, const void* WH, const float* sa,
                   const float* sw, const float* bias, void* partials, int M, int N, int G, int HP, int P,
                   void* workspace, size_t workspace_bytes, void* stream);

/* ---- a11 for weights that the preceding kernel does not write --------------------------------------
 * No counterpart in the reference: reax_sliced_i8 with the same arguments and requirements, for a
 * caller that guarantees that the kernel launched just before this one on the stream does not write W
 * or WH (the usual case: banks are written once and then only read, and the kernel before the
 * projection is its quantizer).  The GEMM then requests its first weight tiles before it waits for
 * that kernel, so the weight stream starts under the tail of the previous launch.  A, AH, sa, sw and
 * bias are still read only after the wait. */
REAX_API int reax_sliced_i8_static(const int8_t* A, const int8_t* W, const void* AH, const void* WH, const float* sa,
                                   const float* sw, const float* bias, void* partials, int M, int N, int G, int HP,
                                   int P, void* workspace, size_t workspace_bytes, void* stream);

/* ---- failure detection -------------------------------------------------------------------------------
 * Runs one kernel that waits on a barrier nothing arrives on, bounded by timeout_ns, and ORs
 * REAX_STATUS_SELFTEST into the status word at `workspace` (a GEMM workspace, or NULL for the status word
 * of reax_gate_up_i8_noalloc's static scratch on the current device) when the wait expires. */
REAX_API int reax_selftest_wait(void* workspace, unsigned long long timeout_ns, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* REAX_B200_H */
