/*
 * h3sk_b200.h -- C-ABI of the B200 (sm_100a) quantized DiT-block linear path.
 *
 * Every entry point takes plain device pointers, sizes and a CUDA stream handle
 * (cast to uintptr_t) and enqueues its work on that stream without a device
 * synchronisation.  No entry point allocates device memory: the caller owns
 * every input and output buffer.  All pointers are device pointers.
 *
 * Two return conventions are kept from the interface each symbol replaces:
 *   - h3_norm_quant_* and h3_convrot_* return a cudaError_t value (0 = success);
 *   - h3_int8* return 1 on success and 0 on failure (the reason is available
 *     through h3_int8_last_error / h3_int8_error).
 * Validation runs on the host before anything is enqueued; a failed check
 * launches nothing.
 *
 * Reference interfaces are cited as path:line inside the H3 SpeedKit sources.
 */
#ifndef H3SK_B200_H
#define H3SK_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------------------ */
/* Fused prologue: RMSNorm -> adaLN x*(1+scale)+shift -> ConvRot256 -> INT8  */
/* ------------------------------------------------------------------------ */

/* Resource report; field order of kernels/norm_quant/norm_quant.cu:215-218. */
typedef struct H3NormQuantResources {
  int64_t abi, bytes, k, threads, warps, num_regs, static_shared_bytes, local_bytes;
  int64_t active_blocks_per_sm, sm_count, max_threads_per_sm, binary_version, ptx_version;
} H3NormQuantResources;

/* Replaces h3_norm_quant_abi (norm_quant.cu:234). Returns 1: the K=5376 ABI. */
int h3_norm_quant_abi(void);
/* Returns 2 when the K-generic extensions (*_k) below are present. */
int h3_norm_quant_abi_ex(void);
/* Replaces h3_norm_quant_resources_size (norm_quant.cu:235). */
size_t h3_norm_quant_resources_size(void);
/* Replaces h3_norm_quant_error (norm_quant.cu:236): cudaGetErrorString. */
const char* h3_norm_quant_error(int code);
/* Replaces h3_norm_quant_query (norm_quant.cu:237-241) for K=5376. */
int h3_norm_quant_query(int table_dtype, int debug, H3NormQuantResources* out, size_t bytes);
/* K-generic query (no reference counterpart; K % 256 == 0, 256 <= K <= 16384). */
int h3_norm_quant_query_k(int64_t k, int table_dtype, int debug, H3NormQuantResources* out,
                          size_t bytes);
/*
 * Replaces h3_norm_quant_run (norm_quant.cu:242-266), K fixed at 5376.
 *   x      BF16 [m, K], row stride xs elements (xs >= K, xs % 4 == 0, 8-byte aligned)
 *   w      BF16 [K] RMSNorm weight
 *   shift  table [T, K] (row stride ss), scale table [T, K] (row stride cs);
 *          table_dtype 0 = FP32, 1 = BF16
 *   rows   int32 [m] table row per token
 *   q      INT8 [m, K] dense, qscale FP32 [m]
 *   debug  1 => also write debug_norm BF16 [m, K], debug_rotated FP32 [m, K],
 *          debug_rstd FP32 [m]; 0 => those must be NULL
 *   eps    finite, >= FLT_MIN
 */
int h3_norm_quant_run(const void* x, const void* w, const void* shift, const void* scale,
                      const void* rows, void* q, void* qscale, void* debug_norm,
                      void* debug_rotated, void* debug_rstd, int64_t m, int64_t xs, int64_t ss,
                      int64_t cs, float eps, int table_dtype, int debug, uintptr_t stream);
/* Same contract with K explicit (K % 256 == 0, 256 <= K <= 16384). The
 * reference fixes K at compile time (norm_quant.cu:16); this is its K-generic form. */
int h3_norm_quant_run_k(const void* x, const void* w, const void* shift, const void* scale,
                        const void* rows, void* q, void* qscale, void* debug_norm,
                        void* debug_rotated, void* debug_rstd, int64_t m, int64_t k, int64_t xs,
                        int64_t ss, int64_t cs, float eps, int table_dtype, int debug,
                        uintptr_t stream);
/* Same contract with the number of modulation-table rows T (shift and scale are
 * [T, >= K]) stated (no reference counterpart: the reference never needs T).
 * Knowing T lets the B200 kernel stage W and all T tables in shared memory when
 * they fit; every entry of `rows` must lie in [0, T), as for the entry points
 * above (an out-of-range entry reads table T - 1 here instead of out of bounds). */
int h3_norm_quant_run_t(const void* x, const void* w, const void* shift, const void* scale,
                        const void* rows, void* q, void* qscale, void* debug_norm,
                        void* debug_rotated, void* debug_rstd, int64_t m, int64_t k, int64_t tables,
                        int64_t xs, int64_t ss, int64_t cs, float eps, int table_dtype, int debug,
                        uintptr_t stream);

/* ------------------------------------------------------------------------ */
/* Fused residual prologue: x = bf(fma(branch, bf(gate[rows]), x)) in place,  */
/* then the prologue above on the updated rows                               */
/* ------------------------------------------------------------------------ */

/* Replaces h3_residual_quant_abi (residual_quant.cu:254). Returns 1. */
int h3_residual_quant_abi(void);
/* Replaces h3_residual_quant_resources_size (residual_quant.cu:255); the report
 * has the field order of H3NormQuantResources (residual_quant.cu:230-233). */
size_t h3_residual_quant_resources_size(void);
/* Replaces h3_residual_quant_error (residual_quant.cu:256): cudaGetErrorString. */
const char* h3_residual_quant_error(int code);
/* Replaces h3_residual_quant_query (residual_quant.cu:257-264) for K=5376;
 * gate_dtype and table_dtype 0 = FP32, 1 = BF16. */
int h3_residual_quant_query(int gate_dtype, int table_dtype, int debug, H3NormQuantResources* out,
                            size_t bytes);
/* K-generic query (no reference counterpart). */
int h3_residual_quant_query_k(int64_t k, int gate_dtype, int table_dtype, int debug,
                              H3NormQuantResources* out, size_t bytes);
/*
 * Replaces h3_residual_quant_run (residual_quant.cu:267-289), K fixed at 5376.
 *   x      BF16 [m, K] contiguous, 8-byte aligned, updated in place:
 *          x = bf(fma(branch, bf(gate[rows[i]]), x))
 *   branch BF16 [m, K] contiguous, 8-byte aligned
 *   gate   table [T, >= K] (row stride gs), gate_dtype 0 = FP32, 1 = BF16
 *   w, shift, scale, rows, q, qscale, debug outputs, eps: as h3_norm_quant_run
 *          (ss, cs row strides; table_dtype for shift/scale)
 * Returns a cudaError_t (0 = success); nothing is launched on a failed check.
 */
int h3_residual_quant_run(void* x, const void* branch, const void* w, const void* gate,
                          const void* shift, const void* scale, const void* rows, void* q, void* qscale,
                          void* debug_norm, void* debug_rotated, void* debug_rstd, int64_t m, int64_t gs,
                          int64_t ss, int64_t cs, float eps, int gate_dtype, int table_dtype, int debug,
                          uintptr_t stream);
/* Same contract with K explicit (K % 256 == 0, 256 <= K <= 16384); the
 * reference fixes K at compile time (residual_quant.cu:16). */
int h3_residual_quant_run_k(void* x, const void* branch, const void* w, const void* gate,
                            const void* shift, const void* scale, const void* rows, void* q, void* qscale,
                            void* debug_norm, void* debug_rotated, void* debug_rstd, int64_t m, int64_t k,
                            int64_t gs, int64_t ss, int64_t cs, float eps, int gate_dtype, int table_dtype,
                            int debug, uintptr_t stream);
/* Same contract with the table count T stated (no reference counterpart), so
 * that W and the shift/scale tables can be staged in shared memory; every entry
 * of `rows` must lie in [0, T) (an out-of-range entry reads table T - 1). */
int h3_residual_quant_run_t(void* x, const void* branch, const void* w, const void* gate,
                            const void* shift, const void* scale, const void* rows, void* q, void* qscale,
                            void* debug_norm, void* debug_rotated, void* debug_rstd, int64_t m, int64_t k,
                            int64_t tables, int64_t gs, int64_t ss, int64_t cs, float eps, int gate_dtype,
                            int table_dtype, int debug, uintptr_t stream);

/* ------------------------------------------------------------------------ */
/* ConvRot256 + per-token INT8 quantiser                                    */
/* ------------------------------------------------------------------------ */

/* Field order of kernels/convrot/convrot_register_v2.cu:140-144. */
typedef struct H3ConvRotResources {
  int64_t abi, bytes, k, threads, warps, num_regs, static_shared_bytes;
  int64_t local_bytes, max_threads_per_block, active_blocks_per_sm;
  int64_t sm_count, max_threads_per_sm, binary_version, ptx_version;
} H3ConvRotResources;

/* Replaces h3_convrot_register_abi (convrot_register_v2.cu:189). Returns 1. */
int h3_convrot_register_abi(void);
/* Replaces h3_convrot_register_resources_size (convrot_register_v2.cu:190). */
size_t h3_convrot_register_resources_size(void);
/* Replaces h3_convrot_register_error (convrot_register_v2.cu:191-193). */
const char* h3_convrot_register_error(int code);
/* Replaces h3_convrot_register_query (convrot_register_v2.cu:194-199); any K % 256 == 0. */
int h3_convrot_register_query(int k, H3ConvRotResources* out, size_t bytes);
/*
 * Replaces h3_convrot_register_run (convrot_register_v2.cu:200-209).
 *   x BF16 [rows, k] dense (16-byte aligned); q INT8 [rows, k] (8-byte aligned);
 *   scale FP32 [rows]; rotated FP32 [rows, k].
 *   mode 0 = production (q, scale), 1 = diagnostic (q, scale and rotated),
 *   2 = rotation only (rotated; q and scale unused).
 *   Any k % 256 == 0 with 256 <= k <= 16384 is accepted (reference: 5376, 7168).
 */
int h3_convrot_register_run(const void* x, void* q, void* scale, void* rotated, int64_t rows,
                            int k, int mode, uintptr_t stream);
/*
 * Replaces Kitchen's quantize_int8_rowwise_convrot64(x, 256, input_act=...) as
 * called at h3_speedkit/runtime.py:159; arithmetic of
 * kernels/convrot/vendor/convrot64_exact.cuh:913-1027.
 *   act 0 = none, 1 = GELU-tanh, 2 = SwiGLU (x row is [gate | up], 2k wide)
 *   x BF16 with row stride xs elements (xs >= k, or >= 2k for SwiGLU;
 *     x and xs*2 bytes 16-byte aligned); q INT8 [rows, k] dense; scale FP32 [rows].
 */
int h3_convrot_quant_act(const void* x, int64_t xs, void* q, void* scale, int64_t rows, int k,
                         int act, uintptr_t stream);
/*
 * The last step of h3_convrot_quant_act (act 0) for rows whose ConvRot256 ran in
 * h3_int8_gelu_rot (no separate reference counterpart; the arithmetic of
 * kernels/convrot/vendor/convrot64_exact.cuh:942-1027 after the rotation):
 *   scale[m] = max(min(rowmax[m], BF16_MAX) / 127, 1e-30) (rowmax: FP32 bits),
 *   q[m, n] = clamp(nearbyint(bf(bf(v[m, n]) / bf(scale[m]))), -128, 127).
 *   v BF16 rotated rows (16-byte aligned, row stride vs >= k, vs % 8 == 0),
 *   rowmax uint32 [rows], q INT8 [rows, k] dense and 16-byte aligned, scale FP32
 *   [rows]; k % 256 == 0, k <= 16384.  Returns a cudaError_t value.
 */
int h3_convrot_codes(const void* v, int64_t vs, const void* rowmax, void* q, void* scale, int64_t rows,
                     int k, uintptr_t stream);

/* ------------------------------------------------------------------------ */
/* INT8 GEMM (tcgen05 kind::i8, int32 accumulators in TMEM) + fused epilogues */
/* ------------------------------------------------------------------------ */

/* Epilogue selectors of h3_int8_ex. */
enum {
  H3_EPI_DEQUANT = 0,      /* D = bf(((acc*xs)*ws)+bias) */
  H3_EPI_DEQUANT_GELU = 1, /* D = bf(gelu_tanh(bf(((acc*xs)*ws)+bias))) */
  H3_EPI_ACC_INT32 = 3     /* D = acc as int32 (debug: bit-exact accumulators) */
};

/*
 * Replaces h3_int8 (kernels/gemm/fc1.cu:119-138):
 *   D[m, n] = bf16( ((float(sum_k A[m,k]*B[n,k]) * xs[m]) * ws[n]) + 0 )
 *   A INT8 [M, K] row-major, B INT8 [N, K] row-major (K-major), xs FP32 [M],
 *   ws FP32 [N], D BF16 [M, N] dense.  K % 16 == 0, N % 8 == 0, A/B/D 16-byte
 *   aligned.  `config` is accepted for ABI compatibility (any value 0..15).
 *   Returns 1 on success, 0 on failure.
 */
int h3_int8(const int8_t* A, const int8_t* B, const float* xs, const float* ws, void* D, int M,
            int N, int K, int config, uintptr_t stream);
/*
 * Replaces h3_int8_gate (kernels/gemm/gate.cu:136-143):
 *   D[m, n] = bf16( fmaf( bf16(((acc*xs[m])*ws[n])+0), gate[rows[m]*N + n], residual[m, n] ) )
 *   gate BF16 table [G, N], rows int32 [M], residual BF16 [M, N].  D may equal
 *   residual (in-place update, h3_speedkit/runtime.py:120).  Returns 1 / 0.
 */
int h3_int8_gate(const int8_t* A, const int8_t* B, const float* xs, const float* ws, void* D,
                 const void* gate, const int32_t* rows, const void* residual, int M, int N, int K,
                 int config, uintptr_t stream);
/*
 * Extended GEMM (no single reference counterpart): optional BF16 bias [N]
 * (NULL = 0), epilogue selector (H3_EPI_*), output row stride ldd in elements
 * (ldd >= N; ldd % 8 == 0).  The bias formula is the explicit
 * __fadd_rn(__fmul_rn(__fmul_rn(acc, xs), ws), bias) of
 * kernels/gemm/r84_kfourwarp.cu:240-241.  Returns 1 / 0.
 */
int h3_int8_ex(const int8_t* A, const int8_t* B, const float* xs, const float* ws,
               const void* bias, void* D, int M, int N, int K, int64_t ldd, int epilogue,
               uintptr_t stream);
/*
 * Extended gate GEMM: optional BF16 bias [N], and an optional requantised copy
 * of the updated rows for the next layer (q INT8 [M, N] + qscale FP32 [M],
 * ConvRot256 + per-token INT8 of D, the arithmetic of
 * kernels/convrot/convrot_register_v2.cu:67-138).  q and qscale both NULL =>
 * no requant.  Returns 1 / 0.
 */
int h3_int8_gate_ex(const int8_t* A, const int8_t* B, const float* xs, const float* ws,
                    const void* bias, void* D, const void* gate, const int32_t* rows,
                    const void* residual, void* q, void* qscale, int M, int N, int K,
                    uintptr_t stream);
/*
 * FC1 + GELU with the FC2-input quantiser's rotation in the epilogue (no single
 * reference counterpart: h3_int8 with the GELU epilogue, kernels/gemm/fc1.cu:119-138,
 * followed by the ConvRot256 of Kitchen's quantize_int8_rowwise_convrot64,
 * convrot64_exact.cuh:942-1027).  Each 256-column group n0..n0+255 of
 * h = bf16(gelu_tanh(bf16(((acc*xs)*ws)+bias))) is rotated:
 *   V[m, n]   = bf16(ConvRot256(h[m, n0 .. n0+255])[n - n0])
 *   rowmax[m] = FP32 bits of max over n of |ConvRot256(...)| (before rounding);
 * rowmax (uint32 [M]) is reset to 0 by the call.  N % 256 == 0; V BF16 with row
 * stride ldv (ldv >= N, ldv % 8 == 0, 16-byte aligned).  Followed by
 * h3_convrot_codes(V, ldv, rowmax, q, scale, M, N) it gives the codes and scales
 * of h3_convrot_quant_act(h, N, q, scale, M, N, act 0) bit for bit.  Returns 1 / 0.
 */
int h3_int8_gelu_rot(const int8_t* A, const int8_t* B, const float* xs, const float* ws,
                     const void* bias, void* V, void* rowmax, int M, int N, int K, int64_t ldv,
                     uintptr_t stream);
/*
 * The same with the plain dequant epilogue when gelu == 0, and the rotation
 * limited to the columns [rot_n0, N) (rot_n0 % 256 == 0): D holds the plain
 * epilogue's BF16 values below rot_n0 and the rotated values from it on, and
 * rowmax the rows' max |rotated value| over those columns.  With gelu == 0 and
 * rot_n0 = 2N/3 this is the QKV projection whose V third feeds the next
 * quantiser: h3_convrot_codes(D + rot_n0, ldd, rowmax, q, scale, M, N - rot_n0)
 * then equals h3_convrot_quant_act(D_plain + rot_n0, ldd, ...) bit for bit.
 * gelu == 1, rot_n0 == 0 is h3_int8_gelu_rot.  Returns 1 / 0.
 */
int h3_int8_rot(const int8_t* A, const int8_t* B, const float* xs, const float* ws, const void* bias,
                void* D, void* rowmax, int M, int N, int K, int64_t ldd, int gelu, int rot_n0,
                uintptr_t stream);
/* cudaError_t-style code of the last failed h3_int8* call on this host thread
 * (0 if the last call succeeded; cudaErrorInvalidValue for a rejected argument). */
int h3_int8_last_error(void);
/* Text for the last failure on this host thread. */
const char* h3_int8_error(void);

/* ------------------------------------------------------------------------ */
/* QKV projection -> pre-quantised attention operands (H3 geometry)          */
/* ------------------------------------------------------------------------ */

/* The H3 geometry the reference's QKV entry points are built for
 * (h3_speedkit/ops/qkv.py:25-28): 56 heads of 128, hidden 5376, N = 21504. */
enum { H3_QKV_HEADS = 56, H3_QKV_HIDDEN = 5376, H3_QKV_SAMPLES = 9 };

/*
 * Replaces h3_qkv_quant_kv (kernels/gemm/r84_kfourwarp.cu:385-388).  Returns 1 on
 * success, 0 on failure (reason in h3_int8_error).
 *   A [M, 5376] INT8, B [21504, 5376] INT8, xs [M] FP32, ws [21504] FP32
 *   D      BF16 [3, 56, M, 128] (16-byte aligned): Q and K RMS-normalised with
 *          qw / kw (BF16 [128]) and roped with freqs (BF16 [M, 48, 2, 2]); V raw
 *   QI     INT8 [56, M, 128], QS FP32 [56, ceil(M/128)*32]  (rotated Q codes/scales)
 *   KI     INT8 [56, M, 128], KS FP32 [56, ceil(M/128)*4]   (K minus its anchor row)
 *   VP     FP32 [56, ceil(M/128), 128] per-tile maxima of |V|
 *   SK     BF16 [56, 9, 128] sampled keys, anchors int32 [56] (row of SK or -1);
 *          both NULL = no centring
 *   1 <= M <= 200000.
 */
int h3_qkv_quant_kv(const int8_t* A, const int8_t* B, const float* xs, const float* ws, void* D,
                    const void* freqs, const void* qw, const void* kw, float eps, int8_t* QI, float* QS,
                    float* VP, int8_t* KI, float* KS, const void* SK, const int* anchors, int M,
                    uintptr_t stream);
/* Same contract for any head count and hidden size (N = 3 * heads * 128, hidden % 16
 * == 0), with an optional rrms [2, heads, M] FP32 debug output (NULL = none).  No
 * reference counterpart (the reference fixes the H3 geometry). */
int h3_qkv_quant_kv_ex(const int8_t* A, const int8_t* B, const float* xs, const float* ws, void* D,
                       const void* freqs, const void* qw, const void* kw, float eps, int8_t* QI,
                       float* QS, float* VP, int8_t* KI, float* KS, const void* SK, const int* anchors,
                       int M, int heads, int hidden, float* rrms, uintptr_t stream);
/*
 * Replaces h3_sample_konly (kernels/gemm/r82_sample_konly.cu:337-341): the K plane of
 * the QKV projection for the nine sample rows, normalised and roped, into plane 1 of
 * D [3, 56, 9, 128] (planes 0 and 2 are not written).  M must be 9; QI, QS and VP are
 * unused, as in the reference.  Returns 1 / 0.
 */
int h3_sample_konly(const int8_t* A, const int8_t* B, const float* xs, const float* ws, void* D,
                    const void* freqs, const void* qw, const void* kw, float eps, int8_t* QI, float* QS,
                    float* VP, int M, uintptr_t stream);
/* Same for any head count, hidden size and row count (no reference counterpart). */
int h3_sample_konly_ex(const int8_t* A, const int8_t* B, const float* xs, const float* ws, void* D,
                       const void* freqs, const void* qw, const void* kw, float eps, int M, int heads,
                       int hidden, float* rrms, uintptr_t stream);
/*
 * Replaces h3_sample_gather (kernels/gemm/r82_sample_konly.cu:352-356): rows
 * s*(M-1)/8, s = 0..8, of Q [M, 5376] INT8, XS [M] FP32 and ROPE [M, 192] BF16 into
 * SQ [9, 5376], SX [9], SR [9, 192].  Returns 1 / 0.
 */
int h3_sample_gather(const void* Q, const void* XS, const void* ROPE, void* SQ, void* SX, void* SR, int M,
                     uintptr_t stream);
/* Same for any hidden size (no reference counterpart). */
int h3_sample_gather_ex(const void* Q, const void* XS, const void* ROPE, void* SQ, void* SX, void* SR,
                        int M, int hidden, uintptr_t stream);
/*
 * Replaces h3_sample_anchor (kernels/gemm/r79_sample_anchor.cu:700-702): K [56, 9, 128]
 * BF16 sampled keys -> anchors int32 [56].  Returns 1 / 0.
 */
int h3_sample_anchor(const void* K, void* anchors, uintptr_t stream);
/* Same for any head count (no reference counterpart). */
int h3_sample_anchor_ex(const void* K, void* anchors, int heads, uintptr_t stream);
/*
 * V quantiser of the QKV op.  No reference C counterpart: it replaces the two Triton
 * kernels the reference launches on the V plane (h3_speedkit/ops/quant_v.py:57-104,
 * launched at ops/qkv.py:70-79).  VP FP32 [heads, ceil(M/128), 128] tile maxima and
 * V BF16 [heads, M, 128] (plane 2 of D) -> VS FP32 [heads*128] scales, VINV FP32
 * [heads*128] their approximate reciprocals, VI INT8 [heads*128, ceil(M/128)*128]
 * (channel-major, tokens permuted inside each run of 16).  Returns 1 / 0.
 */
int h3_quant_v(const float* VP, const void* V, void* VI, float* VS, float* VINV, int M, int heads,
               uintptr_t stream);
/*
 * The whole QKV op in one call, allocating nothing.  It has no counterpart in the
 * reference (which runs the five steps from Python with torch-allocated
 * intermediates).  It is for callers that cannot allocate device memory while
 * they run: a serving loop that must not call cudaMalloc after warm-up (the call
 * can synchronise the device and stall other streams), or a framework that owns
 * all device memory through its own pool.  Same operands and outputs as
 * h3_qkv_quant_kv_ex plus the V quantiser's VI / VS.  The intermediates (nine
 * sample rows, their K plane, the anchors, the V reciprocal scales) live in a
 * 552,960-byte file-scope device array that every GPU loading the library holds
 * until exit; it bounds heads <= 64 and hidden <= 8192, and larger shapes are
 * rejected with an error (h3_int8_error).  The first call on a device looks up
 * the array's device address (cudaGetSymbolAddress) with that device current;
 * make that first call before any stream capture.  The address is cached for
 * the life of the process, so the entry point must not be called after a
 * cudaDeviceReset in the same process (the reset frees the array's context and
 * leaves the cached address stale).  Every operand is checked before the first
 * of the five launches, so a rejected call writes no output.  Every call writes each
 * intermediate before reading it, so nothing needs clearing, but all calls on a
 * device share the array: calls that overlap on the GPU race (issue them on one
 * stream, or order them with events).  Returns 1 / 0.
 */
int h3_qkv_noalloc(const int8_t* A, const int8_t* B, const float* xs, const float* ws, void* D,
                   const void* freqs, const void* qw, const void* kw, float eps, int8_t* QI, float* QS,
                   float* VP, int8_t* KI, float* KS, void* VI, float* VS, int M, int heads, int hidden,
                   uintptr_t stream);

/* ------------------------------------------------------------------------ */
/* INT8 attention on the QKV op's operands (SageAttention-style, D = 128)     */
/* ------------------------------------------------------------------------ */

/* Argument block of kernels/dense/dense_ring.cu:16-24 (same field order and types).
 * Strides are in elements.  q [B, Hq, Sq, 128] and k [B, Hk, Sk, 128] INT8 contiguous;
 * v INT8 [B*Hk*128, v_stride_d] channel-major, v_stride_d >= ceil(Sk/128)*128 tokens,
 * keys permuted in every run of 16 as [0,1,8,9,2,3,10,11,4,5,12,13,6,7,14,15];
 * o BF16 BHSD or BSHD; q_scale FP32 [B, Hq, ceil(Sq/128)*32], k_scale FP32
 * [B, Hk, ceil(Sk/128)*4], v_scale FP32 [B*Hk*128]; sm_scale = head_dim^-0.5. */
typedef struct H3DenseArgs {
  void *q, *k, *v, *o, *q_scale, *k_scale, *v_scale;
  uint32_t batch, qo_len, kv_len, qo_heads, kv_heads;
  uint32_t q_stride_b, q_stride_h, q_stride_s;
  uint32_t k_stride_b, k_stride_h, k_stride_s;
  uint32_t v_stride_b, v_stride_h, v_stride_d;
  uint32_t o_stride_b, o_stride_h, o_stride_s;
  float sm_scale;
} H3DenseArgs;

/* Replaces h3_dense_args_size (dense_ring.cu:26). */
size_t h3_dense_args_size(void);
/* Replaces h3_dense_query_group (dense_ring.cu:27): the arithmetic variant, 8102. */
int h3_dense_query_group(void);
/* Replaces h3_dense_error_string (dense_ring.cu:28-30): cudaGetErrorString. */
const char* h3_dense_error_string(int code);
/*
 * Replaces h3_dense_launch_window (dense_ring.cu:32-94): O = softmax(Q K^T * scales) V
 * with the reference's INT8 arithmetic (u8 probabilities, int32 P.V, FP32 running
 * rescale), rows of query blocks [start, ceil(Sq/128)); the rows before block
 * `start` are set to zero.  Returns a cudaError_t (0 = success); a rejected
 * argument launches nothing.
 */
int h3_dense_launch_window(const H3DenseArgs* args, uintptr_t stream, uint32_t start);
/* Replaces h3_dense_launch (dense_ring.cu:107): the window from block 0. */
int h3_dense_launch(const H3DenseArgs* args, uintptr_t stream);
/* Replaces h3_dense_resources (dense_ring.cu:96-105): out[5] = registers, local
 * bytes, shared bytes, max threads per block, binary version. */
int h3_dense_resources(int* out);

/* ------------------------------------------------------------------------ */
/* Pipeline health and diagnostics                                           */
/* ------------------------------------------------------------------------ */

/*
 * Every mbarrier wait inside the GEMM pipeline is bounded.  A wait that runs
 * out records a nonzero code in a per-device status word, stops the kernel
 * (draining its own copies and releasing TMEM) and leaves the context usable.
 * h3sk_pipeline_status copies that word to *status after synchronising
 * `stream` and, when clear != 0, resets it.  Returns a cudaError_t value.
 */
int h3sk_pipeline_status(int* status, int clear, uintptr_t stream);
/*
 * Self-test of the bounded wait: launches one CTA that waits on an mbarrier no
 * one arrives at, for at most timeout_us microseconds.  The kernel must come
 * back with status H3SK_STATUS_WAIT_TIMEOUT in *status.  Returns cudaError_t.
 */
int h3sk_wait_selftest(int timeout_us, int* status, uintptr_t stream);
/*
 * tcgen05 kind::i8 issue-rate probe: every SM issues `iters` back-to-back
 * 128x256x32 MMAs from shared memory into TMEM; *tops receives the achieved
 * dense INT8 tera-ops per second.  Returns cudaError_t.
 */
int h3sk_int8_mma_peak(int iters, double* tops, uintptr_t stream);
/* The GPU's ex2.approx.ftz.f32 throughput (G ex2 / s), measured by the call:
 * the INT8 attention takes one ex2 per score, and that unit bounds it.  No
 * counterpart in the reference (a measurement aid of this library). */
int h3sk_ex2_peak(int iters, double* gops, uintptr_t stream);
/* Library version string. */
const char* h3sk_version(void);

enum { H3SK_STATUS_OK = 0, H3SK_STATUS_WAIT_TIMEOUT = 1 };

#ifdef __cplusplus
}
#endif

#endif /* H3SK_B200_H */
