// Fused prologue for B200: RMSNorm -> adaLN modulation -> ConvRot256 -> per-token INT8.
//
// One CTA per token row.  The row (K BF16 values) is staged once into shared
// memory with 16-byte (or, for 8-byte-aligned strided rows, 8-byte) coalesced
// loads; the RMS statistics are read from shared memory in the reference's
// accumulation order, and the modulated values are then read in the ConvRot
// register layout, rotated with warp shuffles and quantised in registers.  HBM
// traffic per row: K*2 bytes in, K bytes + 4 bytes out.
//
// Arithmetic follows kernels/norm_quant/norm_quant.cu:51-213:
//  * sum of squares: logical thread t (0..127) fma-accumulates the 4-element
//    chunks t, t+128, ... in element order; a shfl_down tree per warp; the four
//    warp sums fold as (w0+w2)+(w1+w3); variance = div.rn(sum, K)  (:51-78);
//  * rrms = rsqrt.approx(add.rn(var, eps))  (:133-134);
//  * n = bf(w*(rrms*x)); out = bf(bf(n*bf(1+bf(scale))) + bf(shift))  (:164-172);
//  * ConvRot256 + row scale + codes as in rowquant.cuh  (:179-211).
// The reference fixes K = 5376 with 192 threads; this kernel takes K as a
// runtime value (K % 256 == 0, 256 <= K <= 16384) with
// max(128, ceil(K/1024)*32) threads.
#include "rowquant.cuh"
#include "../../include/h3sk_b200.h"

#include <cfloat>
#include <cmath>

namespace h3sk {
namespace {

constexpr int kStatThreads = 128;   // logical reduction width of the reference
constexpr int kMaxK = 16384;
constexpr int kNormK = 5376;        // K of the unsuffixed (reference) entry point

__host__ __device__ constexpr int norm_threads(int k) {
  return ((k + 1023) / 1024) * 32 < kStatThreads ? kStatThreads : ((k + 1023) / 1024) * 32;
}

template <class T> __device__ __forceinline__ float table_value(const T* p);
template <> __device__ __forceinline__ float table_value<float>(const float* p) { return *p; }
template <> __device__ __forceinline__ float table_value<__nv_bfloat16>(const __nv_bfloat16* p) {
  return bf_bits_to_float(*reinterpret_cast<const unsigned short*>(p));
}

template <class ModT, bool kDebug>
__global__ void __launch_bounds__(512) norm_quant_rows(
    const __nv_bfloat16* __restrict__ X, const __nv_bfloat16* __restrict__ W,
    const ModT* __restrict__ Shift, const ModT* __restrict__ Scale,
    const int32_t* __restrict__ Rows, int8_t* __restrict__ Q, float* __restrict__ QScale,
    __nv_bfloat16* __restrict__ DebugNorm, float* __restrict__ DebugRotated,
    float* __restrict__ DebugRstd, int64_t xs, int64_t ss, int64_t cs, float eps, int K,
    int vec16) {
  extern __shared__ __align__(16) unsigned char smem_row[];
  __shared__ float fold[16];
  __shared__ float row_stat;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nthreads = blockDim.x;
  const int64_t row = blockIdx.x;
  const __nv_bfloat16* xr = X + row * xs;

  // 1. Stage the row in shared memory (coalesced vector loads).
  if (vec16) {
    const uint4* src = reinterpret_cast<const uint4*>(xr);
    uint4* dst = reinterpret_cast<uint4*>(smem_row);
    for (int i = tid; i < K / 8; i += nthreads) dst[i] = __ldg(src + i);
  } else {
    const uint2* src = reinterpret_cast<const uint2*>(xr);
    uint2* dst = reinterpret_cast<uint2*>(smem_row);
    for (int i = tid; i < K / 4; i += nthreads) dst[i] = __ldg(src + i);
  }
  __syncthreads();

  // 2. Sum of squares in the reference's order.
  float sum = 0.0f;
  if (tid < kStatThreads) {
    const uint2* chunks = reinterpret_cast<const uint2*>(smem_row);
    for (int i = tid; i < K / 4; i += kStatThreads) {
      const uint2 raw = chunks[i];
      const float a = bf_bits_to_float(raw.x & 0xffffu), b = bf_bits_to_float(raw.x >> 16);
      const float c = bf_bits_to_float(raw.y & 0xffffu), d = bf_bits_to_float(raw.y >> 16);
      sum = ieee_fma(a, a, sum);
      sum = ieee_fma(b, b, sum);
      sum = ieee_fma(c, c, sum);
      sum = ieee_fma(d, d, sum);
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) sum = ieee_add(sum, __shfl_down_sync(kFullMask, sum, off));
    if (lane == 0) fold[warp] = sum;
  }
  __syncthreads();
  if (tid == 0) {
    const float total = ieee_add(ieee_add(fold[0], fold[2]), ieee_add(fold[1], fold[3]));
    row_stat = ieee_div(total, static_cast<float>(K));
  }
  __syncthreads();
  const float rrms = hw_rsqrt(ieee_add(row_stat, eps));

  // 3. Normalise and modulate in the ConvRot register layout.
  const int group = warp * 4 + (lane >> 3), octet = lane & 7;
  const bool active = group < K / 256;
  const int table_row = Rows[row];
  const ModT* shift_row = Shift + static_cast<int64_t>(table_row) * ss;
  const ModT* scale_row = Scale + static_cast<int64_t>(table_row) * cs;
  const int64_t out_row = row * K;
  float v[32];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int col = group * 256 + octet_run_col(octet, j);
    uint4 xv = make_uint4(0, 0, 0, 0);
    uint2 wa = make_uint2(0, 0), wb = make_uint2(0, 0);
    if (active) {
      xv = *reinterpret_cast<const uint4*>(smem_row + 2 * col);
      wa = __ldg(reinterpret_cast<const uint2*>(W + col));
      wb = __ldg(reinterpret_cast<const uint2*>(W + col + 4));
    }
    const uint32_t xw[4] = {xv.x, xv.y, xv.z, xv.w};
    const uint32_t ww[4] = {wa.x, wa.y, wb.x, wb.y};
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      float n = 0.0f;
      if (active) {
        const float x = bf_bits_to_float((xw[e >> 1] >> ((e & 1) * 16)) & 0xffffu);
        const float w = bf_bits_to_float((ww[e >> 1] >> ((e & 1) * 16)) & 0xffffu);
        n = bf_round(ieee_mul(w, ieee_mul(rrms, x)));
        const float sh = bf_round(table_value(shift_row + col + e));
        const float sc = bf_round(table_value(scale_row + col + e));
        const float one_plus = bf_round(ieee_add(1.0f, sc));
        const float prod = bf_round(ieee_mul(n, one_plus));
        n = bf_round(ieee_add(prod, sh));
        if constexpr (kDebug) {
          reinterpret_cast<unsigned short*>(DebugNorm)[out_row + col + e] =
              static_cast<unsigned short>(float_to_bf_bits(n));
        }
      }
      v[j * 8 + e] = n;
    }
  }

  // 4. ConvRot256 in registers, row absmax, scale, codes.
  convrot256_registers(v, lane);
  float local = 0.0f;
#pragma unroll
  for (int r = 0; r < 32; ++r) local = fmaxf(local, fabsf(v[r]));
  local = warp_allmax(local);
  if (lane == 0) fold[warp] = local;
  __syncthreads();
  const int nwarps = nthreads >> 5;
  const float abs_max = warp_allmax(lane < nwarps ? fold[lane] : 0.0f);
  const float scale = int8_row_scale(abs_max);
  if (tid == 0) {
    QScale[row] = scale;
    if constexpr (kDebug) DebugRstd[row] = rrms;
  }
  if (active) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int col = group * 256 + octet_run_col(octet, j);
      if constexpr (kDebug) {
#pragma unroll
        for (int e = 0; e < 8; ++e) DebugRotated[out_row + col + e] = v[j * 8 + e];
      }
      *reinterpret_cast<uint2*>(Q + out_row + col) = pack_codes8(&v[j * 8], scale);
    }
  }
}

template <class T, bool D>
int query_kernel(int k, H3NormQuantResources* out) {
  cudaFuncAttributes a{};
  auto kernel = norm_quant_rows<T, D>;
  const int threads = norm_threads(k);
  int active = 0, device = 0, sms = 0, max_threads = 0;
  cudaError_t e = cudaFuncGetAttributes(&a, kernel);
  if (e != cudaSuccess) return e;
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&active, kernel, threads, size_t(k) * 2);
  if (e != cudaSuccess) return e;
  if ((e = cudaGetDevice(&device)) != cudaSuccess) return e;
  if ((e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device)) != cudaSuccess) return e;
  if ((e = cudaDeviceGetAttribute(&max_threads, cudaDevAttrMaxThreadsPerMultiProcessor, device)) != cudaSuccess)
    return e;
  *out = {1, int64_t(sizeof(H3NormQuantResources)), k, threads, threads / 32, a.numRegs,
          int64_t(a.sharedSizeBytes), int64_t(a.localSizeBytes), active, sms, max_threads,
          a.binaryVersion, a.ptxVersion};
  return cudaSuccess;
}

bool valid_k(int64_t k) { return k >= 256 && k <= kMaxK && k % 256 == 0; }

int run_checked(const void* x, const void* w, const void* shift, const void* scale,
                const void* rows, void* q, void* qscale, void* dn, void* dr, void* drs,
                int64_t m, int64_t k, int64_t xs, int64_t ss, int64_t cs, float eps,
                int table_dtype, int debug, uintptr_t stream_ptr) {
  // Contract of norm_quant.cu:247-255, with K a runtime value.
  if (!valid_k(k)) return cudaErrorInvalidValue;
  if (!x || !w || !shift || !scale || !rows || !q || !qscale || m < 1 || m > INT32_MAX ||
      xs < k || xs % 4 || ss < k || cs < k || table_dtype < 0 || table_dtype > 1 || debug < 0 ||
      debug > 1 || !std::isfinite(eps) || eps < FLT_MIN)
    return cudaErrorInvalidValue;
  if ((uintptr_t(x) & 7u) || (uintptr_t(w) & 7u) || (uintptr_t(q) & 7u) || (uintptr_t(qscale) & 3u) ||
      (uintptr_t(rows) & 3u) || (uintptr_t(shift) % (table_dtype ? 2 : 4)) ||
      (uintptr_t(scale) % (table_dtype ? 2 : 4)))
    return cudaErrorInvalidValue;
  if (debug && (!dn || !dr || !drs || (uintptr_t(dn) & 1u) || (uintptr_t(dr) & 3u) || (uintptr_t(drs) & 3u)))
    return cudaErrorInvalidValue;
  if (!debug && (dn || dr || drs)) return cudaErrorInvalidValue;
  const int vec16 = ((uintptr_t(x) & 15u) == 0 && (xs % 8) == 0) ? 1 : 0;
  const int threads = norm_threads(int(k));
  const size_t smem = size_t(k) * 2;
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_ptr);
#define H3SK_NQ_LAUNCH(T, D)                                                                      \
  norm_quant_rows<T, D><<<dim3(unsigned(m)), threads, smem, stream>>>(                            \
      static_cast<const __nv_bfloat16*>(x), static_cast<const __nv_bfloat16*>(w),               \
      static_cast<const T*>(shift), static_cast<const T*>(scale), static_cast<const int32_t*>(rows), \
      static_cast<int8_t*>(q), static_cast<float*>(qscale), static_cast<__nv_bfloat16*>(dn),     \
      static_cast<float*>(dr), static_cast<float*>(drs), xs, ss, cs, eps, int(k), vec16)
  if (table_dtype == 0) {
    if (debug) H3SK_NQ_LAUNCH(float, true); else H3SK_NQ_LAUNCH(float, false);
  } else {
    if (debug) H3SK_NQ_LAUNCH(__nv_bfloat16, true); else H3SK_NQ_LAUNCH(__nv_bfloat16, false);
  }
#undef H3SK_NQ_LAUNCH
  return cudaGetLastError();
}

int query_checked(int64_t k, int table_dtype, int debug, H3NormQuantResources* out, size_t bytes) {
  if (!out || bytes != sizeof(H3NormQuantResources) || !valid_k(k) || table_dtype < 0 ||
      table_dtype > 1 || debug < 0 || debug > 1)
    return cudaErrorInvalidValue;
  if (table_dtype == 0) return debug ? query_kernel<float, true>(int(k), out) : query_kernel<float, false>(int(k), out);
  return debug ? query_kernel<__nv_bfloat16, true>(int(k), out) : query_kernel<__nv_bfloat16, false>(int(k), out);
}

}  // namespace
}  // namespace h3sk

#define H3SK_EXPORT extern "C" __attribute__((visibility("default")))

H3SK_EXPORT int h3_norm_quant_abi(void) { return 1; }
H3SK_EXPORT int h3_norm_quant_abi_ex(void) { return 2; }
H3SK_EXPORT size_t h3_norm_quant_resources_size(void) { return sizeof(H3NormQuantResources); }
H3SK_EXPORT const char* h3_norm_quant_error(int code) {
  return cudaGetErrorString(static_cast<cudaError_t>(code));
}
H3SK_EXPORT int h3_norm_quant_query(int table_dtype, int debug, H3NormQuantResources* out, size_t bytes) {
  return h3sk::query_checked(h3sk::kNormK, table_dtype, debug, out, bytes);
}
H3SK_EXPORT int h3_norm_quant_query_k(int64_t k, int table_dtype, int debug, H3NormQuantResources* out,
                                      size_t bytes) {
  return h3sk::query_checked(k, table_dtype, debug, out, bytes);
}
H3SK_EXPORT int h3_norm_quant_run(const void* x, const void* w, const void* shift, const void* scale,
                                  const void* rows, void* q, void* qscale, void* debug_norm,
                                  void* debug_rotated, void* debug_rstd, int64_t m, int64_t xs,
                                  int64_t ss, int64_t cs, float eps, int table_dtype, int debug,
                                  uintptr_t stream) {
  return h3sk::run_checked(x, w, shift, scale, rows, q, qscale, debug_norm, debug_rotated, debug_rstd,
                           m, h3sk::kNormK, xs, ss, cs, eps, table_dtype, debug, stream);
}
H3SK_EXPORT int h3_norm_quant_run_k(const void* x, const void* w, const void* shift, const void* scale,
                                    const void* rows, void* q, void* qscale, void* debug_norm,
                                    void* debug_rotated, void* debug_rstd, int64_t m, int64_t k,
                                    int64_t xs, int64_t ss, int64_t cs, float eps, int table_dtype,
                                    int debug, uintptr_t stream) {
  return h3sk::run_checked(x, w, shift, scale, rows, q, qscale, debug_norm, debug_rotated, debug_rstd,
                           m, k, xs, ss, cs, eps, table_dtype, debug, stream);
}
