// ConvRot256 + per-token INT8 quantiser for B200, with an optional input
// activation (none / GELU-tanh / SwiGLU).
//
// One CTA per row, ceil(K/1024) warps; every lane owns 32 values of one 256-wide
// group in the register layout of rowquant.cuh and loads them with 16-byte
// vector loads straight from HBM (each 32-byte sector of the row is consumed by
// one warp instruction, so the row is read exactly once).  The rotation runs in
// registers and warp shuffles; codes leave as 8-byte stores.
//
// Replaces kernels/convrot/convrot_register_v2.cu:67-138 (ACT none, K in
// {5376, 7168}) and Kitchen's quantize_int8_rowwise_convrot64_kernel
// (kernels/convrot/vendor/convrot64_exact.cuh:942-1027, input_act none / GELU-tanh
// / SwiGLU) for any K % 256 == 0 up to 16384.  The per-value results do not
// depend on the thread layout: each FHT output is the same expression of the
// same four inputs, and the absmax is an order-free fmaxf.
#include "rowquant.cuh"
#include "../../include/h3sk_b200.h"

namespace h3sk {
namespace {

constexpr int kMaxK = 16384;

__host__ __device__ constexpr int convrot_threads(int k) { return ((k + 1023) / 1024) * 32; }

enum : int { kModeQuant = 0, kModeDiag = 1, kModeRotate = 2 };

__device__ __forceinline__ void unpack8(const uint4 raw, float* out) {
  const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
  for (int e = 0; e < 8; ++e) out[e] = bf_bits_to_float((w[e >> 1] >> ((e & 1) * 16)) & 0xffffu);
}

template <int kAct, int kMode>
__global__ void __launch_bounds__(512) convrot_quant_rows(
    const __nv_bfloat16* __restrict__ X, int64_t xs, int8_t* __restrict__ Q,
    float* __restrict__ Scales, float* __restrict__ Rotated, int K) {
  __shared__ float warp_max[16];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int group = warp * 4 + (lane >> 3), octet = lane & 7;
  const bool active = group < K / 256;
  const int64_t row = blockIdx.x;
  const __nv_bfloat16* xr = X + row * xs;
  const int64_t out_row = row * K;

  float v[32];
  uint4 raw[4], up_raw[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int col = group * 256 + octet_run_col(octet, j);
    raw[j] = make_uint4(0, 0, 0, 0);
    up_raw[j] = make_uint4(0, 0, 0, 0);
    if (active) {
      raw[j] = __ldg(reinterpret_cast<const uint4*>(xr + col));
      if constexpr (kAct == kActSwiGLU) up_raw[j] = __ldg(reinterpret_cast<const uint4*>(xr + K + col));
    }
  }
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    float a[8];
    unpack8(raw[j], a);
    if constexpr (kAct == kActSwiGLU) {
      float u[8];
      unpack8(up_raw[j], u);
#pragma unroll
      for (int e = 0; e < 8; ++e) v[j * 8 + e] = active ? swiglu(a[e], u[e]) : 0.0f;
    } else if constexpr (kAct == kActGeluTanh) {
#pragma unroll
      for (int e = 0; e < 8; ++e) v[j * 8 + e] = active ? gelu_tanh(a[e]) : 0.0f;
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) v[j * 8 + e] = a[e];
    }
  }

  convrot256_registers(v, lane);

  if constexpr (kMode != kModeQuant) {
    if (active) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int col = group * 256 + octet_run_col(octet, j);
        float4* dst = reinterpret_cast<float4*>(Rotated + out_row + col);
        dst[0] = make_float4(v[j * 8 + 0], v[j * 8 + 1], v[j * 8 + 2], v[j * 8 + 3]);
        dst[1] = make_float4(v[j * 8 + 4], v[j * 8 + 5], v[j * 8 + 6], v[j * 8 + 7]);
      }
    }
  }
  if constexpr (kMode == kModeRotate) return;

  float local = 0.0f;
#pragma unroll
  for (int r = 0; r < 32; ++r) local = fmaxf(local, fabsf(v[r]));
  local = warp_allmax(local);
  if (lane == 0) warp_max[warp] = local;
  __syncthreads();
  const int nwarps = blockDim.x >> 5;
  const float scale = int8_row_scale(warp_allmax(lane < nwarps ? warp_max[lane] : 0.0f));
  if (threadIdx.x == 0) Scales[row] = scale;
  if (active) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int col = group * 256 + octet_run_col(octet, j);
      *reinterpret_cast<uint2*>(Q + out_row + col) = pack_codes8(&v[j * 8], scale);
    }
  }
}

bool valid_k(int64_t k) { return k >= 256 && k <= kMaxK && k % 256 == 0; }

template <int kAct, int kMode>
cudaError_t launch(const void* x, int64_t xs, void* q, void* scale, void* rotated, int64_t rows, int k,
                   cudaStream_t stream) {
  convrot_quant_rows<kAct, kMode><<<dim3(unsigned(rows)), convrot_threads(k), 0, stream>>>(
      static_cast<const __nv_bfloat16*>(x), xs, static_cast<int8_t*>(q), static_cast<float*>(scale),
      static_cast<float*>(rotated), k);
  return cudaGetLastError();
}

}  // namespace

// Shared with the GEMM translation unit (requantisation of a gate-residual output).
cudaError_t convrot_quant_none(const void* x, int64_t xs, void* q, void* scale, int64_t rows, int k,
                               cudaStream_t stream) {
  return launch<kActNone, kModeQuant>(x, xs, q, scale, nullptr, rows, k, stream);
}

}  // namespace h3sk

#define H3SK_EXPORT extern "C" __attribute__((visibility("default")))

H3SK_EXPORT int h3_convrot_register_abi(void) { return 1; }
H3SK_EXPORT size_t h3_convrot_register_resources_size(void) { return sizeof(H3ConvRotResources); }
H3SK_EXPORT const char* h3_convrot_register_error(int code) {
  return cudaGetErrorString(static_cast<cudaError_t>(code));
}

H3SK_EXPORT int h3_convrot_register_query(int k, H3ConvRotResources* out, size_t bytes) {
  using namespace h3sk;
  if (!out || bytes != sizeof(H3ConvRotResources) || !valid_k(k)) return cudaErrorInvalidValue;
  auto kernel = convrot_quant_rows<kActNone, kModeQuant>;
  const int threads = convrot_threads(k);
  cudaFuncAttributes attr{};
  int active = 0, device = 0, sms = 0, max_threads = 0;
  cudaError_t e = cudaFuncGetAttributes(&attr, kernel);
  if (e != cudaSuccess) return e;
  if ((e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&active, kernel, threads, 0)) != cudaSuccess) return e;
  if ((e = cudaGetDevice(&device)) != cudaSuccess) return e;
  if ((e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device)) != cudaSuccess) return e;
  if ((e = cudaDeviceGetAttribute(&max_threads, cudaDevAttrMaxThreadsPerMultiProcessor, device)) != cudaSuccess)
    return e;
  *out = {1, int64_t(sizeof(H3ConvRotResources)), k, threads, threads / 32, attr.numRegs,
          int64_t(attr.sharedSizeBytes), int64_t(attr.localSizeBytes), attr.maxThreadsPerBlock, active,
          sms, max_threads, attr.binaryVersion, attr.ptxVersion};
  return cudaSuccess;
}

H3SK_EXPORT int h3_convrot_register_run(const void* x, void* q, void* scale, void* rotated, int64_t rows,
                                        int k, int mode, uintptr_t stream_ptr) {
  using namespace h3sk;
  // Contract of convrot_register_v2.cu:200-205, with K generic.
  if (!x || rows < 1 || rows > INT32_MAX || mode < 0 || mode > 2 || (mode != 2 && (!q || !scale)) ||
      (mode != 0 && !rotated))
    return cudaErrorInvalidValue;
  if ((uintptr_t(x) & 15u) || (mode != 2 && (uintptr_t(q) & 7u)) || (mode != 2 && (uintptr_t(scale) & 3u)) ||
      (mode != 0 && (uintptr_t(rotated) & 15u)))
    return cudaErrorInvalidValue;
  if (!valid_k(k)) return cudaErrorInvalidValue;
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_ptr);
  if (mode == 0) return launch<kActNone, kModeQuant>(x, k, q, scale, nullptr, rows, k, stream);
  if (mode == 1) return launch<kActNone, kModeDiag>(x, k, q, scale, rotated, rows, k, stream);
  return launch<kActNone, kModeRotate>(x, k, nullptr, nullptr, rotated, rows, k, stream);
}

H3SK_EXPORT int h3_convrot_quant_act(const void* x, int64_t xs, void* q, void* scale, int64_t rows, int k,
                                     int act, uintptr_t stream_ptr) {
  using namespace h3sk;
  if (!x || !q || !scale || rows < 1 || rows > INT32_MAX || !valid_k(k) || act < 0 || act > 2)
    return cudaErrorInvalidValue;
  const int64_t width = act == kActSwiGLU ? 2 * int64_t(k) : int64_t(k);
  if (xs < width || (xs % 8) || (uintptr_t(x) & 15u) || (uintptr_t(q) & 7u) || (uintptr_t(scale) & 3u))
    return cudaErrorInvalidValue;
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_ptr);
  if (act == kActNone) return launch<kActNone, kModeQuant>(x, xs, q, scale, nullptr, rows, k, stream);
  if (act == kActGeluTanh) return launch<kActGeluTanh, kModeQuant>(x, xs, q, scale, nullptr, rows, k, stream);
  return launch<kActSwiGLU, kModeQuant>(x, xs, q, scale, nullptr, rows, k, stream);
}
