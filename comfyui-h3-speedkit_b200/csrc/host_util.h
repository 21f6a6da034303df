// Host-side launch helpers shared by the row-quantiser translation units.
#pragma once
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <cstdint>
#include <map>
#include <mutex>
#include <tuple>

namespace h3sk {

// Device address of the library's pipeline status word on the current device
// (defined with the GEMM); bounded waits that run out record their code there.
int* status_device_ptr();

// The INT8 GEMM with the dequant epilogue bf(((acc*xs)*ws)+0) written head-major:
// D is [N/128, M, 128] BF16 (plane h holds product columns 128h..128h+127).
// Returns 1 on success, 0 on failure (reason in h3_int8_error).
int gemm_dequant_heads(const int8_t* A, const int8_t* B, const float* xs, const float* ws, void* D, int M, int N,
                       int K, cudaStream_t stream);
// Operands of the QKV head epilogue fused into the INT8 GEMM: the GEMM writes the
// dequantised product into D's head-major planes [3, heads, M, 128] and finishes
// every row of every head in its epilogue warps (per-head RMS, weight, RoPE,
// rotation, INT8 codes and scales of Q and K, V tile maxima).
struct HeadsArgs {
  const __nv_bfloat16* freqs;     // [M, 192]: (a, b, c, e) of RoPE pair d < 48
  const __nv_bfloat16* qw;        // [128]
  const __nv_bfloat16* kw;        // [128]
  const __nv_bfloat16* sk;        // [heads, 9, 128] sampled keys, or null (no centring)
  const int* anchors;             // [heads] anchor sample or -1, or null
  int8_t* qi;                     // [heads, M, 128]
  float* qs;                      // [heads, parts * 32]
  int8_t* ki;                     // [heads, M, 128]
  float* ks;                      // [heads, parts * 4]
  float* vp;                      // [heads, parts, 128]
  float eps;
  int heads, parts;
};

// The QKV GEMM with the head epilogue fused (kernels/gemm/r84_kfourwarp.cu:213-375):
// D [3, heads, M, 128] BF16 (Q and K normalised and roped, V raw), Q/K codes and
// scales, V tile maxima, all from the GEMM's epilogue warps.  heads must be even.
// Returns 1 on success, 0 on failure (reason in h3_int8_error).
int gemm_qkv_heads(const int8_t* A, const int8_t* B, const float* xs, const float* ws, void* D, int M, int K,
                   const HeadsArgs& hd, cudaStream_t stream);
int last_gemm_error();
// Set the thread's h3_int8_last_error / h3_int8_error record (returns 0), or clear it.
int record_failure(int code, const char* what);
void record_success();

// Driver entry point of cuTensorMapEncodeTiled, resolved once through the
// runtime (no libcuda link dependency); null if the driver lacks it.
inline PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static std::once_flag once;
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  return fn;
}

// Grid of a persistent kernel: as many CTAs as fit on the device at once
// (occupancy x SM count, computed once per kernel, device, block and smem size),
// but no more than `work_ctas`.  Also opts the kernel into `smem` bytes of
// dynamic shared memory when that exceeds the 48 KB default.
inline cudaError_t rq_persistent_grid(const void* kernel, int threads, int smem, int64_t work_ctas, int* grid) {
  static std::mutex mu;
  static std::map<std::tuple<const void*, int, int, int>, int> resident;
  int device = 0;
  cudaError_t e = cudaGetDevice(&device);
  if (e != cudaSuccess) return e;
  const auto key = std::make_tuple(kernel, device, threads, smem);
  int capacity = 0;
  {
    std::lock_guard<std::mutex> lock(mu);
    auto it = resident.find(key);
    if (it == resident.end()) {
      if (smem > 48 * 1024) {
        e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return e;
      }
      int per_sm = 0, sms = 0;
      e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, threads, smem);
      if (e != cudaSuccess) return e;
      e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
      if (e != cudaSuccess) return e;
      if (per_sm < 1) return cudaErrorInvalidConfiguration;
      it = resident.emplace(key, per_sm * sms).first;
    }
    capacity = it->second;
  }
  *grid = int(work_ctas < capacity ? work_ctas : capacity);
  return cudaSuccess;
}

}  // namespace h3sk
