// GPU-oracle launcher for the reference's vendored Kitchen ConvRot quantiser.
// TEST INFRASTRUCTURE ONLY (built into oracle/_ref/, used by tests as the checker).
//
// It instantiates comfy::quantize_int8_rowwise_convrot64_kernel from the
// reference's own header kernels/convrot/vendor/convrot64_exact.cuh (lines
// 942-1027), found through -I at build time and never copied, and launches it
// the way a caller of quantize_int8_rowwise_convrot64(x, 256, input_act=...)
// does: one CTA per row, shared memory = (K + groups_in_flight*2*256) floats.
// Compiled with --use_fast_math, the flag the reference uses for every
// translation unit that includes this header (tools/build_kernels.py:32-34).
#include "convrot64_exact.cuh"

#include <cstdint>

namespace {
constexpr int kBlockThreads = 256;

template <int ACT>
int launch(const void* x, void* q, void* scale, int64_t rows, int k, cudaStream_t stream) {
  auto kernel = comfy::quantize_int8_rowwise_convrot64_kernel<nv_bfloat16, kBlockThreads, false, ACT>;
  const size_t smem = (size_t(k) + (kBlockThreads / 64) * 2 * 256) * sizeof(float);
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
  if (e != cudaSuccess) return e;
  kernel<<<dim3(unsigned(rows)), kBlockThreads, smem, stream>>>(static_cast<const nv_bfloat16*>(x),
                                                              static_cast<int8_t*>(q), static_cast<float*>(scale),
                                                              k, 0);
  return cudaGetLastError();
}
}  // namespace

// act: 0 none, 1 GELU-tanh, 2 SwiGLU (x is [rows, 2k] for SwiGLU, else [rows, k]).
extern "C" __attribute__((visibility("default"))) int ref_kitchen_convrot64_quant(
    const void* x, void* q, void* scale, int64_t rows, int k, int act, uintptr_t stream) {
  if (!x || !q || !scale || rows < 1 || k < 256 || k % 256) return cudaErrorInvalidValue;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (act == comfy::kActNone) return launch<comfy::kActNone>(x, q, scale, rows, k, s);
  if (act == comfy::kActGeluTanh) return launch<comfy::kActGeluTanh>(x, q, scale, rows, k, s);
  if (act == comfy::kActSwiGLU) return launch<comfy::kActSwiGLU>(x, q, scale, rows, k, s);
  return cudaErrorInvalidValue;
}
