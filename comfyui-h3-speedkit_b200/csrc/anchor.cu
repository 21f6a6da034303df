// K anchor detector of the H3 QKV op (B200, sm_100a).
//
// For each head, nine sampled keys k[s][c] (the rows s*(M-1)/8 of the normalised,
// roped K plane) choose the anchor row the full QKV epilogue subtracts from every
// key before quantising: the sample a that minimises sum_c sum_s (9 k[a][c] -
// sum_s k[s][c])^2 is taken if centring on it lowers the sampled energy and does
// not raise the sampled maximum |k| by more than 12.5 %; otherwise -1
// (kernels/gemm/r79_sample_anchor.cu:452-605, launched by h3_sample_anchor at
// :700-702 with 9 samples, 128 channels, 56 heads).
//
// Arithmetic, the reference's order (the unit is compiled with --use_fast_math,
// as the reference compiles r79_sample_anchor.cu, tools/build_kernels.py:37):
// one channel per thread of 4 warps; per channel an fmaf chain of squares, a
// running max and a running sum over the samples in order; per candidate the
// square of 9*k - sum; shfl_down trees inside each warp; the four warp totals
// added in warp order by thread 0; strict < keeps the first minimum.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "host_util.h"
#include "../../include/h3sk_b200.h"

namespace h3sk {
namespace anchor {

constexpr int kSamples = 9;
constexpr int kChannels = 128;
constexpr int kWarps = kChannels / 32;

__device__ __forceinline__ float tree_sum(float x) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) x += __shfl_down_sync(0xffffffffu, x, off);
  return x;
}
__device__ __forceinline__ float tree_max(float x) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) x = fmaxf(x, __shfl_down_sync(0xffffffffu, x, off));
  return x;
}

__global__ void __launch_bounds__(kChannels) detect_kernel(const __nv_bfloat16* k, int* anchors) {
  __shared__ float w_energy[kWarps], w_max[kWarps], w_dist[kSamples][kWarps], w_best_energy[kWarps],
      w_best_max[kWarps];
  __shared__ int chosen;
  const int h = blockIdx.x, c = threadIdx.x, lane = c & 31, warp = c >> 5;
  const __nv_bfloat16* kh = k + int64_t(h) * kSamples * kChannels;
  float x[kSamples];
#pragma unroll
  for (int s = 0; s < kSamples; ++s) x[s] = __bfloat162float(kh[s * kChannels + c]);

  float energy = 0.f, mx = 0.f, sum = 0.f;
#pragma unroll
  for (int s = 0; s < kSamples; ++s) {
    energy = fmaf(x[s], x[s], energy);
    mx = fmaxf(mx, fabsf(x[s]));
    sum += x[s];
  }
  float dist[kSamples];
#pragma unroll
  for (int a = 0; a < kSamples; ++a) {
    const float d = kSamples * x[a] - sum;
    dist[a] = fmaf(d, d, 0.f);
  }
  energy = tree_sum(energy);
  mx = tree_max(mx);
#pragma unroll
  for (int a = 0; a < kSamples; ++a) dist[a] = tree_sum(dist[a]);
  if (lane == 0) {
    w_energy[warp] = energy;
    w_max[warp] = mx;
#pragma unroll
    for (int a = 0; a < kSamples; ++a) w_dist[a][warp] = dist[a];
  }
  __syncthreads();
  if (c == 0) {
    int best = 0;
    float best_dist = 3.402823466e+38F;
    for (int a = 0; a < kSamples; ++a) {
      float total = 0.f;
      for (int w = 0; w < kWarps; ++w) total += w_dist[a][w];
      if (total < best_dist) {
        best = a;
        best_dist = total;
      }
    }
    chosen = best;
  }
  __syncthreads();

  const float centre = __bfloat162float(kh[chosen * kChannels + c]);
  float best_energy = 0.f, best_max = 0.f;
#pragma unroll
  for (int s = 0; s < kSamples; ++s) {
    const float r = x[s] - centre;
    best_energy = fmaf(r, r, best_energy);
    best_max = fmaxf(best_max, fabsf(r));
  }
  best_energy = tree_sum(best_energy);
  best_max = tree_max(best_max);
  if (lane == 0) {
    w_best_energy[warp] = best_energy;
    w_best_max[warp] = best_max;
  }
  __syncthreads();
  if (c == 0) {
    float e0 = 0.f, m0 = 0.f, e1 = 0.f, m1 = 0.f;
    for (int w = 0; w < kWarps; ++w) {
      e0 += w_energy[w];
      m0 = fmaxf(m0, w_max[w]);
      e1 += w_best_energy[w];
      m1 = fmaxf(m1, w_best_max[w]);
    }
    const bool improves = e1 < e0 && m1 <= m0 * 1.125f;
    anchors[h] = improves ? chosen : -1;
  }
}

}  // namespace anchor
}  // namespace h3sk

#define H3SK_EXPORT extern "C" __attribute__((visibility("default")))

H3SK_EXPORT int h3_sample_anchor_ex(const void* K, void* anchors, int heads, uintptr_t stream) {
  if (!K || !anchors || heads < 1 || heads > 65535 || (reinterpret_cast<uintptr_t>(K) & 1u) ||
      (reinterpret_cast<uintptr_t>(anchors) & 3u))
    return h3sk::record_failure(cudaErrorInvalidValue, "h3_sample_anchor: null, misaligned or heads out of range");
  h3sk::anchor::detect_kernel<<<heads, h3sk::anchor::kChannels, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(K), static_cast<int*>(anchors));
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return h3sk::record_failure(e, "h3_sample_anchor: launch failed");
  h3sk::record_success();
  return 1;
}

H3SK_EXPORT int h3_sample_anchor(const void* K, void* anchors, uintptr_t stream) {
  return h3_sample_anchor_ex(K, anchors, H3_QKV_HEADS, stream);
}
