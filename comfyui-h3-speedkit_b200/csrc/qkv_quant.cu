// QKV head epilogue, sample-row gather and V quantiser of the H3 attention input
// (B200, sm_100a).
//
// The reference's QKV op (h3_speedkit/ops/qkv.py:24-83 of H3 SpeedKit) turns the
// INT8 QKV projection into the pre-quantised operands of its INT8 attention:
//   D   [3, H, M, 128] BF16   Q and K RMS-normalised (per head, weights qw / kw)
//                             and roped (pairs d, d+48 for d < 48); V as produced;
//   QI  [H, M, 128] INT8, QS [H, parts*32]  Q rotated (signed H128) per row, one
//                             scale per 4 rows {base + 8j};
//   KI  [H, M, 128] INT8, KS [H, parts*4]   K minus its anchor row, rotated, one
//                             scale per 32 rows {tr : tr % 8 in {2kg, 2kg+1}};
//   VP  [H, parts, 128]       per-tile |V| maxima, then VI/VS from the V quantiser.
// (parts = ceil(M / 128).)  The reference fuses this into a CUTLASS mma.sync GEMM
// (kernels/gemm/r84_kfourwarp.cu:193-375).  Here the tcgen05 GEMM writes the
// dequantised product straight into D's head-major planes (3D TMA store), and one
// CTA per (128-row tile, head, plane) finishes the plane in place from a 32 KB
// shared-memory copy of the slab: the slab of a head is contiguous in D, so every
// load and store is a 16-byte vector and nothing is staged twice.
//
// Arithmetic (the reference's, which the test suite restates on the CPU):
//   * this unit is compiled WITHOUT fast-math, like the reference's QKV unit
//     (tools/build_kernels.py:35-36): IEEE products, rsqrtf, no flush;
//   * sum of squares: 32 lane chains fmaf(v, v, s) over d = lane + 32i, then the
//     shfl_down tree (r84_kfourwarp.cu:264-267); rrms = rsqrtf(sum/128 + eps);
//   * x = bf((t * rrms) * w); y0 = bf(a*x0 + b*x1), y1 = bf(c*x0 + e*x1) with the
//     RoPE row (a, b, c, e) of pair d (r84:268-279);
//   * rotation (m > 256): sign flips from four fixed 32-bit words, the 4-point
//     block (a0+a2)/2 ... of each lane's channels, five shfl_xor butterflies
//     (lo + hi, lo - hi) and the factor 0.1767766952966369f; m <= 256: the
//     4-point block only (r84:123-186, 286-290, 321-327);
//   * scale = fmaf(max|v|, 1/127, 1e-7); code = cvt.rni.sat.s8.f32(v * rcp(scale))
//     with rcp.approx.ftz.f32 (r84:296-306, 334-347);
//   * V maxima: max of the |BF16| bit patterns of each tile column (r84:352-366).
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "host_util.h"
#include "../../include/h3sk_b200.h"

namespace h3sk {
namespace qkv {

constexpr int kHead = 128;           // channels per head
constexpr int kPairs = 48;           // roped pairs (d, d + 48)
constexpr int kRopeRow = 4 * kPairs; // BF16 values of one token's RoPE row
constexpr int kSamples = 9;
constexpr int kThreads = 256;
constexpr int kTileRows = 128;
constexpr int kMaxRows = 200000;     // the reference's M bound (r84_kfourwarp.cu:386)

struct HeadParams {
  __nv_bfloat16* d;               // [3, heads, m, 128]
  const __nv_bfloat16* freqs;     // [m, 192]
  const __nv_bfloat16* qw;        // [128]
  const __nv_bfloat16* kw;        // [128]
  const __nv_bfloat16* sk;        // [heads, 9, 128] (may be null: no centring)
  const int* anchors;             // [heads] (may be null: no centring)
  int8_t* qi;
  float* qs;
  int8_t* ki;
  float* ks;
  float* vp;
  float* rrms;                    // optional [2, heads, m]
  float eps;
  int m, heads, parts;
  int plane0;                     // plane of blockIdx.z == 0
  int quant;                      // 0: normalise and rope only (the sample form)
};

__device__ __forceinline__ float rcp_approx_ftz(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ uint32_t code_s8(float x) {
  int c;
  asm("cvt.rni.sat.s8.f32 %0, %1;" : "=r"(c) : "f"(x));
  return uint32_t(c) & 0xffu;
}

// The 4-point block of one lane's channels.
__device__ __forceinline__ void block4(float (&v)[4]) {
  const float a0 = v[0] + v[1], a1 = v[0] - v[1], a2 = v[2] + v[3], a3 = v[2] - v[3];
  v[0] = (a0 + a2) * 0.5f;
  v[1] = (a1 + a3) * 0.5f;
  v[2] = (a0 - a2) * 0.5f;
  v[3] = (a1 - a3) * 0.5f;
}

// Rotate one 128-channel row held 4 channels per lane (lane l: channels 4l..4l+3).
// Every lane of the warp must call it (shuffles).
__device__ __forceinline__ void rotate(float (&v)[4], int lane, bool full) {
  if (full) {
    const uint32_t word = lane < 8 ? 0x1035997bu : lane < 16 ? 0x8087f5eeu : lane < 24 ? 0xee2e4e1au : 0x71132418u;
    const int shift = (lane & 7) * 4;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const uint32_t flip = ((word >> (shift + c)) & 1u) ^ 1u;
      v[c] = __uint_as_float(__float_as_uint(v[c]) ^ (flip << 31));
    }
  }
  block4(v);
  if (!full) return;
#pragma unroll
  for (int bit = 1; bit < 32; bit <<= 1) {
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const float other = __shfl_xor_sync(0xffffffffu, v[c], bit);
      v[c] = (lane & bit) ? other - v[c] : v[c] + other;
    }
  }
#pragma unroll
  for (int c = 0; c < 4; ++c) v[c] *= 0.1767766952966369f;
}

__device__ __forceinline__ float warp_max(float x) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) x = fmaxf(x, __shfl_xor_sync(0xffffffffu, x, off));
  return x;
}

__device__ __forceinline__ void load4(const __nv_bfloat16* row, int lane, float (&v)[4]) {
  const uint2 u = *reinterpret_cast<const uint2*>(row + 4 * lane);
  v[0] = __uint_as_float(u.x << 16);
  v[1] = __uint_as_float(u.x & 0xffff0000u);
  v[2] = __uint_as_float(u.y << 16);
  v[3] = __uint_as_float(u.y & 0xffff0000u);
}

__device__ __forceinline__ uint32_t pack_codes(const float (&v)[4], float inv) {
  return code_s8(v[0] * inv) | (code_s8(v[1] * inv) << 8) | (code_s8(v[2] * inv) << 16) | (code_s8(v[3] * inv) << 24);
}

// One CTA per (128-row tile, head, plane).
__global__ void __launch_bounds__(kThreads) heads_kernel(const HeadParams p) {
  __shared__ __align__(16) __nv_bfloat16 tile[kTileRows * kHead];
  __shared__ float group_max[kThreads / 32];
  __shared__ uint32_t v_half[kHead];
  const int tm = blockIdx.x, h = blockIdx.y, g = p.plane0 + int(blockIdx.z);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r0 = tm * kTileRows;
  const int rows = min(kTileRows, p.m - r0);
  __nv_bfloat16* slab = p.d + ((int64_t(g) * p.heads + h) * p.m + r0) * kHead;
  for (int i = threadIdx.x; i < rows * (kHead / 8); i += kThreads)
    reinterpret_cast<uint4*>(tile)[i] = reinterpret_cast<const uint4*>(slab)[i];
  __syncthreads();

  if (g == 2) {
    // V: column maxima of |BF16| bit patterns; two row halves per channel.
    if (p.vp == nullptr) return;
    const int ch = threadIdx.x & (kHead - 1), half = threadIdx.x >> 7;
    uint32_t mx = 0;
    const int end = min(rows, (half + 1) * 64);
    for (int tr = half * 64; tr < end; ++tr) {
      const uint32_t mag = uint32_t(__bfloat16_as_ushort(tile[tr * kHead + ch])) & 0x7fffu;
      mx = mag > mx ? mag : mx;
    }
    if (half) v_half[ch] = mx;
    __syncthreads();
    if (!half) {
      const uint32_t other = v_half[ch];
      mx = other > mx ? other : mx;
      p.vp[(int64_t(h) * p.parts + tm) * kHead + ch] = __uint_as_float(mx << 16);
    }
    return;
  }

  // Q / K: RMS over the head, weight, RoPE; one warp per row.
  const __nv_bfloat16* w = g == 0 ? p.qw : p.kw;
  for (int tr = warp; tr < rows; tr += kThreads / 32) {
    __nv_bfloat16* t = tile + tr * kHead;
    float sum = 0.f;
#pragma unroll
    for (int d = lane; d < kHead; d += 32) {
      const float v = __bfloat162float(t[d]);
      sum = fmaf(v, v, sum);
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) sum += __shfl_down_sync(0xffffffffu, sum, off);
    sum = __shfl_sync(0xffffffffu, sum, 0);
    const float rrms = rsqrtf(sum / 128.f + p.eps);
    const int row = r0 + tr;
    if (p.rrms != nullptr && lane == 0) p.rrms[(int64_t(g) * p.heads + h) * p.m + row] = rrms;
    // Each lane reads and writes only its own channels (2l, 2l+1, +48; 96 + l).
    if (lane < kPairs / 2) {
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const int d = lane * 2 + i;
        float x0 = __bfloat162float(t[d]), x1 = __bfloat162float(t[d + kPairs]);
        x0 = __bfloat162float(__float2bfloat16_rn(x0 * rrms * __bfloat162float(w[d])));
        x1 = __bfloat162float(__float2bfloat16_rn(x1 * rrms * __bfloat162float(w[d + kPairs])));
        const __nv_bfloat16* f = p.freqs + int64_t(row) * kRopeRow + d * 4;
        const float a = __bfloat162float(f[0]), b = __bfloat162float(f[1]);
        const float c = __bfloat162float(f[2]), e = __bfloat162float(f[3]);
        t[d] = __float2bfloat16_rn(a * x0 + b * x1);
        t[d + kPairs] = __float2bfloat16_rn(c * x0 + e * x1);
      }
    }
    const int d = 2 * kPairs + lane;
    t[d] = __float2bfloat16_rn(__bfloat162float(t[d]) * rrms * __bfloat162float(w[d]));
  }
  __syncthreads();
  for (int i = threadIdx.x; i < rows * (kHead / 8); i += kThreads)
    reinterpret_cast<uint4*>(slab)[i] = reinterpret_cast<const uint4*>(tile)[i];
  if (!p.quant) return;

  const bool full = p.m > 256;
  if (g == 0) {
    if (p.qi == nullptr || p.qs == nullptr) return;
    for (int sub = warp; sub < 32; sub += kThreads / 32) {
      const int base = (sub >> 3) * 32 + (sub & 7);
      float v[4][4];
      float mx = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int tr = base + 8 * j;
        if (tr < rows) load4(tile + tr * kHead, lane, v[j]);
        else v[j][0] = v[j][1] = v[j][2] = v[j][3] = 0.f;
        rotate(v[j], lane, full);
#pragma unroll
        for (int c = 0; c < 4; ++c) mx = fmaxf(mx, fabsf(v[j][c]));
      }
      mx = warp_max(mx);
      const float sc = fmaf(mx, 1.f / 127.f, 1e-7f), inv = rcp_approx_ftz(sc);
      if (lane == 0) p.qs[int64_t(h) * p.parts * 32 + tm * 32 + sub] = sc;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int tr = base + 8 * j;
        if (tr < rows)
          *reinterpret_cast<uint32_t*>(p.qi + (int64_t(h) * p.m + r0 + tr) * kHead + 4 * lane) = pack_codes(v[j], inv);
      }
    }
    return;
  }

  // K: centre on the anchor row, rotate, one scale per 32-row group; two warps
  // per group (16 rows each), their maxima combined through shared memory.
  if (p.ki == nullptr || p.ks == nullptr) return;
  float bias[4] = {0.f, 0.f, 0.f, 0.f};
  const int anchor = (p.anchors != nullptr && p.sk != nullptr) ? p.anchors[h] : -1;
  if (anchor >= 0 && anchor < kSamples) {   // an out-of-range anchor reads nothing
#pragma unroll
    for (int c = 0; c < 4; ++c) bias[c] = __bfloat162float(p.sk[(int64_t(h) * kSamples + anchor) * kHead + 4 * lane + c]);
  }
  const int kg = warp >> 1, half = warp & 1;
  float v[16][4];
  float mx = 0.f;
#pragma unroll
  for (int ii = 0; ii < 16; ++ii) {
    const int i = half * 16 + ii;
    const int tr = (i >> 1) * 8 + kg * 2 + (i & 1);
    if (tr < rows) {
      load4(tile + tr * kHead, lane, v[ii]);
#pragma unroll
      for (int c = 0; c < 4; ++c) v[ii][c] = v[ii][c] - bias[c];
    } else {
      v[ii][0] = v[ii][1] = v[ii][2] = v[ii][3] = 0.f;
    }
    rotate(v[ii], lane, full);
#pragma unroll
    for (int c = 0; c < 4; ++c) mx = fmaxf(mx, fabsf(v[ii][c]));
  }
  mx = warp_max(mx);
  if (lane == 0) group_max[warp] = mx;
  __syncthreads();
  mx = fmaxf(group_max[warp & ~1], group_max[warp | 1]);
  const float sc = fmaf(mx, 1.f / 127.f, 1e-7f), inv = rcp_approx_ftz(sc);
  if (lane == 0 && half == 0) p.ks[(int64_t(h) * p.parts + tm) * 4 + kg] = sc;
#pragma unroll
  for (int ii = 0; ii < 16; ++ii) {
    const int i = half * 16 + ii;
    const int tr = (i >> 1) * 8 + kg * 2 + (i & 1);
    if (tr < rows)
      *reinterpret_cast<uint32_t*>(p.ki + (int64_t(h) * p.m + r0 + tr) * kHead + 4 * lane) = pack_codes(v[ii], inv);
  }
}

// Sample rows s*(m-1)/8 (r82_sample_konly.cu:345-351): one CTA per sample.
__global__ void gather_kernel(const int8_t* q, const float* xs, const __nv_bfloat16* rope, int8_t* sq, float* sx,
                              __nv_bfloat16* sr, int m, int hidden) {
  const int s = blockIdx.x;
  const int64_t row = int64_t(s) * (m - 1) / (kSamples - 1);
  const int8_t* src = q + row * hidden;
  int8_t* dst = sq + int64_t(s) * hidden;
  if ((hidden & 15) == 0 && (reinterpret_cast<uintptr_t>(q) & 15u) == 0 && (reinterpret_cast<uintptr_t>(sq) & 15u) == 0) {
    for (int i = threadIdx.x; i < hidden / 16; i += blockDim.x)
      reinterpret_cast<uint4*>(dst)[i] = reinterpret_cast<const uint4*>(src)[i];
  } else {
    for (int i = threadIdx.x; i < hidden; i += blockDim.x) dst[i] = src[i];
  }
  for (int i = threadIdx.x; i < kRopeRow; i += blockDim.x) sr[s * kRopeRow + i] = rope[row * kRopeRow + i];
  if (threadIdx.x == 0) sx[s] = xs[row];
}

// V quantiser, step 1 (h3_speedkit/ops/quant_v.py:57-78): per (head, channel) the
// maximum of the tile maxima, scale = max(RN_ftz(max * 0x3C010204), 0x2B8CBCCC)
// (1/127 and 1e-12 as FP32) and inv = rcp.approx.ftz(scale).
__global__ void v_scales_kernel(const float* vp, float* scale, float* inv, int parts) {
  const int h = blockIdx.x, ch = threadIdx.x;
  float mx = 0.f;
  for (int p = 0; p < parts; ++p) mx = fmaxf(mx, vp[(int64_t(h) * parts + p) * kHead + ch]);
  float sc;
  asm("{ .reg .f32 t; mul.rn.ftz.f32 t, %1, 0f3C010204; max.f32 %0, t, 0f2B8CBCCC; }" : "=f"(sc) : "f"(mx));
  scale[h * kHead + ch] = sc;
  inv[h * kHead + ch] = rcp_approx_ftz(sc);
}

// V quantiser, step 2 (quant_v.py:81-104): vi[h*128 + c, dst] =
// cvt.rni.sat.s8(RN_ftz(v[h, src, c] * inv)) with src = dst's bits (b3 b2 b1 b0)
// taken as (b1 b3 b2 b0) inside each run of 16, 0 past m.  One CTA per
// (128-token block, head): the block is staged token-major, the codes are
// assembled channel-major (word w of channel c at c*32 + (w ^ (c & 31)), so the
// lanes of a warp hit distinct banks both when writing and when reading) and
// written as 128-byte rows.
__global__ void __launch_bounds__(kThreads) v_quant_kernel(const __nv_bfloat16* v, const float* inv, int8_t* vi, int m,
                                                            int64_t padded) {
  __shared__ __align__(16) __nv_bfloat16 tile[kTileRows * kHead];
  __shared__ uint32_t codes[kHead * 32];
  const int b = blockIdx.x, h = blockIdx.y;
  const int t0 = b * kTileRows;
  const int rows = min(kTileRows, m - t0);
  const __nv_bfloat16* src = v + (int64_t(h) * m + t0) * kHead;
  for (int i = threadIdx.x; i < kTileRows * (kHead / 8); i += kThreads)
    reinterpret_cast<uint4*>(tile)[i] = i < rows * (kHead / 8) ? reinterpret_cast<const uint4*>(src)[i] : make_uint4(0, 0, 0, 0);
  __syncthreads();
  const int ch = threadIdx.x & (kHead - 1), half = threadIdx.x >> 7;
  const float s = inv[h * kHead + ch];
#pragma unroll 4
  for (int w = half * 16; w < half * 16 + 16; ++w) {
    uint32_t word = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int dst = 4 * w + j;
      const int from = (dst & ~15) | (dst & 1) | ((dst & 2) << 2) | ((dst & 4) >> 1) | ((dst & 8) >> 1);
      const float x = __bfloat162float(tile[from * kHead + ch]);
      float prod;
      int c;
      asm("mul.rn.ftz.f32 %0, %1, %2;" : "=f"(prod) : "f"(x), "f"(s));
      asm("cvt.rni.sat.s8.f32 %0, %1;" : "=r"(c) : "f"(prod));
      word |= (uint32_t(c) & 0xffu) << (8 * j);
    }
    codes[ch * 32 + (w ^ (ch & 31))] = word;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < kHead * 32; i += kThreads) {
    const int c = i >> 5, w = i & 31;
    *reinterpret_cast<uint32_t*>(vi + (int64_t(h) * kHead + c) * padded + t0 + 4 * w) = codes[c * 32 + (w ^ (c & 31))];
  }
}

bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }

// Head epilogue launch over planes [plane0, plane0 + planes).
int launch_heads(const HeadParams& p, int planes, cudaStream_t stream) {
  dim3 grid(p.parts, p.heads, planes);
  heads_kernel<<<grid, kThreads, 0, stream>>>(p);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? 1 : record_failure(e, "h3_qkv: head epilogue launch failed");
}

int qkv_run(const int8_t* A, const int8_t* B, const float* xs, const float* ws, void* D, const void* freqs,
            const void* qw, const void* kw, float eps, int8_t* QI, float* QS, float* VP, int8_t* KI, float* KS,
            const void* SK, const int* anchors, int M, int heads, int hidden, float* rrms, cudaStream_t stream,
            bool sample) {
  if (!A || !B || !xs || !ws || !D || !freqs || !qw || !kw || M < 1 || M > kMaxRows || heads < 1 || hidden < 16 ||
      hidden % 16)
    return record_failure(cudaErrorInvalidValue, "h3_qkv: null operand or shape out of range");
  if (!(eps >= 0.f) || eps > 3.0e38f) return record_failure(cudaErrorInvalidValue, "h3_qkv: eps must be finite and >= 0");
  if (!aligned(D, 16) || !aligned(freqs, 2) || !aligned(qw, 2) || !aligned(kw, 2))
    return record_failure(cudaErrorInvalidValue, "h3_qkv: D must be 16-byte aligned");
  if (!sample) {
    if (!QI || !QS || !VP || !KI || !KS)
      return record_failure(cudaErrorInvalidValue, "h3_qkv: QI, QS, VP, KI and KS are required");
    if (!aligned(QI, 4) || !aligned(KI, 4) || !aligned(QS, 4) || !aligned(KS, 4) || !aligned(VP, 4))
      return record_failure(cudaErrorInvalidValue, "h3_qkv: misaligned quantised outputs");
    if ((SK == nullptr) != (anchors == nullptr))
      return record_failure(cudaErrorInvalidValue, "h3_qkv: SK and anchors go together");
  }
  const int64_t plane = int64_t(heads) * kHead;
  HeadParams p{};
  p.d = static_cast<__nv_bfloat16*>(D);
  p.freqs = static_cast<const __nv_bfloat16*>(freqs);
  p.qw = static_cast<const __nv_bfloat16*>(qw);
  p.kw = static_cast<const __nv_bfloat16*>(kw);
  p.eps = eps;
  p.m = M;
  p.heads = heads;
  p.parts = (M + kTileRows - 1) / kTileRows;
  p.rrms = rrms;
  if (sample) {
    // K plane only: the K rows of the weight and their scales, into D's plane 1.
    void* dk = static_cast<__nv_bfloat16*>(D) + plane * M;
    if (!gemm_dequant_heads(A, B + plane * hidden, xs, ws + plane, dk, M, int(plane), hidden, stream)) return 0;
    p.plane0 = 1;
    p.quant = 0;
    if (!launch_heads(p, 1, stream)) return 0;
  } else {
    if (!gemm_dequant_heads(A, B, xs, ws, D, M, int(3 * plane), hidden, stream)) return 0;
    p.sk = static_cast<const __nv_bfloat16*>(SK);
    p.anchors = anchors;
    p.qi = QI;
    p.qs = QS;
    p.ki = KI;
    p.ks = KS;
    p.vp = VP;
    p.plane0 = 0;
    p.quant = 1;
    if (!launch_heads(p, 3, stream)) return 0;
  }
  record_success();
  return 1;
}

int gather_run(const void* Q, const void* XS, const void* ROPE, void* SQ, void* SX, void* SR, int M, int hidden,
               cudaStream_t stream) {
  if (!Q || !XS || !ROPE || !SQ || !SX || !SR || M < 1 || M > kMaxRows || hidden < 1)
    return record_failure(cudaErrorInvalidValue, "h3_sample_gather: null operand or M out of range");
  if (!aligned(XS, 4) || !aligned(SX, 4) || !aligned(ROPE, 2) || !aligned(SR, 2))
    return record_failure(cudaErrorInvalidValue, "h3_sample_gather: misaligned operand");
  gather_kernel<<<kSamples, 256, 0, stream>>>(static_cast<const int8_t*>(Q), static_cast<const float*>(XS),
                                              static_cast<const __nv_bfloat16*>(ROPE), static_cast<int8_t*>(SQ),
                                              static_cast<float*>(SX), static_cast<__nv_bfloat16*>(SR), M, hidden);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return record_failure(e, "h3_sample_gather: launch failed");
  record_success();
  return 1;
}

}  // namespace qkv
}  // namespace h3sk

#define H3SK_EXPORT extern "C" __attribute__((visibility("default")))

using h3sk::qkv::qkv_run;

H3SK_EXPORT int h3_qkv_quant_kv(const int8_t* A, const int8_t* B, const float* xs, const float* ws, void* D,
                                const void* freqs, const void* qw, const void* kw, float eps, int8_t* QI, float* QS,
                                float* VP, int8_t* KI, float* KS, const void* SK, const int* anchors, int M,
                                uintptr_t stream) {
  return qkv_run(A, B, xs, ws, D, freqs, qw, kw, eps, QI, QS, VP, KI, KS, SK, anchors, M, H3_QKV_HEADS,
                 H3_QKV_HIDDEN, nullptr, reinterpret_cast<cudaStream_t>(stream), false);
}

H3SK_EXPORT int h3_qkv_quant_kv_ex(const int8_t* A, const int8_t* B, const float* xs, const float* ws, void* D,
                                   const void* freqs, const void* qw, const void* kw, float eps, int8_t* QI,
                                   float* QS, float* VP, int8_t* KI, float* KS, const void* SK, const int* anchors,
                                   int M, int heads, int hidden, float* rrms, uintptr_t stream) {
  return qkv_run(A, B, xs, ws, D, freqs, qw, kw, eps, QI, QS, VP, KI, KS, SK, anchors, M, heads, hidden, rrms,
                 reinterpret_cast<cudaStream_t>(stream), false);
}

H3SK_EXPORT int h3_sample_konly(const int8_t* A, const int8_t* B, const float* xs, const float* ws, void* D,
                                const void* freqs, const void* qw, const void* kw, float eps, int8_t* QI, float* QS,
                                float* VP, int M, uintptr_t stream) {
  (void)QI;
  (void)QS;
  (void)VP;
  if (M != H3_QKV_SAMPLES) return h3sk::record_failure(cudaErrorInvalidValue, "h3_sample_konly: M must be 9");
  return qkv_run(A, B, xs, ws, D, freqs, qw, kw, eps, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr,
                 M, H3_QKV_HEADS, H3_QKV_HIDDEN, nullptr, reinterpret_cast<cudaStream_t>(stream), true);
}

H3SK_EXPORT int h3_sample_konly_ex(const int8_t* A, const int8_t* B, const float* xs, const float* ws, void* D,
                                   const void* freqs, const void* qw, const void* kw, float eps, int M, int heads,
                                   int hidden, float* rrms, uintptr_t stream) {
  return qkv_run(A, B, xs, ws, D, freqs, qw, kw, eps, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr,
                 M, heads, hidden, rrms, reinterpret_cast<cudaStream_t>(stream), true);
}

H3SK_EXPORT int h3_sample_gather(const void* Q, const void* XS, const void* ROPE, void* SQ, void* SX, void* SR, int M,
                                 uintptr_t stream) {
  return h3sk::qkv::gather_run(Q, XS, ROPE, SQ, SX, SR, M, H3_QKV_HIDDEN, reinterpret_cast<cudaStream_t>(stream));
}

H3SK_EXPORT int h3_sample_gather_ex(const void* Q, const void* XS, const void* ROPE, void* SQ, void* SX, void* SR,
                                    int M, int hidden, uintptr_t stream) {
  return h3sk::qkv::gather_run(Q, XS, ROPE, SQ, SX, SR, M, hidden, reinterpret_cast<cudaStream_t>(stream));
}

H3SK_EXPORT int h3_quant_v(const float* VP, const void* V, void* VI, float* VS, float* VINV, int M, int heads,
                           uintptr_t stream) {
  using namespace h3sk::qkv;
  if (!VP || !V || !VI || !VS || !VINV || M < 1 || M > kMaxRows || heads < 1)
    return h3sk::record_failure(cudaErrorInvalidValue, "h3_quant_v: null operand or shape out of range");
  if (!aligned(V, 16) || !aligned(VI, 4) || !aligned(VS, 4) || !aligned(VINV, 4) || !aligned(VP, 4))
    return h3sk::record_failure(cudaErrorInvalidValue, "h3_quant_v: misaligned operand");
  const cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int parts = (M + kTileRows - 1) / kTileRows;
  v_scales_kernel<<<heads, kHead, 0, s>>>(VP, VS, VINV, parts);
  v_quant_kernel<<<dim3(parts, heads), kThreads, 0, s>>>(static_cast<const __nv_bfloat16*>(V), VINV,
                                                        static_cast<int8_t*>(VI), M, int64_t(parts) * kTileRows);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return h3sk::record_failure(e, "h3_quant_v: launch failed");
  h3sk::record_success();
  return 1;
}
