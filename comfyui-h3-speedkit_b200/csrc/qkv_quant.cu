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
#include <mutex>

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

__device__ __forceinline__ float warp_max(float x) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) x = fmaxf(x, __shfl_xor_sync(0xffffffffu, x, off));
  return x;
}

__device__ __forceinline__ float lo_f(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float hi_f(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }
// Two floats -> one BF16 pair word, round to nearest even (low half = lo).
__device__ __forceinline__ uint32_t bf2(float lo, float hi) {
  uint32_t w;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(w) : "f"(hi), "f"(lo));
  return w;
}
__device__ __forceinline__ void unpack8(const uint4 u, float* v) {
  v[0] = lo_f(u.x); v[1] = hi_f(u.x); v[2] = lo_f(u.y); v[3] = hi_f(u.y);
  v[4] = lo_f(u.z); v[5] = hi_f(u.z); v[6] = lo_f(u.w); v[7] = hi_f(u.w);
}
// Codes of four values: cvt.rni.s32 then a saturating pack is cvt.rni.sat.s8
// (round half to even, clamp to [-128, 127], NaN -> 0) four at a time.
__device__ __forceinline__ uint32_t codes4(float a, float b, float c, float d, float inv) {
  int ia, ib, ic, id;
  asm("cvt.rni.s32.f32 %0, %1;" : "=r"(ia) : "f"(a * inv));
  asm("cvt.rni.s32.f32 %0, %1;" : "=r"(ib) : "f"(b * inv));
  asm("cvt.rni.s32.f32 %0, %1;" : "=r"(ic) : "f"(c * inv));
  asm("cvt.rni.s32.f32 %0, %1;" : "=r"(id) : "f"(d * inv));
  uint32_t hi, word;
  asm("cvt.pack.sat.s8.s32.b32 %0, %1, %2, %3;" : "=r"(hi) : "r"(id), "r"(ic), "r"(0));
  asm("cvt.pack.sat.s8.s32.b32 %0, %1, %2, %3;" : "=r"(word) : "r"(ib), "r"(ia), "r"(hi));
  return word;
}

// Rotation of one 128-channel row held by two threads, 64 channels each (thread
// `half` owns channels 64*half + j, j = 0..63); the partner is lane ^ 1.  The
// stages run in the reference's order -- sign flips, the 4-point block on channel
// bits 0-1 ((a0 + a2) * 0.5 ...), butterflies on channel bits 2, 3, 4, 5 in
// registers and bit 6 across the pair, each lo' = lo + hi, hi' = lo - hi, then the
// factor 0.1767766952966369f -- so every value meets the same IEEE operations
// with the same operands as in the reference's 4-channels-per-lane form.
__device__ __forceinline__ void rotate64(float (&v)[64], int half, bool full) {
  if (full) {
    // flip channel ch when bit (ch & 31) of word ch >> 5 is clear.  Per register j
    // both halves' flips are compile-time constants: equal ones become a negation
    // (folded into the adds below), differing ones an XOR with the half's mask.
    const uint32_t hmask = half ? 0x80000000u : 0u;
#pragma unroll
    for (int j = 0; j < 64; ++j) {
      const uint32_t w0 = j < 32 ? 0x1035997bu : 0x8087f5eeu;   // channels j (half 0)
      const uint32_t w1 = j < 32 ? 0xee2e4e1au : 0x71132418u;   // channels 64 + j (half 1)
      const bool f0 = ((w0 >> (j & 31)) & 1u) == 0u, f1 = ((w1 >> (j & 31)) & 1u) == 0u;
      if (f0 && f1) {
        v[j] = -v[j];
      } else if (f0 != f1) {
        v[j] = __uint_as_float(__float_as_uint(v[j]) ^ (f1 ? hmask : (hmask ^ 0x80000000u)));
      }
    }
  }
#pragma unroll
  for (int j = 0; j < 64; j += 4) {
    const float a0 = v[j] + v[j + 1], a1 = v[j] - v[j + 1], a2 = v[j + 2] + v[j + 3], a3 = v[j + 2] - v[j + 3];
    v[j] = (a0 + a2) * 0.5f;
    v[j + 1] = (a1 + a3) * 0.5f;
    v[j + 2] = (a0 - a2) * 0.5f;
    v[j + 3] = (a1 - a3) * 0.5f;
  }
  if (!full) return;
#pragma unroll
  for (int bit = 4; bit < 64; bit <<= 1) {
#pragma unroll
    for (int j = 0; j < 64; ++j) {
      if (j & bit) continue;
      const float lo = v[j], hi = v[j | bit];
      v[j] = lo + hi;
      v[j | bit] = lo - hi;
    }
  }
  // bit 6: the partner holds the other half; lo + hi on half 0, lo - hi on half 1
  // (fmaf(v, -1, other) = RN(other - v): the product is exact).
  const float sgn = half ? -1.f : 1.f;
#pragma unroll
  for (int j = 0; j < 64; ++j) {
    const float other = __shfl_xor_sync(0xffffffffu, v[j], 1);
    v[j] = fmaf(v[j], sgn, other) * 0.1767766952966369f;
  }
}

// uint4 slot of 16-byte chunk c (0..15) of tile row r: the chunk's low three bits
// are XORed with (r ^ (r >> 1) ^ (r >> 2) ^ 3h) & 7, h = c >> 3 the chunk's half.
// A 16-byte shared access is served eight lanes at a time; counted over every
// access pattern below (pairs of threads per row in phase 1, the Q and K row
// groups of phase 2, the V column scan, the row-linear copies) this key needs
// 1920 such wavefronts against a conflict-free floor of 1536 (no swizzle: 6656;
// the key without the 3h term: 2432, as both threads of a row then meet in one
// bank group).
__device__ __forceinline__ int slot(int r, int c) {
  return r * 16 + (c ^ ((r ^ (r >> 1) ^ (r >> 2) ^ (3 * (c >> 3))) & 7));
}

constexpr int kSlabChunks = kTileRows * kHead / 8;   // 16-byte chunks of one slab (32 KB)
constexpr int kHeadsSmem = 2 * kSlabChunks * 16;      // two slabs in flight per CTA

// Work item idx: plane-major, then head, then 128-row tile.
struct Item {
  int g, h, tm;
};
__device__ __forceinline__ Item item_of(const HeadParams& p, int idx) {
  const int per_plane = p.heads * p.parts;
  const int rem = idx % per_plane;
  return Item{p.plane0 + idx / per_plane, rem / p.parts, rem % p.parts};
}
__device__ __forceinline__ __nv_bfloat16* slab_of(const HeadParams& p, const Item& it) {
  return p.d + ((int64_t(it.g) * p.heads + it.h) * p.m + int64_t(it.tm) * kTileRows) * kHead;
}

// Asynchronous copy of item idx's slab into `buf` (16-byte cp.async per chunk,
// swizzled slots); the caller commits the group.
__device__ __forceinline__ void prefetch(const HeadParams& p, int idx, uint4* buf) {
  const Item it = item_of(p, idx);
  const int rows = min(kTileRows, p.m - it.tm * kTileRows);
  const uint4* src = reinterpret_cast<const uint4*>(slab_of(p, it));
  const uint32_t base = uint32_t(__cvta_generic_to_shared(buf));
  for (int i = threadIdx.x; i < rows * (kHead / 8); i += kThreads)
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(base + uint32_t(slot(i >> 4, i & 15)) * 16u),
                 "l"(src + i)
                 : "memory");
}

// Finish one slab already in shared memory.  Every early return is uniform
// across the CTA (it depends on the item and the parameters only).
__device__ __forceinline__ void process(const HeadParams& p, const Item& it, uint4* tile4, float* group_max,
                                        uint4* v_part) {
  const int tm = it.tm, h = it.h, g = it.g;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, half = lane & 1;
  const int r0 = tm * kTileRows;
  const int rows = min(kTileRows, p.m - r0);
  __nv_bfloat16* slab = slab_of(p, it);

  if (g == 2) {
    // V: column maxima of the |BF16| bit patterns.  Thread (chunk c, row group
    // rg) folds 8 rows of 8 channels with packed 16-bit maxima; lanes c and
    // c + 16 of a warp, then the 8 warps through shared memory, are combined.
    if (p.vp == nullptr) return;
    const int c = threadIdx.x & 15, rg = threadIdx.x >> 4;
    uint32_t m4[4] = {0u, 0u, 0u, 0u};
    const int end = min(rows, rg * 8 + 8);
    for (int tr = rg * 8; tr < end; ++tr) {
      const uint4 u = tile4[slot(tr, c)];
      m4[0] = __vmaxu2(m4[0], u.x & 0x7fff7fffu);
      m4[1] = __vmaxu2(m4[1], u.y & 0x7fff7fffu);
      m4[2] = __vmaxu2(m4[2], u.z & 0x7fff7fffu);
      m4[3] = __vmaxu2(m4[3], u.w & 0x7fff7fffu);
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) m4[k] = __vmaxu2(m4[k], __shfl_xor_sync(0xffffffffu, m4[k], 16));
    if (lane < 16) v_part[warp * 16 + c] = make_uint4(m4[0], m4[1], m4[2], m4[3]);
    __syncthreads();
    if (threadIdx.x < kHead) {
      const int ch = threadIdx.x;
      uint32_t mx = 0;
#pragma unroll
      for (int w = 0; w < kThreads / 32; ++w) {
        const uint32_t* part = reinterpret_cast<const uint32_t*>(&v_part[w * 16 + (ch >> 3)]);
        const uint32_t word = part[(ch & 7) >> 1];
        const uint32_t mag = (ch & 1) ? (word >> 16) : (word & 0xffffu);
        mx = mag > mx ? mag : mx;
      }
      p.vp[(int64_t(h) * p.parts + tm) * kHead + ch] = __uint_as_float(mx << 16);
    }
    return;
  }

  // ---- phase 1: RMS over the head, weight, RoPE (row tr, thread half `half`) ----
  const __nv_bfloat16* w = g == 0 ? p.qw : p.kw;
  {
    const int tr = threadIdx.x >> 1;
    const bool live = tr < rows;                       // whole pairs: the pair stays converged
    // chains l = 16*half + j over channels l, l + 32, l + 64, l + 96 in that order
    float ch[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) ch[j] = 0.f;
    if (live) {
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        float x[16];
        unpack8(tile4[slot(tr, 4 * c + 2 * half)], x);
        unpack8(tile4[slot(tr, 4 * c + 2 * half + 1)], x + 8);
#pragma unroll
        for (int j = 0; j < 16; ++j) ch[j] = fmaf(x[j], x[j], ch[j]);
      }
    }
    __syncwarp();   // every RMS read of the row precedes the partner's writes below
    // the shfl_down tree of the reference: off 16 across the pair, 8..1 in registers
#pragma unroll
    for (int j = 0; j < 16; ++j) ch[j] += __shfl_xor_sync(0xffffffffu, ch[j], 1);
#pragma unroll
    for (int off = 8; off > 0; off >>= 1)
#pragma unroll
      for (int j = 0; j < off; ++j) ch[j] += ch[j + off];
    const float sum = __shfl_sync(0xffffffffu, ch[0], lane & ~1);
    const float rrms = rsqrtf(sum / 128.f + p.eps);
    if (live) {
      const int row = r0 + tr;
      if (p.rrms != nullptr && half == 0) p.rrms[(int64_t(g) * p.heads + h) * p.m + row] = rrms;
      const uint4* w4 = reinterpret_cast<const uint4*>(w);
      const uint4* f4 = reinterpret_cast<const uint4*>(p.freqs + int64_t(row) * kRopeRow) + 12 * half;
      // pairs d = 24*half + 8q + i, partner d + 48: one uint4 of x0, x1, w0, w1 and
      // four uint4 of RoPE coefficients (a, b, c, e per pair) per q
#pragma unroll
      for (int q = 0; q < 3; ++q) {
        const int v0 = 3 * half + q, v1 = 6 + 3 * half + q;       // uint4 index of d and d + 48
        float x0[8], x1[8], w0[8], w1[8];
        unpack8(tile4[slot(tr, v0)], x0);
        unpack8(tile4[slot(tr, v1)], x1);
        unpack8(w4[v0], w0);
        unpack8(w4[v1], w1);
        uint32_t y0[4], y1[4];
#pragma unroll
        for (int i = 0; i < 8; i += 2) {
          const uint4 f = f4[4 * q + i / 2];
          float a[2], b[2];
#pragma unroll
          for (int k = 0; k < 2; ++k) {
            a[k] = __bfloat162float(__float2bfloat16_rn(x0[i + k] * rrms * w0[i + k]));
            b[k] = __bfloat162float(__float2bfloat16_rn(x1[i + k] * rrms * w1[i + k]));
          }
          // pair i: (f.x, f.y) = (a_c, b_c | c_c, e_c); pair i + 1: (f.z, f.w)
          y0[i / 2] = bf2(lo_f(f.x) * a[0] + hi_f(f.x) * b[0], lo_f(f.z) * a[1] + hi_f(f.z) * b[1]);
          y1[i / 2] = bf2(lo_f(f.y) * a[0] + hi_f(f.y) * b[0], lo_f(f.w) * a[1] + hi_f(f.w) * b[1]);
        }
        tile4[slot(tr, v0)] = make_uint4(y0[0], y0[1], y0[2], y0[3]);
        tile4[slot(tr, v1)] = make_uint4(y1[0], y1[1], y1[2], y1[3]);
      }
      // tail channels 96 + 16*half .. +16: normalised and weighted only
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        const int vi = 12 + 2 * half + q;
        float x[8], wt[8];
        unpack8(tile4[slot(tr, vi)], x);
        unpack8(w4[vi], wt);
        uint32_t o[4];
#pragma unroll
        for (int i = 0; i < 8; i += 2) o[i / 2] = bf2(x[i] * rrms * wt[i], x[i + 1] * rrms * wt[i + 1]);
        tile4[slot(tr, vi)] = make_uint4(o[0], o[1], o[2], o[3]);
      }
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < rows * (kHead / 8); i += kThreads)
    reinterpret_cast<uint4*>(slab)[i] = tile4[slot(i >> 4, i & 15)];
  if (!p.quant) return;
  if (g == 0 ? (p.qi == nullptr || p.qs == nullptr) : (p.ki == nullptr || p.ks == nullptr)) return;

  // ---- phase 2: rotation and codes; row tr, channels 64*half .. +64 ----
  // Q: lanes 8s..8s+7 of warp w hold the 4 rows {base + 8j} of group 4w + s;
  // K: warps 2kg, 2kg+1 hold the 32 rows {tr : tr % 8 in {2kg, 2kg+1}} of group kg.
  int tr, group;
  if (g == 0) {
    group = 4 * warp + (lane >> 3);
    tr = (group >> 3) * 32 + (group & 7) + 8 * ((lane >> 1) & 3);
  } else {
    group = warp >> 1;
    const int r_in = (warp & 1) * 16 + (lane >> 1);
    tr = (r_in >> 1) * 8 + group * 2 + (r_in & 1);
  }
  const bool live = tr < rows;
  float v[64];
  if (live) {
#pragma unroll
    for (int q = 0; q < 8; ++q) unpack8(tile4[slot(tr, 8 * half + q)], v + 8 * q);
    if (g == 1 && p.anchors != nullptr && p.sk != nullptr) {
      const int anchor = p.anchors[h];
      if (anchor >= 0 && anchor < kSamples) {   // an out-of-range anchor reads nothing
        const uint4* s4 = reinterpret_cast<const uint4*>(p.sk + (int64_t(h) * kSamples + anchor) * kHead) + 8 * half;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          float b[8];
          unpack8(s4[q], b);
#pragma unroll
          for (int i = 0; i < 8; ++i) v[8 * q + i] = v[8 * q + i] - b[i];
        }
      }
    }
  } else {
#pragma unroll
    for (int j = 0; j < 64; ++j) v[j] = 0.f;
  }
  rotate64(v, half, p.m > 256);
  float mx = 0.f;
#pragma unroll
  for (int j = 0; j < 64; ++j) mx = fmaxf(mx, fabsf(v[j]));
  float sc, inv;
  if (g == 0) {
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
    sc = fmaf(mx, 1.f / 127.f, 1e-7f);
    inv = rcp_approx_ftz(sc);
    if ((lane & 7) == 0) p.qs[int64_t(h) * p.parts * 32 + tm * 32 + group] = sc;
  } else {
    mx = warp_max(mx);
    if (lane == 0) group_max[warp] = mx;
    __syncthreads();
    mx = fmaxf(group_max[warp & ~1], group_max[warp | 1]);
    sc = fmaf(mx, 1.f / 127.f, 1e-7f);
    inv = rcp_approx_ftz(sc);
    if (threadIdx.x == 64 * group) p.ks[(int64_t(h) * p.parts + tm) * 4 + group] = sc;
  }
  if (live) {
    int8_t* out = (g == 0 ? p.qi : p.ki) + (int64_t(h) * p.m + r0 + tr) * kHead + 64 * half;
#pragma unroll
    for (int q = 0; q < 4; ++q)
      reinterpret_cast<uint4*>(out)[q] =
          make_uint4(codes4(v[16 * q], v[16 * q + 1], v[16 * q + 2], v[16 * q + 3], inv),
                     codes4(v[16 * q + 4], v[16 * q + 5], v[16 * q + 6], v[16 * q + 7], inv),
                     codes4(v[16 * q + 8], v[16 * q + 9], v[16 * q + 10], v[16 * q + 11], inv),
                     codes4(v[16 * q + 12], v[16 * q + 13], v[16 * q + 14], v[16 * q + 15], inv));
  }
}

// Persistent: CTA b takes items b, b + grid, ...; the slab of the next item is
// copied into the other buffer while this one is finished.
__global__ void __launch_bounds__(kThreads, 2) heads_kernel(const HeadParams p, int items) {
  extern __shared__ __align__(16) uint4 heads_smem[];
  __shared__ float group_max[kThreads / 32];
  __shared__ uint4 v_part[(kThreads / 32) * 16];
  int idx = blockIdx.x;
  if (idx < items) prefetch(p, idx, heads_smem);
  asm volatile("cp.async.commit_group;" ::: "memory");
  for (int k = 0; idx < items; ++k, idx += gridDim.x) {
    const int next = idx + int(gridDim.x);
    if (next < items) prefetch(p, next, heads_smem + ((k + 1) & 1) * kSlabChunks);
    asm volatile("cp.async.commit_group;" ::: "memory");
    asm volatile("cp.async.wait_group 1;" ::: "memory");   // this item's slab has landed
    __syncthreads();
    process(p, item_of(p, idx), heads_smem + (k & 1) * kSlabChunks, group_max, v_part);
    __syncthreads();   // the buffer is free before the next prefetch refills it
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
  const int64_t items = int64_t(planes) * p.heads * p.parts;
  int grid = 0;
  cudaError_t e = rq_persistent_grid(reinterpret_cast<const void*>(heads_kernel), kThreads, kHeadsSmem, items, &grid);
  if (e != cudaSuccess) return record_failure(e, "h3_qkv: head epilogue occupancy query failed");
  heads_kernel<<<grid, kThreads, kHeadsSmem, stream>>>(p, int(items));
  e = cudaGetLastError();
  return e == cudaSuccess ? 1 : record_failure(e, "h3_qkv: head epilogue launch failed");
}

// Every host-side check of one QKV call, the GEMM's operand rules included
// (A, B, D 16-byte aligned; scales 4-byte aligned), so that a caller running
// several launches can validate all of them before it enqueues the first.
// Returns 1, or 0 after recording the reason.
int qkv_check(const int8_t* A, const int8_t* B, const float* xs, const float* ws, const void* D, const void* freqs,
              const void* qw, const void* kw, float eps, const int8_t* QI, const float* QS, const float* VP,
              const int8_t* KI, const float* KS, const void* SK, const int* anchors, int M, int heads, int hidden,
              bool sample) {
  if (!A || !B || !xs || !ws || !D || !freqs || !qw || !kw || M < 1 || M > kMaxRows || heads < 1 || hidden < 16 ||
      hidden % 16)
    return record_failure(cudaErrorInvalidValue, "h3_qkv: null operand or shape out of range");
  if (!(eps >= 0.f) || eps > 3.0e38f) return record_failure(cudaErrorInvalidValue, "h3_qkv: eps must be finite and >= 0");
  if (!aligned(D, 16) || !aligned(freqs, 2) || !aligned(qw, 2) || !aligned(kw, 2))
    return record_failure(cudaErrorInvalidValue, "h3_qkv: D must be 16-byte aligned");
  if (!aligned(A, 16) || !aligned(B, 16) || !aligned(xs, 4) || !aligned(ws, 4))
    return record_failure(cudaErrorInvalidValue, "h3_qkv: A and B must be 16-byte aligned, xs and ws FP32");
  if (!sample) {
    if (!QI || !QS || !VP || !KI || !KS)
      return record_failure(cudaErrorInvalidValue, "h3_qkv: QI, QS, VP, KI and KS are required");
    if (!aligned(QI, 4) || !aligned(KI, 4) || !aligned(QS, 4) || !aligned(KS, 4) || !aligned(VP, 4))
      return record_failure(cudaErrorInvalidValue, "h3_qkv: misaligned quantised outputs");
    if ((SK == nullptr) != (anchors == nullptr))
      return record_failure(cudaErrorInvalidValue, "h3_qkv: SK and anchors go together");
  }
  return 1;
}

int qkv_run(const int8_t* A, const int8_t* B, const float* xs, const float* ws, void* D, const void* freqs,
            const void* qw, const void* kw, float eps, int8_t* QI, float* QS, float* VP, int8_t* KI, float* KS,
            const void* SK, const int* anchors, int M, int heads, int hidden, float* rrms, cudaStream_t stream,
            bool sample) {
  if (!qkv_check(A, B, xs, ws, D, freqs, qw, kw, eps, QI, QS, VP, KI, KS, SK, anchors, M, heads, hidden, sample))
    return 0;
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
  } else if (rrms == nullptr && heads % 2 == 0) {
    // The head epilogue inside the GEMM's epilogue warps: no Q/K plane round trip.
    HeadsArgs hd{};
    hd.freqs = p.freqs;
    hd.qw = p.qw;
    hd.kw = p.kw;
    hd.sk = static_cast<const __nv_bfloat16*>(SK);
    hd.anchors = anchors;
    hd.qi = QI;
    hd.qs = QS;
    hd.ki = KI;
    hd.ks = KS;
    hd.vp = VP;
    hd.eps = eps;
    hd.heads = heads;
    hd.parts = p.parts;
    if (!gemm_qkv_heads(A, B, xs, ws, D, M, hidden, hd, stream)) return 0;
  } else {
    // Odd head counts (a 256-column tile would straddle two heads' planes) and the
    // rrms debug output: the GEMM writes the planes, a second kernel finishes them.
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

// ---- allocation-free whole-op entry point ------------------------------------------
// For callers that may not allocate device memory at run time: a serving loop
// that must not call cudaMalloc after warm-up (the call can synchronise the
// device and stall every other stream), or a host framework that owns all device
// memory through its own pool and hands this library only the operands and
// outputs.  The op's intermediates (sample rows, their K plane, anchors, V
// reciprocal scales) live in one file-scope device array instead of allocated
// buffers.  Its size bounds the geometry: heads <= 64, hidden <= 8192 (the H3
// geometry is 56 x 5376); every GPU that loads the library holds the array
// until the process exits.
namespace h3sk {
namespace qkv {

constexpr int kNoAllocMaxHeads = 64;
constexpr int kNoAllocMaxHidden = 8192;
constexpr size_t pad256(size_t x) { return (x + 255) & ~size_t(255); }
constexpr size_t kSqOff = 0;
constexpr size_t kSxOff = kSqOff + pad256(size_t(kSamples) * kNoAllocMaxHidden);
constexpr size_t kSrOff = kSxOff + pad256(kSamples * 4);
constexpr size_t kSdOff = kSrOff + pad256(size_t(kSamples) * kRopeRow * 2);
constexpr size_t kAnchorOff = kSdOff + pad256(size_t(3) * kNoAllocMaxHeads * kSamples * kHead * 2);
constexpr size_t kVinvOff = kAnchorOff + pad256(size_t(kNoAllocMaxHeads) * 4);
constexpr size_t kScratchBytes = kVinvOff + pad256(size_t(kNoAllocMaxHeads) * kHead * 4);   // 552,960 B

static __device__ __align__(256) unsigned char g_scratch[kScratchBytes];

// Device address of g_scratch on the current device.  In host code the name
// g_scratch is only a host-side stand-in, so the address is looked up with
// cudaGetSymbolAddress, once per device, on the first call made with that
// device current, and cached for the life of the process.  The cache is not
// refreshed: after cudaDeviceReset (which destroys the context holding the
// array) the cached address is stale, so this entry point must not be used
// after a reset in the same process.
unsigned char* scratch_base() {
  static std::mutex mu;
  static unsigned char* base[64] = {};
  int device = 0;
  if (cudaGetDevice(&device) != cudaSuccess || device < 0 || device >= 64) return nullptr;
  std::lock_guard<std::mutex> lock(mu);
  if (base[device] == nullptr) {
    void* ptr = nullptr;
    if (cudaGetSymbolAddress(&ptr, g_scratch) != cudaSuccess) return nullptr;
    base[device] = static_cast<unsigned char*>(ptr);
  }
  return base[device];
}

}  // namespace qkv
}  // namespace h3sk

H3SK_EXPORT int h3_qkv_noalloc(const int8_t* A, const int8_t* B, const float* xs, const float* ws, void* D,
                               const void* freqs, const void* qw, const void* kw, float eps, int8_t* QI, float* QS,
                               float* VP, int8_t* KI, float* KS, void* VI, float* VS, int M, int heads, int hidden,
                               uintptr_t stream) {
  using namespace h3sk::qkv;
  if (heads < 1 || heads > kNoAllocMaxHeads || hidden < 16 || hidden > kNoAllocMaxHidden || hidden % 16)
    return h3sk::record_failure(cudaErrorInvalidValue, "h3_qkv_noalloc: heads <= 64 and hidden <= 8192 (hidden % 16 == 0)");
  // All checks of the five steps run here, before the first launch, so that a
  // rejected call leaves every output untouched.  The sample steps read only
  // caller operands checked below and the aligned scratch array.
  if (!qkv_check(A, B, xs, ws, D, freqs, qw, kw, eps, QI, QS, VP, KI, KS, nullptr, nullptr, M, heads, hidden, false))
    return 0;
  if (!VI || !VS || !aligned(VI, 4) || !aligned(VS, 4))
    return h3sk::record_failure(cudaErrorInvalidValue, "h3_qkv_noalloc: VI and VS must be non-null and 4-byte aligned");
  unsigned char* base = scratch_base();
  if (base == nullptr) return h3sk::record_failure(cudaErrorInvalidSymbol, "h3_qkv_noalloc: scratch address");
  const cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  int8_t* sq = reinterpret_cast<int8_t*>(base + kSqOff);
  float* sx = reinterpret_cast<float*>(base + kSxOff);
  __nv_bfloat16* sr = reinterpret_cast<__nv_bfloat16*>(base + kSrOff);
  __nv_bfloat16* sd = reinterpret_cast<__nv_bfloat16*>(base + kSdOff);
  const __nv_bfloat16* sk = sd + size_t(heads) * kSamples * kHead;   // plane 1 of [3, heads, 9, 128]
  int* anchors = reinterpret_cast<int*>(base + kAnchorOff);
  float* vinv = reinterpret_cast<float*>(base + kVinvOff);
  // Every scratch word is written before it is read, so nothing is cleared.
  if (!gather_run(A, xs, freqs, sq, sx, sr, M, hidden, s)) return 0;
  if (!qkv_run(sq, B, sx, ws, sd, sr, qw, kw, eps, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr,
               kSamples, heads, hidden, nullptr, s, true))
    return 0;
  if (!h3_sample_anchor_ex(sk, anchors, heads, stream)) return 0;
  if (!qkv_run(A, B, xs, ws, D, freqs, qw, kw, eps, QI, QS, VP, KI, KS, sk, anchors, M, heads, hidden, nullptr, s,
               false))
    return 0;
  const void* v_plane = static_cast<const __nv_bfloat16*>(D) + size_t(2) * heads * M * kHead;
  return h3_quant_v(VP, v_plane, VI, VS, vinv, M, heads, stream);
}
