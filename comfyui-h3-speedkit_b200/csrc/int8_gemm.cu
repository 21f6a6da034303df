// INT8 GEMM for B200 (sm_100a): D = epilogue(A[M,K] . B[N,K]^T) with int32
// accumulation in tensor memory.
//
// Design (one persistent CTA per SM, 10 warps; M > 128 runs CTA pairs, see Shape):
//   warp 0      TMA producer: 128x128-byte A tiles and B tiles (256 rows, or the
//               CTA's 128-row half in a pair), 128-byte swizzle, into a shared-
//               memory ring guarded by full/empty mbarriers.  No multicast.
//   warp 1      allocates 512 TMEM columns (two 128x256 int32 accumulators) and
//               issues tcgen05.mma.kind::i8 (N=256, K=32; four per stage; M=256
//               over both CTAs of a pair) from one thread; tcgen05.commit frees
//               each smem stage and publishes each finished accumulator.
//   warps 2-9   epilogue: warp w reads TMEM lane quarter w % 4 and column half
//               (w - 2) / 4, 32 columns per tcgen05.ld; dequantise, apply the
//               fused epilogue (bias, GELU, gate-residual, raw int32, the QKV
//               head epilogue, or the dequant / GELU values followed by the next
//               quantiser's ConvRot256 of the tile's 256-column group) and store.
//               The second accumulator lets the epilogue of tile t overlap the
//               mainloop of tile t+1 (in the dual form a unit's two tiles use
//               both accumulators and the epilogue does not overlap).
// Tiles are visited weight-stationary: in groups of `group_n` N-tiles, whose
// slice of B (group_n x 256 rows x K bytes, at most kBSliceBytes) stays in L2
// while the group sweeps every M-tile, N-tile fastest.  A is then read from
// DRAM once per N-group (once when all of B fits), B about once; a wave of
// CTAs shares each A tile in L2.  Slices of 32 MB measured best (DRAM reads at
// M=98304: QKV 1.05 GB, FC1 1.37 GB, FC2 8.0 GB); 64 MB slices do not stay
// resident (FC1 7.1 GB).  Grouping 16 M-tiles with M fastest, the earlier
// order, re-read B once per group and, at K = 16384, thrashed A (FC2 15.5 GB
// for 2.5 GB of operands); the DRAM power that costs lowers the capped clock.  Every mbarrier wait is bounded; a wait
// that runs out stops the CTA cleanly and records a status code (see
// h3sk_pipeline_status).
//
// Epilogue arithmetic (non-fast-math TU, explicit round-to-nearest intrinsics):
//   y   = bf(__fadd_rn(__fmul_rn(__fmul_rn(float(acc), xs[m]), ws[n]), bias[n]))
//         kernels/gemm/fc1.cu:83-90 (EVT multiplies, plus 0) and the explicit form
//         of kernels/gemm/r84_kfourwarp.cu:240-241;
//   gate: out = bf(__fmaf_rn(y, gate[rows[m]][n], residual[m][n]))
//         kernels/gemm/gate.cu:33-41, 100-104 and indexed_gate.cuh:85-87;
//   GELU: out = bf(gelu_tanh(y)), the formula of convrot64_exact.cuh:913-923.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <cmath>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "host_util.h"
#include "sm100.cuh"
#include "../../include/h3sk_b200.h"

namespace h3sk {

cudaError_t convrot_quant_none(const void* x, int64_t xs, void* q, void* scale, int64_t rows, int k,
                               cudaStream_t stream);

namespace {

using namespace sm100;

constexpr int kBM = 128;            // tile rows per CTA (TMEM lanes)
constexpr int kBN = 256;            // tile columns (TMEM columns per accumulator)
constexpr int kBK = 128;            // K bytes per stage (one 128-byte swizzle row)
constexpr int kUmmaK = 32;          // K of one kind::i8 MMA
constexpr int kATileBytes = kBM * kBK;
constexpr int kEpilogueWarps = 8;    // two per TMEM lane quarter, one per column half
constexpr int kEpilogueThreads = 32 * kEpilogueWarps;
constexpr int kThreads = 64 + kEpilogueThreads;
constexpr int kTmemCols = 512;
constexpr int kDualMinK = 8192;     // K from which the dual (two N-tiles per unit) form is used
constexpr int kDualMinWaves = 8;    // ... when its units fill at least this many waves of pairs
// Pipeline depths (operand stages of the CTA-pair and dual forms), output
// staging buffers per epilogue warp (2: a chunk's store may still be reading one
// buffer while the next chunk fills the other) and TMEM load prefetch (the next
// chunk's tcgen05.ld is issued before the current chunk is computed; 1: every
// form, 2: the dual form only, whose epilogue the MMA waits for).  Measured on
// the cfg5 stack (M = 98304): prefetch shortens the dual FC2 by ~1 % and slows
// the overlapped FC1 by ~2 %; 5 vs 6 stages and double staging are within noise.
#ifndef H3SK_PAIR_STAGES
#define H3SK_PAIR_STAGES 6
#endif
#ifndef H3SK_DUAL_STAGES
#define H3SK_DUAL_STAGES 4
#endif
#ifndef H3SK_STAGE_BUFS
#define H3SK_STAGE_BUFS 1
#endif
#ifndef H3SK_TMEM_PREFETCH
#define H3SK_TMEM_PREFETCH 2
#endif
#ifndef H3SK_BSLICE_MB
#define H3SK_BSLICE_MB 32
#endif
#ifndef H3SK_DUAL_BSLICE_MB
#define H3SK_DUAL_BSLICE_MB 32
#endif
// B bytes an N-group keeps in L2: single-tile units (measured best: 32 MB) and
// dual units (two N-tiles per unit, the long-K form).
constexpr int64_t kBSliceBytes = int64_t(H3SK_BSLICE_MB) << 20;
constexpr int64_t kDualBSliceBytes = int64_t(H3SK_DUAL_BSLICE_MB) << 20;
constexpr uint64_t kWaitTimeoutNs = 2000000000ull;   // 2 s per wait

enum : int {
  kEpiDequant = 0, kEpiGelu = 1, kEpiGate = 2, kEpiAcc = 3, kEpiHeads = 4,
  kEpiGeluRot = 5,      // GELU, then the next quantiser's ConvRot256 of every tile
  kEpiDequantRot = 6,   // dequant, and ConvRot256 of the tiles from column rot_n0 on
  kEpiKinds = 7
};
// Epilogues that rotate 256-column tiles for the next quantiser, and the plain
// epilogue they apply first.
__host__ __device__ constexpr bool is_rot(int epi) { return epi == kEpiGeluRot || epi == kEpiDequantRot; }
__host__ __device__ constexpr int base_epi(int epi) {
  return epi == kEpiGeluRot ? kEpiGelu : (epi == kEpiDequantRot ? kEpiDequant : epi);
}

// Tile geometry of the two kernel shapes.
//   single CTA: a 128 x 256 tile per CTA, B tile 256 rows, 4 stages of 48 KB;
//   CTA pair (cluster of 2, cta_group::2): a 256 x 256 tile per pair, each CTA
//   loads 128 rows of A and 128 rows of B per stage (6 stages of 32 KB) and owns
//   128 accumulator rows; the leader issues M=256 N=256 MMAs over both CTAs'
//   shared memory, so every B byte crosses L2 -> SM once per 256 rows instead of
//   once per 128.
//   dual (CTA pair, long K): each work unit is two N-tiles of one M-tile; a
//   stage holds the A tile and both B halves (48 KB, 4 stages), the leader
//   issues the A stage against both and accumulates into both TMEM
//   accumulators, so A is written into shared memory once per two tiles.
template <bool kPair, bool kDual = false, bool kRot = false>
struct Shape {
  static constexpr int pair = kPair ? 2 : 1;
  static constexpr int dual_n = kDual ? 2 : 1;             // N-tiles per work unit
  static constexpr int tile_m = kBM * pair;               // rows per (pair) tile
  static constexpr int b_rows = kPair ? kBN / 2 : kBN;    // B rows loaded per CTA
  static constexpr int b_tile_bytes = b_rows * kBK;
  static constexpr int stage_bytes = kATileBytes + dual_n * b_tile_bytes;
  // The rotating epilogues store four chunks back to back at the end of a tile:
  // their CTA pairs trade an operand stage for a second staging buffer.
  static constexpr int stages =
      kPair ? (kDual ? H3SK_DUAL_STAGES : (kRot ? H3SK_PAIR_STAGES - 1 : H3SK_PAIR_STAGES)) : 4;
  static constexpr int stage_bufs = (kPair && !kDual) ? (kRot ? 2 : H3SK_STAGE_BUFS) : 1;   // output staging buffers per warp
  static constexpr uint32_t idesc = idesc_i8(kBM * pair, kBN);
};

template <bool kPair, bool kDual = false, bool kRot = false>
struct SmemLayout {
  using S = Shape<kPair, kDual, kRot>;
  // offsets from the 1024-aligned base
  static constexpr int a = 0;
  static constexpr int b = S::stages * kATileBytes;                 // stage s: dual_n B tiles
  static constexpr int bars = b + S::stages * S::dual_n * S::b_tile_bytes;  // full[S], empty[S], tfull[2], tempty[2], drain
  static constexpr int nbars = 2 * S::stages + 5;
  static constexpr int misc = (bars + nbars * 8 + 15) / 16 * 16;  // tmem slot, abort flag, ready flag
  static constexpr int colv = misc + 16;                         // ws[256], bias[256] as float (16-byte aligned)
  static constexpr int hred = colv + 2 * kBN * 4;                // head epilogue: V maxima [2][4][128] u32, K maxima [2][4][4]
  static constexpr int stage = ((hred + 2 * 4 * 128 * 4 + 2 * 4 * 4 * 4) + 1023) / 1024 * 1024;   // per-warp output staging
  static constexpr int stage_warp_bytes = 32 * 32 * 2 * S::stage_bufs;   // stage_bufs x (32 rows x 32 BF16 columns)
  static constexpr int total = stage + kEpilogueWarps * stage_warp_bytes;
  static constexpr int dynamic_bytes = total + 1024;             // slack for 1024 alignment
};
static_assert(SmemLayout<true>::dynamic_bytes <= 227 * 1024, "pair layout exceeds shared memory");
static_assert(SmemLayout<false>::dynamic_bytes <= 227 * 1024, "single layout exceeds shared memory");
static_assert(SmemLayout<true, true>::dynamic_bytes <= 227 * 1024, "dual layout exceeds shared memory");
static_assert(SmemLayout<true, false, true>::dynamic_bytes <= 227 * 1024, "rotating layout exceeds shared memory");

struct GemmParams {
  const float* xs;
  const float* ws;
  const __nv_bfloat16* bias;      // may be null
  void* d;                        // BF16 (or int32 for kEpiAcc)
  int64_t ldd;
  const __nv_bfloat16* gate;      // [G, gate_ld]
  const int32_t* rows;            // [M]
  const __nv_bfloat16* residual;  // [M, ldr]
  int64_t gate_ld;
  int64_t ldr;
  int m, n, k;
  int m_tiles, n_tiles, k_blocks;
  int n_units;                    // work units along N (n_tiles / dual_n)
  int work;                       // m_tiles * n_units
  int group_n;                    // N units per weight-stationary group
  int head_major;                 // 1: D is [N/128, M, 128] (one plane per 128 columns)
  HeadsArgs hd;                   // kEpiHeads only
  uint32_t* rowmax;               // rotating kinds: [M] bits of max |rotated value|, zeroed by the host
  int rot_n0;                     // rotating kinds: first rotated column (tiles from here on rotate)
  int* status;
  uint64_t timeout_ns;
};

__device__ int g_pipeline_status = 0;

__device__ __forceinline__ void tile_coords(int tile, int m_tiles, int n_tiles, int group_n, int& mt, int& nt) {
  const int per_group = group_n * m_tiles;
  const int group = tile / per_group;
  const int first_n = group * group_n;
  const int gn = min(group_n, n_tiles - first_n);
  const int local = tile - group * per_group;
  mt = local / gn;
  nt = first_n + local % gn;
}

// ---- packed FP32 pairs (sm_100 f32x2), round-to-nearest, no flush -------------
// Used for the GELU evaluation, whose contract is 1 BF16 ulp against the CPU
// restatement (checked on every finite BF16 input); packing halves its
// FMA-pipe instructions.
__device__ __forceinline__ uint64_t p2(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ float p2_lo(uint64_t v) { return __uint_as_float(uint32_t(v)); }
__device__ __forceinline__ float p2_hi(uint64_t v) { return __uint_as_float(uint32_t(v >> 32)); }
__device__ __forceinline__ uint64_t p2_mul(uint64_t a, uint64_t b) {
  uint64_t c;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(c) : "l"(a), "l"(b));
  return c;
}
__device__ __forceinline__ uint64_t p2_add(uint64_t a, uint64_t b) {
  uint64_t c;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(c) : "l"(a), "l"(b));
  return c;
}
__device__ __forceinline__ uint64_t p2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
// The two BF16 halves of a word as a packed FP32 pair (low half first).
__device__ __forceinline__ uint64_t p2_from_bf2(uint32_t w) {
  return p2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
}

// Two FP32 values -> one word of two BF16 (round to nearest even), low half = lo.
__device__ __forceinline__ uint32_t pack_bf2(float lo, float hi) {
  uint32_t w;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(w) : "f"(hi), "f"(lo));
  return w;
}
__device__ __forceinline__ uint32_t pack_bf2(uint64_t v) { return pack_bf2(p2_lo(v), p2_hi(v)); }

// GELU-tanh of both BF16 halves of a word, 0.5 v (1 + tanh(u)) with
// u = 0.7978845608028654 (v + 0.044715 v^3) (convrot64_exact.cuh:913-923),
// evaluated left to right with one IEEE rounding per operation, as written:
// ((0.044715 v) v) v, v + that, times 0.7978845608028654.  tanh(u) comes from the
// identity tanh(u) = 2 / (1 + e^(-2u)) - 1: e^(-2u) = 2^(-2u / ln 2) by ex2.approx
// (relative error about 2^-22), the reciprocal by rcp.approx, and the final fma
// rounds tanh(u) to FP32 once.  Near u << 0 that rounding puts 1 + tanh(u) on the
// same FP32 grid (multiples of 2^-24) as 1 + tanhf(u), so the tiny negative-side
// outputs keep the reference's cancellation; elsewhere the relative error of
// 1 + tanh(u) stays below 2^-19, far inside one BF16 ulp.  All 65,280 finite
// BF16 inputs are checked against the CPU restatement (libm tanhf) to 1 BF16 ulp.
// u = +-inf and NaN propagate as in the reference.  Result rounded to BF16.
__device__ __forceinline__ uint32_t gelu_bf2(uint32_t w) {
  const uint64_t v = p2_from_bf2(w);
  const uint64_t cube = p2_mul(p2_mul(p2_mul(p2(0.044715f, 0.044715f), v), v), v);
  const uint64_t inner = p2_mul(p2(0.7978845608028654f, 0.7978845608028654f), p2_add(v, cube));
  const uint64_t arg = p2_mul(inner, p2(-2.8853900817779268f, -2.8853900817779268f));
  float e0, e1, r0, r1;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e0) : "f"(p2_lo(arg)));
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e1) : "f"(p2_hi(arg)));
  const uint64_t den = p2_add(p2(1.0f, 1.0f), p2(e0, e1));
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r0) : "f"(p2_lo(den)));
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r1) : "f"(p2_hi(den)));
  const uint64_t t = p2_fma(p2(2.0f, 2.0f), p2(r0, r1), p2(-1.0f, -1.0f));
  const uint64_t g = p2_mul(p2_mul(p2(0.5f, 0.5f), v), p2_add(p2(1.0f, 1.0f), t));
  return pack_bf2(g);
}

// Named barrier among the eight epilogue warps only.
__device__ __forceinline__ void epilogue_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(kEpilogueThreads) : "memory");
}

// Named barrier among the four epilogue warps of one column half (one head).
__device__ __forceinline__ void half_sync(int half) {
  asm volatile("bar.sync %0, 128;" ::"r"(2 + half) : "memory");
}
// Named barrier between the two epilogue warps of one TMEM lane quarter (the two
// column halves of the same 32 rows).
__device__ __forceinline__ void quarter_sync(int quarter) {
  asm volatile("bar.sync %0, 64;" ::"r"(4 + quarter) : "memory");
}

// ---- ConvRot256 of a tile row (the FC2-input quantiser's rotation) -------------
// The quantiser's arithmetic (kernels/convrot/vendor/convrot64_exact.cuh:202-234,
// 664-677): four radix-4 stages over index bit pairs (0,1), (2,3), (4,5), (6,7);
// every stage output is 0.5 * h4_d(x0, x1, x2, x3) with the additions left to
// right, d=0: ((x0+x1)+x2)-x3, d=1: ((x0+x1)-x2)+x3, d=2: ((x0-x1)+x2)+x3,
// d=3: ((-x0+x1)+x2)+x3, all flushing subnormals (the reference builds its
// quantiser with --use_fast_math).  This unit is built without fast math, so
// every operation is written with its .ftz form.  0.5*RN(t +- x3) is computed as
// fma(t, 0.5, +-0.5*x3) (exact scaling by 0.5 commutes with the rounding) and
// (-x0+x1)+x2 as x2-(x0-x1) (the same rounded value).
__device__ __forceinline__ float z_add(float a, float b) {
  float c;
  asm("add.rn.ftz.f32 %0, %1, %2;" : "=f"(c) : "f"(a), "f"(b));
  return c;
}
__device__ __forceinline__ float z_sub(float a, float b) {
  float c;
  asm("sub.rn.ftz.f32 %0, %1, %2;" : "=f"(c) : "f"(a), "f"(b));
  return c;
}
__device__ __forceinline__ float z_mul(float a, float b) {
  float c;
  asm("mul.rn.ftz.f32 %0, %1, %2;" : "=f"(c) : "f"(a), "f"(b));
  return c;
}
__device__ __forceinline__ float z_fma(float a, float b, float c) {
  float d;
  asm("fma.rn.ftz.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}
__device__ __forceinline__ uint64_t z2_add(uint64_t a, uint64_t b) {
  uint64_t c;
  asm("add.rn.ftz.f32x2 %0, %1, %2;" : "=l"(c) : "l"(a), "l"(b));
  return c;
}
__device__ __forceinline__ uint64_t z2_sub(uint64_t a, uint64_t b) {
  uint64_t c;
  asm("sub.rn.ftz.f32x2 %0, %1, %2;" : "=l"(c) : "l"(a), "l"(b));
  return c;
}
__device__ __forceinline__ uint64_t z2_mul(uint64_t a, uint64_t b) {
  uint64_t c;
  asm("mul.rn.ftz.f32x2 %0, %1, %2;" : "=l"(c) : "l"(a), "l"(b));
  return c;
}
__device__ __forceinline__ uint64_t z2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.ftz.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
// Stage over index bits 0,1 of 64 consecutive values held as 32 pairs (value 2i
// in the low half of v[i]): quads of consecutive values.
__device__ __forceinline__ void rot_stage01(uint64_t (&v)[32]) {
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const float x0 = p2_lo(v[2 * j]), x1 = p2_hi(v[2 * j]);
    const float x2 = p2_lo(v[2 * j + 1]), x3 = p2_hi(v[2 * j + 1]);
    const float a = z_add(x0, x1), b = z_sub(x0, x1);
    const float h = z_mul(0.5f, x3);
    const float t0 = z_add(a, x2), t1 = z_sub(a, x2), t2 = z_add(b, x2), t3 = z_sub(x2, b);
    v[2 * j] = p2(z_fma(t0, 0.5f, -h), z_fma(t1, 0.5f, h));
    v[2 * j + 1] = p2(z_fma(t2, 0.5f, h), z_fma(t3, 0.5f, h));
  }
}
// Stage over the two index bits held at pair strides S and 2S: quads
// {P, P+S, P+2S, P+3S} of pairs, for every P with those bits clear.
template <int S>
__device__ __forceinline__ void rot_stage_pairs(uint64_t (&v)[32]) {
  const uint64_t half = p2(0.5f, 0.5f), nhalf = p2(-0.5f, -0.5f);
#pragma unroll
  for (int q = 0; q < 32; ++q) {
    if ((q / S) & 3) continue;
    const uint64_t x0 = v[q], x1 = v[q + S], x2 = v[q + 2 * S], x3 = v[q + 3 * S];
    const uint64_t a = z2_add(x0, x1), b = z2_sub(x0, x1);
    const uint64_t h = z2_mul(x3, half), nh = z2_mul(x3, nhalf);
    const uint64_t t0 = z2_add(a, x2), t1 = z2_sub(a, x2), t2 = z2_add(b, x2), t3 = z2_sub(x2, b);
    v[q] = z2_fma(t0, half, nh);
    v[q + S] = z2_fma(t1, half, h);
    v[q + 2 * S] = z2_fma(t2, half, h);
    v[q + 3 * S] = z2_fma(t3, half, h);
  }
}
__device__ __forceinline__ void tmem_store_32cols(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]),
      "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]),
      "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
__device__ __forceinline__ void tmem_store_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_load_16cols(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
}
__device__ __forceinline__ uint32_t warp_max_u32(uint32_t x) {
  uint32_t r;
  asm volatile("redux.sync.max.u32 %0, %1, 0xffffffff;" : "=r"(r) : "r"(x));
  return r;
}
__device__ __forceinline__ float bf_at(const uint32_t (&y)[64], int ch) {
  const uint32_t w = y[ch >> 1];
  return __uint_as_float((ch & 1) ? (w & 0xffff0000u) : (w << 16));
}
__device__ __forceinline__ float bf_round(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }
__device__ __forceinline__ uint32_t bf_pair(float lo, float hi) {
  uint32_t w;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(w) : "f"(hi), "f"(lo));
  return w;
}
// Four codes cvt.rni.sat.s8.f32(v * inv), packed little-endian (r84_kfourwarp.cu:300-306).
__device__ __forceinline__ uint32_t codes4_rni(float a, float b, float c, float d, float inv) {
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

// Per-head RMS normalisation, weight and RoPE of one row held by one thread, in
// place on its 64 BF16 pair words (r84_kfourwarp.cu:262-282): the 32 chains
// fmaf(v, v, s) over channels l, l + 32, l + 64, l + 96 in that order, the
// shfl_down tree of the reference folded in registers (s_l += s_{l+off}, off =
// 16 .. 1), rrms = rsqrtf(sum / 128 + eps); then x = bf((t * rrms) * w) and, for
// the pairs (d, d + 48), d < 48: bf(a * x0 + b * x1), bf(c * x0 + e * x1) with the
// row's RoPE coefficients; channels 96..127 are normalised and weighted only.
// The expressions are written as the reference writes them, in a unit compiled
// like the reference's QKV unit (no fast math), so each rounds the same way.
__device__ __forceinline__ void rms_rope_row(uint32_t (&y)[64], const __nv_bfloat16* w, const __nv_bfloat16* f,
                                             float eps) {
  float chain[32];
#pragma unroll
  for (int l = 0; l < 32; ++l) chain[l] = 0.f;
#pragma unroll
  for (int k = 0; k < 4; ++k)
#pragma unroll
    for (int l = 0; l < 32; ++l) {
      const float v = bf_at(y, 32 * k + l);
      chain[l] = fmaf(v, v, chain[l]);
    }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1)
#pragma unroll
    for (int l = 0; l < off; ++l) chain[l] += chain[l + off];
  const float rrms = rsqrtf(chain[0] / 128.f + eps);
  const uint4* w4 = reinterpret_cast<const uint4*>(w);
  const uint4* f4 = reinterpret_cast<const uint4*>(f);
  // pairs: words j (channels 2j, 2j+1) and j + 24 (channels 2j + 48, 2j + 49), j < 24
#pragma unroll
  for (int q = 0; q < 6; ++q) {              // 8 channels d = 8q .. 8q+7 per round
    const uint4 wa = __ldg(w4 + q), wb = __ldg(w4 + 6 + q);
    const uint32_t wlo[4] = {wa.x, wa.y, wa.z, wa.w}, whi[4] = {wb.x, wb.y, wb.z, wb.w};
#pragma unroll
    for (int h = 0; h < 4; ++h) {
      const int j = 4 * q + h;               // word of channels d = 2j, 2j + 1
      const uint4 fc = __ldg(f4 + j);         // (a, b | c, e) of pair 2j, then of pair 2j + 1
      float out0[2], out1[2];
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        const float t0 = bf_at(y, 2 * j + k), t1 = bf_at(y, 2 * j + k + 48);
        const float w0 = __uint_as_float(k ? (wlo[h] & 0xffff0000u) : (wlo[h] << 16));
        const float w1 = __uint_as_float(k ? (whi[h] & 0xffff0000u) : (whi[h] << 16));
        const float x0 = bf_round(t0 * rrms * w0), x1 = bf_round(t1 * rrms * w1);
        const uint32_t ab = k ? fc.z : fc.x, ce = k ? fc.w : fc.y;
        const float a = __uint_as_float(ab << 16), b = __uint_as_float(ab & 0xffff0000u);
        const float c = __uint_as_float(ce << 16), e = __uint_as_float(ce & 0xffff0000u);
        out0[k] = a * x0 + b * x1;
        out1[k] = c * x0 + e * x1;
      }
      y[j] = bf_pair(out0[0], out0[1]);
      y[j + 24] = bf_pair(out1[0], out1[1]);
    }
  }
#pragma unroll
  for (int q = 12; q < 16; ++q) {             // channels 96..127
    const uint4 wt = __ldg(w4 + q);
    const uint32_t ww[4] = {wt.x, wt.y, wt.z, wt.w};
#pragma unroll
    for (int h = 0; h < 4; ++h) {
      const int j = 4 * q + h;
      const float t0 = bf_at(y, 2 * j), t1 = bf_at(y, 2 * j + 1);
      y[j] = bf_pair(t0 * rrms * __uint_as_float(ww[h] << 16), t1 * rrms * __uint_as_float(ww[h] & 0xffff0000u));
    }
  }
}

// The signed H128 rotation of one row held by one thread (r84_kfourwarp.cu:123-191
// in the reference's 4-channels-per-lane form): channel ch is negated where bit
// ch % 32 of sign word ch / 32 is clear, then the 4-point block on channel bits
// 0-1 ((a0 + a2) * 0.5 ...), then butterflies lo' = lo + hi, hi' = lo - hi on
// channel bits 2..6 in that order, then the factor 0.1767766952966369f.  With
// `full` false (M <= 256) only the 4-point block runs (r84:297, 330).
__device__ __forceinline__ void rotate128(float (&v)[128], bool full) {
  if (full) {
    constexpr uint32_t kSigns[4] = {0x1035997bu, 0x8087f5eeu, 0xee2e4e1au, 0x71132418u};
#pragma unroll
    for (int ch = 0; ch < 128; ++ch)
      if (((kSigns[ch >> 5] >> (ch & 31)) & 1u) == 0u) v[ch] = -v[ch];
  }
#pragma unroll
  for (int j = 0; j < 128; j += 4) {
    const float a0 = v[j] + v[j + 1], a1 = v[j] - v[j + 1], a2 = v[j + 2] + v[j + 3], a3 = v[j + 2] - v[j + 3];
    v[j] = (a0 + a2) * 0.5f;
    v[j + 1] = (a1 + a3) * 0.5f;
    v[j + 2] = (a0 - a2) * 0.5f;
    v[j + 3] = (a1 - a3) * 0.5f;
  }
  if (!full) return;
#pragma unroll
  for (int bit = 4; bit < 128; bit <<= 1)
#pragma unroll
    for (int j = 0; j < 128; ++j) {
      if (j & bit) continue;
      const float lo = v[j], hi = v[j | bit];
      v[j] = lo + hi;
      v[j | bit] = lo - hi;
    }
#pragma unroll
  for (int j = 0; j < 128; ++j) v[j] *= 0.1767766952966369f;
}

// Raw int32 accumulators of one row, columns [col0, col0+32) (debug epilogue).
__device__ __forceinline__ void store_chunk_acc(const GemmParams& p, const uint32_t (&r)[32], int row, int col0) {
  int32_t* out = reinterpret_cast<int32_t*>(p.d) + int64_t(row) * p.ldd + col0;
#pragma unroll
  for (int v = 0; v < 8; ++v)
    if (col0 + 4 * v < p.n)
      reinterpret_cast<int4*>(out)[v] = make_int4(int(r[4 * v]), int(r[4 * v + 1]), int(r[4 * v + 2]), int(r[4 * v + 3]));
}

// BF16 epilogue values of 32 consecutive accumulators of one row (columns
// [col0, col0+32), tile-local chunk c) as 16 packed words.  Rows >= M and
// columns >= N produce unused values and read no memory.
// BF16 results of one 32-column chunk of one row: y = bf((acc * xs) * ws + bias)
// (fc1.cu / gate.cu epilogue order), then GELU or the gate-residual update.
// Column scales and bias come from shared memory as 16-byte broadcasts.  The
// dequant and the gate FMA stay scalar: packed f32x2 forms of them were measured
// to differ from the scalar IEEE operations on rare inputs.
template <int kEpi, bool kAddBias = true>
__device__ __forceinline__ void chunk_values(const GemmParams& p, const uint32_t (&r)[32], bool row_ok, int row,
                                             int col0, int c, float xs_row, const __nv_bfloat16* gate_row,
                                             const float* col_ws, const float* col_bias, uint32_t (&packed)[16]) {
  const float4* wsv = reinterpret_cast<const float4*>(col_ws + c * 32);
  const float4* bsv = reinterpret_cast<const float4*>(col_bias + c * 32);
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    const float4 w4 = wsv[q], b4 = bsv[q];
    const float w[4] = {w4.x, w4.y, w4.z, w4.w}, b[4] = {b4.x, b4.y, b4.z, b4.w};
    float y[4];
#pragma unroll
    for (int h = 0; h < 4; ++h) {
      const float prod = __fmul_rn(__fmul_rn(__int2float_rn(int(r[4 * q + h])), xs_row), w[h]);
      y[h] = kAddBias ? __fadd_rn(prod, b[h]) : prod;
    }
    packed[2 * q] = pack_bf2(y[0], y[1]);
    packed[2 * q + 1] = pack_bf2(y[2], y[3]);
  }
  if constexpr (kEpi == kEpiGelu) {
#pragma unroll
    for (int i = 0; i < 16; ++i) packed[i] = gelu_bf2(packed[i]);
  }
  if constexpr (kEpi == kEpiGate) {
    // D may alias the residual: every element is read here, before its store is issued.
    const __nv_bfloat16* res = p.residual + int64_t(row) * p.ldr + col0;
    const __nv_bfloat16* gat = gate_row + col0;
#pragma unroll
    for (int v = 0; v < 4; ++v) {
      if (!row_ok || col0 + 8 * v >= p.n) continue;
      const uint4 rv = *reinterpret_cast<const uint4*>(res + 8 * v);
      const uint4 gv = __ldg(reinterpret_cast<const uint4*>(gat + 8 * v));
      const uint32_t rw[4] = {rv.x, rv.y, rv.z, rv.w};
      const uint32_t gw[4] = {gv.x, gv.y, gv.z, gv.w};
#pragma unroll
      for (int w = 0; w < 4; ++w) {
        const uint32_t yw = packed[4 * v + w];
        const float lo = __fmaf_rn(__uint_as_float(yw << 16), __uint_as_float(gw[w] << 16),
                                   __uint_as_float(rw[w] << 16));
        const float hi = __fmaf_rn(__uint_as_float(yw & 0xffff0000u), __uint_as_float(gw[w] & 0xffff0000u),
                                   __uint_as_float(rw[w] & 0xffff0000u));
        packed[4 * v + w] = pack_bf2(lo, hi);
      }
    }
  }
}

// Persistent warp-specialised INT8 GEMM.  Warp 0: TMA producer; warp 1: MMA
// issuer (TMEM allocation owner); warps 2..9: epilogue (TMEM -> registers ->
// dequant / GELU / gate-residual -> BF16 -> swizzled staging -> TMA store).
// kPair: clusters of two CTAs share one 256 x 256 tile (see Shape); the leader
// (rank 0) issues the MMAs, both CTAs produce their operand halves and run the
// epilogue of their 128 accumulator rows.
template <int kEpi, bool kPair, bool kDual = false>
__global__ void __launch_bounds__(kThreads, 1)
    int8_gemm_persistent(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                         const __grid_constant__ CUtensorMap map_d, const GemmParams p) {
  using S = Shape<kPair, kDual, is_rot(kEpi)>;
  using L = SmemLayout<kPair, kDual, is_rot(kEpi)>;
  constexpr uint32_t kTemptyCount = (kPair ? 2 : 1) * kEpilogueWarps;   // each epilogue warp of each CTA releases
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* smem_a = smem + L::a;
  uint8_t* smem_b = smem + L::b;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::bars);
  uint64_t* empty = full + S::stages;
  uint64_t* tfull = empty + S::stages;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::misc);
  volatile int* abort = reinterpret_cast<volatile int*>(smem + L::misc + 4);
  volatile int* ready = reinterpret_cast<volatile int*>(smem + L::misc + 8);
  float* col_ws = reinterpret_cast<float*>(smem + L::colv);
  float* col_bias = col_ws + kBN;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int* status = p.status;
  const uint32_t rank = kPair ? cluster_ctarank() : 0u;
  const bool leader = rank == 0;
  const int unit = kPair ? int(blockIdx.x >> 1) : int(blockIdx.x);        // tile-walking unit (pair or CTA)
  const int units = kPair ? int(gridDim.x >> 1) : int(gridDim.x);

  if (threadIdx.x == 0) {
    for (int s = 0; s < S::stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], kTemptyCount);
    }
    mbar_init(drain, 1);
    *abort = 0;
    fence_mbar_init();
    tma_prefetch_map(&map_a);
    tma_prefetch_map(&map_b);
    if (kEpi != kEpiAcc) tma_prefetch_map(&map_d);
  }
  if (warp == 1) {
    if constexpr (kPair) {
      tmem_alloc_pair(tmem_slot, kTmemCols);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(tmem_slot, kTmemCols);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  if constexpr (kPair) cluster_sync_all();   // both CTAs' barriers and TMEM exist before any cross-CTA use
  else __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  // Control flow is warp-uniform in every role: lane 0 waits and issues, and
  // __shfl_sync hands its verdict to the other lanes, so every .sync.aligned
  // tcgen05 instruction and every barrier below is reached by converged warps.
  if (warp == 0) {
    // ---------------- TMA producer (both CTAs of a pair) ----------------
    uint64_t policy_a = 0, policy_b = 0;
    uint32_t full_leader = 0;
    if (lane == 0) {
      policy_a = l2_policy_evict_normal();
      policy_b = l2_policy_evict_last();
      if constexpr (kPair) full_leader = map_to_rank(smem_addr(full), 0);
    }
    uint32_t issued_mask = 0, issued_phase_bits = 0;   // per stage: issued at least once / parity of last issue
    int stage = 0;
    uint32_t phase = 0;
    bool ok = true;
    for (int w = unit; ok && w < p.work; w += units) {
      int mt, nu;
      tile_coords(w, p.m_tiles, p.n_units, p.group_n, mt, nu);
      const int a_row = mt * S::tile_m + int(rank) * kBM;
      const int b_row = nu * S::dual_n * kBN + int(rank) * S::b_rows;   // B rows of the unit's first tile
      for (int kb = 0; kb < p.k_blocks; ++kb) {
        int got = 0;
        if (lane == 0) {
          got = mbar_wait_bounded(&empty[stage], phase ^ 1u, abort, status, 11, p.timeout_ns) ? 1 : 0;
          if (got) {
            uint8_t* da = smem_a + stage * kATileBytes;
            uint8_t* db = smem_b + stage * S::dual_n * S::b_tile_bytes;
            if constexpr (kPair) {
              // The leader's full barrier counts both CTAs' bytes; only the leader arms it.
              if (leader) mbar_arrive_expect_tx(&full[stage], 2 * S::stage_bytes);
              const uint32_t bar = full_leader + uint32_t(stage) * 8u;
              tma_load_2d_pair(da, &map_a, bar, kb * kBK, a_row, policy_a);
#pragma unroll
              for (int j = 0; j < S::dual_n; ++j)
                tma_load_2d_pair(db + j * S::b_tile_bytes, &map_b, bar, kb * kBK, b_row + j * kBN, policy_b);
            } else {
              mbar_arrive_expect_tx(&full[stage], S::stage_bytes);
              tma_load_2d(da, &map_a, &full[stage], kb * kBK, a_row, policy_a);
              tma_load_2d(db, &map_b, &full[stage], kb * kBK, b_row, policy_b);
            }
          }
        }
        got = __shfl_sync(0xffffffffu, got, 0);
        if (!got) {
          ok = false;
          break;
        }
        issued_mask |= 1u << stage;
        issued_phase_bits = (issued_phase_bits & ~(1u << stage)) | (phase << stage);
        if (++stage == S::stages) {
          stage = 0;
          phase ^= 1u;
        }
      }
    }
    // Drain: every copy this CTA issued lands before the CTA exits.  A pair's
    // copies complete on the leader's barriers, so the leader drains for both.
    if (lane == 0 && leader) {
      for (int s = 0; s < S::stages; ++s)
        if (issued_mask & (1u << s))
          mbar_wait_bounded(&full[s], (issued_phase_bits >> s) & 1u, nullptr, status, 12, p.timeout_ns);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---------------- MMA issuer (the pair leader only) ----------------
    if (leader) {
      int stage = 0, acc = 0;
      uint32_t phase = 0, acc_phase = 0;
      bool ok = true;
      for (int w = unit; ok && w < p.work; w += units) {
        // the unit's accumulators: acc (one tile) or both (dual)
        int got = 0;
        if (lane == 0) {
          got = mbar_wait_bounded(&tempty[acc], acc_phase ^ 1u, abort, status, 21, p.timeout_ns) ? 1 : 0;
          if (kDual && got)
            got = mbar_wait_bounded(&tempty[1], acc_phase ^ 1u, abort, status, 21, p.timeout_ns) ? 1 : 0;
          if (got) tc_fence_after();
        }
        if (!__shfl_sync(0xffffffffu, got, 0)) break;
        const uint32_t d_tmem = tmem_base + uint32_t(acc * kBN);
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          got = 0;
          if (lane == 0) {
            got = mbar_wait_bounded(&full[stage], phase, abort, status, 22, p.timeout_ns) ? 1 : 0;
            if (got) {
              tc_fence_after();
              const uint64_t a_desc = smem_desc_k_sw128(smem_a + stage * kATileBytes);
#pragma unroll
              for (int j = 0; j < S::dual_n; ++j) {
                const uint64_t b_desc = smem_desc_k_sw128(smem_b + (stage * S::dual_n + j) * S::b_tile_bytes);
                const uint32_t d = d_tmem + uint32_t(j * kBN);
#pragma unroll
                for (int kk = 0; kk < kBK / kUmmaK; ++kk) {
                  // +32 bytes along K inside the swizzle atom = +2 in the 16-byte address field
                  const uint32_t accum = (kb > 0 || kk > 0) ? 1u : 0u;
                  if constexpr (kPair)
                    mma_i8_pair(d, a_desc + uint64_t(2 * kk), b_desc + uint64_t(2 * kk), S::idesc, accum);
                  else
                    mma_i8(d, a_desc + uint64_t(2 * kk), b_desc + uint64_t(2 * kk), S::idesc, accum);
                }
              }
              if constexpr (kPair) mma_commit_pair(&empty[stage], 0x3);   // frees the stage in both CTAs
              else mma_commit(&empty[stage]);
            }
          }
          got = __shfl_sync(0xffffffffu, got, 0);
          if (!got) {
            ok = false;
            break;
          }
          if (++stage == S::stages) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        if (lane == 0) {
          if constexpr (kPair) {
            mma_commit_pair(&tfull[acc], 0x3);   // both CTAs' epilogues
            if constexpr (kDual) mma_commit_pair(&tfull[1], 0x3);
          } else {
            mma_commit(&tfull[acc]);
          }
        }
        __syncwarp();
        if (kDual) {
          acc_phase ^= 1u;   // acc stays 0: the unit used accumulators 0 and 1
        } else if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
      // Drain: every MMA issued by this warp completes before TMEM is released.
      if (lane == 0) {
        if constexpr (kPair) mma_commit_pair(drain, 0x1);
        else mma_commit(drain);
        mbar_wait_bounded(drain, 0, nullptr, status, 23, p.timeout_ns);
      }
      __syncwarp();
    }
  } else {
    // ---------------- epilogue (both CTAs of a pair) ----------------
    const int quarter = warp & 3;            // TMEM lane quarter this warp may access
    const int half = (warp - 2) >> 2;        // column half of the tile
    const int ep_tid = threadIdx.x - 64;     // 0..255
    uint8_t* stage = smem + L::stage + (warp - 2) * L::stage_warp_bytes;
    const uint32_t tempty_leader = kPair ? map_to_rank(smem_addr(tempty), 0) : 0u;
    int acc = 0;
    uint32_t acc_phase = 0;
    uint32_t stored = 0;   // chunks this warp has staged (selects the staging buffer)
    // Tiles in the MMA's order: the dual_n tiles of each work unit in turn, so
    // the accumulators alternate 0, 1, 0, 1 as in the single-tile form.
    for (int it = 0;; ++it) {
      const int w = unit + (it / S::dual_n) * units;
      if (w >= p.work) break;
      int mt, nu;
      tile_coords(w, p.m_tiles, p.n_units, p.group_n, mt, nu);
      const int nt = nu * S::dual_n + it % S::dual_n;
      const int n0 = nt * kBN;
      // Stage this tile's per-column scales (and bias) in shared memory.
      epilogue_sync();   // the previous tile's readers are done
      if (kEpi != kEpiAcc) {
        for (int c = ep_tid; c < kBN; c += kEpilogueThreads) {
          const int n = n0 + c;
          col_ws[c] = n < p.n ? p.ws[n] : 0.0f;
          col_bias[c] = (p.bias != nullptr && n < p.n) ? __bfloat162float(p.bias[n]) : 0.0f;
        }
      }
      // One thread waits for the accumulator; the named barrier hands the
      // outcome to the other 255 so all of them leave or continue together.
      if (ep_tid == 0) *ready = mbar_wait_bounded(&tfull[acc], acc_phase, abort, status, 31, p.timeout_ns) ? 1 : 0;
      epilogue_sync();
      if (*ready == 0) break;
      tc_fence_after();
      const int row_base = mt * S::tile_m + int(rank) * kBM + quarter * 32;
      const int row = row_base + lane;
      const bool row_ok = row < p.m;
      const float xs_row = (kEpi != kEpiAcc && row_ok) ? p.xs[row] : 0.0f;
      const __nv_bfloat16* gate_row = nullptr;
      if (kEpi == kEpiGate && row_ok) gate_row = p.gate + int64_t(p.rows[row]) * p.gate_ld;
      const uint32_t t_row = tmem_base + uint32_t(acc * kBN) + (uint32_t(quarter * 32) << 16);
      const int c_first = half * (kBN / 64), c_last = c_first + kBN / 64 - 1;
      // This warp's last read of the accumulator has landed: release it to the MMA issuer.
      auto release = [&]() {
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          if constexpr (kPair) mbar_arrive_remote(tempty_leader + uint32_t(acc) * 8u);
          else mbar_arrive(&tempty[acc]);
        }
      };
      // BF16 chunk: 32 rows x 32 columns through this warp's staging buffer and
      // one TMA tensor store (rows >= M and columns >= N are clipped by TMA).
      auto store_chunk = [&](int col0, const uint32_t* packed) {
        uint8_t* buf = stage + (stored & (S::stage_bufs - 1)) * (L::stage_warp_bytes / S::stage_bufs);
        ++stored;
        // the store that last read `buf` is done reading it
        if (lane == 0) {
          if constexpr (S::stage_bufs == 2) bulk_wait_read_1();
          else bulk_wait_read_all();
        }
        __syncwarp();
        // 64-byte swizzle: 16-byte chunk v of row i sits at chunk v ^ ((i >> 1) & 3)
        uint8_t* srow = buf + lane * 64;
#pragma unroll
        for (int v = 0; v < 4; ++v)
          *reinterpret_cast<uint4*>(srow + ((v ^ ((lane >> 1) & 3)) << 4)) =
              make_uint4(packed[4 * v], packed[4 * v + 1], packed[4 * v + 2], packed[4 * v + 3]);
        fence_async_shared();
        __syncwarp();
        if (lane == 0) {
          if (p.head_major) tma_store_3d(&map_d, buf, col0 & 127, row_base, col0 >> 7);
          else tma_store_2d(&map_d, buf, col0, row_base);
          bulk_commit();
        }
      };
      auto emit = [&](int c, const uint32_t (&r)[32]) {
        const int col0 = n0 + c * 32;
        if constexpr (kEpi == kEpiAcc) {
          if (row_ok && col0 < p.n) store_chunk_acc(p, r, row, col0);
        } else if (col0 < p.n && row_base < p.m) {
          uint32_t packed[16];
          chunk_values<base_epi(kEpi)>(p, r, row_ok, row, col0, c, xs_row, gate_row, col_ws, col_bias, packed);
          store_chunk(col0, packed);
        }
      };
      if constexpr (kEpi == kEpiHeads) {
        // ---- QKV head epilogue: this thread finishes row `row` of one head ----
        // (128 columns = one head; the tile's two heads are the two column halves)
        const HeadsArgs& hd = p.hd;
        const int plane_w = hd.heads * 128;
        const int g = n0 / plane_w;                          // 0 Q, 1 K, 2 V (a tile never straddles)
        const int head = (n0 - g * plane_w) / 128 + half;
        const int part = (mt * S::tile_m + int(rank) * kBM) / 128;   // this CTA's 128 rows = one part
        // The second CTA of a pair may hold no row < M (the last M-tile): its part
        // does not exist and it writes no scale or maximum.
        const bool part_ok = part < hd.parts;
        uint32_t y[64];                                      // the row's 128 dequantised BF16 values
#pragma unroll
        for (int cc = 0; cc < 4; ++cc) {
          const int c = c_first + cc;
          uint32_t r[32];
          __syncwarp();
          tmem_load_32cols(t_row + uint32_t(c * 32), r);
          tmem_load_wait();
          if (c == c_last) release();
          uint32_t packed[16];
          chunk_values<kEpiDequant>(p, r, row_ok, row, n0 + c * 32, c, xs_row, nullptr, col_ws, col_bias, packed);
#pragma unroll
          for (int i = 0; i < 16; ++i) y[16 * cc + i] = packed[i];
        }
        uint32_t* vred = reinterpret_cast<uint32_t*>(smem + L::hred);   // [2][4][128]
        float* kred = reinterpret_cast<float*>(smem + L::hred + 2 * 4 * 128 * 4);   // [2][4][4]
        if (g == 2) {
          // V: raw values to D, per-channel maxima of |BF16| over the part's 128 rows
          if (row_base < p.m) {
#pragma unroll
            for (int cc = 0; cc < 4; ++cc) store_chunk(n0 + (c_first + cc) * 32, y + 16 * cc);
          }
          uint32_t mine[4] = {0u, 0u, 0u, 0u};
#pragma unroll
          for (int ch = 0; ch < 128; ++ch) {
            const uint32_t w = y[ch >> 1];
            const uint32_t mag = row_ok ? (((ch & 1) ? (w >> 16) : w) & 0x7fffu) : 0u;
            const uint32_t mx = warp_max_u32(mag);
            if (lane == (ch & 31)) mine[ch >> 5] = mx;
          }
#pragma unroll
          for (int k = 0; k < 4; ++k) vred[(half * 4 + quarter) * 128 + 32 * k + lane] = mine[k];
          half_sync(half);
          if (quarter == 0 && part_ok && hd.vp != nullptr) {
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              const int ch = 32 * k + lane;
              uint32_t mx = 0;
#pragma unroll
              for (int qq = 0; qq < 4; ++qq) mx = max(mx, vred[(half * 4 + qq) * 128 + ch]);
              hd.vp[(int64_t(head) * hd.parts + part) * 128 + ch] = __uint_as_float(mx << 16);
            }
          }
        } else {
          // Q / K: normalise and rope, write D, rotate, quantise
          if (row_ok) rms_rope_row(y, g == 0 ? hd.qw : hd.kw, hd.freqs + int64_t(row) * 192, hd.eps);
          if (row_base < p.m) {
#pragma unroll
            for (int cc = 0; cc < 4; ++cc) store_chunk(n0 + (c_first + cc) * 32, y + 16 * cc);
          }
          float v[128];
#pragma unroll
          for (int ch = 0; ch < 128; ++ch) v[ch] = row_ok ? bf_at(y, ch) : 0.f;
          if (g == 1 && row_ok && hd.anchors != nullptr && hd.sk != nullptr) {
            const int anchor = hd.anchors[head];
            if (anchor >= 0 && anchor < 9) {   // an out-of-range anchor reads nothing
              const uint4* s4 = reinterpret_cast<const uint4*>(hd.sk + (int64_t(head) * 9 + anchor) * 128);
#pragma unroll
              for (int q = 0; q < 16; ++q) {
                const uint4 b = __ldg(s4 + q);
                const uint32_t bw[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                  v[8 * q + 2 * i] = v[8 * q + 2 * i] - __uint_as_float(bw[i] << 16);
                  v[8 * q + 2 * i + 1] = v[8 * q + 2 * i + 1] - __uint_as_float(bw[i] & 0xffff0000u);
                }
              }
            }
          }
          rotate128(v, p.m > 256);
          float mx = 0.f;
#pragma unroll
          for (int ch = 0; ch < 128; ++ch) mx = fmaxf(mx, fabsf(v[ch]));
          float sc, inv;
          if (g == 0) {
            // Q group 8 * quarter + lane % 8: rows s, s + 8, s + 16, s + 24 of the quarter
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
            sc = fmaf(mx, 1.f / 127.f, 1e-7f);
            asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(inv) : "f"(sc));
            if (lane < 8 && part_ok && hd.qs != nullptr)
              hd.qs[int64_t(head) * hd.parts * 32 + part * 32 + quarter * 8 + lane] = sc;
          } else {
            // K group kg: rows tr with tr % 8 in {2kg, 2kg + 1}, across the four quarters
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
            const int kg = (lane & 7) >> 1;
            if ((lane & ~6) == 0) kred[(half * 4 + quarter) * 4 + kg] = mx;   // lanes 0, 2, 4, 6
            half_sync(half);
            mx = fmaxf(fmaxf(kred[(half * 4 + 0) * 4 + kg], kred[(half * 4 + 1) * 4 + kg]),
                       fmaxf(kred[(half * 4 + 2) * 4 + kg], kred[(half * 4 + 3) * 4 + kg]));
            sc = fmaf(mx, 1.f / 127.f, 1e-7f);
            asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(inv) : "f"(sc));
            if (quarter == 0 && part_ok && (lane & ~6) == 0 && hd.ks != nullptr)
              hd.ks[(int64_t(head) * hd.parts + part) * 4 + kg] = sc;
          }
          int8_t* codes = g == 0 ? hd.qi : hd.ki;
          if (row_ok && codes != nullptr) {
            uint4* out = reinterpret_cast<uint4*>(codes + (int64_t(head) * p.m + row) * 128);
#pragma unroll
            for (int q = 0; q < 8; ++q)
              out[q] = make_uint4(codes4_rni(v[16 * q], v[16 * q + 1], v[16 * q + 2], v[16 * q + 3], inv),
                                  codes4_rni(v[16 * q + 4], v[16 * q + 5], v[16 * q + 6], v[16 * q + 7], inv),
                                  codes4_rni(v[16 * q + 8], v[16 * q + 9], v[16 * q + 10], v[16 * q + 11], inv),
                                  codes4_rni(v[16 * q + 12], v[16 * q + 13], v[16 * q + 14], v[16 * q + 15], inv));
          }
        }
      } else if constexpr (is_rot(kEpi)) {
        if (n0 < p.rot_n0) {
          // a tile before the rotated columns: the plain epilogue
#pragma unroll 1
          for (int c = c_first; c <= c_last; ++c) {
            uint32_t r[32];
            __syncwarp();
            tmem_load_32cols(t_row + uint32_t(c * 32), r);
            tmem_load_wait();
            if (c == c_last) release();
            emit(c, r);
          }
        } else {
          // ---- the epilogue (GELU for FC1, dequant for the QKV V tiles) + the next
          // quantiser's ConvRot256 ----
          // The tile's 256 columns are one rotation group of each of its rows; the
          // two warps of a lane quarter take the two column halves of its 32 rows.
          // (Four warps per quarter, 18 per CTA, measured slower: 5.9 vs 5.5 ms.)
          constexpr int kBlocks = 2;                  // 64-column blocks per warp in pass 1
          constexpr int kRuns = 2;                    // 16-position runs per warp in pass 2
          const int slice = half;
          // Pass 1: this warp's 64-column blocks: the epilogue's values rounded to
          // BF16 (as the unfused GEMM stores them), widened, the stages over index
          // bits (0,1), (2,3), (4,5), written back over the accumulator columns as
          // FP32.
#pragma unroll 1
          for (int b = 0; b < kBlocks; ++b) {
            const int blk = kBlocks * slice + b;
            uint64_t v[32];
#pragma unroll
            for (int cc = 0; cc < 2; ++cc) {
              const int c = 2 * blk + cc;
              uint32_t r[32];
              __syncwarp();
              tmem_load_32cols(t_row + uint32_t(c * 32), r);
              tmem_load_wait();
              // Without a bias the + 0 is left out: it only turns -0 into +0, and
              // the sign of a zero reaches neither a code nor the row maximum.
              uint32_t packed[16];
              if (p.bias != nullptr)
                chunk_values<base_epi(kEpi), true>(p, r, row_ok, row, n0 + c * 32, c, xs_row, nullptr, col_ws,
                                                   col_bias, packed);
              else
                chunk_values<base_epi(kEpi), false>(p, r, row_ok, row, n0 + c * 32, c, xs_row, nullptr, col_ws,
                                                    col_bias, packed);
#pragma unroll
              for (int i = 0; i < 16; ++i) v[16 * cc + i] = p2_from_bf2(packed[i]);
            }
            rot_stage01(v);
            rot_stage_pairs<2>(v);
            rot_stage_pairs<8>(v);
#pragma unroll
            for (int cc = 0; cc < 2; ++cc) {
              uint32_t w[32];
#pragma unroll
              for (int i = 0; i < 16; ++i) {
                w[2 * i] = uint32_t(v[16 * cc + i]);
                w[2 * i + 1] = uint32_t(v[16 * cc + i] >> 32);
              }
              __syncwarp();
              tmem_store_32cols(t_row + uint32_t((2 * blk + cc) * 32), w);
            }
          }
          tmem_store_wait();
          tc_fence_before();
          quarter_sync(quarter);   // both column halves of these 32 rows are in TMEM
          tc_fence_after();
          // Pass 2: the stage over index bits (6,7) for this warp's positions c of
          // each 64-column block: the four values c + 64 k.
          // The outputs of positions [32 half, 32 half + 32) of block k are one
          // 32-column chunk: the first run's words wait in registers for the second.
          float mx = 0.0f;
          uint32_t first[4][8];
#pragma unroll
          for (int cc = 0; cc < kRuns; ++cc) {
            const int c0 = 16 * (kRuns * slice + cc);
            uint64_t v[32];   // pair 8 k + i: positions c0 + 64 k + 2 i, + 1
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              uint32_t u[16];
              __syncwarp();
              tmem_load_16cols(t_row + uint32_t(c0 + 64 * k), u);
              tmem_load_wait();
#pragma unroll
              for (int i = 0; i < 8; ++i) v[8 * k + i] = p2(__uint_as_float(u[2 * i]), __uint_as_float(u[2 * i + 1]));
            }
            if (cc == kRuns - 1) release();   // every TMEM read of this accumulator is done
            rot_stage_pairs<8>(v);
#pragma unroll
            for (int i = 0; i < 32; i += 2)
              mx = fmaxf(mx, fmaxf(fmaxf(fabsf(p2_lo(v[i])), fabsf(p2_hi(v[i]))),
                                   fmaxf(fabsf(p2_lo(v[i + 1])), fabsf(p2_hi(v[i + 1])))));
            if (cc == 0) {
#pragma unroll
              for (int k = 0; k < 4; ++k)
#pragma unroll
                for (int i = 0; i < 8; ++i) first[k][i] = pack_bf2(v[8 * k + i]);
            } else if (row_base < p.m) {
#pragma unroll
              for (int k = 0; k < 4; ++k) {
                uint32_t packed[16];
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                  packed[i] = first[k][i];
                  packed[8 + i] = pack_bf2(v[8 * k + i]);
                }
                store_chunk(n0 + 32 * slice + 64 * k, packed);
              }
            }
          }
          // max |rotated value| of the row: non-negative and never NaN (fmaxf drops
          // NaN), so its bits order as unsigned integers
          if (row_ok) atomicMax(p.rowmax + row, __float_as_uint(mx));
        }
      } else if constexpr (H3SK_TMEM_PREFETCH == 1 || (H3SK_TMEM_PREFETCH == 2 && kDual)) {
        // chunk c + 1's TMEM load is in flight while chunk c is computed
        uint32_t r[32];
        __syncwarp();
        tmem_load_32cols(t_row + uint32_t(c_first * 32), r);
#pragma unroll
        for (int i = 0; i < kBN / 64; ++i) {
          const int c = c_first + i;
          tmem_load_wait();
          if (c == c_last) release();
          uint32_t cur[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) cur[j] = r[j];
          if (c < c_last) {
            __syncwarp();
            tmem_load_32cols(t_row + uint32_t((c + 1) * 32), r);
          }
          emit(c, cur);
        }
      } else {
#pragma unroll 1
        for (int c = c_first; c <= c_last; ++c) {
          uint32_t r[32];
          __syncwarp();
          tmem_load_32cols(t_row + uint32_t(c * 32), r);
          tmem_load_wait();
          if (c == c_last) release();
          emit(c, r);
        }
      }
      __syncwarp();
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
    if (lane == 0) bulk_wait_all();   // every output store has completed
    __syncwarp();
  }

  // The pair's TMEM is written by the leader's MMAs and its barriers receive the
  // peer's arrivals: neither CTA releases TMEM or exits before both are done.
  tc_fence_before();
  if constexpr (kPair) cluster_sync_all();
  else __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    if constexpr (kPair) tmem_dealloc_pair(tmem_base, kTmemCols);
    else tmem_dealloc(tmem_base, kTmemCols);
  }
}

// ---- bounded-wait self-test and MMA issue-rate probe --------------------------

__global__ void wait_selftest_kernel(int* status, uint64_t timeout_ns) {
  __shared__ uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    // Nothing ever arrives on `bar`: the wait must run out and report.
    mbar_wait_bounded(&bar, 0, reinterpret_cast<volatile int*>(&abort_flag), status, H3SK_STATUS_WAIT_TIMEOUT,
                      timeout_ns);
  }
}

__global__ void __launch_bounds__(128, 1) mma_peak_kernel(int iters, int* status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ uint64_t done;
  __shared__ uint32_t slot;
  for (int i = threadIdx.x; i < Shape<false>::stage_bytes / 16; i += blockDim.x)
    reinterpret_cast<uint4*>(smem)[i] = make_uint4(0x01010101u, 0x01010101u, 0x01010101u, 0x01010101u);
  if (threadIdx.x == 0) {
    mbar_init(&done, 1);
    fence_mbar_init();
  }
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  const int warp = threadIdx.x >> 5;
  if (warp == 0) {
    tmem_alloc(&slot, 256);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = slot;
  if (warp == 0) {
    if (threadIdx.x == 0) {
      const uint64_t a_desc = smem_desc_k_sw128(smem);
      const uint64_t b_desc = smem_desc_k_sw128(smem + kATileBytes);
      for (int i = 0; i < iters; ++i) {
        const int kk = i & 3;
        mma_i8(tmem, a_desc + uint64_t(2 * kk), b_desc + uint64_t(2 * kk), Shape<false>::idesc, i > 0 ? 1u : 0u);
      }
      mma_commit(&done);
      mbar_wait_bounded(&done, 0, nullptr, status, 41, kWaitTimeoutNs);
    }
    __syncwarp();
  }
  __syncthreads();
  if (warp == 0) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 256);
  }
}

// ---- host side -------------------------------------------------------------------

thread_local int t_last_error = 0;
thread_local char t_last_message[256] = "ok";

int fail(int code, const char* what) {
  t_last_error = code;
  std::snprintf(t_last_message, sizeof(t_last_message), "%s (%s)", what,
                cudaGetErrorString(static_cast<cudaError_t>(code)));
  return 0;
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
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

// K-major INT8 operand [rows, k] with row stride k bytes, box of box_rows x 128 bytes.
bool make_operand_map(CUtensorMap* map, const void* base, int rows, int k, int box_rows) {
  auto fn = encode_fn();
  if (!fn) return false;
  const cuuint64_t dims[2] = {cuuint64_t(k), cuuint64_t(rows)};
  const cuuint64_t strides[1] = {cuuint64_t(k)};
  const cuuint32_t box[2] = {cuuint32_t(kBK), cuuint32_t(box_rows)};
  const cuuint32_t elem_strides[2] = {1, 1};
  const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box,
                        elem_strides, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// BF16 output [rows, cols] with row stride ld elements, stored in 32 x 32 boxes
// from a 64-byte-swizzled staging buffer.
bool make_output_map(CUtensorMap* map, const void* base, int rows, int cols, int64_t ld) {
  auto fn = encode_fn();
  if (!fn) return false;
  const cuuint64_t dims[2] = {cuuint64_t(cols), cuuint64_t(rows)};
  const cuuint64_t strides[1] = {cuuint64_t(ld) * 2};
  const cuuint32_t box[2] = {32, 32};
  const cuuint32_t elem_strides[2] = {1, 1};
  const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box,
                        elem_strides, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B,
                        CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// Head-major BF16 output: plane h = columns [128h, 128h + 128) of the product,
// stored as [heads, rows, 128] (plane stride rows * 128 elements), 32 x 32 boxes.
bool make_output_map_heads(CUtensorMap* map, const void* base, int rows, int heads) {
  auto fn = encode_fn();
  if (!fn) return false;
  const cuuint64_t dims[3] = {128, cuuint64_t(rows), cuuint64_t(heads)};
  const cuuint64_t strides[2] = {256, cuuint64_t(rows) * 256};
  const cuuint32_t box[3] = {32, 32, 1};
  const cuuint32_t elem_strides[3] = {1, 1, 1};
  const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box,
                        elem_strides, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B,
                        CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

struct DeviceInfo {
  int sms = 0;
  bool attrs_set[2][2][kEpiKinds] = {};   // [pair][dual][epilogue]
  int max_pairs[2][kEpiKinds] = {};       // co-resident clusters of two CTAs, per [dual][epilogue]
};

DeviceInfo& device_info(int device) {
  static std::mutex mu;
  static DeviceInfo infos[64];
  std::lock_guard<std::mutex> lock(mu);
  DeviceInfo& d = infos[device & 63];
  if (d.sms == 0) cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, device);
  return d;
}

int* status_ptr() {
  int* ptr = nullptr;
  if (cudaGetSymbolAddress(reinterpret_cast<void**>(&ptr), g_pipeline_status) != cudaSuccess) return nullptr;
  return ptr;
}

template <int kEpi, bool kPair, bool kDual = false>
cudaError_t launch_gemm(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& md, GemmParams p,
                        cudaStream_t stream) {
  using L = SmemLayout<kPair, kDual, is_rot(kEpi)>;
  int device = 0;
  cudaError_t e = cudaGetDevice(&device);
  if (e != cudaSuccess) return e;
  DeviceInfo& info = device_info(device);
  auto kernel = int8_gemm_persistent<kEpi, kPair, kDual>;
  if (!info.attrs_set[kPair][kDual][kEpi]) {
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, L::dynamic_bytes);
    if (e != cudaSuccess) return e;
    info.attrs_set[kPair][kDual][kEpi] = true;
  }
  p.status = status_ptr();
  if (!p.status) return cudaErrorInvalidSymbol;
  if constexpr (!kPair) {
    const int grid = p.work < info.sms ? p.work : info.sms;
    kernel<<<grid, kThreads, L::dynamic_bytes, stream>>>(ma, mb, md, p);
    return cudaGetLastError();
  } else {
    // As many clusters of two CTAs as can be resident at once (SMs of a GPC pair
    // up; an odd SM stays idle), no more than there are tiles.
    cudaLaunchConfig_t cfg{};
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = L::dynamic_bytes;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (info.max_pairs[kDual][kEpi] == 0) {
      cfg.gridDim = dim3(unsigned(info.sms & ~1));
      int clusters = 0;
      e = cudaOccupancyMaxActiveClusters(&clusters, kernel, &cfg);
      if (e != cudaSuccess) return e;
      if (clusters < 1) return cudaErrorInvalidConfiguration;
      info.max_pairs[kDual][kEpi] = clusters;
    }
    const int pairs = p.work < info.max_pairs[kDual][kEpi] ? p.work : info.max_pairs[kDual][kEpi];
    cfg.gridDim = dim3(unsigned(2 * pairs));
    return cudaLaunchKernelEx(&cfg, kernel, ma, mb, md, p);
  }
}

int run_gemm(int epi, const int8_t* A, const int8_t* B, const float* xs, const float* ws, const void* bias,
             void* D, int64_t ldd, const void* gate, const int32_t* rows, const void* residual, int M, int N,
             int K, cudaStream_t stream, bool heads = false, const HeadsArgs* hd = nullptr,
             uint32_t* rowmax = nullptr, int rot_n0 = 0) {
  if (!A || !B || !D || M < 1 || N < 1 || K < 16 || K % 16 || N % 8 || ldd < N || ldd % 8)
    return fail(cudaErrorInvalidValue, "h3_int8: invalid shape or null operand");
  if (heads && ((epi != kEpiDequant && epi != kEpiHeads) || N % 128))
    return fail(cudaErrorInvalidValue, "h3_int8: head-major output needs the dequant epilogue and N % 128 == 0");
  if (epi == kEpiHeads && (!heads || !hd || hd->heads < 2 || hd->heads % 2 || N != 3 * hd->heads * 128 ||
                           !hd->freqs || !hd->qw || !hd->kw))
    return fail(cudaErrorInvalidValue, "h3_qkv: the fused head epilogue needs an even head count and N = 3*heads*128");
  if (is_rot(epi) && (heads || !rowmax || (uintptr_t(rowmax) & 3u) || N % kBN || rot_n0 < 0 || rot_n0 >= N ||
                      rot_n0 % kBN))
    return fail(cudaErrorInvalidValue, "h3_int8_rot: needs rowmax, N % 256 == 0 and rot_n0 % 256 == 0 below N");
  if ((uintptr_t(A) & 15u) || (uintptr_t(B) & 15u) || (uintptr_t(D) & 15u))
    return fail(cudaErrorInvalidValue, "h3_int8: A, B and D must be 16-byte aligned");
  if (epi != kEpiAcc && (!xs || !ws || (uintptr_t(xs) & 3u) || (uintptr_t(ws) & 3u)))
    return fail(cudaErrorInvalidValue, "h3_int8: scales must be non-null FP32");
  if (bias && (uintptr_t(bias) & 1u)) return fail(cudaErrorInvalidValue, "h3_int8: misaligned bias");
  if (epi == kEpiGate) {
    if (!gate || !rows || !residual || (uintptr_t(gate) & 15u) || (uintptr_t(residual) & 15u) ||
        (uintptr_t(rows) & 3u))
      return fail(cudaErrorInvalidValue, "h3_int8_gate: gate/rows/residual null or misaligned");
  }
  // CTA pairs whenever the problem has more than one 128-row tile row.
  const bool pair = M > kBM;
  CUtensorMap ma, mb, md;
  if (!make_operand_map(&ma, A, M, K, kBM) ||
      !make_operand_map(&mb, B, N, K, pair ? Shape<true>::b_rows : Shape<false>::b_rows))
    return fail(cudaErrorInvalidValue, "h3_int8: tensor map encoding failed");
  std::memset(&md, 0, sizeof(md));
  if (epi != kEpiAcc && !(heads ? make_output_map_heads(&md, D, M, N / 128) : make_output_map(&md, D, M, N, ldd)))
    return fail(cudaErrorInvalidValue, "h3_int8: output tensor map encoding failed");
  GemmParams p{};
  p.xs = xs;
  p.ws = ws;
  p.bias = static_cast<const __nv_bfloat16*>(bias);
  p.d = D;
  p.ldd = ldd;
  p.gate = static_cast<const __nv_bfloat16*>(gate);
  p.rows = rows;
  p.residual = static_cast<const __nv_bfloat16*>(residual);
  p.gate_ld = N;
  p.ldr = N;
  p.m = M;
  p.n = N;
  p.k = K;
  p.head_major = heads ? 1 : 0;
  if (hd) p.hd = *hd;
  p.rowmax = rowmax;
  p.rot_n0 = rot_n0;
  p.m_tiles = (M + (pair ? 2 * kBM : kBM) - 1) / (pair ? 2 * kBM : kBM);
  p.n_tiles = (N + kBN - 1) / kBN;
  p.k_blocks = (K + kBK - 1) / kBK;
  // The dual form (two N-tiles per work unit, one A stage for both) where K is
  // long enough for its unoverlapped epilogue to be small against the mainloop
  // and there are enough units (>= kDualMinWaves per co-resident pair) for the
  // larger units not to lose a partial last wave.
  int device = 0;
  if (cudaGetDevice(&device) != cudaSuccess) return fail(cudaErrorInvalidDevice, "h3_int8: no device");
  const int approx_pairs = device_info(device).sms / 2;
  const bool dual = pair && epi != kEpiHeads && !is_rot(epi) && K >= kDualMinK && p.n_tiles % 2 == 0 &&
                    int64_t(p.m_tiles) * (p.n_tiles / 2) >= int64_t(kDualMinWaves) * approx_pairs;
  const int dual_n = dual ? 2 : 1;
  p.n_units = p.n_tiles / dual_n;
  p.work = p.m_tiles * p.n_units;
  {
    const int64_t slice = int64_t(kBN) * dual_n * K;   // B bytes of one work unit's N-tiles
    const int64_t g = (dual ? kDualBSliceBytes : kBSliceBytes) / (slice > 0 ? slice : 1);
    p.group_n = int(g < 1 ? 1 : (g > p.n_units ? p.n_units : g));
  }
  p.timeout_ns = kWaitTimeoutNs;
  cudaError_t e;
  if (is_rot(epi)) {   // the row maxima accumulate from zero (after every check above)
    e = cudaMemsetAsync(rowmax, 0, size_t(M) * sizeof(uint32_t), stream);
    if (e != cudaSuccess) return fail(e, "h3_int8_gelu_rot: row maxima reset failed");
  }
  if (dual) {
    switch (epi) {
      case kEpiDequant: e = launch_gemm<kEpiDequant, true, true>(ma, mb, md, p, stream); break;
      case kEpiGelu: e = launch_gemm<kEpiGelu, true, true>(ma, mb, md, p, stream); break;
      case kEpiGate: e = launch_gemm<kEpiGate, true, true>(ma, mb, md, p, stream); break;
      default: e = launch_gemm<kEpiAcc, true, true>(ma, mb, md, p, stream); break;
    }
  } else if (pair) {
    switch (epi) {
      case kEpiDequant: e = launch_gemm<kEpiDequant, true>(ma, mb, md, p, stream); break;
      case kEpiGelu: e = launch_gemm<kEpiGelu, true>(ma, mb, md, p, stream); break;
      case kEpiGate: e = launch_gemm<kEpiGate, true>(ma, mb, md, p, stream); break;
      case kEpiHeads: e = launch_gemm<kEpiHeads, true>(ma, mb, md, p, stream); break;
      case kEpiGeluRot: e = launch_gemm<kEpiGeluRot, true>(ma, mb, md, p, stream); break;
      case kEpiDequantRot: e = launch_gemm<kEpiDequantRot, true>(ma, mb, md, p, stream); break;
      default: e = launch_gemm<kEpiAcc, true>(ma, mb, md, p, stream); break;
    }
  } else {
    switch (epi) {
      case kEpiDequant: e = launch_gemm<kEpiDequant, false>(ma, mb, md, p, stream); break;
      case kEpiGelu: e = launch_gemm<kEpiGelu, false>(ma, mb, md, p, stream); break;
      case kEpiGate: e = launch_gemm<kEpiGate, false>(ma, mb, md, p, stream); break;
      case kEpiHeads: e = launch_gemm<kEpiHeads, false>(ma, mb, md, p, stream); break;
      case kEpiGeluRot: e = launch_gemm<kEpiGeluRot, false>(ma, mb, md, p, stream); break;
      case kEpiDequantRot: e = launch_gemm<kEpiDequantRot, false>(ma, mb, md, p, stream); break;
      default: e = launch_gemm<kEpiAcc, false>(ma, mb, md, p, stream); break;
    }
  }
  if (e != cudaSuccess) return fail(e, "h3_int8: launch failed");
  t_last_error = 0;
  std::snprintf(t_last_message, sizeof(t_last_message), "ok");
  return 1;
}

}  // namespace

int* status_device_ptr() { return status_ptr(); }

int gemm_dequant_heads(const int8_t* A, const int8_t* B, const float* xs, const float* ws, void* D, int M, int N,
                       int K, cudaStream_t stream) {
  return run_gemm(kEpiDequant, A, B, xs, ws, nullptr, D, N, nullptr, nullptr, nullptr, M, N, K, stream, true);
}

int gemm_qkv_heads(const int8_t* A, const int8_t* B, const float* xs, const float* ws, void* D, int M, int K,
                   const HeadsArgs& hd, cudaStream_t stream) {
  return run_gemm(kEpiHeads, A, B, xs, ws, nullptr, D, 3 * hd.heads * 128, nullptr, nullptr, nullptr, M,
                  3 * hd.heads * 128, K, stream, true, &hd);
}

int last_gemm_error() { return t_last_error; }
int record_failure(int code, const char* what) { return fail(code, what); }
void record_success() {
  t_last_error = 0;
  std::snprintf(t_last_message, sizeof(t_last_message), "ok");
}

}  // namespace h3sk

#define H3SK_EXPORT extern "C" __attribute__((visibility("default")))

H3SK_EXPORT int h3_int8(const int8_t* A, const int8_t* B, const float* xs, const float* ws, void* D, int M,
                        int N, int K, int config, uintptr_t stream) {
  if (config < 0 || config > 15) return h3sk::fail(cudaErrorInvalidValue, "h3_int8: config out of range");
  return h3sk::run_gemm(h3sk::kEpiDequant, A, B, xs, ws, nullptr, D, N, nullptr, nullptr, nullptr, M, N, K,
                        reinterpret_cast<cudaStream_t>(stream));
}

H3SK_EXPORT int h3_int8_gate(const int8_t* A, const int8_t* B, const float* xs, const float* ws, void* D,
                             const void* gate, const int32_t* rows, const void* residual, int M, int N, int K,
                             int config, uintptr_t stream) {
  if (config < 0 || config > 15) return h3sk::fail(cudaErrorInvalidValue, "h3_int8_gate: config out of range");
  return h3sk::run_gemm(h3sk::kEpiGate, A, B, xs, ws, nullptr, D, N, gate, rows, residual, M, N, K,
                        reinterpret_cast<cudaStream_t>(stream));
}

H3SK_EXPORT int h3_int8_ex(const int8_t* A, const int8_t* B, const float* xs, const float* ws, const void* bias,
                           void* D, int M, int N, int K, int64_t ldd, int epilogue, uintptr_t stream) {
  if (epilogue != H3_EPI_DEQUANT && epilogue != H3_EPI_DEQUANT_GELU && epilogue != H3_EPI_ACC_INT32)
    return h3sk::fail(cudaErrorInvalidValue, "h3_int8_ex: unknown epilogue");
  if (epilogue == H3_EPI_ACC_INT32 && (ldd % 4)) return h3sk::fail(cudaErrorInvalidValue, "h3_int8_ex: ldd");
  return h3sk::run_gemm(epilogue, A, B, xs, ws, bias, D, ldd, nullptr, nullptr, nullptr, M, N, K,
                        reinterpret_cast<cudaStream_t>(stream));
}

H3SK_EXPORT int h3_int8_gelu_rot(const int8_t* A, const int8_t* B, const float* xs, const float* ws,
                                 const void* bias, void* V, void* rowmax, int M, int N, int K, int64_t ldv,
                                 uintptr_t stream) {
  return h3sk::run_gemm(h3sk::kEpiGeluRot, A, B, xs, ws, bias, V, ldv, nullptr, nullptr, nullptr, M, N, K,
                        reinterpret_cast<cudaStream_t>(stream), false, nullptr, static_cast<uint32_t*>(rowmax));
}

H3SK_EXPORT int h3_int8_rot(const int8_t* A, const int8_t* B, const float* xs, const float* ws, const void* bias,
                            void* D, void* rowmax, int M, int N, int K, int64_t ldd, int gelu, int rot_n0,
                            uintptr_t stream) {
  if (gelu != 0 && gelu != 1) return h3sk::fail(cudaErrorInvalidValue, "h3_int8_rot: gelu is 0 or 1");
  return h3sk::run_gemm(gelu ? h3sk::kEpiGeluRot : h3sk::kEpiDequantRot, A, B, xs, ws, bias, D, ldd, nullptr,
                        nullptr, nullptr, M, N, K, reinterpret_cast<cudaStream_t>(stream), false, nullptr,
                        static_cast<uint32_t*>(rowmax), rot_n0);
}

H3SK_EXPORT int h3_int8_gate_ex(const int8_t* A, const int8_t* B, const float* xs, const float* ws,
                                const void* bias, void* D, const void* gate, const int32_t* rows,
                                const void* residual, void* q, void* qscale, int M, int N, int K,
                                uintptr_t stream) {
  if ((q == nullptr) != (qscale == nullptr))
    return h3sk::fail(cudaErrorInvalidValue, "h3_int8_gate_ex: q and qscale go together");
  if (q && (N % 256 || N > 16384 || (uintptr_t(q) & 7u) || (uintptr_t(qscale) & 3u)))
    return h3sk::fail(cudaErrorInvalidValue, "h3_int8_gate_ex: requant needs N % 256 == 0, N <= 16384");
  const cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (!h3sk::run_gemm(h3sk::kEpiGate, A, B, xs, ws, bias, D, N, gate, rows, residual, M, N, K, s)) return 0;
  if (q) {
    const cudaError_t e = h3sk::convrot_quant_none(D, N, q, qscale, M, N, s);
    if (e != cudaSuccess) return h3sk::fail(e, "h3_int8_gate_ex: requant launch failed");
  }
  return 1;
}

H3SK_EXPORT int h3_int8_last_error(void) { return h3sk::t_last_error; }
H3SK_EXPORT const char* h3_int8_error(void) { return h3sk::t_last_message; }

H3SK_EXPORT int h3sk_pipeline_status(int* status, int clear, uintptr_t stream) {
  if (!status) return cudaErrorInvalidValue;
  const cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  int value = 0;
  cudaError_t e = cudaMemcpyFromSymbolAsync(&value, h3sk::g_pipeline_status, sizeof(int), 0,
                                            cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return e;
  *status = value;
  if (clear && value) {
    const int zero = 0;
    e = cudaMemcpyToSymbolAsync(h3sk::g_pipeline_status, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  }
  return e;
}

H3SK_EXPORT int h3sk_wait_selftest(int timeout_us, int* status, uintptr_t stream) {
  if (!status || timeout_us < 1 || timeout_us > 1000000) return cudaErrorInvalidValue;
  const cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  int* dev = h3sk::status_ptr();
  if (!dev) return cudaErrorInvalidSymbol;
  cudaError_t e = cudaMemsetAsync(dev, 0, sizeof(int), s);
  if (e != cudaSuccess) return e;
  h3sk::wait_selftest_kernel<<<1, 32, 0, s>>>(dev, uint64_t(timeout_us) * 1000ull);
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  return h3sk_pipeline_status(status, 1, stream);
}

H3SK_EXPORT int h3sk_int8_mma_peak(int iters, double* tops, uintptr_t stream) {
  if (!tops || iters < 64 || iters > (1 << 24)) return cudaErrorInvalidValue;
  const cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  int device = 0, sms = 0;
  cudaError_t e = cudaGetDevice(&device);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
  if (e != cudaSuccess) return e;
  int* dev = h3sk::status_ptr();
  if (!dev) return cudaErrorInvalidSymbol;
  // 120 KB of dynamic shared memory keeps the probe at one CTA per SM (only the
  // first 48 KB are read).
  const int smem = 120 * 1024;
  e = cudaFuncSetAttribute(h3sk::mma_peak_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  cudaEvent_t t0, t1;
  cudaEventCreate(&t0);
  cudaEventCreate(&t1);
  h3sk::mma_peak_kernel<<<sms, 128, smem, s>>>(64, dev);   // warm-up
  cudaEventRecord(t0, s);
  h3sk::mma_peak_kernel<<<sms, 128, smem, s>>>(iters, dev);
  cudaEventRecord(t1, s);
  e = cudaGetLastError();
  if (e == cudaSuccess) e = cudaEventSynchronize(t1);
  float ms = 0.0f;
  if (e == cudaSuccess) e = cudaEventElapsedTime(&ms, t0, t1);
  cudaEventDestroy(t0);
  cudaEventDestroy(t1);
  if (e != cudaSuccess) return e;
  const double ops = 2.0 * h3sk::kBM * h3sk::kBN * h3sk::kUmmaK * double(iters) * double(sms);
  *tops = ops / (double(ms) * 1e-3) / 1e12;
  return cudaSuccess;
}

H3SK_EXPORT const char* h3sk_version(void) { return "h3sk_b200 0.1.0 (sm_100a)"; }
