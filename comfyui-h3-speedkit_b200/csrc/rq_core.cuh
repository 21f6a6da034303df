// Register/shared-memory core of the B200 row quantisers: ConvRot256 of a row
// held 64 values per thread, row absmax, and INT8 codes.
//
// Thread layout.  A 256-value group is owned by 4 consecutive lanes (a "quad
// team"); thread q of the team owns 64 values.  Index bits of a value inside its
// group: b0..b7.
//   layout A  (loads, FHT stages 1-3): registers hold b0..b5, the team index q
//             is b6,b7 -- i.e. thread q owns the 64 consecutive values [64q, 64q+64).
//   layout B  (FHT stage 4, absmax, codes, stores): registers hold b0..b3 and
//             b6,b7, the team index is b4,b5 -- four runs of 16 consecutive values.
// One exchange through shared memory moves the data from A to B; every access is
// a 16-byte vector and the buffer is XOR-swizzled so that a warp's 32 accesses
// hit 8 distinct 16-byte bank groups 4 times each (the minimum, 4 wavefronts).
// Registers are paired on b0 (float2) so FHT stages 2-4 run as packed f32x2
// instructions; stage 1 (b0,b1) runs on scalars.
//
// Arithmetic is the reference's (see rowquant.cuh for the contract), restated in
// an exactly equal form:
//   * every stage output 0.5*RN(((x0 +- x1) +- x2) -+ x3) is computed as
//     fma(t, 0.5, +-0.5*x3) with t = RN((x0 +- x1) +- x2): scaling by 0.5 is exact
//     and commutes with round-to-nearest, so RN(0.5*t +- 0.5*x3) =
//     0.5*RN(t +- x3) bit for bit for normal values (all operations flush
//     subnormals as the reference's --use_fast_math translation unit does);
//   * (-x0 + x1) + x2 is evaluated as x2 - (x0 - x1), the same rounded value;
//   * codes: bf(v) / bf(scale) is the same C division as the reference; the
//     quotient is rounded to BF16 (cvt.rn.bf16x2), NaN is mapped to -128 by a
//     BF16 max with -128 (the reference's fmaxf(-128, NaN)), rounded to an
//     integer half-to-even (cvt.rni.s32.bf16) and saturated to [-128, 127] while
//     packing (cvt.pack.sat.s8.s32) -- equal to clamp(nearbyintf(.), -128, 127).
#pragma once
#include "rowquant.cuh"

namespace h3sk {
namespace rq {

constexpr int kTeam = 4;        // threads per 256-value group
constexpr int kVals = 64;       // values per thread
constexpr int kGroupBytes = 1024;

// ---- packed FP32 (sm_100 f32x2) -----------------------------------------------
__device__ __forceinline__ uint64_t f2_pack(float lo, float hi) {
  return (uint64_t(__float_as_uint(hi)) << 32) | __float_as_uint(lo);
}
__device__ __forceinline__ float f2_lo(uint64_t p) { return __uint_as_float(uint32_t(p)); }
__device__ __forceinline__ float f2_hi(uint64_t p) { return __uint_as_float(uint32_t(p >> 32)); }
// Flush-to-zero forms: the quantiser translation unit semantics.
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
  uint64_t c; asm("add.rn.ftz.f32x2 %0, %1, %2;" : "=l"(c) : "l"(a), "l"(b)); return c;
}
__device__ __forceinline__ uint64_t f2_sub(uint64_t a, uint64_t b) {
  uint64_t c; asm("sub.rn.ftz.f32x2 %0, %1, %2;" : "=l"(c) : "l"(a), "l"(b)); return c;
}
__device__ __forceinline__ uint64_t f2_mul(uint64_t a, uint64_t b) {
  uint64_t c; asm("mul.rn.ftz.f32x2 %0, %1, %2;" : "=l"(c) : "l"(a), "l"(b)); return c;
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d; asm("fma.rn.ftz.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c)); return d;
}
// IEEE (no flush) multiply, for the RMSNorm prefix (norm_quant.cu:22-45).
__device__ __forceinline__ uint64_t f2_mul_ieee(uint64_t a, uint64_t b) {
  uint64_t c; asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(c) : "l"(a), "l"(b)); return c;
}
__device__ __forceinline__ uint64_t f2_fma_ieee(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d; asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c)); return d;
}
__device__ __forceinline__ uint64_t f2_add_ieee(uint64_t a, uint64_t b) {
  uint64_t c; asm("add.rn.f32x2 %0, %1, %2;" : "=l"(c) : "l"(a), "l"(b)); return c;
}

// acc + x*x for both BF16 halves of `w` in element order (low half first), each an
// IEEE round-to-nearest FMA without flush (fma.rn.f32.bf16: the BF16 product is
// exact in FP32, so this is fma.rn.f32 on the widened value, unwidened).
__device__ __forceinline__ float fma_sq_bf2(uint32_t w, float acc) {
  float d;
  asm("{\n\t.reg .b16 lo, hi;\n\tmov.b32 {lo, hi}, %1;\n\t"
      "fma.rn.f32.bf16 %0, lo, lo, %2;\n\tfma.rn.f32.bf16 %0, hi, hi, %0;\n\t}"
      : "=f"(d) : "r"(w), "f"(acc));
  return d;
}

// Residual update of two BF16 elements (residual_quant.cu:59-71):
// bf(fma(b, g, x)) per half, where the FMA is the IEEE round-to-nearest
// fma.rn.f32.bf16 (exact BF16 product, FP32 addend x widened, one rounding, no
// flush) and the FP32 result is rounded once more to BF16.  b, g, x: BF16 pair
// words, element 2i in the low half; g already rounded to BF16.
__device__ __forceinline__ uint32_t residual_bf2(uint32_t b, uint32_t g, uint32_t x) {
  float lo, hi;
  asm("{\n\t.reg .b16 bl, bh, gl, gh;\n\tmov.b32 {bl, bh}, %2;\n\tmov.b32 {gl, gh}, %3;\n\t"
      "fma.rn.f32.bf16 %0, bl, gl, %4;\n\tfma.rn.f32.bf16 %1, bh, gh, %5;\n\t}"
      : "=f"(lo), "=f"(hi)
      : "r"(b), "r"(g), "f"(__uint_as_float(x << 16)), "f"(__uint_as_float(x & 0xffff0000u)));
  uint32_t w;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(w) : "f"(hi), "f"(lo));
  return w;
}

// ---- BF16 pairs ------------------------------------------------------------------
// A 32-bit word of two BF16 values (element 2i in the low half) -> float pair.
__device__ __forceinline__ uint64_t bf2_to_f2(uint32_t w) { return f2_pack(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u)); }
// float pair -> BF16 pair, round to nearest even (low half = lo).
__device__ __forceinline__ uint32_t f2_to_bf2(uint64_t p) {
  uint32_t w; asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(w) : "f"(f2_hi(p)), "f"(f2_lo(p))); return w;
}
__device__ __forceinline__ uint32_t bf2_add(uint32_t a, uint32_t b) {
  uint32_t c; asm("add.rn.bf16x2 %0, %1, %2;" : "=r"(c) : "r"(a), "r"(b)); return c;
}
__device__ __forceinline__ uint32_t bf2_mul(uint32_t a, uint32_t b) {
  uint32_t c; asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(c) : "r"(a), "r"(b)); return c;
}
__device__ __forceinline__ uint32_t bf2_max(uint32_t a, uint32_t b) {
  uint32_t c; asm("max.bf16x2 %0, %1, %2;" : "=r"(c) : "r"(a), "r"(b)); return c;
}

// ---- FHT stages -------------------------------------------------------------------
// Stage over b0,b1 on scalars: quads (4j .. 4j+3).
__device__ __forceinline__ void stage_b01(uint64_t (&v)[32]) {
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const float x0 = f2_lo(v[2 * j]), x1 = f2_hi(v[2 * j]);
    const float x2 = f2_lo(v[2 * j + 1]), x3 = f2_hi(v[2 * j + 1]);
    const float a = x0 + x1, b = x0 - x1;
    const float h = 0.5f * x3;
    const float t0 = a + x2, t1 = a - x2, t2 = b + x2, t3 = x2 - b;
    v[2 * j] = f2_pack(__fmaf_rn(t0, 0.5f, -h), __fmaf_rn(t1, 0.5f, h));
    v[2 * j + 1] = f2_pack(__fmaf_rn(t2, 0.5f, h), __fmaf_rn(t3, 0.5f, h));
  }
}

// Stage over the two index bits held at pair-index strides S and 2S (S >= 1):
// quads {P, P+S, P+2S, P+3S} of pairs, for every P with those bits clear.
template <int S>
__device__ __forceinline__ void stage_pairs(uint64_t (&v)[32]) {
  const uint64_t half = f2_pack(0.5f, 0.5f), nhalf = f2_pack(-0.5f, -0.5f);
#pragma unroll
  for (int p = 0; p < 32; ++p) {
    if ((p / S) & 3) continue;
    const uint64_t x0 = v[p], x1 = v[p + S], x2 = v[p + 2 * S], x3 = v[p + 3 * S];
    const uint64_t a = f2_add(x0, x1), b = f2_sub(x0, x1);
    const uint64_t h = f2_mul(x3, half), nh = f2_mul(x3, nhalf);
    const uint64_t t0 = f2_add(a, x2), t1 = f2_sub(a, x2), t2 = f2_add(b, x2), t3 = f2_sub(x2, b);
    v[p] = f2_fma(t0, half, nh);
    v[p + S] = f2_fma(t1, half, h);
    v[p + 2 * S] = f2_fma(t2, half, h);
    v[p + 3 * S] = f2_fma(t3, half, h);
  }
}

// Layout A: stages over (b0,b1), (b2,b3), (b4,b5).  Pair index = value index / 2,
// so b2,b3 sit at pair strides 2,4 and b4,b5 at 8,16.
__device__ __forceinline__ void fht_layout_a(uint64_t (&v)[32]) {
  stage_b01(v);
  stage_pairs<2>(v);
  stage_pairs<8>(v);
}
// Layout B: registers r = (b0..b3) | (b6,b7) << 4; b6,b7 sit at pair strides 8,16.
__device__ __forceinline__ void fht_layout_b(uint64_t (&v)[32]) { stage_pairs<8>(v); }

// ---- exchange A -> B through a 1 KB per-group buffer ----------------------------
// Logical value p of the group: line L = p >> 5, chunk C = (p >> 2) & 7, word p & 3.
// Physical chunk = C ^ L ^ (3 for odd groups): conflict-free for both sides.
__device__ __forceinline__ uint32_t swz_offset(int p, int odd) {
  const int line = p >> 5, chunk = (p >> 2) & 7;
  return uint32_t(line * 128 + ((chunk ^ line ^ (odd ? 3 : 0)) << 4));
}

// q = team index, buf = this group's 1 KB; the 4 team threads are lanes of one warp.
__device__ __forceinline__ void exchange_a_to_b(uint64_t (&v)[32], float* buf, int q, int odd) {
  char* base = reinterpret_cast<char*>(buf);
#pragma unroll
  for (int k = 0; k < 16; ++k) {
    const int p = 64 * q + 4 * k;   // layout A: registers 4k..4k+3
    *reinterpret_cast<uint4*>(base + swz_offset(p, odd)) =
        make_uint4(uint32_t(v[2 * k]), uint32_t(v[2 * k] >> 32), uint32_t(v[2 * k + 1]), uint32_t(v[2 * k + 1] >> 32));
  }
  __syncwarp();
#pragma unroll
  for (int m = 0; m < 16; ++m) {
    // layout B: registers r = 4m..4m+3 hold b0..b3 = 4(m&3)+w, b4,b5 = q, b6,b7 = m>>2
    const int p = 4 * (m & 3) + 16 * q + 64 * (m >> 2);
    const uint4 c = *reinterpret_cast<const uint4*>(base + swz_offset(p, odd));
    v[2 * m] = (uint64_t(c.y) << 32) | c.x;
    v[2 * m + 1] = (uint64_t(c.w) << 32) | c.z;
  }
  __syncwarp();
}

// ---- absmax, scale, codes ---------------------------------------------------------
// Three-input max (sm_100 max.f32 with three sources; NaN inputs are ignored like
// fmaxf's).  The order of a max reduction does not change its value.
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}
__device__ __forceinline__ float absmax64(const uint64_t (&v)[32]) {
  float m0 = 0.0f, m1 = 0.0f;
#pragma unroll
  for (int p = 0; p < 32; p += 2) {
    m0 = fmax3(m0, fabsf(f2_lo(v[p])), fabsf(f2_hi(v[p])));
    m1 = fmax3(m1, fabsf(f2_lo(v[p + 1])), fabsf(f2_hi(v[p + 1])));
  }
  return fmaxf(m0, m1);
}

// Codes of four consecutive values (two pairs) packed little-endian.
__device__ __forceinline__ uint32_t codes4(uint64_t p01, uint64_t p23, float scale_bf) {
  const uint32_t neg128 = 0xC300C300u;   // BF16 -128, -128
  uint32_t w01 = f2_to_bf2(p01), w23 = f2_to_bf2(p23);
  const float q0 = __uint_as_float(w01 << 16) / scale_bf;
  const float q1 = __uint_as_float(w01 & 0xffff0000u) / scale_bf;
  const float q2 = __uint_as_float(w23 << 16) / scale_bf;
  const float q3 = __uint_as_float(w23 & 0xffff0000u) / scale_bf;
  uint32_t b01, b23;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(b01) : "f"(q1), "f"(q0));
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(b23) : "f"(q3), "f"(q2));
  b01 = bf2_max(b01, neg128);
  b23 = bf2_max(b23, neg128);
  int c0, c1, c2, c3;
  asm("{\n\t.reg .b16 lo, hi;\n\tmov.b32 {lo, hi}, %2;\n\t"
      "cvt.rni.s32.bf16 %0, lo;\n\tcvt.rni.s32.bf16 %1, hi;\n\t}" : "=r"(c0), "=r"(c1) : "r"(b01));
  asm("{\n\t.reg .b16 lo, hi;\n\tmov.b32 {lo, hi}, %2;\n\t"
      "cvt.rni.s32.bf16 %0, lo;\n\tcvt.rni.s32.bf16 %1, hi;\n\t}" : "=r"(c2), "=r"(c3) : "r"(b23));
  uint32_t hi16, word;
  asm("cvt.pack.sat.s8.s32.b32 %0, %1, %2, %3;" : "=r"(hi16) : "r"(c3), "r"(c2), "r"(0));
  asm("cvt.pack.sat.s8.s32.b32 %0, %1, %2, %3;" : "=r"(word) : "r"(c1), "r"(c0), "r"(hi16));
  return word;
}

// Layout B: codes of run j (16 values, registers 16j..16j+15) as one uint4.
__device__ __forceinline__ uint4 codes_run(const uint64_t (&v)[32], int j, float scale_bf) {
  return make_uint4(codes4(v[8 * j + 0], v[8 * j + 1], scale_bf), codes4(v[8 * j + 2], v[8 * j + 3], scale_bf),
                    codes4(v[8 * j + 4], v[8 * j + 5], scale_bf), codes4(v[8 * j + 6], v[8 * j + 7], scale_bf));
}

// Column (within the group) of layout-B run j of team thread q.
__device__ __forceinline__ int run_col_b(int q, int j) { return 16 * q + 64 * j; }

// Store the 64 codes of a layout-B thread: four 16-byte runs (16-byte aligned
// output) or eight 8-byte halves (output aligned to 8 bytes only).
__device__ __forceinline__ void store_codes(int8_t* group_out, int q, const uint64_t (&v)[32], float scale_bf,
                                            int vec16) {
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint4 c = codes_run(v, j, scale_bf);
    int8_t* dst = group_out + run_col_b(q, j);
    if (vec16) {
      *reinterpret_cast<uint4*>(dst) = c;
    } else {
      reinterpret_cast<uint2*>(dst)[0] = make_uint2(c.x, c.y);
      reinterpret_cast<uint2*>(dst)[1] = make_uint2(c.z, c.w);
    }
  }
}

}  // namespace rq
}  // namespace h3sk
