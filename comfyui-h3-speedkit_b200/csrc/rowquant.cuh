// Shared device arithmetic of the row quantisers (prologue and ConvRot quantiser).
//
// Arithmetic contract (the reference's, restated):
//  * ConvRot256 is the normalised 256-point Hadamard transform H4^(x)4 / 16, run
//    as four radix-4 stages over index bit pairs (0,1), (2,3), (4,5), (6,7).  Every
//    output of a stage is 0.5f * h4_d(x0, x1, x2, x3) with the additions taken left
//    to right:  d=0: ((x0+x1)+x2)-x3   d=1: ((x0+x1)-x2)+x3
//               d=2: ((x0-x1)+x2)+x3   d=3: ((-x0+x1)+x2)+x3
//    (kernels/convrot/vendor/convrot64_exact.cuh:202-234, 664-677).
//  * Row scale: max(min(absmax, BF16_MAX) * (1/127), 1e-30), stored unrounded
//    (kernels/norm_quant/norm_quant.cu:189-192).
//  * Code: clamp(nearbyint(bf(bf(v) / bf(scale))), -128, 127)
//    (convrot64_exact.cuh:53-57; convrot_register_v2.cu:126-128).
//
// The reference compiles its quantiser translation units with --use_fast_math
// (tools/build_kernels.py:32-34), which makes the quotient above the compiler's
// fast division with flush-to-zero.  Any TU including this header must be built
// with the same flag so `/` means the same operation; the build passes
// -DH3SK_QUANT_FAST_MATH together with --use_fast_math and this header refuses
// to compile without it.
#pragma once
#ifndef H3SK_QUANT_FAST_MATH
#error "rowquant.cuh must be compiled with --use_fast_math -DH3SK_QUANT_FAST_MATH (reference quantiser semantics)"
#endif

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

namespace h3sk {

constexpr unsigned kFullMask = 0xffffffffu;
constexpr float kBf16Max = 3.38953139e38f;

// ---- BF16 bit helpers -------------------------------------------------------
__device__ __forceinline__ float bf_bits_to_float(uint32_t bits16) {
  return __uint_as_float(bits16 << 16);
}
// Round-to-nearest-even FP32 -> BF16 bits (cvt.rn.bf16.f32).
__device__ __forceinline__ uint32_t float_to_bf_bits(float a) {
  unsigned short b;
  asm("cvt.rn.bf16.f32 %0, %1;" : "=h"(b) : "f"(a));
  return b;
}
__device__ __forceinline__ float bf_round(float a) { return bf_bits_to_float(float_to_bf_bits(a)); }

// ---- IEEE round-to-nearest FP32 operations without FTZ or contraction -------
// Inline PTX is untouched by --use_fast_math, so these keep subnormals and the
// operation boundaries the RMSNorm prefix needs (norm_quant.cu:19-38).
__device__ __forceinline__ float ieee_add(float a, float b) {
  float c; asm("add.rn.f32 %0, %1, %2;" : "=f"(c) : "f"(a), "f"(b)); return c;
}
__device__ __forceinline__ float ieee_mul(float a, float b) {
  float c; asm("mul.rn.f32 %0, %1, %2;" : "=f"(c) : "f"(a), "f"(b)); return c;
}
__device__ __forceinline__ float ieee_fma(float a, float b, float c) {
  float d; asm("fma.rn.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c)); return d;
}
__device__ __forceinline__ float ieee_div(float a, float b) {
  float c; asm("div.rn.f32 %0, %1, %2;" : "=f"(c) : "f"(a), "f"(b)); return c;
}
// Hardware reciprocal square root (MUFU), the instruction the reference uses for
// rrms; its input is positive and normal because eps >= FLT_MIN.
__device__ __forceinline__ float hw_rsqrt(float a) {
  float b; asm("rsqrt.approx.f32 %0, %1;" : "=f"(b) : "f"(a)); return b;
}

// ---- Register-resident ConvRot256 -------------------------------------------
// Layout: a 256-value group lives in 8 consecutive lanes ("octet"), 32 values per
// lane.  For value index p (8 bits) of the group:
//   register r = (p & 7) | ((p >> 4) & 1) << 3 | ((p >> 6) & 1) << 4
//   octet lane = ((p >> 3) & 1) | ((p >> 5) & 1) << 1 | ((p >> 7) & 1) << 2
// so index bits {0,1,2,4,6} are register bits and {3,5,7} are lane bits.  The
// 8-element run of register block j (j = 0..3) in octet lane o starts at
// group column octet_run_col(o, j) and is contiguous in memory.
__device__ __forceinline__ int octet_run_col(int o, int j) {
  return ((o & 1) << 3) | ((j & 1) << 4) | ((o & 2) << 4) | ((j & 2) << 5) | ((o & 4) << 5);
}

// One output of a radix-4 stage: row d of the regular H4 block, halved.
__device__ __forceinline__ float h4_half(int d, float x0, float x1, float x2, float x3) {
  float s;
  if (d == 0)      s = x0 + x1 + x2 - x3;
  else if (d == 1) s = x0 + x1 - x2 + x3;
  else if (d == 2) s = x0 - x1 + x2 + x3;
  else             s = -x0 + x1 + x2 + x3;
  return 0.5f * s;
}

// Stage over index bits (0,1): both bits are register bits 0 and 1.
__device__ __forceinline__ void fht_stage_in_lane(float (&v)[32]) {
#pragma unroll
  for (int r = 0; r < 32; r += 4) {
    const float x0 = v[r], x1 = v[r + 1], x2 = v[r + 2], x3 = v[r + 3];
    v[r]     = h4_half(0, x0, x1, x2, x3);
    v[r + 1] = h4_half(1, x0, x1, x2, x3);
    v[r + 2] = h4_half(2, x0, x1, x2, x3);
    v[r + 3] = h4_half(3, x0, x1, x2, x3);
  }
}

// Stage whose low index bit is register bit RBIT and high index bit is octet
// lane bit LBIT: the quadruple (x0..x3) is {(own, r), (own, r|RBIT),
// (peer, r), (peer, r|RBIT)} ordered by (lane bit, register bit).  The lane with
// the lane bit clear produces rows 0/1, its partner rows 2/3; both evaluate the
// canonical x0..x3 order so rounding and signed zeros match.
template <int RBIT, int LBIT>
__device__ __forceinline__ void fht_stage_cross_lane(float (&v)[32], int lane) {
  const bool upper = (lane & LBIT) != 0;
#pragma unroll
  for (int r = 0; r < 32; ++r) {
    if (r & RBIT) continue;
    const float a = v[r], b = v[r | RBIT];
    const float pa = __shfl_xor_sync(kFullMask, a, LBIT);
    const float pb = __shfl_xor_sync(kFullMask, b, LBIT);
    const float x0 = upper ? pa : a, x1 = upper ? pb : b;
    const float x2 = upper ? a : pa, x3 = upper ? b : pb;
    v[r]        = h4_half(upper ? 2 : 0, x0, x1, x2, x3);
    v[r | RBIT] = h4_half(upper ? 3 : 1, x0, x1, x2, x3);
  }
}

__device__ __forceinline__ void convrot256_registers(float (&v)[32], int lane) {
  fht_stage_in_lane(v);               // index bits 0,1
  fht_stage_cross_lane<4, 1>(v, lane);   // index bits 2 (reg bit 2), 3 (lane bit 0)
  fht_stage_cross_lane<8, 2>(v, lane);   // index bits 4 (reg bit 3), 5 (lane bit 1)
  fht_stage_cross_lane<16, 4>(v, lane);  // index bits 6 (reg bit 4), 7 (lane bit 2)
}

// ---- Row scale and codes ----------------------------------------------------
__device__ __forceinline__ float warp_allmax(float value) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) value = fmaxf(value, __shfl_xor_sync(kFullMask, value, off));
  return value;
}

__device__ __forceinline__ float int8_row_scale(float abs_max) {
  return fmaxf(fminf(abs_max, kBf16Max) * (1.0f / 127.0f), 1.0e-30f);
}

// INT8 code of one rotated value given the row scale (see the header comment).
__device__ __forceinline__ uint32_t int8_code(float value, float scale) {
  const float scale_bf = __bfloat162float(__float2bfloat16_rn(scale));
  const float value_bf = __bfloat162float(__float2bfloat16_rn(value));
  const float scaled = __bfloat162float(__float2bfloat16_rn(value_bf / scale_bf));
  float code = nearbyintf(scaled);
  code = fminf(127.0f, fmaxf(-128.0f, code));
  return static_cast<uint32_t>(static_cast<unsigned char>(static_cast<int8_t>(code)));
}

// Pack the codes of eight consecutive values into two little-endian words.
__device__ __forceinline__ uint2 pack_codes8(const float* v8, float scale) {
  uint32_t lo = 0, hi = 0;
#pragma unroll
  for (int e = 0; e < 4; ++e) lo |= int8_code(v8[e], scale) << (8 * e);
#pragma unroll
  for (int e = 0; e < 4; ++e) hi |= int8_code(v8[4 + e], scale) << (8 * e);
  return make_uint2(lo, hi);
}

// Input activations the quantiser can absorb (codes of input_act_codes.h:13).
enum : int { kActNone = 0, kActGeluTanh = 1, kActSwiGLU = 2 };

// GELU-tanh as torch.nn.functional.gelu(approximate="tanh"), the expression of
// convrot64_exact.cuh:913-923.
__device__ __forceinline__ float gelu_tanh(float v) {
  const float inner = 0.7978845608028654f * (v + 0.044715f * v * v * v);
  return 0.5f * v * (1.0f + tanhf(inner));
}
// silu(gate) * up, the expression of convrot64_exact.cuh:928-937.
__device__ __forceinline__ float swiglu(float gate, float up) {
  return (gate / (1.0f + expf(-gate))) * up;
}

}  // namespace h3sk
