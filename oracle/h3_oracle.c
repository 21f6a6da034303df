/*
 * h3_oracle.c -- CPU restatement of the H3 SpeedKit quantized DiT-block linear
 * path.  TEST INFRASTRUCTURE ONLY: tests/, the smoke check and bench.py's
 * cpu_baseline / reference arm use it as the checker and CPU baseline; the
 * product path never calls it.
 *
 * Every function states the reference lines it restates.  Built with
 * -ffp-contract=off and without fast-math, so each C float operation is one
 * IEEE round-to-nearest FP32 operation and fmaf is the correctly rounded fused
 * multiply-add.  Known, documented departures from the GPU reference:
 *   - rrms: the reference uses the hardware rsqrt.approx.f32; here it is
 *     1/sqrt evaluated in double and rounded (callers may inject the GPU's rrms);
 *   - the quantiser quotient: the reference divides with the compiler's fast
 *     division (its quantiser TUs use --use_fast_math); here IEEE division;
 *   - tanhf/expf in the activations are libm's.
 * Flush-to-zero of the fast-math quantiser TUs is reproduced on the operations
 * of the rotation and the code computation (ftz_* helpers).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define H3O_EXPORT __attribute__((visibility("default")))

/* ---- BF16 / FP32 bit helpers ------------------------------------------------ */
static inline float f_from_u(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
static inline uint32_t u_from_f(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float bf_to_f(uint16_t b) { return f_from_u((uint32_t)b << 16); }
/* Round-to-nearest-even FP32 -> BF16 (cvt.rn.bf16.f32); NaN stays NaN. */
static inline uint16_t f_to_bf(float f) {
  uint32_t u = u_from_f(f);
  if ((u & 0x7f800000u) == 0x7f800000u && (u & 0x007fffffu)) return (uint16_t)((u >> 16) | 0x0040u);
  u += 0x7fffu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}
static inline float bf_round(float f) { return bf_to_f(f_to_bf(f)); }
/* Flush a subnormal to a zero of the same sign. */
static inline float ftz(float f) {
  uint32_t u = u_from_f(f);
  return ((u & 0x7f800000u) == 0 && (u & 0x007fffffu)) ? f_from_u(u & 0x80000000u) : f;
}
static inline float ftz_add(float a, float b) { return ftz(ftz(a) + ftz(b)); }
static inline float ftz_sub(float a, float b) { return ftz(ftz(a) - ftz(b)); }
static inline float ftz_mul(float a, float b) { return ftz(ftz(a) * ftz(b)); }

static int set_threads(int threads) {
#ifdef _OPENMP
  if (threads > 0) omp_set_num_threads(threads);
  return omp_get_max_threads();
#else
  (void)threads;
  return 1;
#endif
}

/* ---- ConvRot256 ---------------------------------------------------------------
 * Four radix-4 stages with strides 1, 4, 16, 64 over one 256-value group; output
 * i of a stage is 0.5f * h4_d(x0..x3) with d = (i / s) & 3, base = i - d*s,
 * x_j = v[base + j*s], and the additions taken left to right
 * (kernels/convrot/vendor/convrot64_exact.cuh:202-234, 664-677).            */
static inline float h4_half(int d, float x0, float x1, float x2, float x3) {
  float s;
  switch (d) {
    case 0: s = ftz_sub(ftz_add(ftz_add(x0, x1), x2), x3); break;
    case 1: s = ftz_add(ftz_sub(ftz_add(x0, x1), x2), x3); break;
    case 2: s = ftz_add(ftz_add(ftz_sub(x0, x1), x2), x3); break;
    default: s = ftz_add(ftz_add(ftz_add(-x0, x1), x2), x3); break;
  }
  return ftz_mul(0.5f, s);
}

static void convrot256(float* g) {
  float tmp[256];
  static const int strides[4] = {1, 4, 16, 64};
  for (int st = 0; st < 4; ++st) {
    const int s = strides[st];
    for (int i = 0; i < 256; ++i) {
      const int d = (i / s) & 3, base = i - d * s;
      tmp[i] = h4_half(d, g[base], g[base + s], g[base + 2 * s], g[base + 3 * s]);
    }
    memcpy(g, tmp, sizeof(tmp));
  }
}

/* ---- Row scale and INT8 codes ---------------------------------------------------
 * scale = max(min(absmax, BF16_MAX) * (1/127), 1e-30), stored unrounded
 * (kernels/norm_quant/norm_quant.cu:183-192); code = clamp(nearbyint(
 * bf(bf(v) / bf(scale))), -128, 127) (convrot64_exact.cuh:53-57,
 * convrot_register_v2.cu:126-129).                                          */
static float row_scale(const float* v, int64_t k) {
  float amax = 0.0f;
  for (int64_t i = 0; i < k; ++i) amax = fmaxf(amax, fabsf(ftz(v[i])));
  return fmaxf(ftz_mul(fminf(amax, 3.38953139e38f), 1.0f / 127.0f), 1.0e-30f);
}

static inline int8_t int8_code(float v, float scale) {
  const float sb = bf_round(ftz(scale));
  const float vb = bf_round(ftz(v));
  const float q = bf_round(ftz(ftz(vb) / ftz(sb)));
  float c = nearbyintf(q);
  c = fminf(127.0f, fmaxf(-128.0f, c));
  return (int8_t)c;
}

/* Public: quantise already-rotated rows (used by tests that inject values). */
H3O_EXPORT void h3o_quant_rows(const float* rot, int64_t m, int64_t k, int8_t* q, float* scale, int threads) {
  set_threads(threads);
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < m; ++r) {
    const float* v = rot + r * k;
    const float s = row_scale(v, k);
    scale[r] = s;
    for (int64_t i = 0; i < k; ++i) q[r * k + i] = int8_code(v[i], s);
  }
}

/* Public: ConvRot256 of each group of each row, FP32 in/out. */
H3O_EXPORT void h3o_convrot_rows(float* v, int64_t m, int64_t k, int threads) {
  set_threads(threads);
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < m; ++r)
    for (int64_t g = 0; g < k / 256; ++g) convrot256(v + r * k + g * 256);
}

/* ---- Fused prologue (kernels/norm_quant/norm_quant.cu:51-213) -------------------
 * sum of squares: logical thread t in 0..127 fma-accumulates the 4-element
 * chunks t, t+128, ... of the row in element order (:56-65); each 32-thread
 * warp folds with shfl_down offsets 16, 8, 4, 2, 1 (:66-67); the warp sums fold
 * as (w0+w2)+(w1+w3) (:69-74); variance = sum / K (:75).
 * rrms = rsqrt(var + eps) (:134).
 * n = bf(w * (rrms * x)); s = bf(shift); c = bf(scale); one_c = bf(1 + c);
 * out = bf(bf(n * one_c) + s) (:164-172), table row = rows[token] (:138-140). */
static float rms_variance(const uint16_t* x, int64_t k) {
  float lane_sum[128];
  const int64_t chunks = k / 4;
  for (int t = 0; t < 128; ++t) {
    float s = 0.0f;
    for (int64_t i = t; i < chunks; i += 128)
      for (int e = 0; e < 4; ++e) {
        const float v = bf_to_f(x[4 * i + e]);
        s = fmaf(v, v, s);
      }
    lane_sum[t] = s;
  }
  float warp_sum[4];
  for (int w = 0; w < 4; ++w) {
    float s[32];
    for (int l = 0; l < 32; ++l) s[l] = lane_sum[32 * w + l];
    for (int off = 16; off > 0; off >>= 1) {
      float nxt[32];
      for (int l = 0; l < 32; ++l) nxt[l] = (l + off < 32) ? s[l] + s[l + off] : s[l] + s[l];
      /* lanes whose source is out of range add their own value, as shfl_down
       * returns the caller's own register; only lane 0's result is used. */
      memcpy(s, nxt, sizeof(s));
    }
    warp_sum[w] = s[0];
  }
  const float total = (warp_sum[0] + warp_sum[2]) + (warp_sum[1] + warp_sum[3]);
  return total / (float)k;
}

H3O_EXPORT float h3o_rms_variance(const uint16_t* x, int64_t k) { return rms_variance(x, k); }

H3O_EXPORT int h3o_norm_quant(const uint16_t* x, int64_t xs, const uint16_t* w, const void* shift,
                              const void* scale, int table_dtype, int64_t ss, int64_t cs,
                              const int32_t* rows, int64_t m, int64_t k, float eps,
                              const float* rrms_in, int8_t* q, float* qscale, uint16_t* dbg_norm,
                              float* dbg_rot, float* dbg_rstd, int threads) {
  if (k % 256 || k < 256 || xs < k) return 1;
  set_threads(threads);
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < m; ++r) {
    const uint16_t* xr = x + r * xs;
    float rrms;
    if (rrms_in) {
      rrms = rrms_in[r];
    } else {
      const float var = rms_variance(xr, k);
      rrms = (float)(1.0 / sqrt((double)(var + eps)));
    }
    const int64_t tr = rows[r];
    float* v = (float*)malloc(sizeof(float) * (size_t)k);
    for (int64_t i = 0; i < k; ++i) {
      const float xv = bf_to_f(xr[i]);
      const float wv = bf_to_f(w[i]);
      float sh, sc;
      if (table_dtype == 0) {
        sh = ((const float*)shift)[tr * ss + i];
        sc = ((const float*)scale)[tr * cs + i];
      } else {
        sh = bf_to_f(((const uint16_t*)shift)[tr * ss + i]);
        sc = bf_to_f(((const uint16_t*)scale)[tr * cs + i]);
      }
      float n = bf_round(wv * (rrms * xv));
      const float sb = bf_round(sh), cb = bf_round(sc);
      const float one_c = bf_round(1.0f + cb);
      const float p = bf_round(n * one_c);
      n = bf_round(p + sb);
      v[i] = n;
      if (dbg_norm) dbg_norm[r * k + i] = f_to_bf(n);
    }
    for (int64_t g = 0; g < k / 256; ++g) convrot256(v + g * 256);
    const float s = row_scale(v, k);
    qscale[r] = s;
    if (dbg_rstd) dbg_rstd[r] = rrms;
    for (int64_t i = 0; i < k; ++i) {
      if (dbg_rot) dbg_rot[r * k + i] = v[i];
      q[r * k + i] = int8_code(v[i], s);
    }
    free(v);
  }
  return 0;
}

/* ---- residual update of the fused residual prologue ----------------------------
 * residual_quant.cu:59-78: x[i] <- bf(fma(branch[i], bf(gate[rows[r]][i]), x[i]))
 * (IEEE fused multiply-add, no flush), in place; the prologue (h3o_norm_quant)
 * then runs on the updated rows.  gate_dtype 0 = FP32 table, 1 = BF16 bits.   */
H3O_EXPORT int h3o_residual_update(uint16_t* x, const uint16_t* branch, const void* gate, int gate_dtype,
                                   int64_t gs, const int32_t* rows, int64_t m, int64_t k, int threads) {
  if (k < 1 || gs < k) return 1;
  set_threads(threads);
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < m; ++r) {
    const int64_t tr = rows[r];
    for (int64_t i = 0; i < k; ++i) {
      const float g = gate_dtype ? bf_to_f(((const uint16_t*)gate)[tr * gs + i])
                                 : bf_round(((const float*)gate)[tr * gs + i]);
      x[r * k + i] = f_to_bf(fmaf(bf_to_f(branch[r * k + i]), g, bf_to_f(x[r * k + i])));
    }
  }
  return 0;
}

/* ---- ConvRot quantiser with input activation --------------------------------------
 * convrot64_exact.cuh:913-1027 (act none / GELU-tanh / SwiGLU) and
 * convrot_register_v2.cu:67-138 (act none).  x rows have stride xs elements;
 * for SwiGLU the row is [gate | up], 2k wide.                               */
static inline float act_value(const uint16_t* xr, int64_t i, int64_t k, int act) {
  if (act == 2) {
    const float g = bf_to_f(xr[i]), u = bf_to_f(xr[k + i]);
    return (g / (1.0f + expf(-g))) * u;
  }
  const float v = bf_to_f(xr[i]);
  if (act == 1) {
    const float inner = 0.7978845608028654f * (v + 0.044715f * v * v * v);
    return 0.5f * v * (1.0f + tanhf(inner));
  }
  return v;
}

H3O_EXPORT int h3o_convrot_quant(const uint16_t* x, int64_t xs, int64_t m, int64_t k, int act, int8_t* q,
                                 float* scale, float* rotated, int threads) {
  if (k % 256 || k < 256 || act < 0 || act > 2) return 1;
  set_threads(threads);
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < m; ++r) {
    const uint16_t* xr = x + r * xs;
    float* v = (float*)malloc(sizeof(float) * (size_t)k);
    for (int64_t i = 0; i < k; ++i) v[i] = act_value(xr, i, k, act);
    for (int64_t g = 0; g < k / 256; ++g) convrot256(v + g * 256);
    if (rotated) memcpy(rotated + r * k, v, sizeof(float) * (size_t)k);
    if (q) {
      const float s = row_scale(v, k);
      scale[r] = s;
      for (int64_t i = 0; i < k; ++i) q[r * k + i] = int8_code(v[i], s);
    }
    free(v);
  }
  return 0;
}

/* ---- INT8 GEMM, exact int32 (kernels/gemm/fc1.cu:60-101: A row-major [M,K],
 * B [N,K] "ColumnMajor" = K-major, int32 accumulator).                         */
H3O_EXPORT void h3o_gemm_s32(const int8_t* a, const int8_t* b, int64_t m, int64_t n, int64_t k, int32_t* c,
                             int threads) {
  set_threads(threads);
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < m; ++i) {
    const int8_t* ar = a + i * k;
    for (int64_t j = 0; j < n; ++j) {
      const int8_t* br = b + j * k;
      int32_t s = 0;
      for (int64_t t = 0; t < k; ++t) s += (int32_t)ar[t] * (int32_t)br[t];
      c[i * n + j] = s;
    }
  }
}

/* ---- Epilogues --------------------------------------------------------------------
 * dequant: y = bf(((float(acc) * xs[m]) * ws[n]) + bias[n])   fc1.cu:83-90 and
 *          the explicit __fadd_rn(__fmul_rn(__fmul_rn(..))) of r84_kfourwarp.cu:240-241
 * gelu:    out = bf(gelu_tanh(y))                               convrot64_exact.cuh:913-923
 * gate:    out = bf(fmaf(y, gate[rows[m]*gate_ld + n], residual[m, n]))
 *                                                              gate.cu:172-180, 239-242     */
static inline float dequant_value(int32_t acc, float xs, float ws, float bias) {
  const float a = (float)acc;
  return bf_round(((a * xs) * ws) + bias);
}

H3O_EXPORT void h3o_dequant(const int32_t* acc, const float* xs, const float* ws, const uint16_t* bias,
                            int64_t m, int64_t n, int gelu, uint16_t* out, int64_t ldo, int threads) {
  set_threads(threads);
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < m; ++i)
    for (int64_t j = 0; j < n; ++j) {
      float y = dequant_value(acc[i * n + j], xs[i], ws[j], bias ? bf_to_f(bias[j]) : 0.0f);
      if (gelu) {
        const float inner = 0.7978845608028654f * (y + 0.044715f * y * y * y);
        y = 0.5f * y * (1.0f + tanhf(inner));
      }
      out[i * ldo + j] = f_to_bf(y);
    }
}

H3O_EXPORT void h3o_gate(const int32_t* acc, const float* xs, const float* ws, const uint16_t* bias,
                         const uint16_t* gate, int64_t gate_ld, const int32_t* rows, const uint16_t* residual,
                         int64_t m, int64_t n, uint16_t* out, int threads) {
  set_threads(threads);
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < m; ++i) {
    const uint16_t* g = gate + (int64_t)rows[i] * gate_ld;
    for (int64_t j = 0; j < n; ++j) {
      const float y = dequant_value(acc[i * n + j], xs[i], ws[j], bias ? bf_to_f(bias[j]) : 0.0f);
      out[i * n + j] = f_to_bf(fmaf(y, bf_to_f(g[j]), bf_to_f(residual[i * n + j])));
    }
  }
}

H3O_EXPORT int h3o_max_threads(void) { return set_threads(0); }

/* ---- QKV head epilogue -------------------------------------------------------------
 * The epilogue of the reference's fused QKV kernel after its int32 mainloop
 * (kernels/gemm/r84_kfourwarp.cu:228-375; the K-plane-only sample form is
 * r82_sample_konly.cu:230-330).  Input: the dequantised BF16 rows y [m, 3*H*128]
 * (plane g = Q, K, V; head h; 128 channels), i.e. bf(((acc*xs)*ws)+0).
 * The reference TU is built without fast-math, so nothing flushes here.
 *   - per (row, Q/K head): sum = 32 lane chains fmaf(v, v, s) over d = l + 32i,
 *     then the shfl_down tree; rrms = rsqrtf(sum/128 + eps) (hardware
 *     approximation: 1/sqrt in double here, or the caller's injected value);
 *     x = bf((t*rrms)*w); RoPE on d < 48 with partner d + 48:
 *     y0 = bf(a*x0 + b*x1), y1 = bf(c*x0 + e*x1) (every product of two BF16 values
 *     is exact in FP32, so contraction cannot change the sum); tail d >= 96 is x.
 *   - Q codes: per 128-row tile, 32 groups of 4 rows {base + 8j}, base =
 *     (sub/8)*32 + sub%8; K codes: 4 groups of 32 rows {tr : tr%8 in {2kg, 2kg+1}}
 *     after subtracting the anchor row of sk; each row is rotated by the signed
 *     128-point Hadamard (m > 256) or by 4-point blocks only (m <= 256);
 *     scale = fmaf(max|v|, 1/127, 1e-7); code = cvt.rni.sat.s8(v * rcp(scale))
 *     (rcp.approx.ftz on the GPU: IEEE 1/scale here).
 *   - V: vp = max over each tile's rows of the |BF16| bit patterns.           */
static const uint32_t kQkvSigns[4] = {0x1035997bu, 0x8087f5eeu, 0xee2e4e1au, 0x71132418u};

static void qkv_convrot4(float* v) {
  const float a0 = v[0] + v[1], a1 = v[0] - v[1], a2 = v[2] + v[3], a3 = v[2] - v[3];
  v[0] = (a0 + a2) * 0.5f;
  v[1] = (a1 + a3) * 0.5f;
  v[2] = (a0 - a2) * 0.5f;
  v[3] = (a1 - a3) * 0.5f;
}

/* One 128-channel row as the reference's warp holds it: lane l owns channels 4l..4l+3. */
static void qkv_rotate(float* v, int full) {
  if (full) {
    for (int ch = 0; ch < 128; ++ch) {
      const int lane = ch >> 2, c = ch & 3;
      const uint32_t flip = ((kQkvSigns[lane >> 3] >> ((lane & 7) * 4 + c)) & 1u) ^ 1u;
      v[ch] = f_from_u(u_from_f(v[ch]) ^ (flip << 31));
    }
  }
  for (int lane = 0; lane < 32; ++lane) qkv_convrot4(v + 4 * lane);
  if (!full) return;
  for (int bit = 1; bit < 32; bit <<= 1)
    for (int lane = 0; lane < 32; ++lane) {
      if (lane & bit) continue;
      for (int c = 0; c < 4; ++c) {
        const float lo = v[4 * lane + c], hi = v[4 * (lane | bit) + c];
        v[4 * lane + c] = lo + hi;
        v[4 * (lane | bit) + c] = lo - hi;
      }
    }
  for (int ch = 0; ch < 128; ++ch) v[ch] *= 0.1767766952966369f;
}

/* cvt.rni.sat.s8.f32: round half to even, saturate, NaN -> 0. */
static inline int8_t qkv_code(float x) {
  if (x != x) return 0;
  const float r = nearbyintf(x);
  return (int8_t)(r > 127.0f ? 127 : (r < -128.0f ? -128 : (int)r));
}

static float qkv_rrms(const uint16_t* t, float eps) {
  float p[32];
  for (int l = 0; l < 32; ++l) {
    float s = 0.0f;
    for (int i = 0; i < 4; ++i) {
      const float v = bf_to_f(t[l + 32 * i]);
      s = fmaf(v, v, s);
    }
    p[l] = s;
  }
  for (int off = 16; off > 0; off >>= 1)
    for (int l = 0; l < off; ++l) p[l] = p[l] + p[l + off];
  return (float)(1.0 / sqrt((double)(p[0] / 128.0f + eps)));
}

/* Normalise + RoPE one Q/K head row t -> u (both BF16 bits). */
static void qkv_norm_rope(const uint16_t* t, const uint16_t* w, const uint16_t* f, float rrms, uint16_t* u) {
  for (int d = 0; d < 48; ++d) {
    const float x0 = bf_round((bf_to_f(t[d]) * rrms) * bf_to_f(w[d]));
    const float x1 = bf_round((bf_to_f(t[d + 48]) * rrms) * bf_to_f(w[d + 48]));
    const float a = bf_to_f(f[4 * d]), b = bf_to_f(f[4 * d + 1]), c = bf_to_f(f[4 * d + 2]), e = bf_to_f(f[4 * d + 3]);
    u[d] = f_to_bf(fmaf(a, x0, b * x1));
    u[d + 48] = f_to_bf(fmaf(c, x0, e * x1));
  }
  for (int d = 96; d < 128; ++d) u[d] = f_to_bf((bf_to_f(t[d]) * rrms) * bf_to_f(w[d]));
}

/* planes: bit g set => produce plane g (Q=1, K=2, V=4).  d: [3, H, m, 128] (only the
 * requested planes are written).  qi/ki: [H, m, 128]; qs: [H, parts*32];
 * ks: [H, parts*4]; vp: [H, parts, 128]; any may be NULL to skip it.
 * rrms_in / rrms_out: optional [2, H, m].  sk: [H, 9, 128]; anchors: [H].     */
H3O_EXPORT void h3o_qkv_heads(const uint16_t* y, int64_t m, int64_t heads, const uint16_t* freqs,
                              const uint16_t* qw, const uint16_t* kw, float eps, const uint16_t* sk,
                              const int32_t* anchors, const float* rrms_in, int planes, uint16_t* d,
                              int8_t* qi, float* qs, int8_t* ki, float* ks, float* vp, float* rrms_out,
                              int threads) {
  set_threads(threads);
  const int64_t n = 3 * heads * 128, parts = (m + 127) / 128;
  const int full = m > 256;
#pragma omp parallel for schedule(dynamic, 1) collapse(2)
  for (int64_t tm = 0; tm < parts; ++tm)
    for (int64_t h = 0; h < heads; ++h) {
      const int64_t r0 = tm * 128, rows = (m - r0) < 128 ? (m - r0) : 128;
      uint16_t u[2][128][128];
      for (int g = 0; g < 2; ++g) {
        if (!(planes & (1 << g))) continue;
        const uint16_t* w = g == 0 ? qw : kw;
        for (int64_t tr = 0; tr < rows; ++tr) {
          const int64_t row = r0 + tr;
          const uint16_t* t = y + row * n + (g * heads + h) * 128;
          const float rrms = rrms_in ? rrms_in[(g * heads + h) * m + row] : qkv_rrms(t, eps);
          if (rrms_out) rrms_out[(g * heads + h) * m + row] = rrms;
          qkv_norm_rope(t, w, freqs + row * 192, rrms, u[g][tr]);
          if (d) memcpy(d + ((g * heads + h) * m + row) * 128, u[g][tr], 256);
        }
      }
      if ((planes & 1) && qi && qs) {
        for (int sub = 0; sub < 32; ++sub) {
          const int base = (sub / 8) * 32 + sub % 8;
          float v[4][128], mx = 0.0f;
          for (int j = 0; j < 4; ++j) {
            const int64_t tr = base + 8 * j;
            for (int ch = 0; ch < 128; ++ch) v[j][ch] = tr < rows ? bf_to_f(u[0][tr][ch]) : 0.0f;
            qkv_rotate(v[j], full);
            for (int ch = 0; ch < 128; ++ch) mx = fmaxf(mx, fabsf(v[j][ch]));
          }
          const float sc = fmaf(mx, 1.0f / 127.0f, 1e-7f), inv = 1.0f / sc;
          qs[h * parts * 32 + tm * 32 + sub] = sc;
          for (int j = 0; j < 4; ++j) {
            const int64_t tr = base + 8 * j;
            if (tr >= rows) continue;
            for (int ch = 0; ch < 128; ++ch) qi[(h * m + r0 + tr) * 128 + ch] = qkv_code(v[j][ch] * inv);
          }
        }
      }
      if ((planes & 2) && ki && ks) {
        float bias[128];
        const int a = anchors ? anchors[h] : -1;
        for (int ch = 0; ch < 128; ++ch) bias[ch] = a >= 0 ? bf_to_f(sk[(h * 9 + a) * 128 + ch]) : 0.0f;
        for (int kg = 0; kg < 4; ++kg) {
          float v[32][128], mx = 0.0f;
          for (int i = 0; i < 32; ++i) {
            const int64_t tr = (i / 2) * 8 + kg * 2 + (i & 1);
            for (int ch = 0; ch < 128; ++ch) v[i][ch] = tr < rows ? bf_to_f(u[1][tr][ch]) - bias[ch] : 0.0f;
            qkv_rotate(v[i], full);
            for (int ch = 0; ch < 128; ++ch) mx = fmaxf(mx, fabsf(v[i][ch]));
          }
          const float sc = fmaf(mx, 1.0f / 127.0f, 1e-7f), inv = 1.0f / sc;
          ks[(h * parts + tm) * 4 + kg] = sc;
          for (int i = 0; i < 32; ++i) {
            const int64_t tr = (i / 2) * 8 + kg * 2 + (i & 1);
            if (tr >= rows) continue;
            for (int ch = 0; ch < 128; ++ch) ki[(h * m + r0 + tr) * 128 + ch] = qkv_code(v[i][ch] * inv);
          }
        }
      }
      if (planes & 4) {
        for (int ch = 0; ch < 128; ++ch) {
          uint32_t mx = 0;
          for (int64_t tr = 0; tr < rows; ++tr) {
            const uint16_t b = y[(r0 + tr) * n + (2 * heads + h) * 128 + ch];
            if (d) d[((2 * heads + h) * m + r0 + tr) * 128 + ch] = b;
            const uint32_t mag = b & 0x7fffu;
            mx = mag > mx ? mag : mx;
          }
          if (vp) vp[(h * parts + tm) * 128 + ch] = bf_to_f((uint16_t)mx);
        }
      }
    }
}

/* ---- K anchor detector -----------------------------------------------------------
 * kernels/gemm/r79_sample_anchor.cu:467-605 as launched by h3_sample_anchor
 * (:700-702): per head, nine sampled keys k[s][c] (c < 128), one channel per
 * thread of 4 warps, shfl_down trees, warp totals added in warp order.  The TU
 * uses --use_fast_math: FTZ on every operation; 9*x - sum contracts to one
 * fma, exact here because 9*x is exact for a BF16 x.                          */
static float warp_tree_sum(float* p) {
  for (int off = 16; off > 0; off >>= 1)
    for (int l = 0; l < off; ++l) p[l] = ftz_add(p[l], p[l + off]);
  return p[0];
}
static float warp_tree_max(float* p) {
  for (int off = 16; off > 0; off >>= 1)
    for (int l = 0; l < off; ++l) p[l] = fmaxf(p[l], p[l + off]);
  return p[0];
}

H3O_EXPORT void h3o_sample_anchor(const uint16_t* k, int64_t heads, int32_t* anchors) {
  for (int64_t h = 0; h < heads; ++h) {
    const uint16_t* kh = k + h * 9 * 128;
    float e[128], mxv[128], dist[9][128], sum[128];
    for (int c = 0; c < 128; ++c) {
      float en = 0.0f, mx = 0.0f, cs = 0.0f;
      for (int s = 0; s < 9; ++s) {
        const float v = ftz(bf_to_f(kh[s * 128 + c]));
        en = ftz(fmaf(v, v, en));
        mx = fmaxf(mx, fabsf(v));
        cs = ftz_add(cs, v);
      }
      e[c] = en;
      mxv[c] = mx;
      sum[c] = cs;
      for (int s = 0; s < 9; ++s) {
        const float dd = ftz(fmaf(9.0f, ftz(bf_to_f(kh[s * 128 + c])), -cs));
        dist[s][c] = ftz(fmaf(dd, dd, 0.0f));
      }
    }
    (void)sum;
    float we[4], wm[4], wd[9][4];
    for (int w = 0; w < 4; ++w) {
      float p[32];
      memcpy(p, e + 32 * w, sizeof p);
      we[w] = warp_tree_sum(p);
      memcpy(p, mxv + 32 * w, sizeof p);
      wm[w] = warp_tree_max(p);
      for (int s = 0; s < 9; ++s) {
        memcpy(p, dist[s] + 32 * w, sizeof p);
        wd[s][w] = warp_tree_sum(p);
      }
    }
    int best = 0;
    float best_d = 3.402823466e+38f;
    for (int s = 0; s < 9; ++s) {
      float dsum = 0.0f;
      for (int w = 0; w < 4; ++w) dsum = ftz_add(dsum, wd[s][w]);
      if (dsum < best_d) {
        best = s;
        best_d = dsum;
      }
    }
    float be[128], bm[128];
    for (int c = 0; c < 128; ++c) {
      const float a = ftz(bf_to_f(kh[best * 128 + c]));
      float en = 0.0f, mx = 0.0f;
      for (int s = 0; s < 9; ++s) {
        const float r = ftz_sub(bf_to_f(kh[s * 128 + c]), a);
        en = ftz(fmaf(r, r, en));
        mx = fmaxf(mx, fabsf(r));
      }
      be[c] = en;
      bm[c] = mx;
    }
    float toe = 0.0f, tom = 0.0f, tbe = 0.0f, tbm = 0.0f;
    for (int w = 0; w < 4; ++w) {
      float p[32];
      memcpy(p, be + 32 * w, sizeof p);
      const float wbe = warp_tree_sum(p);
      memcpy(p, bm + 32 * w, sizeof p);
      const float wbm = warp_tree_max(p);
      toe = ftz_add(toe, we[w]);
      tom = fmaxf(tom, wm[w]);
      tbe = ftz_add(tbe, wbe);
      tbm = fmaxf(tbm, wbm);
    }
    const int improves = tbe < toe && tbm <= ftz_mul(tom, 1.125f);
    anchors[h] = improves ? best : -1;
  }
}

/* ---- V quantiser -------------------------------------------------------------------
 * The Triton kernels the reference's QKV op runs on the V plane
 * (h3_speedkit/ops/quant_v.py:57-110, launched at ops/qkv.py:70-79):
 *   scale[h,c] = max(RN_ftz(max_p vp[h,p,c] * (1/127)), 1e-12); inv = rcp(scale)
 *   (rcp.approx.ftz on the GPU: IEEE 1/scale here);
 *   vi[h*128 + c, dst] = cvt.rni.sat.s8(RN_ftz(v[h, src(dst), c] * inv)) for
 *   dst < padded = parts*128, src = dst with bits (b3 b2 b1 b0) -> (b1 b3 b2 b0)
 *   inside each run of 16 tokens, and 0 for src >= m.                           */
H3O_EXPORT void h3o_quant_v(const uint16_t* v, int64_t m, int64_t heads, const float* vp, int8_t* vi,
                            float* scale, int threads) {
  set_threads(threads);
  const int64_t parts = (m + 127) / 128, padded = parts * 128;
  const float k127 = f_from_u(0x3C010204u), floor_ = f_from_u(0x2B8CBCCCu);
#pragma omp parallel for schedule(static)
  for (int64_t hc = 0; hc < heads * 128; ++hc) {
    const int64_t h = hc / 128, c = hc % 128;
    float mx = 0.0f;
    for (int64_t p = 0; p < parts; ++p) mx = fmaxf(mx, vp[(h * parts + p) * 128 + c]);
    const float sc = fmaxf(ftz_mul(mx, k127), floor_), inv = ftz(1.0f / sc);
    scale[hc] = sc;
    for (int64_t dst = 0; dst < padded; ++dst) {
      const int64_t src = (dst & ~(int64_t)15) | (dst & 1) | ((dst & 2) << 2) | ((dst & 4) >> 1) | ((dst & 8) >> 1);
      const float x = src < m ? bf_to_f(v[(h * m + src) * 128 + c]) : 0.0f;
      vi[hc * padded + dst] = qkv_code(ftz_mul(x, inv));
    }
  }
}
