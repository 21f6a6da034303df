// Fused prologue for B200: RMSNorm -> adaLN modulation -> ConvRot256 -> per-token INT8.
//
// One CTA per token row; the ConvRot/quantisation core is rq_core.cuh (4 threads
// per 256-value group, 64 consecutive values per thread, one swizzled
// shared-memory exchange).  HBM traffic per row: K*2 bytes in, K bytes + 4 out.
//
// Arithmetic follows kernels/norm_quant/norm_quant.cu:51-213:
//  * sum of squares: logical thread t (0..127) fma-accumulates the 4-element
//    chunks t, t+128, ... in element order; a shfl_down tree per 32-thread
//    logical warp; the four warp sums fold as (w0+w2)+(w1+w3);
//    variance = div.rn(sum, K)  (:51-78).  Here physical thread p < 64 runs the
//    logical threads p and p+64 as the two halves of packed f32x2 FMAs (IEEE, no
//    flush), so physical warp 0 carries logical warps 0 and 2, warp 1 carries 1 and 3;
//  * rrms = rsqrt.approx(add.rn(var, eps))  (:133-134);
//  * n = bf(w*(rrms*x)) with IEEE f32x2 multiplies; out = bf(bf(n*bf(1+bf(scale))) +
//    bf(shift))  (:164-172) with BF16x2 add/multiply: for BF16 operands the FP32
//    result rounded to BF16 equals the directly rounded BF16 result (the FP32
//    product of two BF16 values is exact, and FP32 has more than 2*8+2 bits, so
//    rounding the FP32 sum again to BF16 is the correctly rounded BF16 sum);
//  * ConvRot256 + row scale + codes as in rq_core.cuh  (:179-211).
// The reference fixes K = 5376 with 192 threads; this kernel takes any
// K % 256 == 0 up to 16384 with max(64, K/64 rounded up to a warp) threads.
#include "row_stream.cuh"
#include "../../include/h3sk_b200.h"

#include <cfloat>
#include <cmath>

namespace h3sk {
namespace {

constexpr int kMaxK = 16384;
constexpr int kNormK = 5376;        // K of the unsuffixed (reference) entry point
constexpr int kModBatch = 2;        // chunks per modulation round of the streaming prologue
constexpr int kResBatch = 2;        // chunks per round of the residual pass (staged form; 1 otherwise)

__host__ __device__ constexpr int norm_threads(int k) {
  return ((k / 64 + 31) / 32) * 32 < 64 ? 64 : ((k / 64 + 31) / 32) * 32;
}
__host__ __device__ constexpr int norm_smem(int k) { return (norm_threads(k) / rq::kTeam) * rq::kGroupBytes; }

// Eight consecutive BF16 values of a row as four words (16-byte or 2x8-byte loads).
__device__ __forceinline__ uint4 load8(const __nv_bfloat16* p, int vec16) {
  if (vec16) return __ldg(reinterpret_cast<const uint4*>(p));
  const uint2 a = __ldg(reinterpret_cast<const uint2*>(p)), b = __ldg(reinterpret_cast<const uint2*>(p + 4));
  return make_uint4(a.x, a.y, b.x, b.y);
}

// Eight modulation-table values (BF16 or FP32) as four BF16 pair words, each
// value rounded to BF16 (an identity for BF16 tables).  vec: the eight values
// start on a 16-byte boundary.
template <class T> __device__ __forceinline__ uint4 table8(const T* p, int vec);
template <> __device__ __forceinline__ uint4 table8<__nv_bfloat16>(const __nv_bfloat16* p, int vec) {
  if (vec) return __ldg(reinterpret_cast<const uint4*>(p));
  const unsigned short* h = reinterpret_cast<const unsigned short*>(p);
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) w[i] = uint32_t(__ldg(h + 2 * i)) | (uint32_t(__ldg(h + 2 * i + 1)) << 16);
  return make_uint4(w[0], w[1], w[2], w[3]);
}
template <> __device__ __forceinline__ uint4 table8<float>(const float* p, int vec) {
  float f[8];
  if (vec) {
    const float4 a = __ldg(reinterpret_cast<const float4*>(p)), b = __ldg(reinterpret_cast<const float4*>(p + 4));
    f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w; f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) f[i] = __ldg(p + i);
  }
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) w[i] = rq::f2_to_bf2(rq::f2_pack(f[2 * i], f[2 * i + 1]));
  return make_uint4(w[0], w[1], w[2], w[3]);
}

// Eight consecutive BF16 values through plain (coherent) loads, for rows this
// kernel also writes.
__device__ __forceinline__ uint4 load8_rw(const __nv_bfloat16* p, int vec16) {
  if (vec16) return *reinterpret_cast<const uint4*>(p);
  const uint2 a = reinterpret_cast<const uint2*>(p)[0], b = reinterpret_cast<const uint2*>(p)[1];
  return make_uint4(a.x, a.y, b.x, b.y);
}
__device__ __forceinline__ void store8(__nv_bfloat16* p, uint4 v, int vec16) {
  if (vec16) {
    *reinterpret_cast<uint4*>(p) = v;
  } else {
    reinterpret_cast<uint2*>(p)[0] = make_uint2(v.x, v.y);
    reinterpret_cast<uint2*>(p)[1] = make_uint2(v.z, v.w);
  }
}
// bf(fma(branch, bf(gate), x)) of eight elements (residual_quant.cu:59-71).
__device__ __forceinline__ uint4 residual8(uint4 b, uint4 g, uint4 x) {
  return make_uint4(rq::residual_bf2(b.x, g.x, x.x), rq::residual_bf2(b.y, g.y, x.y),
                    rq::residual_bf2(b.z, g.z, x.z), rq::residual_bf2(b.w, g.w, x.w));
}

// One CTA per row.  kResidual (the fused residual prologue of
// kernels/residual_quant/residual_quant.cu:134-224): the row is first updated
// in place, XOut[row] = bf(fma(Branch[row], bf(Gate[Rows[row]]), XOut[row]))
// (contiguous rows of K), into a shared-memory copy that the prologue below
// then reads instead of X.
template <class ModT, bool kDebug, class GateT = float, bool kResidual = false>
__global__ void __launch_bounds__(256) norm_quant_rows(
    const __nv_bfloat16* __restrict__ X, const __nv_bfloat16* __restrict__ W,
    const ModT* __restrict__ Shift, const ModT* __restrict__ Scale,
    const int32_t* __restrict__ Rows, int8_t* __restrict__ Q, float* __restrict__ QScale,
    __nv_bfloat16* __restrict__ DebugNorm, float* __restrict__ DebugRotated,
    float* __restrict__ DebugRstd, int64_t xs, int64_t ss, int64_t cs, float eps, int K,
    int x_vec16, int w_vec16, int t_vec16, int q_vec16, __nv_bfloat16* __restrict__ XOut = nullptr,
    const __nv_bfloat16* __restrict__ Branch = nullptr, const GateT* __restrict__ Gate = nullptr,
    int64_t gs = 0, int b_vec16 = 0, int g_vec16 = 0) {
  extern __shared__ __align__(16) float exch[];
  __shared__ float fold[8];
  __shared__ float row_stat;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t row = blockIdx.x;
  const __nv_bfloat16* xr = kResidual ? nullptr : X + row * xs;
  // kResidual: the updated row, after the exchange buffers
  uint4* xrow = reinterpret_cast<uint4*>(reinterpret_cast<unsigned char*>(exch) + norm_smem(K));

  // 0. Residual update (kResidual).
  if constexpr (kResidual) {
    __nv_bfloat16* xw = XOut + row * K;
    const __nv_bfloat16* br = Branch + row * K;
    const GateT* gr = Gate + int64_t(Rows[row]) * gs;
    for (int c = tid; c < K / 8; c += int(blockDim.x)) {
      const uint4 nv = residual8(load8(br + 8 * c, b_vec16), table8<GateT>(gr + 8 * c, g_vec16),
                                 load8_rw(xw + 8 * c, x_vec16));
      xrow[c] = nv;
      store8(xw + 8 * c, nv, x_vec16);
    }
    __syncthreads();
  }

  // 1. Sum of squares in the reference's order: logical threads tid and tid+64.
  if (tid < 64) {
    const uint2* chunks = kResidual ? reinterpret_cast<const uint2*>(xrow) : reinterpret_cast<const uint2*>(xr);
    const int nchunks = K / 4;
    uint64_t acc = 0;   // (+0.0f, +0.0f)
#pragma unroll 4
    for (int base = 0; base < nchunks; base += 128) {
      const int c0 = base + tid, c1 = base + tid + 64;
      uint2 r0 = make_uint2(0, 0), r1 = make_uint2(0, 0);
      if constexpr (kResidual) {
        if (c0 < nchunks) r0 = chunks[c0];
        if (c1 < nchunks) r1 = chunks[c1];
      } else {
        if (c0 < nchunks) r0 = __ldg(chunks + c0);
        if (c1 < nchunks) r1 = __ldg(chunks + c1);
      }
      // element order inside a chunk: r.x low, r.x high, r.y low, r.y high
      uint64_t e;
      e = rq::f2_pack(__uint_as_float(r0.x << 16), __uint_as_float(r1.x << 16));
      acc = rq::f2_fma_ieee(e, e, acc);
      e = rq::f2_pack(__uint_as_float(r0.x & 0xffff0000u), __uint_as_float(r1.x & 0xffff0000u));
      acc = rq::f2_fma_ieee(e, e, acc);
      e = rq::f2_pack(__uint_as_float(r0.y << 16), __uint_as_float(r1.y << 16));
      acc = rq::f2_fma_ieee(e, e, acc);
      e = rq::f2_pack(__uint_as_float(r0.y & 0xffff0000u), __uint_as_float(r1.y & 0xffff0000u));
      acc = rq::f2_fma_ieee(e, e, acc);
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      const float lo = __shfl_down_sync(kFullMask, rq::f2_lo(acc), off);
      const float hi = __shfl_down_sync(kFullMask, rq::f2_hi(acc), off);
      acc = rq::f2_add_ieee(acc, rq::f2_pack(lo, hi));
    }
    if (lane == 0) {
      fold[warp] = rq::f2_lo(acc);        // logical warp `warp`
      fold[warp + 2] = rq::f2_hi(acc);    // logical warp `warp + 2`
    }
  }
  __syncthreads();
  if (tid == 0) {
    const float total = ieee_add(ieee_add(fold[0], fold[2]), ieee_add(fold[1], fold[3]));
    row_stat = ieee_div(total, static_cast<float>(K));
  }
  __syncthreads();
  const float rrms = hw_rsqrt(ieee_add(row_stat, eps));

  // 2. Normalise and modulate in layout A (64 consecutive values per thread).
  const int group = tid >> 2, q = tid & 3;
  const bool active = group < K / 256;
  const int col0 = group * 256 + 64 * q;
  const int64_t out_row = row * K;
  uint64_t v[32];
  if (active) {
    const int table_row = Rows[row];
    const ModT* shift_row = Shift + static_cast<int64_t>(table_row) * ss + col0;
    const ModT* scale_row = Scale + static_cast<int64_t>(table_row) * cs + col0;
    const uint64_t rr = rq::f2_pack(rrms, rrms);
    const uint32_t one2 = 0x3F803F80u;   // BF16 (1, 1)
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const uint4 xv = kResidual ? xrow[(col0 >> 3) + i] : load8(xr + col0 + 8 * i, x_vec16);
      const uint4 wv = load8(W + col0 + 8 * i, w_vec16);
      const uint4 sv = table8<ModT>(shift_row + 8 * i, t_vec16);
      const uint4 cv = table8<ModT>(scale_row + 8 * i, t_vec16);
      const uint32_t xw[4] = {xv.x, xv.y, xv.z, xv.w}, ww[4] = {wv.x, wv.y, wv.z, wv.w};
      const uint32_t sw[4] = {sv.x, sv.y, sv.z, sv.w}, cw[4] = {cv.x, cv.y, cv.z, cv.w};
      uint32_t nw[4];
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        const uint64_t t = rq::f2_mul_ieee(rq::bf2_to_f2(ww[h]), rq::f2_mul_ieee(rr, rq::bf2_to_f2(xw[h])));
        const uint32_t n = rq::f2_to_bf2(t);
        const uint32_t one_c = rq::bf2_add(one2, cw[h]);
        nw[h] = rq::bf2_add(rq::bf2_mul(n, one_c), sw[h]);
        v[4 * i + h] = rq::bf2_to_f2(nw[h]);
      }
      if constexpr (kDebug) {
        unsigned short* dst = reinterpret_cast<unsigned short*>(DebugNorm) + out_row + col0 + 8 * i;
#pragma unroll
        for (int h = 0; h < 4; ++h) {
          dst[2 * h] = static_cast<unsigned short>(nw[h] & 0xffffu);
          dst[2 * h + 1] = static_cast<unsigned short>(nw[h] >> 16);
        }
      }
    }
  } else {
#pragma unroll
    for (int p = 0; p < 32; ++p) v[p] = 0;
  }

  // 3. ConvRot256, row absmax, scale, codes.
  rq::fht_layout_a(v);
  rq::exchange_a_to_b(v, exch + group * 256, q, group & 1);
  rq::fht_layout_b(v);
  const float local = warp_allmax(rq::absmax64(v));
  if (lane == 0) fold[warp] = local;
  __syncthreads();
  const int nwarps = blockDim.x >> 5;
  const float scale = int8_row_scale(warp_allmax(lane < nwarps ? fold[lane] : 0.0f));
  if (tid == 0) {
    QScale[row] = scale;
    if constexpr (kDebug) DebugRstd[row] = rrms;
  }
  if (active) {
    if constexpr (kDebug) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float* dst = DebugRotated + out_row + group * 256 + rq::run_col_b(q, j);
#pragma unroll
        for (int h = 0; h < 8; ++h) {
          dst[2 * h] = rq::f2_lo(v[8 * j + h]);
          dst[2 * h + 1] = rq::f2_hi(v[8 * j + h]);
        }
      }
    }
    const float scale_bf = __bfloat162float(__float2bfloat16_rn(scale));
    rq::store_codes(Q + out_row + group * 256, q, v, scale_bf, q_vec16);
  }
}

// Persistent streaming prologue (row_stream.cuh).  Per row, a team:
//  1. waits for the row in its ring slot (swizzled BF16, one TMA box);
//  2. sum of squares in the reference's order (team threads 0..63 run the
//     logical threads p and p+64 as f32x2 halves, reading 8-byte chunks);
//     barrier A (AND of the wait flags), then every thread folds the four
//     logical-warp sums and computes rrms itself;
//  3. modulation pass: thread t takes the 16-byte chunks t, t + team, ... of the
//     row, reads W / shift / scale for those 8 columns with coalesced global
//     loads (they stay in L1: every row of the CTA uses the same columns), and
//     writes the modulated BF16 values back into the slot; barrier B;
//  4. reads its 64 layout-A values from the slot (the slot is then free), FHT
//     stages 1-3, two-half exchange, stage 4, absmax; barrier C, after which
//     thread 0 refills the slot with the team's next-but-D row;
//  5. row scale and codes.
// kStaged (the number of tables T is known and W plus T tables fit in shared
// memory): every CTA first stages W, bf(1 + bf(scale_t)) and bf(shift_t) for all
// tables in shared memory with the rows' 128-byte swizzle, and step 3 happens in
// layout A straight from shared memory -- no modulation pass, no barrier B.
// kResidual (the fused residual prologue, residual_quant.cu:134-224): each slot
// also receives the Branch row (second TMA box at byte `boff`); before step 2 the
// team rewrites the row in the slot as bf(fma(branch, bf(Gate[Rows[row]]), x))
// and stores it to XOut (contiguous rows of K), then barrier R.
// The arithmetic is that of norm_quant_rows, value for value.
template <class ModT, bool kStaged, bool kInSlot, class GateT = float, bool kResidual = false>
__global__ void __launch_bounds__(512, 1) norm_quant_stream(
    const __grid_constant__ CUtensorMap map_x, const __nv_bfloat16* __restrict__ W,
    const ModT* __restrict__ Shift, const ModT* __restrict__ Scale, const int32_t* __restrict__ Rows,
    int8_t* __restrict__ Q, float* __restrict__ QScale, int64_t ss, int64_t cs, float eps, int64_t M,
    const rs::Plan plan, int tables, int w_vec16, int t_vec16, int q_vec16, int* status,
    const __grid_constant__ CUtensorMap map_b, __nv_bfloat16* __restrict__ XOut,
    const GateT* __restrict__ Gate, int64_t gs, int g_vec16, uint32_t boff) {
  extern __shared__ unsigned char smem_raw[];
  __shared__ rs::RingState st;
  unsigned char* smem =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int K = plan.k, D = plan.slots_per_team, teams = plan.teams, team_threads = plan.team_threads;
  const int tid = threadIdx.x, lane = tid & 31;
  const int team = tid / team_threads, tt = tid - team * team_threads;
  const int g = tt >> 2, q = tt & 3, twarp = tt >> 5, nwarps = team_threads >> 5;
  const bool active = g < K / 256;
  const int grid = int(gridDim.x);
  const int n_local = int((M - int64_t(blockIdx.x) + grid - 1) / grid);
  const int n_team = team < n_local ? (n_local - team + teams - 1) / teams : 0;
  unsigned char* ring = smem + size_t(team) * size_t(D) * plan.slot_bytes;
  const uint32_t ring_a = sm100::smem_addr(ring);
  // This group's 512-byte exchange region: its own buffer after the rings, or
  // (exch_bytes == 0) its part of the row slot it has just read.
  const uint32_t group_off = uint32_t(g * rs::kHalfGroupBytes);
  const uint32_t xbuf_a = sm100::smem_addr(smem) + uint32_t(plan.ring_bytes + team * plan.exch_bytes) + group_off;
  uint64_t* full = st.full + team * D;
  const int bar_id = 1 + team;
  const int nchunks = K / 4;       // 8-byte chunks of the sum of squares
  const int nchunks16 = K / 8;     // 16-byte chunks of the modulation pass

  // Staged arrays (kStaged): W, then (onec, shift) per table, each K BF16 values
  // in its own 1024-byte aligned block, 16-byte chunk c at swz128(16 c).
  const uint32_t arr_bytes = uint32_t((K * 2 + 1023) / 1024 * 1024);
  const uint32_t w_a = sm100::smem_addr(smem) + uint32_t(plan.ring_bytes + plan.teams * plan.exch_bytes);
  if constexpr (kStaged) {
    const uint32_t one2 = 0x3F803F80u;   // BF16 (1, 1)
    const int per_array = K / 8;
    for (int j = tid; j < per_array * (1 + 2 * tables); j += blockDim.x) {
      const int arr = j / per_array, c = j - arr * per_array;
      uint4 val;
      if (arr == 0) {
        val = load8(W + 8 * c, w_vec16);
      } else {
        const int t = (arr - 1) >> 1;
        if ((arr - 1) & 1) {
          val = table8<ModT>(Shift + int64_t(t) * ss + 8 * c, t_vec16);
        } else {
          const uint4 cv = table8<ModT>(Scale + int64_t(t) * cs + 8 * c, t_vec16);
          val = make_uint4(rq::bf2_add(one2, cv.x), rq::bf2_add(one2, cv.y), rq::bf2_add(one2, cv.z),
                           rq::bf2_add(one2, cv.w));
        }
      }
      rs::sts128(w_a + uint32_t(arr) * arr_bytes + rs::swz128(16u * uint32_t(c)), val.x, val.y, val.z, val.w);
    }
    __syncthreads();
  }

  // One row (and, kResidual, its branch row) into a slot.
  auto issue = [&](unsigned char* slot, uint64_t* bar, int r) {
    if constexpr (kResidual) {
      const uint64_t policy = rs::l2_policy_evict_first();
      sm100::mbar_arrive_expect_tx(bar, uint32_t(K) * 4u);
      rs::tma_load_3d(slot, &map_x, bar, 0, 0, r, policy);
      rs::tma_load_3d(slot + boff, &map_b, bar, 0, 0, r, policy);
    } else {
      rs::issue_row(&map_x, slot, bar, r, K, K);
    }
  };

  int issued = 0;
  if (tt == 0) {
    for (int d = 0; d < D; ++d) sm100::mbar_init(&full[d], 1);
    sm100::fence_mbar_init();
    sm100::tma_prefetch_map(&map_x);
    if constexpr (kResidual) sm100::tma_prefetch_map(&map_b);
    for (; issued < D && issued < n_team; ++issued)
      issue(ring + size_t(issued) * plan.slot_bytes, &full[issued], int(blockIdx.x) + (team + issued * teams) * grid);
  }
  rs::team_sync(bar_id, team_threads);

  int d = 0;
  uint32_t ph = 0;
  int parity = 0;
  int k = 0;
  for (; k < n_team; ++k, parity ^= 1) {
    const int64_t row = int64_t(blockIdx.x) + int64_t(team + k * teams) * grid;
    const bool ok = sm100::mbar_wait_bounded(&full[d], ph, nullptr, status, rs::kCodeFull, rs::kWaitNs);
    const uint32_t row_a = ring_a + uint32_t(d * plan.slot_bytes);

    // 1b. residual update in the slot and in XOut (kResidual)
    if constexpr (kResidual) {
      const int gate_row = kStaged ? min(max(__ldg(Rows + row), 0), tables - 1) : __ldg(Rows + row);
      const GateT* grow = Gate + int64_t(gate_row) * gs;
      if (ok) {
        // kB chunks per round, every load of a round before its math: the gate
        // loads go to L1/L2 and would otherwise stall one at a time.
        constexpr int kB = kStaged ? kResBatch : 1;   // wider rounds spill in the modulation-pass form
        for (int c0 = tt; c0 < nchunks16; c0 += kB * team_threads) {
          uint4 gv[kB], xv[kB], bv[kB];
#pragma unroll
          for (int u = 0; u < kB; ++u) {
            const int c = c0 + u * team_threads;
            if (c < nchunks16) {
              const uint32_t off = rs::swz128(16u * uint32_t(c));
              gv[u] = table8<GateT>(grow + 8 * c, g_vec16);
              xv[u] = rs::lds128(row_a + off);
              bv[u] = rs::lds128(row_a + boff + off);
            }
          }
#pragma unroll
          for (int u = 0; u < kB; ++u) {
            const int c = c0 + u * team_threads;
            if (c >= nchunks16) continue;
            const uint4 nv = residual8(bv[u], gv[u], xv[u]);
            rs::sts128(row_a + rs::swz128(16u * uint32_t(c)), nv.x, nv.y, nv.z, nv.w);
            *reinterpret_cast<uint4*>(XOut + row * K + 8 * c) = nv;
          }
        }
      }
      if (!rs::team_sync_and(bar_id, team_threads, ok)) break;   // barrier R
    }

    // 2. sum of squares
    if (kStaged && tt < 64) {
      // logical thread tt in acc0, logical thread tt + 64 in acc1; BF16 operands
      // go straight into the FMAs (fma.rn.f32.bf16, see rq_core.cuh)
      float acc0 = 0.0f, acc1 = 0.0f;
#pragma unroll 4
      for (int base = 0; base < nchunks; base += 128) {
        const int c0 = base + tt, c1 = base + tt + 64;
        const uint2 r0 = c0 < nchunks ? rs::lds64(row_a + rs::swz128(8u * c0)) : make_uint2(0, 0);
        const uint2 r1 = c1 < nchunks ? rs::lds64(row_a + rs::swz128(8u * c1)) : make_uint2(0, 0);
        acc0 = rq::fma_sq_bf2(r0.y, rq::fma_sq_bf2(r0.x, acc0));
        acc1 = rq::fma_sq_bf2(r1.y, rq::fma_sq_bf2(r1.x, acc1));
      }
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) {
        acc0 = ieee_add(acc0, __shfl_down_sync(kFullMask, acc0, off));
        acc1 = ieee_add(acc1, __shfl_down_sync(kFullMask, acc1, off));
      }
      if (lane == 0) {
        st.stat_fold[team][twarp] = acc0;       // logical warp twarp
        st.stat_fold[team][twarp + 2] = acc1;   // logical warp twarp + 2
      }
    } else if (!kStaged && tt < 64) {
      // the same sums as packed f32x2 FMAs (fewer registers for this variant)
      uint64_t acc = 0;
#pragma unroll 4
      for (int base = 0; base < nchunks; base += 128) {
        const int c0 = base + tt, c1 = base + tt + 64;
        const uint2 r0 = c0 < nchunks ? rs::lds64(row_a + rs::swz128(8u * c0)) : make_uint2(0, 0);
        const uint2 r1 = c1 < nchunks ? rs::lds64(row_a + rs::swz128(8u * c1)) : make_uint2(0, 0);
        uint64_t e;
        e = rq::f2_pack(__uint_as_float(r0.x << 16), __uint_as_float(r1.x << 16));
        acc = rq::f2_fma_ieee(e, e, acc);
        e = rq::f2_pack(__uint_as_float(r0.x & 0xffff0000u), __uint_as_float(r1.x & 0xffff0000u));
        acc = rq::f2_fma_ieee(e, e, acc);
        e = rq::f2_pack(__uint_as_float(r0.y << 16), __uint_as_float(r1.y << 16));
        acc = rq::f2_fma_ieee(e, e, acc);
        e = rq::f2_pack(__uint_as_float(r0.y & 0xffff0000u), __uint_as_float(r1.y & 0xffff0000u));
        acc = rq::f2_fma_ieee(e, e, acc);
      }
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) {
        const float lo = __shfl_down_sync(kFullMask, rq::f2_lo(acc), off);
        const float hi = __shfl_down_sync(kFullMask, rq::f2_hi(acc), off);
        acc = rq::f2_add_ieee(acc, rq::f2_pack(lo, hi));
      }
      if (lane == 0) {
        st.stat_fold[team][twarp] = rq::f2_lo(acc);
        st.stat_fold[team][twarp + 2] = rq::f2_hi(acc);
      }
    }
    if (!rs::team_sync_and(bar_id, team_threads, ok)) break;   // barrier A
    const float* f = st.stat_fold[team];
    const float total = ieee_add(ieee_add(f[0], f[2]), ieee_add(f[1], f[3]));
    const float rrms = hw_rsqrt(ieee_add(ieee_div(total, static_cast<float>(K)), eps));

    uint64_t v[32];
    if constexpr (kStaged) {
      // 3+4. modulation in layout A from the staged arrays
      const int table_row = min(max(__ldg(Rows + row), 0), tables - 1);   // memory-safe for bad row maps
      const uint32_t c_a = w_a + uint32_t(1 + 2 * table_row) * arr_bytes;
      const uint32_t s_a = c_a + arr_bytes;
      if (active) {
        const uint64_t rr = rq::f2_pack(rrms, rrms);
        const uint32_t line = uint32_t(4 * g + q), key = (line & 7u) << 4;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const uint32_t off = line * 128u + ((16u * uint32_t(i)) ^ key);
          const uint4 xv = rs::lds128(row_a + off), wv = rs::lds128(w_a + off);
          const uint4 cv = rs::lds128(c_a + off), sv = rs::lds128(s_a + off);
          const uint32_t xw[4] = {xv.x, xv.y, xv.z, xv.w}, ww[4] = {wv.x, wv.y, wv.z, wv.w};
          const uint32_t cw[4] = {cv.x, cv.y, cv.z, cv.w}, sw[4] = {sv.x, sv.y, sv.z, sv.w};
#pragma unroll
          for (int h = 0; h < 4; ++h) {
            const uint64_t t = rq::f2_mul_ieee(rq::bf2_to_f2(ww[h]), rq::f2_mul_ieee(rr, rq::bf2_to_f2(xw[h])));
            v[4 * i + h] = rq::bf2_to_f2(rq::bf2_add(rq::bf2_mul(rq::f2_to_bf2(t), cw[h]), sw[h]));
          }
        }
      } else {
#pragma unroll
        for (int p = 0; p < 32; ++p) v[p] = 0;
      }
    } else {
      // 3. modulation pass, in place
      {
        const int table_row = __ldg(Rows + row);
        const ModT* shift_row = Shift + static_cast<int64_t>(table_row) * ss;
        const ModT* scale_row = Scale + static_cast<int64_t>(table_row) * cs;
        const uint64_t rr = rq::f2_pack(rrms, rrms);
        const uint32_t one2 = 0x3F803F80u;   // BF16 (1, 1)
        // kModBatch chunks per round, all loads first: the shared stores are ordered
        // asm, so batching is what lets the loads of a round overlap.
        for (int c0 = tt; c0 < nchunks16; c0 += kModBatch * team_threads) {
          uint4 xv[kModBatch], wv[kModBatch], sv[kModBatch], cv[kModBatch];
          uint32_t pa[kModBatch];
  #pragma unroll
          for (int u = 0; u < kModBatch; ++u) {
            const int c = c0 + u * team_threads;
            if (c < nchunks16) {
              pa[u] = row_a + rs::swz128(16u * c);
              xv[u] = rs::lds128(pa[u]);
              wv[u] = load8(W + 8 * c, w_vec16);
              sv[u] = table8<ModT>(shift_row + 8 * c, t_vec16);
              cv[u] = table8<ModT>(scale_row + 8 * c, t_vec16);
            }
          }
  #pragma unroll
          for (int u = 0; u < kModBatch; ++u) {
            if (c0 + u * team_threads >= nchunks16) continue;
            const uint32_t xw[4] = {xv[u].x, xv[u].y, xv[u].z, xv[u].w};
            const uint32_t ww[4] = {wv[u].x, wv[u].y, wv[u].z, wv[u].w};
            const uint32_t sw[4] = {sv[u].x, sv[u].y, sv[u].z, sv[u].w};
            const uint32_t cw[4] = {cv[u].x, cv[u].y, cv[u].z, cv[u].w};
            uint32_t nw[4];
  #pragma unroll
            for (int h = 0; h < 4; ++h) {
              const uint64_t t = rq::f2_mul_ieee(rq::bf2_to_f2(ww[h]), rq::f2_mul_ieee(rr, rq::bf2_to_f2(xw[h])));
              nw[h] = rq::bf2_add(rq::bf2_mul(rq::f2_to_bf2(t), rq::bf2_add(one2, cw[h])), sw[h]);
            }
            rs::sts128(pa[u], nw[0], nw[1], nw[2], nw[3]);
          }
        }
      }
      rs::team_sync(bar_id, team_threads);   // barrier B: the modulated row is complete

      // 4. ConvRot256 + absmax
      if (active) {
        uint4 raw[8];
        rs::load_row_a(row_a, g, q, raw);
  #pragma unroll
        for (int i = 0; i < 8; ++i) {
          v[4 * i + 0] = rq::bf2_to_f2(raw[i].x);
          v[4 * i + 1] = rq::bf2_to_f2(raw[i].y);
          v[4 * i + 2] = rq::bf2_to_f2(raw[i].z);
          v[4 * i + 3] = rq::bf2_to_f2(raw[i].w);
        }
      } else {
  #pragma unroll
        for (int p = 0; p < 32; ++p) v[p] = 0;
      }
    }
    rq::fht_layout_a(v);
    if constexpr (kInSlot) {
      __syncwarp();   // the group's layout-A reads of its region come first
      rs::exchange_a_to_b_halves(v, row_a + group_off, q, g & 1);
    } else {
      rs::exchange_a_to_b_halves(v, xbuf_a, q, g & 1);
    }
    // This thread's generic-proxy writes to the slot (modulation pass, in-slot
    // exchange) are ordered before the TMA (async proxy) that refills it.
    if constexpr (!kStaged || kInSlot || kResidual) sm100::fence_async_shared();
    rq::fht_layout_b(v);
    const float local = warp_allmax(rq::absmax64(v));
    if (lane == 0) st.max_fold[team][parity][twarp] = local;
    rs::team_sync(bar_id, team_threads);   // barrier C
    if (tt == 0 && issued < n_team) {
      issue(ring + size_t(d) * plan.slot_bytes, &full[d], int(blockIdx.x) + (team + issued * teams) * grid);
      ++issued;
    }
    if (++d == D) { d = 0; ph ^= 1u; }

    // 5. scale and codes
    float m = 0.0f;
    for (int w = 0; w < nwarps; ++w) m = fmaxf(m, st.max_fold[team][parity][w]);
    const float scale = int8_row_scale(m);
    if (tt == 0) QScale[row] = scale;
    if (active) {
      const float scale_bf = __bfloat162float(__float2bfloat16_rn(scale));
      rq::store_codes(Q + row * K + g * 256, q, v, scale_bf, q_vec16);
    }
  }
  // After an abort: no box may still be landing in this team's ring at exit.
  if (tt == 0)
    for (int j = k; j < issued; ++j)
      sm100::mbar_wait_bounded(&full[j % D], uint32_t((j / D) & 1), nullptr, status, rs::kCodeFull, rs::kWaitNs);
}

template <class T, bool D, class G = float, bool R = false>
int query_kernel(int k, H3NormQuantResources* out) {
  cudaFuncAttributes a{};
  auto kernel = norm_quant_rows<T, D, G, R>;
  const int threads = norm_threads(k);
  int active = 0, device = 0, sms = 0, max_threads = 0;
  cudaError_t e = cudaFuncGetAttributes(&a, kernel);
  if (e != cudaSuccess) return e;
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&active, kernel, threads, norm_smem(k) + (R ? 2 * k : 0));
  if (e != cudaSuccess) return e;
  if ((e = cudaGetDevice(&device)) != cudaSuccess) return e;
  if ((e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device)) != cudaSuccess) return e;
  if ((e = cudaDeviceGetAttribute(&max_threads, cudaDevAttrMaxThreadsPerMultiProcessor, device)) != cudaSuccess)
    return e;
  *out = {1, int64_t(sizeof(H3NormQuantResources)), k, threads, threads / 32, a.numRegs,
          int64_t(a.sharedSizeBytes), int64_t(a.localSizeBytes), active, sms, max_threads,
          a.binaryVersion, a.ptxVersion};
  return cudaSuccess;
}

bool valid_k(int64_t k) { return k >= 256 && k <= kMaxK && k % 256 == 0; }

// Operands of the fused residual prologue (residual_quant.cu:238-289): x is
// updated in place (contiguous rows of K) from branch (contiguous rows of K)
// and the gate table [T, >= gs] (gate_dtype 0 = FP32, 1 = BF16).
struct ResidualArgs {
  void* x;
  const void* branch;
  const void* gate;
  int64_t gs;
  int gate_dtype;
};

// tables: number of table rows T (shift/scale are [T, >=K]); 0 = not known.
// res: the residual operands, or null for the plain prologue.
int run_checked(const void* x, const void* w, const void* shift, const void* scale,
                const void* rows, void* q, void* qscale, void* dn, void* dr, void* drs,
                int64_t m, int64_t k, int64_t tables, int64_t xs, int64_t ss, int64_t cs, float eps,
                int table_dtype, int debug, uintptr_t stream_ptr, const ResidualArgs* res = nullptr) {
  // Contract of norm_quant.cu:247-255 (residual_quant.cu:259-270), with K a runtime value.
  if (!valid_k(k)) return cudaErrorInvalidValue;
  if (!x || !w || !shift || !scale || !rows || !q || !qscale || m < 1 || m > INT32_MAX ||
      xs < k || xs % 4 || ss < k || cs < k || table_dtype < 0 || table_dtype > 1 || debug < 0 ||
      debug > 1 || !std::isfinite(eps) || eps < FLT_MIN)
    return cudaErrorInvalidValue;
  if ((uintptr_t(x) & 7u) || (uintptr_t(w) & 7u) || (uintptr_t(q) & 7u) || (uintptr_t(qscale) & 3u) ||
      (uintptr_t(rows) & 3u) || (uintptr_t(shift) % (table_dtype ? 2 : 4)) ||
      (uintptr_t(scale) % (table_dtype ? 2 : 4)))
    return cudaErrorInvalidValue;
  if (res && (!res->branch || !res->gate || res->gs < k || res->gate_dtype < 0 || res->gate_dtype > 1 ||
              xs != k || (uintptr_t(res->branch) & 7u) || (uintptr_t(res->gate) % (res->gate_dtype ? 2 : 4))))
    return cudaErrorInvalidValue;
  if (debug && (!dn || !dr || !drs || (uintptr_t(dn) & 1u) || (uintptr_t(dr) & 3u) || (uintptr_t(drs) & 3u)))
    return cudaErrorInvalidValue;
  if (!debug && (dn || dr || drs)) return cudaErrorInvalidValue;
  const int x_vec16 = ((uintptr_t(x) & 15u) == 0 && (xs % 8) == 0) ? 1 : 0;
  const int w_vec16 = (uintptr_t(w) & 15u) == 0 ? 1 : 0;
  const int q_vec16 = (uintptr_t(q) & 15u) == 0 ? 1 : 0;
  const int64_t tsz = table_dtype ? 2 : 4;
  const int t_vec16 = ((uintptr_t(shift) & 15u) == 0 && (uintptr_t(scale) & 15u) == 0 && (ss * tsz) % 16 == 0 &&
                       (cs * tsz) % 16 == 0) ? 1 : 0;
  const int b_vec16 = res && (uintptr_t(res->branch) & 15u) == 0 ? 1 : 0;
  const int64_t gsz = res && res->gate_dtype ? 2 : 4;
  const int g_vec16 = res && (uintptr_t(res->gate) & 15u) == 0 && (res->gs * gsz) % 16 == 0 ? 1 : 0;
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_ptr);
  if (tables < 0 || tables > INT32_MAX) return cudaErrorInvalidValue;
  if (!debug && x_vec16 && (!res || b_vec16)) {
    // Streaming kernel: TMA needs 16-byte aligned rows, which x_vec16 (and, for the
    // residual form, b_vec16) states.  With T known and W plus T tables fitting
    // beside two ring slots per team, the tables are staged in shared memory.
    // The residual form's slot holds the row and its branch row at `boff`.
    const uint32_t boff = uint32_t((k * 2 + 1023) / 1024 * 1024);
    const int width = res ? int(boff / 2 + k) : int(k);
    const int arr_bytes = int((k * 2 + 1023) / 1024 * 1024);
    const int64_t staged_bytes = tables > 0 ? int64_t(arr_bytes) * (1 + 2 * tables) : -1;
    rs::Plan plan = rs::make_plan(int(k), width, 64);
    bool staged = false;
    if (staged_bytes > 0 && staged_bytes <= rs::kSmemBudget) {
      // Stage only when it costs no row team.
      const rs::Plan sp = rs::make_plan(int(k), width, 64, int(staged_bytes));
      if (sp.teams >= 1 && sp.teams == plan.teams && sp.smem <= rs::kSmemBudget) {
        plan = sp;
        staged = true;
      }
    }
    CUtensorMap map, map_b;
    bool maps = plan.teams >= 1 && plan.slots_per_team >= 2 && rs::make_row_map(&map, x, m, int(k), int(k), xs);
    if (maps && res) maps = rs::make_row_map(&map_b, res->branch, m, int(k), int(k), k);
    if (maps) {
      if (!res) map_b = map;
      int* status = status_device_ptr();
      if (!status) return cudaErrorInvalidDevicePointer;
      int grid = 0;
#define H3SK_NQ_STREAM(T, S, G, R)                                                                          \
  do {                                                                                                      \
    auto kernel = plan.exch_bytes ? norm_quant_stream<T, S, false, G, R> : norm_quant_stream<T, S, true, G, R>; \
    const cudaError_t e = rs::stream_grid(reinterpret_cast<const void*>(kernel), plan.smem, m, &grid);      \
    if (e != cudaSuccess) return e;                                                                         \
    kernel<<<grid, plan.threads, plan.smem, stream>>>(                                                      \
        map, static_cast<const __nv_bfloat16*>(w), static_cast<const T*>(shift), static_cast<const T*>(scale), \
        static_cast<const int32_t*>(rows), static_cast<int8_t*>(q), static_cast<float*>(qscale), ss, cs, eps, m, \
        plan, int(tables), w_vec16, t_vec16, q_vec16, status, map_b,                                        \
        static_cast<__nv_bfloat16*>(res ? res->x : nullptr), static_cast<const G*>(res ? res->gate : nullptr), \
        res ? res->gs : 0, g_vec16, boff);                                                                  \
  } while (0)
#define H3SK_NQ_STREAM_T(T, G, R)                                                                            \
  do {                                                                                                      \
    if (staged) H3SK_NQ_STREAM(T, true, G, R); else H3SK_NQ_STREAM(T, false, G, R);                         \
  } while (0)
#define H3SK_NQ_STREAM_G(G, R)                                                                               \
  do {                                                                                                      \
    if (table_dtype == 0) H3SK_NQ_STREAM_T(float, G, R); else H3SK_NQ_STREAM_T(__nv_bfloat16, G, R);        \
  } while (0)
      if (!res) H3SK_NQ_STREAM_G(float, false);
      else if (res->gate_dtype == 0) H3SK_NQ_STREAM_G(float, true);
      else H3SK_NQ_STREAM_G(__nv_bfloat16, true);
#undef H3SK_NQ_STREAM_G
#undef H3SK_NQ_STREAM_T
#undef H3SK_NQ_STREAM
      return cudaGetLastError();
    }
  }
  const int threads = norm_threads(int(k));
  const int smem = norm_smem(int(k)) + (res ? int(k) * 2 : 0);
#define H3SK_NQ_LAUNCH(T, D, G, R)                                                                 \
  do {                                                                                             \
    auto kernel = norm_quant_rows<T, D, G, R>;                                                     \
    if (smem > 48 * 1024) {                                                                        \
      const cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem); \
      if (e != cudaSuccess) return e;                                                              \
    }                                                                                              \
    kernel<<<dim3(unsigned(m)), threads, smem, stream>>>(                                          \
        static_cast<const __nv_bfloat16*>(res ? nullptr : x), static_cast<const __nv_bfloat16*>(w), \
        static_cast<const T*>(shift), static_cast<const T*>(scale), static_cast<const int32_t*>(rows), \
        static_cast<int8_t*>(q), static_cast<float*>(qscale), static_cast<__nv_bfloat16*>(dn),     \
        static_cast<float*>(dr), static_cast<float*>(drs), xs, ss, cs, eps, int(k), x_vec16, w_vec16, \
        t_vec16, q_vec16, static_cast<__nv_bfloat16*>(res ? res->x : nullptr),                      \
        static_cast<const __nv_bfloat16*>(res ? res->branch : nullptr),                            \
        static_cast<const G*>(res ? res->gate : nullptr), res ? res->gs : 0, b_vec16, g_vec16);    \
  } while (0)
#define H3SK_NQ_LAUNCH_T(T, G, R)                                                                  \
  do {                                                                                             \
    if (debug) H3SK_NQ_LAUNCH(T, true, G, R); else H3SK_NQ_LAUNCH(T, false, G, R);                 \
  } while (0)
#define H3SK_NQ_LAUNCH_G(G, R)                                                                     \
  do {                                                                                             \
    if (table_dtype == 0) H3SK_NQ_LAUNCH_T(float, G, R); else H3SK_NQ_LAUNCH_T(__nv_bfloat16, G, R); \
  } while (0)
  if (!res) H3SK_NQ_LAUNCH_G(float, false);
  else if (res->gate_dtype == 0) H3SK_NQ_LAUNCH_G(float, true);
  else H3SK_NQ_LAUNCH_G(__nv_bfloat16, true);
#undef H3SK_NQ_LAUNCH_G
#undef H3SK_NQ_LAUNCH_T
#undef H3SK_NQ_LAUNCH
  return cudaGetLastError();
}

int query_checked(int64_t k, int table_dtype, int debug, H3NormQuantResources* out, size_t bytes) {
  if (!out || bytes != sizeof(H3NormQuantResources) || !valid_k(k) || table_dtype < 0 ||
      table_dtype > 1 || debug < 0 || debug > 1)
    return cudaErrorInvalidValue;
  if (table_dtype == 0) return debug ? query_kernel<float, true>(int(k), out) : query_kernel<float, false>(int(k), out);
  return debug ? query_kernel<__nv_bfloat16, true>(int(k), out) : query_kernel<__nv_bfloat16, false>(int(k), out);
}

// Resources of the one-CTA-per-row residual kernel (residual_quant.cu:230-252).
int query_residual(int64_t k, int gate_dtype, int table_dtype, int debug, H3NormQuantResources* out, size_t bytes) {
  if (!out || bytes != sizeof(H3NormQuantResources) || !valid_k(k) || gate_dtype < 0 || gate_dtype > 1 ||
      table_dtype < 0 || table_dtype > 1 || debug < 0 || debug > 1)
    return cudaErrorInvalidValue;
  const int kk = int(k);
#define H3SK_RQ_QUERY(G, T) \
  return debug ? query_kernel<T, true, G, true>(kk, out) : query_kernel<T, false, G, true>(kk, out)
  if (gate_dtype == 0) {
    if (table_dtype == 0) H3SK_RQ_QUERY(float, float);
    H3SK_RQ_QUERY(float, __nv_bfloat16);
  }
  if (table_dtype == 0) H3SK_RQ_QUERY(__nv_bfloat16, float);
  H3SK_RQ_QUERY(__nv_bfloat16, __nv_bfloat16);
#undef H3SK_RQ_QUERY
}

int run_residual(void* x, const void* branch, const void* w, const void* gate, const void* shift, const void* scale,
                 const void* rows, void* q, void* qscale, void* dn, void* dr, void* drs, int64_t m, int64_t k,
                 int64_t tables, int64_t gs, int64_t ss, int64_t cs, float eps, int gate_dtype, int table_dtype,
                 int debug, uintptr_t stream) {
  const ResidualArgs res{x, branch, gate, gs, gate_dtype};
  return run_checked(x, w, shift, scale, rows, q, qscale, dn, dr, drs, m, k, tables, k, ss, cs, eps, table_dtype,
                     debug, stream, &res);
}

}  // namespace
}  // namespace h3sk

#define H3SK_EXPORT extern "C" __attribute__((visibility("default")))

H3SK_EXPORT int h3_norm_quant_abi(void) { return 1; }
H3SK_EXPORT int h3_norm_quant_abi_ex(void) { return 2; }
H3SK_EXPORT size_t h3_norm_quant_resources_size(void) { return sizeof(H3NormQuantResources); }
H3SK_EXPORT const char* h3_norm_quant_error(int code) {
  return cudaGetErrorString(static_cast<cudaError_t>(code));
}
H3SK_EXPORT int h3_norm_quant_query(int table_dtype, int debug, H3NormQuantResources* out, size_t bytes) {
  return h3sk::query_checked(h3sk::kNormK, table_dtype, debug, out, bytes);
}
H3SK_EXPORT int h3_norm_quant_query_k(int64_t k, int table_dtype, int debug, H3NormQuantResources* out,
                                      size_t bytes) {
  return h3sk::query_checked(k, table_dtype, debug, out, bytes);
}
H3SK_EXPORT int h3_norm_quant_run(const void* x, const void* w, const void* shift, const void* scale,
                                  const void* rows, void* q, void* qscale, void* debug_norm,
                                  void* debug_rotated, void* debug_rstd, int64_t m, int64_t xs,
                                  int64_t ss, int64_t cs, float eps, int table_dtype, int debug,
                                  uintptr_t stream) {
  return h3sk::run_checked(x, w, shift, scale, rows, q, qscale, debug_norm, debug_rotated, debug_rstd,
                           m, h3sk::kNormK, 0, xs, ss, cs, eps, table_dtype, debug, stream);
}
H3SK_EXPORT int h3_norm_quant_run_k(const void* x, const void* w, const void* shift, const void* scale,
                                    const void* rows, void* q, void* qscale, void* debug_norm,
                                    void* debug_rotated, void* debug_rstd, int64_t m, int64_t k,
                                    int64_t xs, int64_t ss, int64_t cs, float eps, int table_dtype,
                                    int debug, uintptr_t stream) {
  return h3sk::run_checked(x, w, shift, scale, rows, q, qscale, debug_norm, debug_rotated, debug_rstd,
                           m, k, 0, xs, ss, cs, eps, table_dtype, debug, stream);
}
H3SK_EXPORT int h3_norm_quant_run_t(const void* x, const void* w, const void* shift, const void* scale,
                                    const void* rows, void* q, void* qscale, void* debug_norm,
                                    void* debug_rotated, void* debug_rstd, int64_t m, int64_t k,
                                    int64_t tables, int64_t xs, int64_t ss, int64_t cs, float eps,
                                    int table_dtype, int debug, uintptr_t stream) {
  if (tables < 1) return cudaErrorInvalidValue;
  return h3sk::run_checked(x, w, shift, scale, rows, q, qscale, debug_norm, debug_rotated, debug_rstd,
                           m, k, tables, xs, ss, cs, eps, table_dtype, debug, stream);
}

// Fused residual prologue: x <- bf(fma(branch, bf(gate[rows]), x)) in place, then
// the prologue on the updated rows (kernels/residual_quant/residual_quant.cu).
H3SK_EXPORT int h3_residual_quant_abi(void) { return 1; }
H3SK_EXPORT size_t h3_residual_quant_resources_size(void) { return sizeof(H3NormQuantResources); }
H3SK_EXPORT const char* h3_residual_quant_error(int code) {
  return cudaGetErrorString(static_cast<cudaError_t>(code));
}
H3SK_EXPORT int h3_residual_quant_query(int gate_dtype, int table_dtype, int debug, H3NormQuantResources* out,
                                        size_t bytes) {
  return h3sk::query_residual(h3sk::kNormK, gate_dtype, table_dtype, debug, out, bytes);
}
H3SK_EXPORT int h3_residual_quant_query_k(int64_t k, int gate_dtype, int table_dtype, int debug,
                                          H3NormQuantResources* out, size_t bytes) {
  return h3sk::query_residual(k, gate_dtype, table_dtype, debug, out, bytes);
}
H3SK_EXPORT int h3_residual_quant_run(void* x, const void* branch, const void* w, const void* gate,
                                      const void* shift, const void* scale, const void* rows, void* q,
                                      void* qscale, void* debug_norm, void* debug_rotated, void* debug_rstd,
                                      int64_t m, int64_t gs, int64_t ss, int64_t cs, float eps, int gate_dtype,
                                      int table_dtype, int debug, uintptr_t stream) {
  return h3sk::run_residual(x, branch, w, gate, shift, scale, rows, q, qscale, debug_norm, debug_rotated, debug_rstd,
                            m, h3sk::kNormK, 0, gs, ss, cs, eps, gate_dtype, table_dtype, debug, stream);
}
H3SK_EXPORT int h3_residual_quant_run_k(void* x, const void* branch, const void* w, const void* gate,
                                        const void* shift, const void* scale, const void* rows, void* q,
                                        void* qscale, void* debug_norm, void* debug_rotated, void* debug_rstd,
                                        int64_t m, int64_t k, int64_t gs, int64_t ss, int64_t cs, float eps,
                                        int gate_dtype, int table_dtype, int debug, uintptr_t stream) {
  return h3sk::run_residual(x, branch, w, gate, shift, scale, rows, q, qscale, debug_norm, debug_rotated, debug_rstd,
                            m, k, 0, gs, ss, cs, eps, gate_dtype, table_dtype, debug, stream);
}
H3SK_EXPORT int h3_residual_quant_run_t(void* x, const void* branch, const void* w, const void* gate,
                                        const void* shift, const void* scale, const void* rows, void* q,
                                        void* qscale, void* debug_norm, void* debug_rotated, void* debug_rstd,
                                        int64_t m, int64_t k, int64_t tables, int64_t gs, int64_t ss, int64_t cs,
                                        float eps, int gate_dtype, int table_dtype, int debug, uintptr_t stream) {
  if (tables < 1) return cudaErrorInvalidValue;
  return h3sk::run_residual(x, branch, w, gate, shift, scale, rows, q, qscale, debug_norm, debug_rotated, debug_rstd,
                            m, k, tables, gs, ss, cs, eps, gate_dtype, table_dtype, debug, stream);
}
