// ConvRot256 + per-token INT8 quantiser for B200, with an optional input
// activation (none / GELU-tanh / SwiGLU).
//
// One CTA per row, 4 threads per 256-value group, 64 values per thread (see
// rq_core.cuh): 16-byte vector loads of 64 consecutive BF16 values per thread,
// FHT stages 1-3 in registers, one swizzled shared-memory exchange, stage 4 in
// registers, row absmax (one block barrier), packed codes as 16-byte stores.
// HBM traffic per row: 2K bytes in (4K for SwiGLU), K + 4 bytes out.
//
// Replaces kernels/convrot/convrot_register_v2.cu:67-138 (ACT none, K in
// {5376, 7168}) and Kitchen's quantize_int8_rowwise_convrot64_kernel
// (kernels/convrot/vendor/convrot64_exact.cuh:942-1027, input_act none / GELU-tanh
// / SwiGLU) for any K % 256 == 0 up to 16384.  The per-value results do not
// depend on the thread layout: each FHT output is the same expression of the
// same four inputs, and the absmax is an order-free fmaxf.
#include "row_stream.cuh"
#include "../../include/h3sk_b200.h"

namespace h3sk {
namespace {

constexpr int kMaxK = 16384;

__host__ __device__ constexpr int convrot_threads(int k) { return ((k / 64 + 31) / 32) * 32; }
__host__ __device__ constexpr int convrot_smem(int k) { return (convrot_threads(k) / rq::kTeam) * rq::kGroupBytes; }

enum : int { kModeQuant = 0, kModeDiag = 1, kModeRotate = 2 };

template <int kAct>
__device__ __forceinline__ void load_act_a(const __nv_bfloat16* xr, int col0, int K, uint64_t (&v)[32]) {
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const uint4 raw = __ldg(reinterpret_cast<const uint4*>(xr + col0 + 8 * i));
    const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
    if constexpr (kAct == kActNone) {
#pragma unroll
      for (int h = 0; h < 4; ++h) v[4 * i + h] = rq::bf2_to_f2(w[h]);
    } else if constexpr (kAct == kActGeluTanh) {
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        const uint64_t x = rq::bf2_to_f2(w[h]);
        v[4 * i + h] = rq::f2_pack(gelu_tanh(rq::f2_lo(x)), gelu_tanh(rq::f2_hi(x)));
      }
    } else {
      const uint4 up = __ldg(reinterpret_cast<const uint4*>(xr + K + col0 + 8 * i));
      const uint32_t u[4] = {up.x, up.y, up.z, up.w};
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        const uint64_t g = rq::bf2_to_f2(w[h]), x = rq::bf2_to_f2(u[h]);
        v[4 * i + h] = rq::f2_pack(swiglu(rq::f2_lo(g), rq::f2_lo(x)), swiglu(rq::f2_hi(g), rq::f2_hi(x)));
      }
    }
  }
}

template <int kAct, int kMode>
__global__ void __launch_bounds__(256) convrot_quant_rows(
    const __nv_bfloat16* __restrict__ X, int64_t xs, int8_t* __restrict__ Q,
    float* __restrict__ Scales, float* __restrict__ Rotated, int K, int q_vec16) {
  extern __shared__ __align__(16) float exch[];
  __shared__ float warp_max[8];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int group = tid >> 2, q = tid & 3;
  const bool active = group < K / 256;
  const int64_t row = blockIdx.x;
  const __nv_bfloat16* xr = X + row * xs;

  uint64_t v[32];
  if (active) {
    load_act_a<kAct>(xr, group * 256 + 64 * q, K, v);
  } else {
#pragma unroll
    for (int p = 0; p < 32; ++p) v[p] = 0;
  }
  rq::fht_layout_a(v);
  rq::exchange_a_to_b(v, exch + group * 256, q, group & 1);
  rq::fht_layout_b(v);

  const int64_t out_row = row * K;
  if constexpr (kMode != kModeQuant) {
    if (active) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float4* dst = reinterpret_cast<float4*>(Rotated + out_row + group * 256 + rq::run_col_b(q, j));
#pragma unroll
        for (int h = 0; h < 4; ++h) {
          const uint64_t a = v[8 * j + 2 * h], b = v[8 * j + 2 * h + 1];
          dst[h] = make_float4(rq::f2_lo(a), rq::f2_hi(a), rq::f2_lo(b), rq::f2_hi(b));
        }
      }
    }
  }
  if constexpr (kMode == kModeRotate) return;

  const float local = warp_allmax(rq::absmax64(v));
  if (lane == 0) warp_max[warp] = local;
  __syncthreads();
  const int nwarps = blockDim.x >> 5;
  const float scale = int8_row_scale(warp_allmax(lane < nwarps ? warp_max[lane] : 0.0f));
  if (tid == 0) Scales[row] = scale;
  if (active) {
    const float scale_bf = __bfloat162float(__float2bfloat16_rn(scale));
    rq::store_codes(Q + out_row + group * 256, q, v, scale_bf, q_vec16);
  }
}

// Layout-A values of one thread from its 8 raw input words (and, for SwiGLU,
// the 8 words of the up half), through the input activation.
template <int kAct>
__device__ __forceinline__ void activate_raw(const uint4 (&raw)[8], const uint4 (&up)[8], uint64_t (&v)[32]) {
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const uint32_t w[4] = {raw[i].x, raw[i].y, raw[i].z, raw[i].w};
    if constexpr (kAct == kActNone) {
#pragma unroll
      for (int h = 0; h < 4; ++h) v[4 * i + h] = rq::bf2_to_f2(w[h]);
    } else if constexpr (kAct == kActGeluTanh) {
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        const uint64_t x = rq::bf2_to_f2(w[h]);
        v[4 * i + h] = rq::f2_pack(gelu_tanh(rq::f2_lo(x)), gelu_tanh(rq::f2_hi(x)));
      }
    } else {
      const uint32_t u[4] = {up[i].x, up[i].y, up[i].z, up[i].w};
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        const uint64_t g = rq::bf2_to_f2(w[h]), x = rq::bf2_to_f2(u[h]);
        v[4 * i + h] = rq::f2_pack(swiglu(rq::f2_lo(g), rq::f2_lo(x)), swiglu(rq::f2_hi(g), rq::f2_hi(x)));
      }
    }
  }
}

// Persistent streaming quantiser (row_stream.cuh): each row team reads its
// rows from its TMA-fed ring in layout A and runs the same ConvRot / absmax /
// code steps as convrot_quant_rows.  One team barrier per row (the absmax),
// after which thread 0 refills the slot just read.
template <int kAct>
__global__ void __launch_bounds__(512, 1) convrot_quant_stream(
    const __grid_constant__ CUtensorMap map_x, int8_t* __restrict__ Q, float* __restrict__ Scales, int64_t M,
    const rs::Plan plan, int q_vec16, int* status) {
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
  // This group's 512-byte exchange buffer after the rings (the host only takes
  // this kernel with plan.exch_bytes > 0): the slots see generic reads only.
  const uint32_t xbuf_a =
      sm100::smem_addr(smem) + uint32_t(plan.ring_bytes + team * plan.exch_bytes + g * rs::kHalfGroupBytes);
  uint64_t* full = st.full + team * D;
  const int bar_id = 1 + team;

  int issued = 0;
  if (tt == 0) {
    for (int d = 0; d < D; ++d) sm100::mbar_init(&full[d], 1);
    sm100::fence_mbar_init();
    sm100::tma_prefetch_map(&map_x);
    for (; issued < D && issued < n_team; ++issued)
      rs::issue_row(&map_x, ring + size_t(issued) * plan.slot_bytes, &full[issued],
                    int(blockIdx.x) + (team + issued * teams) * grid, K, plan.width);
  }
  rs::team_sync(bar_id, team_threads);

  int d = 0;
  uint32_t ph = 0;
  int parity = 0;
  int k = 0;
  for (; k < n_team; ++k, parity ^= 1) {
    const bool ok = sm100::mbar_wait_bounded(&full[d], ph, nullptr, status, rs::kCodeFull, rs::kWaitNs);
    const uint32_t row_a = ring_a + uint32_t(d * plan.slot_bytes);
    uint64_t v[32];
    if (active) {
      uint4 raw[8], up[8];
      rs::load_row_a(row_a, g, q, raw);
      if constexpr (kAct == kActSwiGLU) rs::load_row_a(row_a + uint32_t(2 * K), g, q, up);
      activate_raw<kAct>(raw, up, v);
    } else {
#pragma unroll
      for (int p = 0; p < 32; ++p) v[p] = 0;
    }
    rq::fht_layout_a(v);
    rs::exchange_a_to_b_halves(v, xbuf_a, q, g & 1);
    rq::fht_layout_b(v);
    const float local = warp_allmax(rq::absmax64(v));
    if (lane == 0) st.max_fold[team][parity][twarp] = local;
    if (!rs::team_sync_and(bar_id, team_threads, ok)) break;
    // Slot d has been read by the whole team: refill it.
    if (tt == 0 && issued < n_team) {
      rs::issue_row(&map_x, ring + size_t(d) * plan.slot_bytes, &full[d],
                    int(blockIdx.x) + (team + issued * teams) * grid, K, plan.width);
      ++issued;
    }
    if (++d == D) { d = 0; ph ^= 1u; }
    float m = 0.0f;
    for (int w = 0; w < nwarps; ++w) m = fmaxf(m, st.max_fold[team][parity][w]);
    const float scale = int8_row_scale(m);
    const int64_t row = int64_t(blockIdx.x) + int64_t(team + k * teams) * grid;
    if (tt == 0) Scales[row] = scale;
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

bool valid_k(int64_t k) { return k >= 256 && k <= kMaxK && k % 256 == 0; }

// The streaming kernel needs 16-byte aligned rows (TMA); anything else takes the
// one-CTA-per-row kernel.
template <int kAct>
cudaError_t launch_stream(const void* x, int64_t xs, void* q, void* scale, int64_t rows, int k,
                          cudaStream_t stream, bool* launched) {
  *launched = false;
  if ((uintptr_t(x) & 15u) || (xs % 8)) return cudaSuccess;
  const int width = kAct == kActSwiGLU ? 2 * k : k;
  const rs::Plan plan = rs::make_plan(k, width, 32);
  if (plan.teams < 1 || plan.slots_per_team < 2 || plan.exch_bytes == 0) return cudaSuccess;
  CUtensorMap map;
  if (!rs::make_row_map(&map, x, rows, width, k, xs)) return cudaSuccess;
  auto kernel = convrot_quant_stream<kAct>;
  int grid = 0;
  cudaError_t e = rs::stream_grid(reinterpret_cast<const void*>(kernel), plan.smem, rows, &grid);
  if (e != cudaSuccess) return e;
  int* status = status_device_ptr();
  if (!status) return cudaErrorInvalidDevicePointer;
  kernel<<<grid, plan.threads, plan.smem, stream>>>(map, static_cast<int8_t*>(q), static_cast<float*>(scale), rows,
                                                    plan, (uintptr_t(q) & 15u) == 0 ? 1 : 0, status);
  *launched = true;
  return cudaGetLastError();
}

template <int kAct, int kMode>
cudaError_t launch(const void* x, int64_t xs, void* q, void* scale, void* rotated, int64_t rows, int k,
                   cudaStream_t stream) {
  if constexpr (kMode == kModeQuant) {
    bool launched = false;
    const cudaError_t e = launch_stream<kAct>(x, xs, q, scale, rows, k, stream, &launched);
    if (launched || e != cudaSuccess) return e;
  }
  auto kernel = convrot_quant_rows<kAct, kMode>;
  const int smem = convrot_smem(k);
  if (smem > 48 * 1024) {
    const cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
  }
  kernel<<<dim3(unsigned(rows)), convrot_threads(k), smem, stream>>>(
      static_cast<const __nv_bfloat16*>(x), xs, static_cast<int8_t*>(q), static_cast<float*>(scale),
      static_cast<float*>(rotated), k, (uintptr_t(q) & 15u) == 0 ? 1 : 0);
  return cudaGetLastError();
}

// The quantiser's last step for rows whose ConvRot256 ran elsewhere (the FC1
// epilogue of h3_int8_gelu_rot): the row scale from the row's max |rotated value|
// and the codes of the rotated values, already rounded to BF16 (the code rounds
// each value to BF16 first, so nothing is lost).  One CTA per row, 16 values per
// thread and step: two 16-byte streaming loads, one 16-byte store.
__global__ void __launch_bounds__(256) codes_from_rotated(const __nv_bfloat16* __restrict__ v, int64_t vs,
                                                          const uint32_t* __restrict__ rowmax, int8_t* __restrict__ q,
                                                          float* __restrict__ scale, int k) {
  const int64_t row = blockIdx.x;
  const float s = int8_row_scale(__uint_as_float(__ldg(rowmax + row)));
  if (threadIdx.x == 0) scale[row] = s;
  const float scale_bf = __bfloat162float(__float2bfloat16_rn(s));
  const uint4* src = reinterpret_cast<const uint4*>(v + row * vs);
  uint4* dst = reinterpret_cast<uint4*>(q + row * int64_t(k));
  for (int j = threadIdx.x; j < k / 16; j += blockDim.x) {
    const uint4 a = __ldcs(src + 2 * j), b = __ldcs(src + 2 * j + 1);
    dst[j] = make_uint4(rq::codes4(rq::bf2_to_f2(a.x), rq::bf2_to_f2(a.y), scale_bf),
                        rq::codes4(rq::bf2_to_f2(a.z), rq::bf2_to_f2(a.w), scale_bf),
                        rq::codes4(rq::bf2_to_f2(b.x), rq::bf2_to_f2(b.y), scale_bf),
                        rq::codes4(rq::bf2_to_f2(b.z), rq::bf2_to_f2(b.w), scale_bf));
  }
}

}  // namespace

// Shared with the GEMM translation unit (requantisation of a gate-residual output).
cudaError_t convrot_quant_none(const void* x, int64_t xs, void* q, void* scale, int64_t rows, int k,
                               cudaStream_t stream) {
  return launch<kActNone, kModeQuant>(x, xs, q, scale, nullptr, rows, k, stream);
}

}  // namespace h3sk

#define H3SK_EXPORT extern "C" __attribute__((visibility("default")))

H3SK_EXPORT int h3_convrot_register_abi(void) { return 1; }
H3SK_EXPORT size_t h3_convrot_register_resources_size(void) { return sizeof(H3ConvRotResources); }
H3SK_EXPORT const char* h3_convrot_register_error(int code) {
  return cudaGetErrorString(static_cast<cudaError_t>(code));
}

H3SK_EXPORT int h3_convrot_register_query(int k, H3ConvRotResources* out, size_t bytes) {
  using namespace h3sk;
  if (!out || bytes != sizeof(H3ConvRotResources) || !valid_k(k)) return cudaErrorInvalidValue;
  auto kernel = convrot_quant_rows<kActNone, kModeQuant>;
  const int threads = convrot_threads(k);
  cudaFuncAttributes attr{};
  int active = 0, device = 0, sms = 0, max_threads = 0;
  cudaError_t e = cudaFuncGetAttributes(&attr, kernel);
  if (e != cudaSuccess) return e;
  if ((e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&active, kernel, threads, convrot_smem(k))) != cudaSuccess)
    return e;
  if ((e = cudaGetDevice(&device)) != cudaSuccess) return e;
  if ((e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device)) != cudaSuccess) return e;
  if ((e = cudaDeviceGetAttribute(&max_threads, cudaDevAttrMaxThreadsPerMultiProcessor, device)) != cudaSuccess)
    return e;
  *out = {1, int64_t(sizeof(H3ConvRotResources)), k, threads, threads / 32, attr.numRegs,
          int64_t(attr.sharedSizeBytes), int64_t(attr.localSizeBytes), attr.maxThreadsPerBlock, active,
          sms, max_threads, attr.binaryVersion, attr.ptxVersion};
  return cudaSuccess;
}

H3SK_EXPORT int h3_convrot_register_run(const void* x, void* q, void* scale, void* rotated, int64_t rows,
                                        int k, int mode, uintptr_t stream_ptr) {
  using namespace h3sk;
  // Contract of convrot_register_v2.cu:200-205, with K generic.
  if (!x || rows < 1 || rows > INT32_MAX || mode < 0 || mode > 2 || (mode != 2 && (!q || !scale)) ||
      (mode != 0 && !rotated))
    return cudaErrorInvalidValue;
  if ((uintptr_t(x) & 15u) || (mode != 2 && (uintptr_t(q) & 7u)) || (mode != 2 && (uintptr_t(scale) & 3u)) ||
      (mode != 0 && (uintptr_t(rotated) & 15u)))
    return cudaErrorInvalidValue;
  if (!valid_k(k)) return cudaErrorInvalidValue;
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_ptr);
  if (mode == 0) return launch<kActNone, kModeQuant>(x, k, q, scale, nullptr, rows, k, stream);
  if (mode == 1) return launch<kActNone, kModeDiag>(x, k, q, scale, rotated, rows, k, stream);
  return launch<kActNone, kModeRotate>(x, k, nullptr, nullptr, rotated, rows, k, stream);
}

H3SK_EXPORT int h3_convrot_codes(const void* v, int64_t vs, const void* rowmax, void* q, void* scale, int64_t rows,
                                 int k, uintptr_t stream_ptr) {
  using namespace h3sk;
  if (!v || !rowmax || !q || !scale || rows < 1 || rows > INT32_MAX || !valid_k(k) || vs < k || (vs % 8) ||
      (uintptr_t(v) & 15u) || (uintptr_t(q) & 15u) || (uintptr_t(rowmax) & 3u) || (uintptr_t(scale) & 3u))
    return cudaErrorInvalidValue;
  codes_from_rotated<<<unsigned(rows), 256, 0, reinterpret_cast<cudaStream_t>(stream_ptr)>>>(
      static_cast<const __nv_bfloat16*>(v), vs, static_cast<const uint32_t*>(rowmax), static_cast<int8_t*>(q),
      static_cast<float*>(scale), k);
  return cudaGetLastError();
}

H3SK_EXPORT int h3_convrot_quant_act(const void* x, int64_t xs, void* q, void* scale, int64_t rows, int k,
                                     int act, uintptr_t stream_ptr) {
  using namespace h3sk;
  if (!x || !q || !scale || rows < 1 || rows > INT32_MAX || !valid_k(k) || act < 0 || act > 2)
    return cudaErrorInvalidValue;
  const int64_t width = act == kActSwiGLU ? 2 * int64_t(k) : int64_t(k);
  if (xs < width || (xs % 8) || (uintptr_t(x) & 15u) || (uintptr_t(q) & 7u) || (uintptr_t(scale) & 3u))
    return cudaErrorInvalidValue;
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_ptr);
  if (act == kActNone) return launch<kActNone, kModeQuant>(x, xs, q, scale, nullptr, rows, k, stream);
  if (act == kActGeluTanh) return launch<kActGeluTanh, kModeQuant>(x, xs, q, scale, nullptr, rows, k, stream);
  return launch<kActSwiGLU, kModeQuant>(x, xs, q, scale, nullptr, rows, k, stream);
}
