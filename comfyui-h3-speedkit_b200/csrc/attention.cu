// INT8 attention of the H3 block on B200 (sm_100a): the consumer of the QKV op's
// pre-quantised operands (kernels/dense/dense_ring.cu:32-94 and
// qk_int_sv_i8_cuda.cuh of H3 SpeedKit, a SageAttention-derived mma.sync kernel
// for SM120).  Same C ABI (H3DenseArgs, h3_dense_*), same arithmetic, written
// for tcgen05: S = Q K^T and O_blk = P V run as kind::i8 MMAs with int32
// accumulators in TMEM, and one thread owns one query row for the softmax.
// Operand layouts are the reference's; the int32 -> float conversions are exact.
//
// Operands (one batch, any head count; qo_heads % kv_heads == 0):
//   Q  INT8 [B, Hq, Sq, 128], one FP32 scale per 4 rows {32b + s + 8j} of a
//      128-row block:           QS [B, Hq, ceil(Sq/128) * 32]
//   K  INT8 [B, Hk, Sk, 128], one FP32 scale per 128-key block and key class
//      t = (key % 8) / 2:       KS [B, Hk, ceil(Sk/128) * 4]
//   V  INT8 [B*Hk*128, ceil(Sk/128)*128] channel-major, keys permuted inside
//      every run of 16 as [0,1,8,9,2,3,10,11,4,5,12,13,6,7,14,15];  VS [B*Hk*128]
//   O  BF16, BHSD or BSHD strides.
//
// Arithmetic, per query row and 128-key block j (the reference's, exactly):
//   s = int32 Q.K (exact; float(s) is exact, |s| < 2^22);  (all int32 accumulators
//   start at zero: the first K=32 step of each MMA overwrites its slot)
//   per key class t: scale_t = (sm_scale * log2e) * (q_scale * k_scale[j][t]);
//   m_t = fmaf(max_t(s), scale_t, -7.9943534), tile_m = max_t m_t,
//   m = max(m_prev, tile_m), r = ex2(-|m_prev - tile_m|),
//   o_scale = m_prev < tile_m ? r : 1, tile_scale = tile_m < m_prev ? r : 1;
//   d_t *= o_scale (but see the last block), O *= o_scale;
//   p = ex2(fmaf(s, scale_t, -tile_m)), P = u8(rni, saturated);
//   blocks before the last: d_t = fmaf(sum of the 4 P of (16-key tile, t), tile_scale, d_t)
//   (the integer sum dp4a gives, as a float), tile by tile;
//   the last block: keys >= Sk score -1e30, the row maximum starts at -50000,
//   and d_t = fmaf((p0 + p1) + (p8 + p9), tile_scale, d_t) on the unrounded p,
//   except that its first 16-key tile folds the rescale in:
//   d_t = fmaf(d_t, o_scale, round(((p0 + p1) + (p8 + p9)) * tile_scale)) -- the
//   contraction the reference's compiler picks on that straight-line path;
//   O = fmaf(float(int32 P.V), tile_scale, O);
//   at the end d = (d_0 + d_1) + (d_2 + d_3), O = (O * rcp.approx(d)) * v_scale, BF16.
// The 4 "key classes" t are the 4 threads of a quad of the reference's mma.sync
// layout; their partial maxima and denominators are kept apart here so that
// every FP32 operation has the reference's operands in the reference's order.
// The unit is compiled with --use_fast_math, like the reference's dense unit.
//
// Roles (20 warps, five warpgroups):
//   * warpgroup 0: warp 0 the TMA producer (lane 0: Q once and the K ring, lane
//     1: the V ring, both 4 stages), warp 1 the TMEM owner and the MMA issuers
//     (lane 0: S(j) into TMEM slot j % 4; lane 1: P.V(j) into the same slot
//     once P(j) is written), warps 2-3 idle;
//   * warpgroups 1-2: 8 correction warps, thread = (query row, 64 output
//     channels) with O in registers: each block's P.V joins O, then the
//     normalised BF16 output;
//   * warpgroups 3-4: 8 softmax warps, two per TMEM lane quadrant taking
//     alternate blocks, thread = query row; a short chain step per block
//     carries the running maximum and the four class denominators from block
//     to block in the reference's order.
// setmaxnreg moves registers from warpgroup 0 to the others.  The four TMEM
// slots let S run up to four blocks ahead of the softmax.  Every mbarrier wait
// is bounded (2 s) and reports a status code instead of hanging.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <climits>
#include <cstdint>

#include "host_util.h"
#include "sm100.cuh"

namespace h3sk {
namespace attn {

using namespace sm100;

constexpr int kRows = 128;             // query rows per CTA (TMEM lanes)
constexpr int kKeys = 128;             // keys per block
constexpr int kDim = 128;              // head dimension
constexpr int kTileBytes = 128 * 128;  // one INT8 [128 x 128] tile
constexpr int kStages = 4;             // K and V ring depth
constexpr int kSlots = 4;              // TMEM slots: block j's S, then its P.V, in slot j % 4
constexpr int kSoftWarps = 8;          // two per TMEM lane quadrant (alternate blocks): thread = query row
constexpr int kCorrWarps = 8;          // two per quadrant: thread = (query row, 64 output channels)
// Warpgroups: 0 = TMA producer, MMA issuer and two idle warps; 1-2 = correction;
// 3-4 = softmax.  setmaxnreg moves registers from warpgroup 0 to the others.
constexpr int kCorrWarp0 = 4, kSoftWarp0 = kCorrWarp0 + kCorrWarps;
constexpr int kThreads = 32 * (kSoftWarp0 + kSoftWarps);
constexpr int kRegsLaunch = 96;        // per thread at launch (the compiler's cap for kThreads)
constexpr int kRegsSetup = 32, kRegsCorr = 104, kRegsSoft = 120;
static_assert(kRegsSetup * 128 + kRegsCorr * 32 * kCorrWarps + kRegsSoft * 32 * kSoftWarps <=
                  kRegsLaunch * kThreads,
              "setmaxnreg shares must fit in the block's launch registers");
constexpr float kExpOffset = 7.9943534f;          // attn_utils.cuh:40 (S_U8_OFFSET)
constexpr float kLog2e = 1.44269504088896340736f;
constexpr uint64_t kTimeoutNs = 2000000000ull;

struct Args {
  int q_heads, kv_heads, batch;
  int q_len, kv_len, q_blocks, kv_blocks;
  int q_block_start;
  const float* qs;   // [B, Hq, q_blocks * 32]
  const float* ks;   // [B, Hk, kv_blocks * 4]
  const float* vs;   // [B * Hk * 128]
  __nv_bfloat16* o;
  int64_t o_sb, o_sh, o_ss;   // element strides
  float sm_scale;
  int* status;
};

struct Smem {
  // 1024-aligned operand tiles (128-byte swizzle)
  uint8_t q[kTileBytes];
  uint8_t k[kStages][kTileBytes];
  uint8_t v[kStages][kTileBytes];
  uint8_t p[kSlots][kTileBytes];  // P of block j in buffer j % 4
  float2 sc[kSlots][kRows];       // [block % 4][row]: (o_scale, tile_scale) to the correction warps
  float xinv[kRows];              // 1 / d, from the softmax to the correction warps
  float cm[kRows];                // the running maximum after the last chained block
  float4 cd[kRows];               // the four class denominators after it
  uint64_t q_full;
  uint64_t k_full[kStages], k_empty[kStages];
  uint64_t v_full[kStages], v_empty[kStages];
  uint64_t s_full[kSlots], p_full[kSlots], pv_full[kSlots], slot_free[kSlots];
  uint64_t sc_full[kSlots], inv_full, drain;
  uint64_t cbar[4];               // [quadrant]: the chain step of the previous block is done
  uint32_t tmem;
  int abort;
};

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float rcp(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float max3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}
__device__ __forceinline__ float as_f(uint32_t x) { return __uint_as_float(x); }
// Four probabilities -> four u8 codes (cvt.rni.s32 then a saturating pack;
// mma.cuh:769-786), low byte = a.
__device__ __forceinline__ uint32_t u8x4(float a, float b, float c, float d) {
  uint32_t qa, qb, qc, qd, hi, w;
  asm("cvt.rni.s32.f32 %0, %1;" : "=r"(qa) : "f"(a));
  asm("cvt.rni.s32.f32 %0, %1;" : "=r"(qb) : "f"(b));
  asm("cvt.rni.s32.f32 %0, %1;" : "=r"(qc) : "f"(c));
  asm("cvt.rni.s32.f32 %0, %1;" : "=r"(qd) : "f"(d));
  asm("cvt.pack.sat.u8.s32.b32 %0, %1, %2, 0;" : "=r"(hi) : "r"(qd), "r"(qc));
  asm("cvt.pack.sat.u8.s32.b32 %0, %1, %2, %3;" : "=r"(w) : "r"(qb), "r"(qa), "r"(hi));
  return w;
}
// ---- packed FP32 pairs (sm_100 f32x2), flushing subnormals like the unit's scalar math ----
__device__ __forceinline__ uint64_t pk(uint32_t lo, uint32_t hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "r"(lo), "r"(hi));
  return r;
}
__device__ __forceinline__ uint64_t pkf(float lo, float hi) { return pk(__float_as_uint(lo), __float_as_uint(hi)); }
__device__ __forceinline__ void upk(uint64_t x, uint32_t& lo, uint32_t& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=r"(lo), "=r"(hi) : "l"(x));
}
__device__ __forceinline__ uint64_t add2(uint64_t a, uint64_t b) {
  uint64_t c;
  asm("add.rn.ftz.f32x2 %0, %1, %2;" : "=l"(c) : "l"(a), "l"(b));
  return c;
}
__device__ __forceinline__ uint64_t mul2(uint64_t a, uint64_t b) {
  uint64_t c;
  asm("mul.rn.ftz.f32x2 %0, %1, %2;" : "=l"(c) : "l"(a), "l"(b));
  return c;
}
__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.ftz.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
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
// 32 lanes x 16 consecutive 32-bit columns (load, store, fill).
__device__ __forceinline__ void tmem_load_16cols(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
}
__device__ __forceinline__ void tmem_store_16cols(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}
__device__ __forceinline__ void tmem_fill_16cols(uint32_t taddr, uint32_t x) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1};" ::"r"(taddr),
      "r"(x)
      : "memory");
}
// The same 32-bit value into 32 consecutive columns of the warp's 32 lanes.
__device__ __forceinline__ void tmem_fill_32cols(uint32_t taddr, uint32_t x) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,"
      "%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1};" ::"r"(taddr),
      "r"(x)
      : "memory");
}
__device__ __forceinline__ void tmem_store_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void regs_dec() { asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N)); }
template <int N>
__device__ __forceinline__ void regs_inc() { asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N)); }
// this warpgroup's share, from the launch count
template <int N>
__device__ __forceinline__ void regs_set() {
  if constexpr (N < kRegsLaunch)
    regs_dec<N>();
  else if constexpr (N > kRegsLaunch)
    regs_inc<N>();
}
template <int N>
__device__ __forceinline__ void tmem_load_cols(uint32_t taddr, uint32_t (&r)[N]);
template <>
__device__ __forceinline__ void tmem_load_cols<32>(uint32_t taddr, uint32_t (&r)[32]) {
  tmem_load_32cols(taddr, r);
}
// 32 lanes x 64 consecutive 32-bit columns.
__device__ __forceinline__ void tmem_load_64cols(uint32_t taddr, uint32_t (&r)[64]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x64.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,"
      "%32,%33,%34,%35,%36,%37,%38,%39,%40,%41,%42,%43,%44,%45,%46,%47,"
      "%48,%49,%50,%51,%52,%53,%54,%55,%56,%57,%58,%59,%60,%61,%62,%63}, [%64];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31]),
        "=r"(r[32]), "=r"(r[33]), "=r"(r[34]), "=r"(r[35]), "=r"(r[36]), "=r"(r[37]), "=r"(r[38]), "=r"(r[39]),
        "=r"(r[40]), "=r"(r[41]), "=r"(r[42]), "=r"(r[43]), "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47]),
        "=r"(r[48]), "=r"(r[49]), "=r"(r[50]), "=r"(r[51]), "=r"(r[52]), "=r"(r[53]), "=r"(r[54]), "=r"(r[55]),
        "=r"(r[56]), "=r"(r[57]), "=r"(r[58]), "=r"(r[59]), "=r"(r[60]), "=r"(r[61]), "=r"(r[62]), "=r"(r[63])
      : "r"(taddr)
      : "memory");
}
template <>
__device__ __forceinline__ void tmem_load_cols<64>(uint32_t taddr, uint32_t (&r)[64]) {
  tmem_load_64cols(taddr, r);
}

// Bounded mbarrier wait that sleeps: try_wait with a suspend-time hint parks the
// warp until the phase completes (or the hint runs out) instead of spinning, so a
// waiting warp leaves its scheduler's issue slots to the warps still computing.
// Gives up after kTimeoutNs (raising *abort, recording `code`) or once another
// role raised *abort.
constexpr uint32_t kSuspendHintNs = 10000000u;
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(done)
      : "r"(smem_addr(bar)), "r"(parity), "r"(kSuspendHintNs)
      : "memory");
  return done != 0;
}
__device__ __forceinline__ bool mbar_test_wait(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(done)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return done != 0;
}
__device__ __forceinline__ bool wait_sleep(uint64_t* bar, uint32_t parity, volatile int* abort, int* status,
                                           int code) {
  if (mbar_test_wait(bar, parity)) return true;   // the common case: already complete
  if (mbar_try_wait_sleep(bar, parity)) return true;
  const uint64_t start = global_timer_ns();
  for (;;) {
    if (mbar_try_wait_sleep(bar, parity)) return true;
    if (abort != nullptr && *abort) return false;
    if (global_timer_ns() - start > kTimeoutNs) {
      if (abort != nullptr) *abort = 1;
      if (status != nullptr) atomicExch(status, code);
      return false;
    }
  }
}

// mbarrier wait by a whole warp; the warp's verdict is unanimous.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, Smem& sm, int* status, int code) {
  // every lane tests the barrier (one instruction for the warp, no divergent branch)
  const bool ok = wait_sleep(bar, parity, reinterpret_cast<volatile int*>(&sm.abort), status, code);
  return __all_sync(0xffffffffu, ok);
}

// Instruction descriptors (sm100.cuh idesc_i8 fields): s8 x s8 and u8 x s8, M=N=128.
constexpr uint32_t kIdescQK = idesc_i8(kRows, kKeys);
constexpr uint32_t kIdescPV = idesc_i8(kRows, kDim) & ~(7u << 7);   // A format 0 = u8

__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_addr(bar)), "r"(x), "r"(y), "r"(z)
      : "memory");
}

__global__ void __launch_bounds__(kThreads, 1)
    attention_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_k,
                     const __grid_constant__ CUtensorMap map_v, const Args a) {
  extern __shared__ uint8_t smem_raw[];
  Smem& sm = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int bx = int(blockIdx.x) + a.q_block_start;     // 128-row query block
  const int head = int(blockIdx.y), batch = int(blockIdx.z);
  const int kv_head = head / (a.q_heads / a.kv_heads);
  const int bh_q = batch * a.q_heads + head, bh_k = batch * a.kv_heads + kv_head;
  const int nblk = a.kv_blocks;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(&sm.abort);

  if (threadIdx.x == 0) {
    mbar_init(&sm.q_full, 1);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&sm.k_full[s], 1);
      mbar_init(&sm.k_empty[s], 1);
      mbar_init(&sm.v_full[s], 1);
      mbar_init(&sm.v_empty[s], 1);
    }
    for (int s = 0; s < kSlots; ++s) {
      mbar_init(&sm.s_full[s], 1);
      mbar_init(&sm.p_full[s], 4);
      mbar_init(&sm.pv_full[s], 1);
      mbar_init(&sm.slot_free[s], kCorrWarps);
      mbar_init(&sm.sc_full[s], 4);
    }
    mbar_init(&sm.inv_full, 4);
    for (int q = 0; q < 4; ++q) mbar_init(&sm.cbar[q], 1);
    mbar_init(&sm.drain, 2);
    sm.abort = 0;
    fence_mbar_init();
    tma_prefetch_map(&map_q);
    tma_prefetch_map(&map_k);
    tma_prefetch_map(&map_v);
  }
  if (warp == 1) {
    tmem_alloc(&sm.tmem, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem;

  // Each warpgroup's branch opens with its register share (setmaxnreg, executed
  // by all four warps of the warpgroup at one site).
  if (warp < kCorrWarp0) {
    regs_set<kRegsSetup>();
    if (warp == 0) {
      // ---------------- TMA producer: lane 0 Q and the K ring, lane 1 the V ring ----------------
      // (two independent threads, so that a K load never waits behind a V stage)
      if (lane < 2) {
        const bool is_k = lane == 0;
        uint64_t* full = is_k ? sm.k_full : sm.v_full;
        uint64_t* empty = is_k ? sm.k_empty : sm.v_empty;
        int issued = 0;
        bool ok = true;
        if (is_k) {
          mbar_arrive_expect_tx(&sm.q_full, kTileBytes);
          tma_load_3d(sm.q, &map_q, &sm.q_full, 0, bx * kRows, bh_q);
        }
        for (int j = 0; ok && j < nblk; ++j) {
          const int s = j % kStages;
          const uint32_t ph = uint32_t(j / kStages) & 1u;
          if (j >= kStages) ok = wait_sleep(&empty[s], ph ^ 1u, abort_flag, a.status, is_k ? 41 : 42);
          if (!ok) break;
          mbar_arrive_expect_tx(&full[s], kTileBytes);
          if (is_k)
            tma_load_3d(sm.k[s], &map_k, &full[s], 0, j * kKeys, bh_k);
          else
            tma_load_3d(sm.v[s], &map_v, &full[s], j * kKeys, 0, bh_k);
          issued = j + 1;
        }
        // every copy this thread issued lands before the CTA exits
        if (is_k) mbar_wait_bounded(&sm.q_full, 0, nullptr, a.status, 43, kTimeoutNs);
        for (int j = (issued > kStages ? issued - kStages : 0); j < issued; ++j)
          mbar_wait_bounded(&full[j % kStages], uint32_t(j / kStages) & 1u, nullptr, a.status, 43, kTimeoutNs);
      }
      __syncwarp();
    } else if (warp == 1) {
      // ---------------- MMA issuers: lane 0 the S stream, lane 1 the P.V stream ----------------
      // S(j) goes into TMEM slot j % 4 once the correction warps are done with
      // P.V(j - 4) there; P.V(j) goes into the same slot once P(j) is written
      // (the softmax has finished reading S(j)).  Two independent threads, so
      // that neither stream waits behind the other's inputs.  Both MMAs start
      // from a zero accumulator.
      if (lane == 0) {
        bool ok = wait_sleep(&sm.q_full, 0, abort_flag, a.status, 51);
        const uint64_t qd = smem_desc_k_sw128(sm.q);
        for (int j = 0; ok && j < nblk; ++j) {
          const int s = j % kStages, slot = j % kSlots;
          ok = wait_sleep(&sm.k_full[s], uint32_t(j / kStages) & 1u, abort_flag, a.status, 52) &&
               (j < kSlots || wait_sleep(&sm.slot_free[slot], uint32_t(j / kSlots - 1) & 1u, abort_flag, a.status, 53));
          if (!ok) break;
          tc_fence_after();
          const uint64_t kd = smem_desc_k_sw128(sm.k[s]);
#pragma unroll
          for (int kk = 0; kk < kDim / 32; ++kk)
            mma_i8(tmem + 128u * slot, qd + uint64_t(2 * kk), kd + uint64_t(2 * kk), kIdescQK, kk);
          mma_commit(&sm.k_empty[s]);
          mma_commit(&sm.s_full[slot]);
        }
        // every MMA this thread issued completes before TMEM is released
        mma_commit(&sm.drain);
      } else if (lane == 1) {
        bool ok = true;
        for (int j = 0; ok && j < nblk; ++j) {
          const int s = j % kStages, slot = j % kSlots;
          ok = wait_sleep(&sm.p_full[slot], uint32_t(j / kSlots) & 1u, abort_flag, a.status, 54) &&
               wait_sleep(&sm.v_full[s], uint32_t(j / kStages) & 1u, abort_flag, a.status, 55);
          if (!ok) break;
          tc_fence_after();
          const uint64_t pd = smem_desc_k_sw128(sm.p[slot]), vd = smem_desc_k_sw128(sm.v[s]);
#pragma unroll
          for (int kk = 0; kk < kKeys / 32; ++kk)
            mma_i8(tmem + 128u * slot, pd + uint64_t(2 * kk), vd + uint64_t(2 * kk), kIdescPV, kk);
          mma_commit(&sm.v_empty[s]);
          mma_commit(&sm.pv_full[slot]);
        }
        mma_commit(&sm.drain);
      }
      if (lane < 2) mbar_wait_bounded(&sm.drain, 0, nullptr, a.status, 57, kTimeoutNs);
      __syncwarp();
    }   // warps 2 and 3: idle
  } else if (warp < kSoftWarp0) {
    regs_set<kRegsCorr>();
    // ---------------- correction: O <- fmaf(float(P.V), tile_scale, O * o_scale) ----------------
    // Thread = (query row, half): TMEM lane r of quadrant warp % 4 and output
    // channels [64 h, 64 h + 64), O of them in registers.  Block j's P.V joins O
    // here while the softmax works on later blocks; o_scale and tile_scale come
    // from the block's chain step.  x * 1 == x for every value O takes (FTZ
    // arithmetic makes no subnormals), so a warp rescales all of its rows when
    // any of them needs it.
    const int quarter = warp & 3;
    const int half = (warp - kCorrWarp0) >> 2;
    const int r = quarter * 32 + lane;
    const int row = bx * kRows + r;
    const uint32_t lane_off = uint32_t(quarter * 32) << 16;
    const uint32_t col0 = uint32_t(64 * half);
    uint64_t o2[32];   // O of channels col0 + [0, 64), as FP32 pairs
#pragma unroll
    for (int i = 0; i < 32; ++i) o2[i] = 0ull;
    bool ok = true;
    for (int j = 0; j < nblk; ++j) {
      const int slot = j % kSlots;
      const uint32_t ph = uint32_t(j / kSlots) & 1u;
      if (!warp_wait(&sm.sc_full[slot], ph, sm, a.status, 71)) {
        ok = false;
        break;
      }
      const float2 sc = sm.sc[slot][r];
      if (!warp_wait(&sm.pv_full[slot], ph, sm, a.status, 72)) {
        ok = false;
        break;
      }
      tc_fence_after();
      if (j > 0 && __any_sync(0xffffffffu, sc.x != 1.0f)) {
        const uint64_t os2 = pkf(sc.x, sc.x);
#pragma unroll
        for (int i = 0; i < 32; ++i) o2[i] = mul2(o2[i], os2);
      }
      const uint64_t ts2 = pkf(sc.y, sc.y);
      const uint32_t t_pv = tmem + 128u * slot + lane_off + col0;
#pragma unroll
      for (int g = 0; g < 2; ++g) {
        uint32_t pv[32];
        tmem_load_32cols(t_pv + 32 * g, pv);
        tmem_load_wait();
        if (g == 1) {
          // every P.V value of the slot is in registers: release it for S(j + 4)
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&sm.slot_free[slot]);
        }
#pragma unroll
        for (int i = 0; i < 16; ++i)
          o2[16 * g + i] = fma2(pkf(float(int(pv[2 * i])), float(int(pv[2 * i + 1]))), ts2, o2[16 * g + i]);
      }
    }
    // O = (O / d) * v_scale in BF16
    if (ok && warp_wait(&sm.inv_full, 0, sm, a.status, 73) && row < a.q_len) {
      const float inv = sm.xinv[r];
      const float* vs = a.vs + int64_t(bh_k) * kDim + col0;
      __nv_bfloat16* out =
          a.o + int64_t(batch) * a.o_sb + int64_t(head) * a.o_sh + int64_t(row) * a.o_ss + col0;
#pragma unroll
      for (int g = 0; g < 8; ++g) {
        uint32_t w[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          uint32_t lo, hi;
          upk(o2[4 * g + q], lo, hi);
          const float o0 = (as_f(lo) * inv) * __ldg(vs + 8 * g + 2 * q);
          const float o1 = (as_f(hi) * inv) * __ldg(vs + 8 * g + 2 * q + 1);
          __nv_bfloat162 h = __floats2bfloat162_rn(o0, o1);
          w[q] = *reinterpret_cast<uint32_t*>(&h);
        }
        reinterpret_cast<uint4*>(out)[g] = make_uint4(w[0], w[1], w[2], w[3]);
      }
    }
  } else {
    regs_set<kRegsSoft>();
    // ---------------- softmax ----------------
    // Two warps per TMEM lane quadrant, thread = query row: warp `sub` takes the
    // blocks j with j % 2 == sub.  A block's probabilities, P codes and
    // denominators depend only on its own maximum, so the two warps compute
    // them side by side; the running maximum and the class-denominator chain --
    // the reference's sequential part -- pass from block to block, and so from
    // warp to warp, in a short chain step through shared memory.  The four
    // class denominators take the 16-key runs in key order, as the reference's
    // four quad threads do.
    const int quarter = warp & 3;
    const int sub = (warp - kSoftWarp0) >> 2;
    const int r = quarter * 32 + lane;                  // row within the block (TMEM lane)
    const uint32_t lane_off = uint32_t(quarter * 32) << 16;
    const float q_scale = a.qs[int64_t(bh_q) * a.q_blocks * 32 + bx * 32 + (r >> 5) * 8 + (r & 7)];
    const float sm_base = a.sm_scale * kLog2e;
    const float* kscale = a.ks + int64_t(bh_k) * nblk * 4;
    bool return_early = false;
    float kn[4];                              // the K scales of this warp's next block
#pragma unroll
    for (int t = 0; t < 4; ++t) kn[t] = sub < nblk ? __ldg(kscale + sub * 4 + t) : 0.0f;
    // The odd-block warps start once P(0) is written, which staggers the two
    // warps' first exp2 streams (measured a few per cent faster).
    if (sub == 1 && nblk > 1 && !warp_wait(&sm.p_full[0], 0, sm, a.status, 60)) return_early = true;
    for (int j = sub; !return_early && j < nblk; j += 2) {
      const bool last = j == nblk - 1;
      const int slot = j % kSlots;
      const uint32_t t_s = tmem + 128u * slot + lane_off;
      if (!warp_wait(&sm.s_full[slot], uint32_t(j / kSlots) & 1u, sm, a.status, 61)) break;
      tc_fence_after();
      float scale[4];
#pragma unroll
      for (int t = 0; t < 4; ++t) scale[t] = sm_base * (q_scale * kn[t]);
      if (j + 2 < nblk) {
#pragma unroll
        for (int t = 0; t < 4; ++t) kn[t] = __ldg(kscale + (j + 2) * 4 + t);
      }
      // per-class maxima: class t holds keys 2t, 2t+1, 2t+8, 2t+9 of every run
      // of 16 (integers; in the last block floats, with the keys past Sk at
      // -1e30 and the maximum starting at -50000)
      float mx[4];
      uint32_t v[32];
      if (!last) {
        int mb[4][2];   // two chains per class
#pragma unroll
        for (int q4 = 0; q4 < 4; ++q4) {
          tmem_load_32cols(t_s + 32 * q4, v);
          tmem_load_wait();
#pragma unroll
          for (int t = 0; t < 4; ++t) {
#pragma unroll
            for (int e = 0; e < 2; ++e) {
              const int o = 2 * t + 8 * e;
              int x = max(max(int(v[o]), int(v[o + 1])), max(int(v[16 + o]), int(v[17 + o])));
              mb[t][e] = q4 == 0 ? x : max(mb[t][e], x);
            }
          }
        }
#pragma unroll
        for (int t = 0; t < 4; ++t) mx[t] = float(max(mb[t][0], mb[t][1]));
      } else {
#pragma unroll
        for (int t = 0; t < 4; ++t) mx[t] = -50000.0f;
#pragma unroll
        for (int q4 = 0; q4 < 4; ++q4) {
          tmem_load_32cols(t_s + 32 * q4, v);
          tmem_load_wait();
          const int key0 = j * kKeys + 32 * q4;
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const float sc = key0 + i < a.kv_len ? float(int(v[i])) : -1.0e30f;
            mx[(i & 7) >> 1] = fmaxf(mx[(i & 7) >> 1], sc);
          }
        }
      }
      float mt[4];
#pragma unroll
      for (int t = 0; t < 4; ++t) mt[t] = fmaf(mx[t], scale[t], -kExpOffset);
      const float tile_m = fmaxf(fmaxf(mt[0], mt[1]), fmaxf(mt[2], mt[3]));
      // probabilities -> u8 P (key order of V: the four keys of class t of each
      // 16-key run in one word at byte 4t) and the runs' class denominators.
      // P buffer j % 4 was last read by P.V(j - 4), complete since S(j) is.
      const float neg_m = -tile_m;
      const uint64_t negm2 = pkf(neg_m, neg_m);
      uint64_t scale2[4];
#pragma unroll
      for (int t = 0; t < 4; ++t) scale2[t] = pkf(scale[t], scale[t]);
      uint8_t* const prow = sm.p[slot] + (r >> 3) * 1024 + (r & 7) * 128;
      float den[8][4];
      // (two copies of the loop, so that neither has a branch inside)
      if (!last) {
#pragma unroll
        for (int q4 = 0; q4 < 4; ++q4) {
          tmem_load_32cols(t_s + 32 * q4, v);
          tmem_load_wait();
#pragma unroll
          for (int c2 = 0; c2 < 2; ++c2) {
            uint32_t words[4];
            const int chunk = 2 * q4 + c2;        // 16-key run = 16-byte chunk of the P row
#pragma unroll
            for (int t = 0; t < 4; ++t) {
              const int i0 = 16 * c2 + 2 * t;
              // x = fmaf(float(s), scale_t, -tile_m), two keys per instruction
              uint32_t x0, x1, x2, x3;
              upk(fma2(pkf(float(int(v[i0])), float(int(v[i0 + 1]))), scale2[t], negm2), x0, x1);
              upk(fma2(pkf(float(int(v[i0 + 8])), float(int(v[i0 + 9]))), scale2[t], negm2), x2, x3);
              words[t] = u8x4(ex2(as_f(x0)), ex2(as_f(x1)), ex2(as_f(x2)), ex2(as_f(x3)));
              // the integer sum of the four codes, exact as a float
              den[chunk][t] = float(int(__dp4a(words[t], 0x01010101u, 0u)));
            }
            *reinterpret_cast<uint4*>(prow + ((chunk ^ (r & 7)) << 4)) = make_uint4(words[0], words[1], words[2],
                                                                                   words[3]);
          }
        }
      } else {
#pragma unroll
        for (int q4 = 0; q4 < 4; ++q4) {
          tmem_load_32cols(t_s + 32 * q4, v);
          tmem_load_wait();
#pragma unroll
          for (int c2 = 0; c2 < 2; ++c2) {
            uint32_t words[4];
            const int chunk = 2 * q4 + c2;
#pragma unroll
            for (int t = 0; t < 4; ++t) {
              const int i0 = 16 * c2 + 2 * t;
              const int k0 = j * kKeys + 32 * q4 + i0;
              const float s0 = k0 < a.kv_len ? float(int(v[i0])) : -1.0e30f;
              const float s1 = k0 + 1 < a.kv_len ? float(int(v[i0 + 1])) : -1.0e30f;
              const float s2 = k0 + 8 < a.kv_len ? float(int(v[i0 + 8])) : -1.0e30f;
              const float s3 = k0 + 9 < a.kv_len ? float(int(v[i0 + 9])) : -1.0e30f;
              const float p0 = ex2(fmaf(s0, scale[t], neg_m)), p1 = ex2(fmaf(s1, scale[t], neg_m));
              const float p2 = ex2(fmaf(s2, scale[t], neg_m)), p3 = ex2(fmaf(s3, scale[t], neg_m));
              words[t] = u8x4(p0, p1, p2, p3);
              den[chunk][t] = (p0 + p1) + (p2 + p3);   // the last block sums the unrounded p
            }
            *reinterpret_cast<uint4*>(prow + ((chunk ^ (r & 7)) << 4)) = make_uint4(words[0], words[1], words[2],
                                                                                   words[3]);
          }
        }
      }
      fence_async_shared();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.p_full[slot]);
      // chain step: the running maximum and the denominators, block after block
      float m_prev = -50000.0f;
      float d[4] = {1.0f, 1.0f, 1.0f, 1.0f};
      if (j > 0) {
        if (!warp_wait(&sm.cbar[quarter], uint32_t(j - 1) & 1u, sm, a.status, 62)) break;
        m_prev = sm.cm[r];
        const float4 dd = sm.cd[r];
        d[0] = dd.x;
        d[1] = dd.y;
        d[2] = dd.z;
        d[3] = dd.w;
      }
      const float m = fmaxf(m_prev, tile_m);
      const float smaller = ex2(-fabsf(m_prev - tile_m));
      const float o_scale = m_prev < tile_m ? smaller : 1.0f;
      const float tile_scale = tile_m < m_prev ? smaller : 1.0f;
      // o_scale and tile_scale of this block to the row's correction threads.
      // Slot j % 4 was last read for block j - 4, before the correction released
      // that block's TMEM slot for S(j) (waited on above).
      sm.sc[slot][r] = make_float2(o_scale, tile_scale);
      // blocks before the last rescale d on their own (the reference applies
      // o_scale under a branch); the last block folds d * o_scale into its
      // first denominator update, as the reference's straight-line float path
      // compiles: fma(d, o_scale, round(sum * tile_scale))
      if (!last) {
#pragma unroll
        for (int t = 0; t < 4; ++t) d[t] *= o_scale;
      }
#pragma unroll
      for (int c = 0; c < 8; ++c) {
#pragma unroll
        for (int t = 0; t < 4; ++t)
          d[t] = (last && c == 0) ? fmaf(d[t], o_scale, __fmul_rn(den[c][t], tile_scale))
                                  : fmaf(den[c][t], tile_scale, d[t]);
      }
      if (!last) {
        sm.cm[r] = m;
        sm.cd[r] = make_float4(d[0], d[1], d[2], d[3]);
      } else {
        sm.xinv[r] = rcp((d[0] + d[1]) + (d[2] + d[3]));
      }
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&sm.sc_full[slot]);
        mbar_arrive(last ? &sm.inv_full : &sm.cbar[quarter]);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// The exp2 roofline: every score of the attention takes one ex2.approx (the
// reference's arithmetic; no other unit computes it bit for bit), and the SFU
// that executes it is the attention's bound.  Eight independent chains per thread,
// eight 256-thread CTAs per SM.
// Each chain runs x <- -2^x, which stays in [-1, 0).
__global__ void __launch_bounds__(256) ex2_peak_kernel(int iters, float* sink) {
  float x[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) x[i] = -1.0e-3f * float(threadIdx.x + i);
  for (int it = 0; it < iters; ++it) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      asm volatile("ex2.approx.ftz.f32 %0, %0;" : "+f"(x[i]));
      x[i] = -x[i];
    }
  }
  float acc = 0.0f;
#pragma unroll
  for (int i = 0; i < 8; ++i) acc += x[i];
  if (sink != nullptr) sink[blockIdx.x * blockDim.x + threadIdx.x] = acc;
}

}  // namespace attn
}  // namespace h3sk

// ---- C ABI: the reference's h3_dense_* (dense_ring.cu:16-107) -------------------------

struct H3DenseArgs {
  void *q, *k, *v, *o, *q_scale, *k_scale, *v_scale;
  uint32_t batch, qo_len, kv_len, qo_heads, kv_heads;
  uint32_t q_stride_b, q_stride_h, q_stride_s;
  uint32_t k_stride_b, k_stride_h, k_stride_s;
  uint32_t v_stride_b, v_stride_h, v_stride_d;
  uint32_t o_stride_b, o_stride_h, o_stride_s;
  float sm_scale;
};

#define H3SK_EXPORT extern "C" __attribute__((visibility("default")))

namespace {

bool encode_3d(CUtensorMap* map, const void* base, uint64_t d0, uint64_t d1, uint64_t d2, uint64_t s1, uint64_t s2) {
  auto fn = h3sk::tensor_map_encoder();
  if (!fn) return false;
  const cuuint64_t dims[3] = {d0, d1, d2};
  const cuuint64_t strides[2] = {s1, s2};
  const cuuint32_t box[3] = {128, 128, 1};
  const cuuint32_t es[3] = {1, 1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(base), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

H3SK_EXPORT size_t h3_dense_args_size(void) { return sizeof(H3DenseArgs); }
// The reference reports its build's experiment id here (H3_VARIANT_ID); this
// library implements the arithmetic of variant 8102.
H3SK_EXPORT int h3_dense_query_group(void) { return 8102; }
H3SK_EXPORT const char* h3_dense_error_string(int code) {
  return cudaGetErrorString(static_cast<cudaError_t>(code));
}

H3SK_EXPORT int h3_dense_launch_window(const H3DenseArgs* a, uintptr_t stream_ptr, uint32_t start) {
  using namespace h3sk::attn;
  if (!a || !a->q || !a->k || !a->v || !a->o || !a->q_scale || !a->k_scale || !a->v_scale || !a->batch ||
      !a->qo_len || !a->kv_len || !a->qo_heads || !a->kv_heads || a->qo_heads % a->kv_heads != 0)
    return cudaErrorInvalidValue;
  const uint64_t q_blocks = (a->qo_len + 127) / 128, kv_blocks = (a->kv_len + 127) / 128;
  // the operand layouts of the QKV op (and of the reference's own checks,
  // dense_ring.cu:44-47): Q and K contiguous [B, H, S, 128], V [B*Hk*128, padded Sk]
  if (a->q_stride_s != 128 || a->q_stride_h != a->qo_len * 128 || a->q_stride_b != a->qo_heads * a->q_stride_h ||
      a->k_stride_s != 128 || a->k_stride_h != a->kv_len * 128 || a->k_stride_b != a->kv_heads * a->k_stride_h ||
      a->v_stride_h != 128 * a->v_stride_d || a->v_stride_b != a->kv_heads * a->v_stride_h ||
      a->v_stride_d < kv_blocks * 128 || a->v_stride_d % 16)
    return cudaErrorInvalidValue;
  const bool bhsd = a->o_stride_s == 128 && a->o_stride_h == a->qo_len * 128;
  const bool bshd = a->o_stride_s == a->qo_heads * 128 && a->o_stride_h == 128;
  if (!bhsd && !bshd) return cudaErrorInvalidValue;
  if (!aligned16(a->q) || !aligned16(a->k) || !aligned16(a->v) || !aligned16(a->o) ||
      (reinterpret_cast<uintptr_t>(a->q_scale) & 3u) || (reinterpret_cast<uintptr_t>(a->k_scale) & 3u) ||
      (reinterpret_cast<uintptr_t>(a->v_scale) & 3u))
    return cudaErrorInvalidValue;
  if (!(a->sm_scale == a->sm_scale) || start >= q_blocks) return cudaErrorInvalidValue;
  if (q_blocks > 65535u * 65535u || a->qo_heads > 65535u || a->batch > 65535u) return cudaErrorInvalidValue;
  const cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_ptr);
  CUtensorMap mq, mk, mv;
  if (!encode_3d(&mq, a->q, 128, a->qo_len, uint64_t(a->batch) * a->qo_heads, a->q_stride_s, a->q_stride_h) ||
      !encode_3d(&mk, a->k, 128, a->kv_len, uint64_t(a->batch) * a->kv_heads, a->k_stride_s, a->k_stride_h) ||
      !encode_3d(&mv, a->v, a->v_stride_d, 128, uint64_t(a->batch) * a->kv_heads, a->v_stride_d, a->v_stride_h))
    return cudaErrorInvalidValue;
  int* status = h3sk::status_device_ptr();
  if (!status) return cudaErrorInvalidSymbol;
  if (start) {
    // rows before the window are zero (dense_ring.cu:68-80)
    const size_t rows = size_t(start) * 128;
    for (uint32_t b = 0; b < a->batch; ++b) {
      char* base = static_cast<char*>(a->o) + size_t(b) * a->o_stride_b * 2;
      cudaError_t e = bshd ? cudaMemsetAsync(base, 0, rows * a->qo_heads * 128 * 2, stream)
                           : cudaMemset2DAsync(base, size_t(a->o_stride_h) * 2, 0, rows * 128 * 2, a->qo_heads, stream);
      if (e != cudaSuccess) return e;
    }
  }
  Args args{};
  args.q_heads = int(a->qo_heads);
  args.kv_heads = int(a->kv_heads);
  args.batch = int(a->batch);
  args.q_len = int(a->qo_len);
  args.kv_len = int(a->kv_len);
  args.q_blocks = int(q_blocks);
  args.kv_blocks = int(kv_blocks);
  args.q_block_start = int(start);
  args.qs = static_cast<const float*>(a->q_scale);
  args.ks = static_cast<const float*>(a->k_scale);
  args.vs = static_cast<const float*>(a->v_scale);
  args.o = static_cast<__nv_bfloat16*>(a->o);
  args.o_sb = a->o_stride_b;
  args.o_sh = a->o_stride_h;
  args.o_ss = a->o_stride_s;
  args.sm_scale = a->sm_scale;
  args.status = status;
  const int smem = int(sizeof(Smem)) + 1024;
  // the warpgroups' setmaxnreg shares need the block's launch registers; refuse
  // (never launch) a build whose launch register count would leave them short
  static int launch_regs = -1;
  if (launch_regs < 0) {
    cudaFuncAttributes attr;
    const cudaError_t fe = cudaFuncGetAttributes(&attr, attention_kernel);
    if (fe != cudaSuccess) return fe;
    launch_regs = attr.numRegs;
  }
  if (launch_regs < kRegsLaunch) return cudaErrorInvalidConfiguration;
  cudaError_t e = cudaFuncSetAttribute(attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  const dim3 grid(unsigned(q_blocks - start), a->qo_heads, a->batch);
  attention_kernel<<<grid, kThreads, smem, stream>>>(mq, mk, mv, args);
  return cudaGetLastError();
}

H3SK_EXPORT int h3_dense_launch(const H3DenseArgs* a, uintptr_t stream) { return h3_dense_launch_window(a, stream, 0); }

// numRegs, localSizeBytes, sharedSizeBytes (dynamic), maxThreadsPerBlock, binaryVersion
// (the reference's field order, dense_ring.cu:96-104).
H3SK_EXPORT int h3_dense_resources(int* out) {
  if (!out) return cudaErrorInvalidValue;
  cudaFuncAttributes attr;
  const cudaError_t e = cudaFuncGetAttributes(&attr, h3sk::attn::attention_kernel);
  if (e != cudaSuccess) return e;
  out[0] = attr.numRegs;
  out[1] = int(attr.localSizeBytes);
  out[2] = int(sizeof(h3sk::attn::Smem)) + 1024;
  out[3] = attr.maxThreadsPerBlock;
  out[4] = attr.binaryVersion;
  return 0;
}

// ex2.approx throughput of the whole GPU (G ex2 / s), measured now: the attention's roofline denominator.
H3SK_EXPORT int h3sk_ex2_peak(int iters, double* gops, uintptr_t stream) {
  if (!gops || iters < 64 || iters > (1 << 20)) return cudaErrorInvalidValue;
  const cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  int device = 0, sms = 0;
  cudaError_t e = cudaGetDevice(&device);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
  if (e != cudaSuccess) return e;
  cudaEvent_t t0, t1;
  cudaEventCreate(&t0);
  cudaEventCreate(&t1);
  h3sk::attn::ex2_peak_kernel<<<sms * 8, 256, 0, s>>>(64, nullptr);   // warm-up
  cudaEventRecord(t0, s);
  h3sk::attn::ex2_peak_kernel<<<sms * 8, 256, 0, s>>>(iters, nullptr);
  cudaEventRecord(t1, s);
  e = cudaGetLastError();
  if (e == cudaSuccess) e = cudaEventSynchronize(t1);
  float ms = 0.0f;
  if (e == cudaSuccess) e = cudaEventElapsedTime(&ms, t0, t1);
  cudaEventDestroy(t0);
  cudaEventDestroy(t1);
  if (e != cudaSuccess) return e;
  *gops = double(sms) * 8 * 256 * 8 * double(iters) / (double(ms) * 1e-3) / 1e9;
  return cudaSuccess;
}
