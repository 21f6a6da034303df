// Streaming machinery of the persistent B200 row kernels (prologue and ConvRot
// quantiser): TMA-fed shared-memory rings of whole token rows, row teams that
// consume them, a conflict-free two-half A->B exchange, and the host-side plan.
//
// CTA = `teams` row teams of `team_threads` threads (4 per 256-value group), one
// CTA per SM.  Each team owns a private ring of `slots_per_team` row slots; its
// thread 0 loads the team's rows into the ring with one 3D TMA box per row (no
// multicast):
//   tensor [rows][width/64][64] BF16, box {64, K/64, 1}, 128-byte swizzle,
// so a row occupies K*2 bytes of its slot as K/64 "lines" of 128 bytes whose
// 16-byte chunks are XOR-permuted by (line & 7).  Every read of the slot uses
// the same permutation (swz128), which makes both the 8-byte stats reads and the
// 16-byte layout-A reads of a warp conflict-free.  While a team works on one
// row, its next rows are already landing, so every SM keeps HBM reads in flight
// all the time (the one-CTA-per-row kernels only had loads outstanding during
// their first phase).
//
// Team t's k-th row is local row i = t + k * teams of the CTA, token row
// blockIdx.x + i * gridDim.x, in slot d = k % slots_per_team; full[t][d]
// completes (parity (k / slots_per_team) & 1) when its bytes have landed.  The
// team refills slot d with row k + slots_per_team right after the team barrier
// that follows the last read of row k, so no "empty" barrier is needed.
//
// Every wait is bounded (2 s); a wait that runs out records its code in the
// library status word.  Teams decide to stop only at a team barrier that
// AND-reduces the threads' flags, so a team never splits around a barrier, and
// thread 0 waits (bounded) for its outstanding boxes before the CTA exits.
#pragma once
#include "host_util.h"
#include "rq_core.cuh"
#include "sm100.cuh"

#include <map>
#include <mutex>

namespace h3sk {
namespace rs {

constexpr int kMaxSlots = 32;
constexpr int kMaxTeams = 15;                   // named barriers 1..15
constexpr int kMaxK = 16384;
constexpr int kSmemBudget = 224 * 1024;         // dynamic shared memory per CTA (227 KB less static state)
constexpr int kHalfGroupBytes = 512;            // exchange region per 256-value group
constexpr uint64_t kWaitNs = 2000000000ull;
enum : int { kCodeFull = 0x301 };

// 128-byte swizzle of a byte offset inside a 1024-byte aligned buffer (the TMA
// CU_TENSOR_MAP_SWIZZLE_128B pattern: bits 4..6 ^= bits 7..9).
__device__ __forceinline__ uint32_t swz128(uint32_t byte) { return byte ^ (((byte >> 7) & 7u) << 4); }

// 3D tiled TMA load with an L2 cache hint, completion on an mbarrier.
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y, int z,
                                            uint64_t cache_hint) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4, %5}], [%2], %6;" ::"r"(sm100::smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(sm100::smem_addr(bar)), "r"(x), "r"(y), "r"(z), "l"(cache_hint)
      : "memory");
}
__device__ __forceinline__ uint64_t l2_policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// Thread 0 of a team: load token row `row` into ring slot `slot` (evict-first:
// every input row is read exactly once).
__device__ __forceinline__ void issue_row(const CUtensorMap* map, unsigned char* slot, uint64_t* bar, int row, int k,
                                          int width) {
  const uint64_t policy = l2_policy_evict_first();
  sm100::mbar_arrive_expect_tx(bar, uint32_t(width) * 2u);
  tma_load_3d(slot, map, bar, 0, 0, row, policy);
  if (width != k) tma_load_3d(slot + 2 * k, map, bar, 0, k / 64, row, policy);
}

// Barrier of one row team (named barrier `id`, `threads` threads).
__device__ __forceinline__ void team_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}
// Team barrier that returns whether `ok` holds on every thread of the team.
__device__ __forceinline__ bool team_sync_and(int id, int threads, bool ok) {
  uint32_t all;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.and.pred q, %2, %3, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}\n"
      : "=r"(all)
      : "r"(ok ? 1u : 0u), "r"(id), "r"(threads)
      : "memory");
  return all != 0;
}

// Shared-memory vector access through 32-bit shared-window addresses (keeps
// addresses in one register each).
__device__ __forceinline__ uint4 lds128(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
  return v;
}
__device__ __forceinline__ void sts128(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}
__device__ __forceinline__ uint2 lds64(uint32_t addr) {
  uint2 v;
  asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(addr));
  return v;
}

// Layout-A inputs of team thread (group g, q) from a swizzled row at shared
// address `row`: the 64 consecutive BF16 values [256g + 64q, +64) as 8 16-byte
// words (line 4g + q).
__device__ __forceinline__ void load_row_a(uint32_t row, int g, int q, uint4 (&raw)[8]) {
  const uint32_t line = uint32_t(4 * g + q);
  const uint32_t base = row + line * 128u, key = (line & 7u) << 4;
#pragma unroll
  for (int i = 0; i < 8; ++i) raw[i] = lds128(base + ((16u * uint32_t(i)) ^ key));
}

// ---- exchange A -> B in two halves through a 512-byte buffer per group --------
// Half h moves the chunks (4 consecutive values) whose index bit 3 equals h; bit 3
// is a register bit in both layouts, so each half is balanced: every thread
// writes 8 chunks and reads 8 chunks.  A chunk is named by index bits b2, b4b5,
// b6b7; its 16-byte slot in the buffer is
//   line b4b5, bank slot (b4b5 ^ b6b7) | ((b2 ^ odd) << 2)
// so the 8 lanes of each quarter-warp phase (two groups x four threads) hit 8
// distinct bank slots on both the writing and the reading side.
// `buf` = shared address of the group's 512-byte buffer.  With q and odd fixed
// per thread, the writer's slot for (b2, b45) is  b45*128 + (wkey ^ (b45 << 4 | b2 << 6))
// with wkey = q << 4 | odd << 6, and the reader's slot for (b2, b67) is
// q*128 + (wkey ^ (b67 << 4 | b2 << 6)) -- one XOR and one add per access.
template <int kHalf>
__device__ __forceinline__ void exchange_half(uint64_t (&v)[32], uint32_t buf, uint32_t wkey, uint32_t rbase) {
  // layout A (thread q = b6b7): chunk k = b2 | b3 << 1 | b4b5 << 2 in registers 2k, 2k+1
#pragma unroll
  for (int b45 = 0; b45 < 4; ++b45) {
#pragma unroll
    for (int b2 = 0; b2 < 2; ++b2) {
      const int k = b2 | (kHalf << 1) | (b45 << 2);
      const uint32_t addr = buf + uint32_t(b45 * 128) + (wkey ^ uint32_t((b45 << 4) | (b2 << 6)));
      sts128(addr, uint32_t(v[2 * k]), uint32_t(v[2 * k] >> 32), uint32_t(v[2 * k + 1]), uint32_t(v[2 * k + 1] >> 32));
    }
  }
  __syncwarp();
  // layout B (thread q = b4b5): chunk m = b2 | b3 << 1 | b6b7 << 2 in registers 2m, 2m+1
#pragma unroll
  for (int b67 = 0; b67 < 4; ++b67) {
#pragma unroll
    for (int b2 = 0; b2 < 2; ++b2) {
      const int m = b2 | (kHalf << 1) | (b67 << 2);
      const uint4 c = lds128(rbase + (wkey ^ uint32_t((b67 << 4) | (b2 << 6))));
      v[2 * m] = (uint64_t(c.y) << 32) | c.x;
      v[2 * m + 1] = (uint64_t(c.w) << 32) | c.z;
    }
  }
  __syncwarp();
}

// buf: shared address of this group's 512-byte region; q: team index; odd: group
// parity.  The region is either the group's own exchange buffer or the group's
// part of the row slot it has just read in layout A (lines 4g .. 4g+3 belong to
// the group's four threads, all in one warp; slots are sized so that inactive
// groups past K / 256 also stay inside their slot).  For the in-slot form the
// caller puts a __syncwarp between its layout-A reads and this call.
__device__ __forceinline__ void exchange_a_to_b_halves(uint64_t (&v)[32], uint32_t buf, int q, int odd) {
  const uint32_t wkey = (uint32_t(q) << 4) | (uint32_t(odd) << 6);
  const uint32_t rbase = buf + uint32_t(q) * 128u;
  exchange_half<0>(v, buf, wkey, rbase);
  exchange_half<1>(v, buf, wkey, rbase);
}

// ---- shared state of a streaming CTA ---------------------------------------------
struct alignas(16) RingState {
  uint64_t full[kMaxSlots];            // team t, ring slot d: full[t * slots_per_team + d]
  float stat_fold[kMaxTeams][4];       // prologue: the four logical-warp sums of squares
  float max_fold[kMaxTeams][2][8];     // per-warp absmax, double-buffered by row parity
};

// Geometry shared by host and device.
struct Plan {
  int k;               // values per row (the quantised width)
  int width;           // BF16 input values per row (2k for SwiGLU)
  int team_threads;    // multiple of 32, >= k / 64
  int teams;           // <= kMaxTeams
  int threads;         // teams * team_threads
  int slots_per_team;  // 2: one row being read, the next one landing
  int slot_bytes;      // max(width * 2, groups * 512) rounded up to 1024
  int ring_bytes;      // teams * slots_per_team * slot_bytes
  int exch_bytes;      // per team: groups * 512, or 0 = exchange inside the row slot
  int extra_bytes;     // caller's shared arrays after the rings and exchange buffers
  int smem;            // dynamic shared memory incl. 1024-byte alignment slack
};

// Up to 512 threads (16 warps: 4 per SM sub-partition, so 128 registers a thread)
// and two ring slots per team (deeper rings measured slower), `extra` bytes
// reserved after the rings.  The A->B exchange gets its own buffers when they fit
// (measured faster); otherwise it runs inside the row slot just read.
inline Plan make_plan(int k, int width, int min_team_threads, int extra = 0) {
  Plan p{};
  p.k = k;
  p.width = width;
  int team = ((k / 64 + 31) / 32) * 32;
  if (team < min_team_threads) team = min_team_threads;
  p.team_threads = team;
  const int exch = (team / 4) * kHalfGroupBytes;
  // A slot holds the row and, for an in-slot exchange, every group's 512 bytes.
  p.slot_bytes = ((max(width * 2, exch) + 1023) / 1024) * 1024;
  p.extra_bytes = ((extra + 1023) / 1024) * 1024;
  int teams = 512 / team;
  if (teams < 1) teams = 1;
  if (teams > kMaxTeams) teams = kMaxTeams;
  if (2 * teams > kMaxSlots) teams = kMaxSlots / 2;
  for (; teams >= 1; --teams) {
    const int ring = teams * 2 * p.slot_bytes;
    const int rest = kSmemBudget - 1024 - p.extra_bytes - ring;
    if (rest >= teams * exch) { p.exch_bytes = exch; break; }
    if (rest >= 0) { p.exch_bytes = 0; break; }
  }
  p.teams = teams;
  p.slots_per_team = teams >= 1 ? 2 : 0;
  p.threads = teams * team;
  p.ring_bytes = teams * 2 * p.slot_bytes;
  p.smem = 1024 + p.ring_bytes + teams * p.exch_bytes + p.extra_bytes;
  return p;
}

// ---- host side ----------------------------------------------------------------------
// Tensor map of BF16 rows viewed as [rows][width / 64][64] with row stride `ld`
// elements (ld % 8 == 0, base 16-byte aligned), box {64, k / 64, 1}.
inline bool make_row_map(CUtensorMap* map, const void* base, int64_t rows, int width, int k, int64_t ld) {
  auto fn = tensor_map_encoder();
  if (!fn) return false;
  const cuuint64_t dims[3] = {64, cuuint64_t(width / 64), cuuint64_t(rows)};
  const cuuint64_t strides[2] = {128, cuuint64_t(ld) * 2};
  const cuuint32_t box[3] = {64, cuuint32_t(k / 64), 1};
  const cuuint32_t elem_strides[3] = {1, 1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, elem_strides,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Opt `kernel` into `smem` bytes of dynamic shared memory (once per kernel and
// device) and return the grid: one CTA per SM, no more CTAs than rows.
inline cudaError_t stream_grid(const void* kernel, int smem, int64_t rows, int* grid) {
  static std::mutex mu;
  static std::map<std::pair<const void*, int>, int> ready;   // (kernel, device) -> SM count
  int device = 0;
  cudaError_t e = cudaGetDevice(&device);
  if (e != cudaSuccess) return e;
  int sms = 0;
  {
    std::lock_guard<std::mutex> lock(mu);
    auto it = ready.find({kernel, device});
    if (it == ready.end()) {
      e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBudget);
      if (e != cudaSuccess) return e;
      e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
      if (e != cudaSuccess) return e;
      it = ready.emplace(std::make_pair(kernel, device), sms).first;
    }
    sms = it->second;
  }
  if (smem > kSmemBudget) return cudaErrorInvalidValue;
  *grid = int(rows < sms ? rows : sms);
  return cudaSuccess;
}

}  // namespace rs
}  // namespace h3sk
