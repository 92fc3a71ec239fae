// Device-side building blocks shared by the minicpm5_mk sm_100a kernels:
// bounded mbarrier waits, TMA 2D loads, tcgen05 (TMEM alloc / MMA / commit / ld) wrappers,
// shared-memory matrix descriptors, and bf16 packing helpers.
//
// Every wait on an mbarrier is bounded by a wall-clock limit read from %globaltimer.  When a
// wait runs out, the waiting role raises the CTA-wide abort flag (in shared memory), every other
// role's wait then returns early, the kernel drains what it issued, frees TMEM and records an
// error code in the library's device error word.  No kernel traps or spins forever.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace mk {

// Device error codes (written into the library's device error word, first error wins).
enum : int {
  DEV_OK = 0,
  DEV_ERR_TIMEOUT_GEMM = 0x100,
  DEV_ERR_TIMEOUT_ATTN = 0x200,
  DEV_ERR_BAD_TOKEN_ID = 0x300,
  DEV_ERR_TIMEOUT_ATTN_TC = 0x400,
};

// Wall-clock limit of one mbarrier wait.  Legitimate waits are microseconds long.
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s

// Zig-zag sequence-parallel layout of one sequence over `world` ranks (sp_global_block,
// plugin/minicpm5_mk/mk_attn.py:721-724, generalised from 2 to `world` ranks): the sequence is cut
// into blocks of `blk` tokens; in every group of 2 * world consecutive blocks, rank r owns block r
// and block 2 * world - 1 - r, which balances the causal attention work.  A rank stores its blocks
// in sequence order (`rows_per_rank` rows); an all-gather stacks the ranks' rows rank by rank.
// blk == 0 is the identity (one rank, rows = positions).
struct SpLayout {
  int blk = 0, rank = 0, world = 1, rows_per_rank = 0;
};

// Sequence position of local row `row`.
__host__ __device__ __forceinline__ int sp_pos(const SpLayout& l, int row) {
  if (l.blk == 0) return row;
  const int i = row / l.blk, k = i >> 1;
  const int b = 2 * l.world * k + ((i & 1) ? 2 * l.world - 1 - l.rank : l.rank);
  return b * l.blk + row % l.blk;
}

// Row of sequence position `pos` in the rank-by-rank all-gathered buffer.
__host__ __device__ __forceinline__ int sp_row(const SpLayout& l, int pos) {
  if (l.blk == 0) return pos;
  const int b = pos / l.blk, k = b / (2 * l.world), m = b % (2 * l.world);
  const bool second = m >= l.world;
  const int r = second ? 2 * l.world - 1 - m : m;
  return r * l.rows_per_rank + (2 * k + (second ? 1 : 0)) * l.blk + pos % l.blk;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---------------------------------------------------------------------------------- launch overlap
// Programmatic dependent launch: the forward launches each kernel with programmatic stream serialization,
// so it may start (barrier set-up, TMEM allocation, descriptor prefetch, loads of the constant weights)
// while the previous kernel drains.  pdl_wait() blocks the calling thread until every earlier kernel of
// the stream has completed and its writes are visible; every thread calls it before its first access to
// memory an earlier kernel writes or reads.  Without the launch attribute it returns at once.
// pdl_trigger() lets the next kernel's CTAs be scheduled once every CTA of this grid has issued it (or
// exited); they still wait in pdl_wait() for this grid to finish.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ---------------------------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

// A waiting thread is suspended until the phase completes (or this long), instead of re-polling and
// taking issue slots from the warps that do the work.
constexpr uint32_t kSuspendHintNs = 10000000;
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity), "r"(kSuspendHintNs)
      : "memory");
  return ok != 0;
}

// Wait until the phase with the given parity has completed.  Returns false when the CTA-wide
// abort flag is (or becomes) set, or when the wait exceeds kWaitLimitNs (then it sets the flag).
// The clock and the flag are read only every kWaitPoll unsuccessful tries: reading %globaltimer
// costs a few hundred nanoseconds, which would otherwise be added to every hand-off that finds
// its barrier not yet complete.
constexpr uint32_t kWaitPoll = 16;
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
  const uint32_t a = smem_u32(bar);
  uint64_t t0 = 0;
  for (uint32_t n = 1;; ++n) {
    if (mbar_try_wait(a, parity)) return true;
    if (n % kWaitPoll == 0) {
      if (*abort_flag) return false;
      const uint64_t t = globaltimer_ns();
      if (t0 == 0) {
        t0 = t;
      } else if (t - t0 > kWaitLimitNs) {
        *abort_flag = 1;
        return false;
      }
    }
  }
}

// Bounded wait that ignores the abort flag (used while draining on the way out).
__device__ __forceinline__ bool mbar_wait_drain(uint64_t* bar, uint32_t parity) {
  const uint32_t a = smem_u32(bar);
  uint64_t t0 = 0;
  for (uint32_t n = 1;; ++n) {
    if (mbar_try_wait(a, parity)) return true;
    if (n % kWaitPoll == 0) {
      const uint64_t t = globaltimer_ns();
      if (t0 == 0) {
        t0 = t;
      } else if (t - t0 > kWaitLimitNs) {
        return false;
      }
    }
  }
}

// One lane of the (fully active) warp returns true.
__device__ __forceinline__ bool elect_one() {
  uint32_t pred;
  asm volatile(
      "{\n\t.reg .pred p;\n\t.reg .b32 r;\n\t"
      "elect.sync r|p, 0xffffffff;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(pred));
  return pred != 0;
}

// ---------------------------------------------------------------------------------- TMA
// 2D tiled bulk tensor load global -> shared, completion signalled on `bar` (complete_tx bytes).
// c0 is the innermost coordinate: callers keep c0 * element size a multiple of 16 bytes.
__device__ __forceinline__ void tma_load_2d(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int c0,
                                            int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], "
      "[%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}

__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// Make this thread's generic-proxy shared-memory writes visible to the async proxy
// (tcgen05.mma operand reads, TMA).
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---------------------------------------------------------------------------------- CTA pairs
// A cluster of two CTAs runs one 2-SM UMMA (tcgen05 .cta_group::2): the even CTA issues the MMAs and
// waits for both CTAs' operands; signals cross the pair as mbarrier arrivals on shared::cluster
// addresses obtained with mapa.  No copy is multicast.
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// shared::cluster address of this CTA's shared variable at `smem_addr` in CTA `rank` of the cluster
__device__ __forceinline__ uint32_t mapa_cluster(uint32_t smem_addr, uint32_t rank) {
  uint32_t d;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(d) : "r"(smem_addr), "r"(rank));
  return d;
}
// All threads of both CTAs; release / acquire order the shared-memory writes around it.
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Arrive on a barrier of either CTA of the pair.  What the arrival publishes is TMEM content (converted
// weights) or the end of TMEM reads (a drained accumulator), which tcgen05 fences order, so the default
// CTA-scope release suffices; cluster scope cost about 1000 cycles per arrival.
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cl_addr) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(cl_addr) : "memory");
}
// 2D tiled load into this CTA's shared memory whose completion (complete_tx) is counted on the barrier
// at shared::cluster address `bar_cl`, which may belong to the pair's even CTA.
__device__ __forceinline__ void tma_load_2d_pair(void* smem_dst, const CUtensorMap* map, uint32_t bar_cl, int c0,
                                                 int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, "
      "%4}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cl), "r"(c0), "r"(c1)
      : "memory");
}
// TMEM allocation of a CTA pair: the same warp of both CTAs executes it; both receive the same address.
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* smem_slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_slot)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
// D (+)= A * B over the pair: M = 256 rows, the even CTA's TMEM holds rows [0, 128) of A and D, the odd
// CTA's rows [128, 256); B's N columns are split in halves over the two CTAs' shared memory.
__device__ __forceinline__ void mma_f16_ts_pair(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc,
                                                uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive (once) on the barrier at shared::cluster address `bar_cl` when the pair MMAs issued so far by
// this thread have completed.
__device__ __forceinline__ void mma_commit_pair(uint32_t bar_cl) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar_cl)
               : "memory");
}

// ---------------------------------------------------------------------------------- tcgen05
__device__ __forceinline__ void tmem_alloc(uint32_t* smem_slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_slot)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D(tmem) (+)= A(smem desc) * B(smem desc)^T, kind::f16 (bf16 inputs, f32 accumulate).
__device__ __forceinline__ void mma_f16_ss(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                           uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive (once) on `bar` when every tcgen05 async op issued so far by this thread has completed.
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

// 32 lanes x 32 consecutive 32-bit columns: thread i of the warp receives row (lane base + i).
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]),
        "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]),
        "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
}
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// 32 lanes x 32 consecutive 32-bit columns from registers (thread i writes row lane base + i).
__device__ __forceinline__ void tmem_st_32x32b_x32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
      "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]),
      "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]),
      "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
// 32 lanes x 16 consecutive 32-bit columns from registers.
__device__ __forceinline__ void tmem_st_32x32b_x16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// D(tmem) (+)= A(tmem) * B(smem desc), kind::f16.  A is M x K bf16 with row m in lane m and two
// consecutive K elements packed per 32-bit column.
__device__ __forceinline__ void mma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc,
                                           uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// 3D tiled bulk tensor load global -> shared (c0 innermost).
__device__ __forceinline__ void tma_load_3d(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1,
                                            int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], "
      "[%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm volatile("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Shared-memory matrix descriptor (sm_100 UMMA format): K-major operand, 128-byte swizzle,
// rows of 128 bytes, 8-row core groups 1024 bytes apart (stride byte offset), version 1.
// The tile base must be 1024-byte aligned; stepping K by 16 bf16 inside the swizzle row adds
// 32 bytes (2 in the >>4 address field).
__device__ __forceinline__ uint64_t sdesc_kmajor_sw128(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr >> 4) & 0x3FFF);  // start address
  d |= static_cast<uint64_t>(1) << 16;                     // leading byte offset (unused for swizzled K-major)
  d |= static_cast<uint64_t>(1024 >> 4) << 32;             // stride byte offset: 8 rows * 128 B
  d |= static_cast<uint64_t>(1) << 46;                     // descriptor version (sm_100)
  d |= static_cast<uint64_t>(2) << 61;                     // layout: SWIZZLE_128B
  return d;
}

// MN-major operand with 128-byte swizzle: 64 MN-contiguous elements per 128-byte row, rows along K,
// 8-row (K) groups 1024 bytes apart (stride byte offset), 64-element MN blocks `lbo` bytes apart.
__device__ __forceinline__ uint64_t sdesc_mnmajor_sw128(uint32_t smem_addr, uint32_t lbo) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr >> 4) & 0x3FFF);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFF) << 16;
  d |= static_cast<uint64_t>(1024 >> 4) << 32;
  d |= static_cast<uint64_t>(1) << 46;
  d |= static_cast<uint64_t>(2) << 61;
  return d;
}

// Instruction descriptor for kind::f16: bf16 A/B, f32 D, both K-major, shape M x N.
__host__ __device__ constexpr uint32_t idesc_bf16_f32(int M, int N) {
  return (1u << 4)                                   // D format f32
         | (1u << 7)                                 // A format bf16
         | (1u << 10)                                // B format bf16
         | (static_cast<uint32_t>(N >> 3) << 17)     // N / 8
         | (static_cast<uint32_t>(M >> 4) << 24);    // M / 16
}
// Same with B MN-major.
__host__ __device__ constexpr uint32_t idesc_bf16_f32_bmn(int M, int N) { return idesc_bf16_f32(M, N) | (1u << 16); }

// ---------------------------------------------------------------------------------- numerics
// Four signed int8 (one 32-bit word) -> four bf16 (two 32-bit words), exact; lo = (x0, x1),
// hi = (x2, x3), lower K in the low half.
// Each byte b goes into the low byte of a 16-bit lane under 0x43 (the bf16 exponent of 128).  With
// bit 7 cleared the lane is bf16(128 + (b & 0x7F)); the two's-complement value is
// x = (b & 0x7F) - 128 * b7 = that - 128 - 128 * b7, so one bf16x2 add of c = bf16(-128) or
// bf16(-256) (0xC300 with bit 7 of b copied in) gives x.  Every operand and the sum are integers of
// at most 8 significant bits, so the add is exact.  8 instructions per 4 values.
__device__ __forceinline__ void i8x4_to_bf16x4(uint32_t w, uint32_t& lo, uint32_t& hi) {
  asm("{\n\t"
      ".reg .b32 r0, r1, v0, v1, c0, c1;\n\t"
      "prmt.b32 r0, %2, 0x43434343, 0x4140;\n\t"             // [b0, 0x43, b1, 0x43]
      "prmt.b32 r1, %2, 0x43434343, 0x4342;\n\t"             // [b2, 0x43, b3, 0x43]
      "and.b32 v0, r0, 0xFF7FFF7F;\n\t"
      "and.b32 v1, r1, 0xFF7FFF7F;\n\t"
      "lop3.b32 c0, r0, 0x00800080, 0xC300C300, 0xEA;\n\t"   // (r & 0x80) | 0xC300 per lane
      "lop3.b32 c1, r1, 0x00800080, 0xC300C300, 0xEA;\n\t"
      "add.rn.bf16x2 %0, v0, c0;\n\t"
      "add.rn.bf16x2 %1, v1, c1;\n\t"
      "}"
      : "=r"(lo), "=r"(hi)
      : "r"(w));
}

// max(a, b, c) in one instruction.
__device__ __forceinline__ float max3f(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}
// (a0, a1) * s + c for two lanes in one packed f32x2 FMA.
__device__ __forceinline__ void fma2_sc(float a0, float a1, float s, float c, float& d0, float& d1) {
  asm("{\n\t.reg .b64 x, y, z, r;\n\t"
      "mov.b64 x, {%2, %3};\n\tmov.b64 y, {%4, %4};\n\tmov.b64 z, {%5, %5};\n\t"
      "fma.rn.f32x2 r, x, y, z;\n\tmov.b64 {%0, %1}, r;\n\t}"
      : "=f"(d0), "=f"(d1)
      : "f"(a0), "f"(a1), "f"(s), "f"(c));
}
// (d0, d1) += (a0, a1) in one packed f32x2 add.
__device__ __forceinline__ void add2_acc(float& d0, float& d1, float a0, float a1) {
  asm("{\n\t.reg .b64 x, y;\n\t"
      "mov.b64 x, {%0, %1};\n\tmov.b64 y, {%2, %3};\n\t"
      "add.rn.f32x2 x, x, y;\n\tmov.b64 {%0, %1}, x;\n\t}"
      : "+f"(d0), "+f"(d1)
      : "f"(a0), "f"(a1));
}

__device__ __forceinline__ uint32_t pack_bf16x2(float a, float b) {
  __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&v);
}

__device__ __forceinline__ float2 unpack_bf16x2(uint32_t w) {
  __nv_bfloat162 v = *reinterpret_cast<__nv_bfloat162*>(&w);
  return __bfloat1622float2(v);
}

// silu(g) = g * sigmoid(g), with sigmoid(g) = (1 + tanh(g / 2)) / 2: one MUFU operation (tanh.approx,
// relative error about 2^-11, below the bf16 rounding of the result) instead of an exponential and a
// reciprocal.  Measured 1 % faster on the gate/up GEMM, cold and under the power cap.
__device__ __forceinline__ float silu_f(float g) {
  float t;
  asm("tanh.approx.f32 %0, %1;" : "=f"(t) : "f"(0.5f * g));
  return 0.5f * g * (1.0f + t);
}

// v[j] summed over the 32 lanes of the warp; lane l returns the sum of v[l].
// Butterfly transpose-reduction: 31 shuffles for 32 sums, in a fixed order.
__device__ __forceinline__ float warp_transpose_sum32(float (&v)[32], int lane) {
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) {
    const bool up = (lane & off) != 0;
#pragma unroll
    for (int i = 0; i < off; ++i) {
      const float send = up ? v[i] : v[i + off];
      const float keep = up ? v[i + off] : v[i];
      v[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
    }
  }
  return v[0];
}

}  // namespace mk
