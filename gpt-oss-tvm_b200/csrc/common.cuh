// common.cuh -- sm_100a building blocks shared by the gpt-oss B200 kernels:
// bf16 bit helpers, bounded mbarrier waits, TMA tile loads, tcgen05 (TMEM
// allocation, MMA, loads/stores) and the device-side error flag.
//
// Every spin-wait is bounded.  A wait that runs out records an error code in
// the caller-supplied device flag and returns false; the kernel then skips
// its remaining work, drains what it has in flight and frees its TMEM, so a
// stuck pipeline never hangs the GPU.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace gptoss {

// ---------------------------------------------------------------- errors --
enum DeviceError : uint32_t {
  kErrNone = 0,
  kErrTimeoutFull = 1u << 0,     // consumer waited too long for a full stage
  kErrTimeoutEmpty = 1u << 1,    // producer waited too long for an empty stage
  kErrTimeoutAccum = 1u << 2,    // epilogue waited too long for an accumulator
  kErrBadRouting = 1u << 3,      // expert index outside [0, E)
  kErrTimeoutOther = 1u << 4,
  kErrTimeoutFlag = 1u << 5,     // generic bounded flag wait ran out
  kErrBadTilePlan = 1u << 6,     // a token tile larger than the GEMM variant holds
};

// Token rows of one grouped-GEMM tile (the MMA N dimension).  With few rows
// per expert (decode) the tiles are at most 32 rows and the GEMM runs its
// weight-streaming variant; otherwise at most 160 (two 160-column
// accumulators leave TMEM room for four one-chunk weight slots; a multiple
// of 32, the granularity of a CTA-pair MMA's N).  The permutation plans its
// token tiles with the same rule as the GEMM launch.
constexpr int kMoeTileMaxRows = 160;
constexpr int kMoeTileRowsSmall = 32;
__host__ __device__ __forceinline__ int moe_tile_rows_max(int64_t rows, int32_t num_experts) {
  return rows <= 8 * (int64_t)num_experts ? kMoeTileRowsSmall : kMoeTileMaxRows;
}

// Poll budget for one mbarrier wait.  try_wait itself blocks for a bounded,
// hardware-defined window, so this is several seconds of waiting at most.
constexpr uint32_t kWaitPolls = 1u << 22;

__device__ __forceinline__ void raise_error(uint32_t* flag, uint32_t code) {
  if (flag) atomicOr(flag, code);
}

// ------------------------------------------------------------------ bf16 --
__device__ __forceinline__ float bf16_bits_to_f32(uint16_t h) {
  return __uint_as_float(((uint32_t)h) << 16);
}
// Round-to-nearest-even fp32 -> bf16 bits (finite values).
__device__ __forceinline__ uint16_t f32_to_bf16_bits(float f) {
  uint32_t u = __float_as_uint(f);
  u = u + (((u >> 16) & 1u) + 0x7FFFu);
  return (uint16_t)(u >> 16);
}
__device__ __forceinline__ float round_bf16(float f) { return bf16_bits_to_f32(f32_to_bf16_bits(f)); }

__host__ __device__ __forceinline__ int64_t min64(int64_t a, int64_t b) { return a < b ? a : b; }
__host__ __device__ __forceinline__ int64_t max64(int64_t a, int64_t b) { return a > b ? a : b; }

// ------------------------------------------------------------- smem addr --
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

// ------------------------------------------------------------- mbarriers --
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(
                   smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait for the phase with the given parity to complete.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, uint32_t* err, uint32_t code) {
  for (uint32_t i = 0; i < kWaitPolls; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
  }
  raise_error(err, code);
  return false;
}

// ------------------------------------------------------------------- TMA --
__device__ __forceinline__ void tma_prefetch_desc(const void* tmap) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(tmap) : "memory");
}
// 2-D tiled load (no multicast), completion signalled on `bar` as tx bytes.
__device__ __forceinline__ void tma_load_2d(void* smem_dst, const void* tmap, int32_t x, int32_t y,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cta.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(smem_dst)),
      "l"(tmap), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

// 3-D tiled load (no multicast), completion signalled on `bar` as tx bytes.
__device__ __forceinline__ void tma_load_3d(void* smem_dst, const void* tmap, int32_t x, int32_t y, int32_t z,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cta.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::
          "r"(smem_u32(smem_dst)),
      "l"(tmap), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
      : "memory");
}

// --------------------------------------------------------------- tcgen05 --
// TMEM allocation is warp-wide; the allocated base address is written to smem.
__device__ __forceinline__ void tmem_alloc(uint32_t* smem_dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_dst)),
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
// D[tmem] (+)= A[tmem] * B[smem]^T, kind::f16 (bf16 inputs, fp32 accumulate).
__device__ __forceinline__ void tc_mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// One 64-wide K chunk: four K=16 steps, A columns a_tmem + 0/8/16/24 and B
// 32 bytes further along the 128-byte swizzled rows per step (descriptor start
// address + 2).  `accumulate` == 0 only for the first chunk of a tile.  One asm
// block keeps the per-instruction issue cost (descriptor arithmetic,
// predicates) off the single issuing thread's critical path.
__device__ __forceinline__ void tc_mma4_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                           uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "setp.eq.b32 q, 0, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%5], %6, %3, q;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%7], %8, %3, q;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%9], %10, %3, q;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(a_tmem + 8), "l"(b_desc + 2), "r"(a_tmem + 16),
      "l"(b_desc + 4), "r"(a_tmem + 24), "l"(b_desc + 6)
      : "memory");
}
// D[tmem] (+)= A[smem] * B[smem]^T, kind::f16.
__device__ __forceinline__ void tc_mma_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive on `bar` once every previously issued tcgen05.mma of this thread has completed.
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// Instruction descriptor for kind::f16: bf16 A/B, fp32 D, both K-major.
__host__ __device__ constexpr uint32_t make_idesc_bf16(uint32_t M, uint32_t N) {
  return (1u << 4)            // D format f32
         | (1u << 7)          // A format bf16
         | (1u << 10)         // B format bf16
         | ((N >> 3) << 17)   // N / 8
         | ((M >> 4) << 24);  // M / 16
}

// Instruction descriptor for kind::f16: f16 A/B, fp32 D, both K-major.
__host__ __device__ constexpr uint32_t make_idesc_f16(uint32_t M, uint32_t N) {
  return (1u << 4) | ((N >> 3) << 17) | ((M >> 4) << 24);
}

// Shared-memory matrix descriptor: K-major operand, 128-byte swizzle,
// rows of 128 bytes, 8-row groups 1024 bytes apart.
__device__ __forceinline__ uint64_t make_sdesc_sw128(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= (uint64_t)((smem_addr & 0x3FFFF) >> 4);  // start address
  d |= (uint64_t)(16 >> 4) << 16;                // leading byte offset (unused with swizzle)
  d |= (uint64_t)(1024 >> 4) << 32;              // stride byte offset: 8 rows * 128 B
  d |= (uint64_t)1 << 46;                        // descriptor version (sm_100)
  d |= (uint64_t)2 << 61;                        // SWIZZLE_128B
  return d;
}

// 32 lanes x 32 bit, 32 consecutive columns per thread.
__device__ __forceinline__ void tmem_st_x32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
      "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
      "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld_x32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
}
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// ------------------------------------------------- CTA pairs (clusters of 2) --
// Kernels built on these run as clusters of two CTAs on the two SMs of a TPC;
// rank 0 issues the pair's tensor-core work.  Every tcgen05 instruction that
// names a CTA group in such a kernel names cta_group::2.
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// The shared::cluster address of the same variable in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t smem_addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_addr), "r"(rank));
  return r;
}
// All threads of both CTAs; orders everything before it cluster-wide.
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}
// Arrive on an mbarrier of another CTA of the cluster (address from
// mapa_shared).  Default (CTA-scope release) semantics: what the barrier
// publishes between the CTAs of a pair is TMEM contents, ordered by
// tcgen05.wait::st / tcgen05.ld waits and tcgen05.fence::before_thread_sync on
// the arriving side and tcgen05.fence::after_thread_sync after the wait.  A
// cluster-scope release here costs ~1.6 k cycles per arrive (measured).
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
// 2-D tiled load into this CTA's shared memory whose completion (tx bytes) is
// signalled on a barrier of either CTA of the pair (`bar_cluster` from
// mapa_shared).  No multicast.
__device__ __forceinline__ void tma_load_2d_pair(void* smem_dst, const void* tmap, int32_t x, int32_t y,
                                                 uint32_t bar_cluster) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
      "[%4];" ::"r"(smem_u32(smem_dst)),
      "l"(tmap), "r"(x), "r"(y), "r"(bar_cluster)
      : "memory");
}
// TMEM allocation for a CTA pair: the same warp of both CTAs issues it and
// both get the same column range.
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* smem_dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_dst)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
// Pair MMA (M = 256: 128 A rows from each CTA's TMEM, B rows split in halves
// between the two CTAs' shared memory at the same offset, D rows in each
// CTA's TMEM).  Four K=16 steps of one 64-wide K chunk, as tc_mma4_ts.
__device__ __forceinline__ void tc_mma4_ts_pair(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                                uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "setp.eq.b32 q, 0, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], [%1], %2, %3, {%11, %11, %11, %11, %11, %11, %11, %11}, p;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], [%5], %6, %3, {%11, %11, %11, %11, %11, %11, %11, %11}, q;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], [%7], %8, %3, {%11, %11, %11, %11, %11, %11, %11, %11}, q;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], [%9], %10, %3, {%11, %11, %11, %11, %11, %11, %11, %11}, q;\n\t}" ::
          "r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(a_tmem + 8), "l"(b_desc + 2), "r"(a_tmem + 16),
      "l"(b_desc + 4), "r"(a_tmem + 24), "l"(b_desc + 6), "r"(0u)
      : "memory");
}
// Arrive once on the barrier at this offset in every CTA of `cta_mask` when
// the pair MMAs issued so far by this thread have completed.
__device__ __forceinline__ void tc_commit_pair(uint64_t* bar, uint16_t cta_mask) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          smem_u32(bar)),
      "h"(cta_mask)
      : "memory");
}

// ------------------------------------------------------------- misc PTX --
__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
}
__device__ __forceinline__ uint32_t lane_id() {
  uint32_t l;
  asm volatile("mov.u32 %0, %%laneid;" : "=r"(l));
  return l;
}
__device__ __forceinline__ bool elect_one() {
  uint32_t pred = 0;
  asm volatile(
      "{\n\t.reg .pred p;\n\t.reg .b32 r;\n\t"
      "elect.sync r|p, 0xffffffff;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(pred));
  return pred != 0;
}
__device__ __forceinline__ uint4 ldg_nc_v4(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

// ------------------------------------------------------------- MXFP4 -----
// E2M1 -> bf16 decode of 8 nibbles (one 32-bit word: nibble j = element j,
// low nibble of each byte first) scaled by 2^(scale-127).  Exact: every
// product of an E2M1 value and a power of two is representable in bf16.
//
// Magnitude codes 0..7 map to bf16 {0, 0.5, 1, 1.5, 2, 3, 4, 6}; their high
// bytes {00,3F,3F,3F,40,40,40,40} and low bytes {00,00,80,C0,00,40,80,C0}
// are looked up with byte permutes, the nibble sign bits are moved to bit
// 15/31, and the result is multiplied by the scale as packed bf16 (exact).
struct Fp4Tables {
  static constexpr uint32_t kHbLo = 0x3F3F3F00u, kHbHi = 0x40404040u;
  static constexpr uint32_t kLbLo = 0xC0800000u, kLbHi = 0xC0804000u;
};

__device__ __forceinline__ uint32_t bf16x2_mul(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

// out[0..3] = bf16x2 words for elements (0,1), (2,3), (4,5), (6,7).
__device__ __forceinline__ void fp4x8_to_bf16x8(uint32_t w, uint32_t scale2, uint32_t (&out)[4]) {
  const uint32_t m = w & 0x77777777u;
  const uint32_t m_hi = m >> 16;
  const uint32_t hb0 = prmt(Fp4Tables::kHbLo, Fp4Tables::kHbHi, m);
  const uint32_t lb0 = prmt(Fp4Tables::kLbLo, Fp4Tables::kLbHi, m);
  const uint32_t hb1 = prmt(Fp4Tables::kHbLo, Fp4Tables::kHbHi, m_hi);
  const uint32_t lb1 = prmt(Fp4Tables::kLbLo, Fp4Tables::kLbHi, m_hi);
  const uint32_t w4 = w << 4;  // even-element sign (bit 3 of each byte) -> bit 7
  uint32_t o0 = prmt(lb0, hb0, 0x5140u), o1 = prmt(lb0, hb0, 0x7362u);
  uint32_t o2 = prmt(lb1, hb1, 0x5140u), o3 = prmt(lb1, hb1, 0x7362u);
  // byte1 <- w4.byte k (sign of element 2k at bit 7), byte3 <- w.byte k (sign of element 2k+1)
  o0 |= prmt(w4, w, 0x4000u) & 0x80008000u;
  o1 |= prmt(w4, w, 0x5010u) & 0x80008000u;
  o2 |= prmt(w4, w, 0x6020u) & 0x80008000u;
  o3 |= prmt(w4, w, 0x7030u) & 0x80008000u;
  out[0] = bf16x2_mul(o0, scale2);
  out[1] = bf16x2_mul(o1, scale2);
  out[2] = bf16x2_mul(o2, scale2);
  out[3] = bf16x2_mul(o3, scale2);
}

// 2^(s-127) as a bf16 pair; exact for 1 <= s <= 254.
__device__ __forceinline__ uint32_t e8m0_scale_bf16x2(uint32_t s) {
  uint32_t h = (s & 0xFFu) << 7;
  return h | (h << 16);
}

// e2m1 -> f16 decode of 8 nibbles with the hardware converter, scaled by the
// E8M0 power of two as packed f16 (exact for scale codes 104..140: every
// product is an f16 normal or subnormal number).
__device__ __forceinline__ void fp4x8_to_f16x8(uint32_t w, uint32_t scale2, uint32_t& o0, uint32_t& o1, uint32_t& o2,
                                               uint32_t& o3) {
  asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\t"
      "mov.b32 {b0, b1, b2, b3}, %4;\n\t"
      "cvt.rn.f16x2.e2m1x2 %0, b0;\n\t"
      "cvt.rn.f16x2.e2m1x2 %1, b1;\n\t"
      "cvt.rn.f16x2.e2m1x2 %2, b2;\n\t"
      "cvt.rn.f16x2.e2m1x2 %3, b3;\n\t}"
      : "=r"(o0), "=r"(o1), "=r"(o2), "=r"(o3)
      : "r"(w));
  asm("mul.rn.f16x2 %0, %0, %1;" : "+r"(o0) : "r"(scale2));
  asm("mul.rn.f16x2 %0, %0, %1;" : "+r"(o1) : "r"(scale2));
  asm("mul.rn.f16x2 %0, %0, %1;" : "+r"(o2) : "r"(scale2));
  asm("mul.rn.f16x2 %0, %0, %1;" : "+r"(o3) : "r"(scale2));
}

// 2^(s-127) as an f16 pair (normal for s >= 113, subnormal for 103..112).
__device__ __forceinline__ uint32_t e8m0_scale_f16x2(uint32_t s) {
  const uint32_t h = s >= 113u ? ((s - 112u) << 10) : (1u << (s - 103u));
  return h | (h << 16);
}

// Clamped SwiGLU of one (glu, linear) pair (model/mlp.py:29-60):
// min(glu, limit) * sigmoid(alpha * min(glu, limit)) * (clamp(linear, -limit, limit) + 1).
__device__ __forceinline__ float swiglu_f32(float glu, float lin, float alpha, float limit) {
  const float g = fminf(glu, limit);
  const float l = fmaxf(fminf(lin, limit), -limit);
  // g * sigmoid(alpha * g); a huge denominator gives 0, the limit
  const float gs = __fdividef(g, 1.0f + __expf(-(alpha * g)));
  return gs * (l + 1.0f);
}

}  // namespace gptoss
