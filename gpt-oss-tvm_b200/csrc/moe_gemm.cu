// moe_gemm.cu -- grouped MXFP4 expert GEMMs on the 5th-generation tensor cores.
//
// Computes, for every expert e and every permuted row r of that expert
// (rows indptr[e] .. indptr[e+1] of the expert-major activation matrix),
//     h[r, n] = bias[e, n] + sum_k W_e[n, k] * act[r, k]
// with W_e decoded from the checkpoint's native MXFP4 layout
// (blocks [E, N, K/32, 16] e2m1 nibbles, scales [E, N, K/32] e8m0), i.e. the
// run_einsum of model/mlp.py:238-326 and the grouped kernels of
// model/mlp_optimized.py:214-460, and fuses the epilogue:
//   mode 0 (gate/up):  y[r, n/2] = bf16(swiglu(h[r, 2j], h[r, 2j+1]))
//                      (clamped SwiGLU, model/mlp.py:29-60)
//   mode 1 (down):     out[r, n] = h[r, n]   (fp32, combined later)
//
// Design (sm_100a, persistent: one CTA per SM, or one cluster of two CTAs
// per TPC for prefill-sized tiles):
//   * The weights are the MMA "A" operand and live in TMEM: dequant warps (one
//     TMEM lane = one weight row each) turn e2m1 nibbles into exact bf16 and
//     write them with tcgen05.st.  This keeps the shared-memory bandwidth for
//     the activation operand only.
//   * The activations (expert-major rows, bf16, K-major) are the "B" operand,
//     brought into 128-byte-swizzled shared memory by TMA.
//   * tcgen05.mma.kind::f16 (K = 16 per instruction) accumulates fp32 in
//     TMEM: cta_group::2 with M = 256 weight rows (128 per CTA of a pair) for
//     prefill-sized tiles of up to 128 token rows, cta_group::1 with M = 128
//     for decode-sized tiles of up to 32 token rows (and for prefill tiles
//     when GPTOSS_MOE_PAIR=0).
//   * Nibbles are streamed by TMA (128-byte swizzle, 4 K chunks per stage);
//     each tile's 128 x K/32 scale bytes arrive with one bulk copy.
// Warp roles: 0-15 dequant (four warpgroups), 16-19 epilogue (double-buffered
// TMEM accumulator, so the epilogue of tile i overlaps the main loop of tile
// i+1), 20 activation TMA, 21 MMA issuer (also owns TMEM), 22 weight TMA.
#include "common.cuh"
#include "launch.h"
#include "moe_tile.cuh"

namespace gptoss {

constexpr int kGemmThreads = 736;
constexpr int kBoxRows = 16;        // activation TMA box heights: 16 rows, and 64 rows for the
constexpr int kBigBoxRows = 64;     // bulk of large tiles (fewer, larger TMA requests)
constexpr int kBK = 64;             // K per pipeline chunk (one 128 B swizzle row of bf16)
constexpr int kWChunks = 4;                        // K chunks per nibble stage
constexpr int kWRowBytes = kWChunks * kBK / 2;     // 128 nibble bytes of a weight row per stage
constexpr int kWStageBytes = kBM * kWRowBytes;     // 16 KB (128 rows x 128 B, 128-byte swizzle)
constexpr int kMaxGroups = 96;                     // K/32 upper bound (K <= 3072)
constexpr int kScaleBytes = kBM * kMaxGroups;      // per-tile scale buffer (row stride = G)
constexpr int kTmemCols = 512;
constexpr int kDequantWarps = 16;  // 4 warpgroups
constexpr int kEpiWarp0 = 16;
constexpr int kActWarp = 20, kMmaWarp = 21, kWWarp = 22;

// Three shapes of one pipeline (kVar):
//   kVarSmall (decode, few rows per expert): up to 32 token rows; the MMA is
//     nearly free and the weights must stream at HBM speed: 6 nibble stages
//     and 6 activation stages of 4 chunks (96 KB + up to 96 KB in flight per
//     SM; an activation stream only a few chunks deep would queue behind the
//     weights in the SM's TMA unit and pace the MMA); 4 TMEM A slots of 2
//     chunks.
//   kVarPair (prefill): clusters of two CTAs on the two SMs of a TPC and
//     tcgen05.mma.cta_group::2 -- one MMA covers 256 weight rows (128 from
//     each CTA's TMEM) x up to 128 token rows, and each CTA stages only half
//     of the token rows (the MMA reads the other half from the peer's shared
//     memory), so per MMA cycle an SM takes in half the activation bytes of
//     the single-CTA form.  That L2 -> SM stream, not DRAM or the issue
//     slots, bounds the single-CTA form on prefill.  Rank 0's MMA thread
//     issues every MMA of the pair and its commits arrive on both CTAs'
//     barriers; rank 1's dequant and epilogue warps arrive on rank 0's
//     barriers and its activation loads complete on rank 0's.
//   kVarLarge: the single-CTA form of the same tiles (GPTOSS_MOE_PAIR=0, or
//     when no CTA pair fits).
// Prefill tiles hold up to 160 token rows: two 160-column accumulators and
// four one-chunk TMEM A slots fill TMEM.  Measured on B200 (8192-token
// layer): 160-row tiles with one-chunk A stages beat 128-row tiles with eight
// one-chunk or four two-chunk A slots (smaller N leaves the single MMA
// thread's per-chunk waits and commits, not the tensor pipe, as the pace),
// and prefetching the next tile into L2 slows the loads it competes with.
// Two-chunk activation stages for the pair (one stage-empty commit per two
// chunks) are 9 % faster than one-chunk stages; two-chunk TMEM A stages
// written by two warpgroups (half the full-barrier waits) were not.
// A nibble stage is one TMA box of 128 weight rows x 128 bytes (4 K chunks):
// wide rows keep the TMA request rate, not HBM, from bounding the stream.
enum GemmVariant { kVarSmall = 0, kVarLarge = 1, kVarPair = 2 };

template <int kVar>
struct GemmCfg {
  static constexpr bool kPair = kVar == kVarPair;
  static constexpr bool kSmall = kVar == kVarSmall;
  static constexpr int kMaxBN = kSmall ? kMoeTileRowsSmall : kMoeTileMaxRows;  // token rows per tile (MMA N)
  static constexpr int kRowsCta = kPair ? kMaxBN / 2 : kMaxBN;  // token rows staged per CTA
  static constexpr int kMmaM = kPair ? 2 * kBM : kBM;           // weight rows per MMA
  static constexpr int kNRound = kPair ? 32 : 16;               // MMA N granularity
  static constexpr int kBStages = kPair ? 5 : 6;
  static constexpr int kBChunks = kSmall ? 4 : (kPair ? 2 : 1);  // K chunks per activation stage
  static constexpr int kAChunks = kSmall ? 2 : 1;  // K chunks per TMEM A stage (one warpgroup's round)
  // TMEM A slots, a multiple of 4: slot s is written only by warpgroup s % 4
  static constexpr int kASlots = 4;
  static constexpr int kASlotCols = kAChunks * kBK / 2;  // TMEM columns of an A slot (f16/bf16 pairs)
  static constexpr int kAPerW = kWChunks / kAChunks;    // A stages per nibble stage = its reader warpgroups
  static constexpr int kWStages = kSmall ? 6 : (kPair ? 4 : 3);
  static_assert(kBChunks % kAChunks == 0 && kWChunks % kAChunks == 0, "A stages nest in both rings");
  static constexpr int kActChunkBytes = kRowsCta * kBK * 2;  // one chunk of this CTA's token rows
  static constexpr int kActStageBytes = kBChunks * kActChunkBytes;
  static constexpr int kAccCols = kMaxBN;
  static constexpr int kAColBase = 2 * kAccCols;
  static_assert(kAColBase + kASlots * kASlotCols <= kTmemCols, "TMEM budget");
  static_assert(kASlots % 4 == 0 && kDequantWarps == 16, "A slots divide among the four dequant warpgroups");
  static_assert(kMaxBN % kNRound == 0 && (kRowsCta % kBoxRows) == 0, "whole TMA boxes per CTA");
  // shared memory offsets from the 1024-aligned base
  static constexpr int kAct = 0;
  static constexpr int kW = kAct + kBStages * kActStageBytes;
  static constexpr int kScale = kW + kWStages * kWStageBytes;
  static constexpr int kBar = kScale + 2 * kScaleBytes;
  static constexpr int kNumBars = 2 * kASlots + 2 * kBStages + 2 * kWStages + 4 + 4 + 1;
  static constexpr int kMisc = kBar + kNumBars * 8;
  static constexpr int kEpi = (kMisc + 64 + 15) & ~15;  // 4 epilogue warps x (32 tokens x 32 features x 2 B)
  static constexpr int kAlloc = kEpi + 4 * 2048 + 1024;  // + slack for manual 1024 B alignment
  static_assert(kW % 1024 == 0 && kActChunkBytes % 1024 == 0, "128-byte swizzle atoms stay 1024-aligned");
  static_assert(kAlloc <= 227 * 1024, "shared memory budget");
};

__device__ __forceinline__ void tmem_st_x16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}

// 16 words (32 elements, one MXFP4 group) of decoded weights.
template <bool kF16>
__device__ __forceinline__ void decode_group(const uint4 nb, uint32_t sc, bool row_ok, uint32_t (&r)[16]) {
  if (!row_ok) {
#pragma unroll
    for (int j = 0; j < 16; ++j) r[j] = 0u;
    return;
  }
  if (kF16) {
    const uint32_t sc2 = e8m0_scale_f16x2(sc);
    fp4x8_to_f16x8(nb.x, sc2, r[0], r[1], r[2], r[3]);
    fp4x8_to_f16x8(nb.y, sc2, r[4], r[5], r[6], r[7]);
    fp4x8_to_f16x8(nb.z, sc2, r[8], r[9], r[10], r[11]);
    fp4x8_to_f16x8(nb.w, sc2, r[12], r[13], r[14], r[15]);
  } else {
    const uint32_t sc2 = e8m0_scale_bf16x2(sc);
    uint32_t o[4];
    fp4x8_to_bf16x8(nb.x, sc2, o); r[0] = o[0]; r[1] = o[1]; r[2] = o[2]; r[3] = o[3];
    fp4x8_to_bf16x8(nb.y, sc2, o); r[4] = o[0]; r[5] = o[1]; r[6] = o[2]; r[7] = o[3];
    fp4x8_to_bf16x8(nb.z, sc2, o); r[8] = o[0]; r[9] = o[1]; r[10] = o[2]; r[11] = o[3];
    fp4x8_to_bf16x8(nb.w, sc2, o); r[12] = o[0]; r[13] = o[1]; r[14] = o[2]; r[15] = o[3];
  }
}

// kF16: weights decoded to f16 by the hardware converter and activations in
// f16 (the fast path, valid when every scale code is in 104..140); otherwise
// exact bf16 decode and bf16 activations.  kVar: GemmVariant.
template <int kMode, bool kF16, int kVar>
__global__ void __launch_bounds__(kGemmThreads, 1)
    moe_gemm_tc_kernel(const __grid_constant__ CUtensorMap tmap_act, const __grid_constant__ CUtensorMap tmap_act64,
                       const __grid_constant__ CUtensorMap tmap_w, const GemmParams p) {
  using C = GemmCfg<kVar>;
  constexpr bool kPair = C::kPair;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint8_t* act_s = smem + C::kAct;
  uint8_t* w_s = smem + C::kW;
  uint8_t* sc_s = smem + C::kScale;
  uint64_t* bars = (uint64_t*)(smem + C::kBar);
  uint64_t* full_bar = bars;                        // [kASlots] A slot written (both CTAs) and its activations landed
  uint64_t* empty_bar = full_bar + C::kASlots;      // [kASlots] MMA commit
  uint64_t* bfull_bar = empty_bar + C::kASlots;     // [kBStages] activation TMA tx (both halves on rank 0)
  uint64_t* bempty_bar = bfull_bar + C::kBStages;   // [kBStages] MMA commit
  uint64_t* wfull_bar = bempty_bar + C::kBStages;   // [kWStages] nibble TMA tx
  uint64_t* wempty_bar = wfull_bar + C::kWStages;   // [kWStages] the dequant warps that read it
  uint64_t* scfull_bar = wempty_bar + C::kWStages;  // [2] scale bulk copy tx
  uint64_t* scempty_bar = scfull_bar + 2;           // [2] all 16 dequant warps
  uint64_t* accfull_bar = scempty_bar + 2;          // [2] MMA commit
  uint64_t* accempty_bar = accfull_bar + 2;         // [2] the epilogue warps (both CTAs)
  uint64_t* drain_bar = accempty_bar + 2;           // [1] every MMA complete
  uint32_t* misc = (uint32_t*)(smem + C::kMisc);
  volatile uint32_t* tmem_slot = misc;
  volatile uint32_t* abort_s = misc + 1;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  // a pair of CTAs (cluster of two, rank 0 issues the MMAs) or one CTA works a tile
  const uint32_t rank = kPair ? cluster_ctarank() : 0u;
  const int32_t unit = kPair ? (int32_t)(blockIdx.x >> 1) : (int32_t)blockIdx.x;
  const int32_t nunits = kPair ? (int32_t)(gridDim.x >> 1) : (int32_t)gridDim.x;
  const int32_t fstride = kPair ? 2 * kBM : kBM;  // weight rows per tile
  const int32_t fofs = (int32_t)rank * kBM;       // this CTA's first weight row in the tile
  const int32_t G = p.K >> 5;
  const int32_t nchunks = p.K / kBK;
  const int32_t nstages = (nchunks + kWChunks - 1) / kWChunks;  // nibble stages per tile
  const int32_t nastages = (nchunks + C::kAChunks - 1) / C::kAChunks;  // TMEM A stages per tile
  const int32_t nbstages = (nchunks + C::kBChunks - 1) / C::kBChunks;  // activation stages per tile
  const int32_t ftiles = (p.N + fstride - 1) / fstride;
  const int32_t total_tiles = __ldg(p.tile_ptr + p.num_experts) * ftiles;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::kASlots; ++s) {
      mbar_init(&full_bar[s], kPair ? 8 : 4);
      mbar_init(&empty_bar[s], 1);
    }
    for (int s = 0; s < C::kBStages; ++s) {
      mbar_init(&bfull_bar[s], 1);
      mbar_init(&bempty_bar[s], 1);
    }
    for (int s = 0; s < C::kWStages; ++s) {
      mbar_init(&wfull_bar[s], 1);
      mbar_init(&wempty_bar[s], 4 * C::kAPerW);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&scfull_bar[s], 1);
      mbar_init(&scempty_bar[s], kDequantWarps);
      mbar_init(&accfull_bar[s], 1);
      mbar_init(&accempty_bar[s], kPair ? 8 : 4);
    }
    mbar_init(drain_bar, 1);
    *abort_s = 0;
    fence_mbar_init();
  }
  if (warp == kMmaWarp) {
    if (kPair) {
      tmem_alloc_pair((uint32_t*)tmem_slot, kTmemCols);
      tmem_relinquish_pair();
    } else {
      tmem_alloc((uint32_t*)tmem_slot, kTmemCols);
      tmem_relinquish();
    }
  }
  if (warp == kActWarp && lane == 0) {
    tma_prefetch_desc(&tmap_act);
    tma_prefetch_desc(&tmap_act64);
    tma_prefetch_desc(&tmap_w);
  }
  // barrier initialisation and the TMEM address visible to every role (and,
  // for a pair, to the other CTA)
  tc_fence_before();
  if (kPair) cluster_sync_all();
  else __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == kActWarp) {
    // ------------------------------------------------ activation producer
    if (elect_one()) {
      const uint32_t bfull0 = kPair ? mapa_shared(smem_u32(bfull_bar), 0) : 0u;
      uint32_t bit = 0;
      for (int32_t t = unit; t < total_tiles && !*abort_s; t += nunits) {
        TileInfo ti;
        if (!decode_tile<C::kMaxBN>(p, t, ftiles, ti, fstride, fofs)) continue;
        // this CTA's token rows: all of the tile, or for a pair its half of
        // the MMA's N (rows rounded up to 32)
        int32_t r0 = ti.row0, rows = ti.nrows;
        if (kPair) {
          rows = ((ti.nrows + 31) & ~31) >> 1;
          r0 += (int32_t)rank * rows;
        }
        const int32_t nbig = C::kSmall ? 0 : rows / kBigBoxRows;
        const int32_t nbox = (rows - nbig * kBigBoxRows + kBoxRows - 1) / kBoxRows;
        const int32_t brows = nbig * kBigBoxRows + nbox * kBoxRows;  // rows landed per chunk

        for (int32_t c0 = 0; c0 < nchunks; c0 += C::kBChunks, ++bit) {
          const uint32_t s = bit % C::kBStages, ph = (bit / C::kBStages) & 1;
          const int32_t nq = min(C::kBChunks, nchunks - c0);
          if (!mbar_wait(&bempty_bar[s], ph ^ 1, p.err, kErrTimeoutEmpty)) { *abort_s = 1; break; }
          // rank 0's barrier counts both halves
          if (rank == 0) mbar_arrive_expect_tx(&bfull_bar[s], (uint32_t)(nq * brows * 128 * (kPair ? 2 : 1)));
          for (int32_t q = 0; q < nq; ++q) {
            uint8_t* dst = act_s + s * C::kActStageBytes + q * C::kActChunkBytes;
            const int32_t x = (c0 + q) * kBK;
            for (int32_t b = 0; b < nbig; ++b) {
              if (kPair)
                tma_load_2d_pair(dst + b * kBigBoxRows * 128, &tmap_act64, x, r0 + b * kBigBoxRows, bfull0 + s * 8);
              else
                tma_load_2d(dst + b * kBigBoxRows * 128, &tmap_act64, x, r0 + b * kBigBoxRows, &bfull_bar[s]);
            }
            for (int32_t b = 0; b < nbox; ++b) {
              uint8_t* d = dst + (nbig * kBigBoxRows + b * kBoxRows) * 128;
              const int32_t y = r0 + nbig * kBigBoxRows + b * kBoxRows;
              if (kPair) tma_load_2d_pair(d, &tmap_act, x, y, bfull0 + s * 8);
              else tma_load_2d(d, &tmap_act, x, y, &bfull_bar[s]);
            }
          }
        }
      }
    }
  } else if (warp == kWWarp) {
    // ------------------------------------- weight producer (this CTA's rows)
    if (elect_one()) {
      uint32_t wit = 0, tl = 0;
      for (int32_t t = unit; t < total_tiles && !*abort_s; t += nunits) {
        TileInfo ti;
        if (!decode_tile<C::kMaxBN>(p, t, ftiles, ti, fstride, fofs)) continue;
        const uint32_t sb = tl & 1, sph = (tl >> 1) & 1;
        ++tl;
        if (!mbar_wait(&scempty_bar[sb], sph ^ 1, p.err, kErrTimeoutEmpty)) { *abort_s = 1; break; }
        // rows past N (a pair's last tile when N is not a multiple of 256)
        // load nothing; their TMEM rows decode to zeros
        const int32_t frows = min(kBM, p.N - ti.f0);
        if (frows > 0) {
          const uint32_t sbytes = (uint32_t)(frows * G);
          mbar_arrive_expect_tx(&scfull_bar[sb], sbytes);
          const uint8_t* src = p.scales + ((size_t)ti.expert * p.N + ti.f0) * G;
          asm volatile(
              "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                  smem_u32(sc_s + sb * kScaleBytes)),
              "l"(src), "r"(sbytes), "r"(smem_u32(&scfull_bar[sb]))
              : "memory");
        } else {
          mbar_arrive(&scfull_bar[sb]);
        }
        const int32_t wrow = ti.expert * p.N + ti.f0;
        bool ok = true;
        for (int32_t j = 0; j < nstages; ++j, ++wit) {
          const uint32_t s = wit % C::kWStages, ph = (wit / C::kWStages) & 1;
          if (!mbar_wait(&wempty_bar[s], ph ^ 1, p.err, kErrTimeoutEmpty)) { ok = false; break; }
          if (frows > 0) {
            mbar_arrive_expect_tx(&wfull_bar[s], kWStageBytes);  // the zero-filled tail counts too
            tma_load_2d(w_s + s * kWStageBytes, &tmap_w, j * kWRowBytes, wrow, &wfull_bar[s]);
          } else {
            mbar_arrive(&wfull_bar[s]);
          }
        }
        if (!ok) { *abort_s = 1; break; }
      }
    }
  } else if (warp == kMmaWarp) {
    // ------------------------------------------ MMA issuer (a pair: rank 0)
    if (rank == 0 && elect_one()) {
      // slot / activation-stage cursors run on across tiles, in step with the
      // dequant warpgroups (A stages) and the activation producer (stages)
      uint32_t s = 0, ph = 0, sb = 0, tl = 0;
      bool ok = true;
      const uint64_t bdesc0 = make_sdesc_sw128(smem_u32(act_s));
      for (int32_t t = unit; t < total_tiles && !*abort_s; t += nunits) {
        TileInfo ti;
        if (!decode_tile<C::kMaxBN>(p, t, ftiles, ti, fstride, fofs)) continue;
        const uint32_t n_mma = (uint32_t)((ti.nrows + C::kNRound - 1) & ~(C::kNRound - 1));
        const uint32_t idesc = kF16 ? make_idesc_f16(C::kMmaM, n_mma) : make_idesc_bf16(C::kMmaM, n_mma);
        const uint32_t ab = tl & 1, aph = (tl >> 1) & 1;
        if (!mbar_wait(&accempty_bar[ab], aph ^ 1, p.err, kErrTimeoutAccum)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + ab * C::kAccCols;
        int32_t sub = 0, q = 0;
        for (int32_t c = 0; c < nchunks; ++c) {
          if (sub == 0) {
            // the owning warpgroup(s) arrive once the weights are in TMEM and
            // the activation stage holding this A stage has landed
            if (!mbar_wait(&full_bar[s], ph, p.err, kErrTimeoutFull)) { ok = false; break; }
            tc_fence_after();
          }
          // start-address field of the descriptor: (byte offset >> 4), no carry out of its 14 bits
          const uint64_t bdesc = bdesc0 + (uint64_t)((uint32_t)(sb * C::kActStageBytes + q * C::kActChunkBytes) >> 4);
          const uint32_t a_tmem = tmem_base + C::kAColBase + s * C::kASlotCols + sub * 32;
          if (kPair) tc_mma4_ts_pair(d_tmem, a_tmem, bdesc, idesc, c > 0 ? 1u : 0u);
          else tc_mma4_ts(d_tmem, a_tmem, bdesc, idesc, c > 0 ? 1u : 0u);
          const bool last = c == nchunks - 1;
          if (++sub == C::kAChunks || last) {
            if (kPair) tc_commit_pair(&empty_bar[s], 3);
            else tc_commit(&empty_bar[s]);
            sub = 0;
            if (++s == (uint32_t)C::kASlots) { s = 0; ph ^= 1u; }
          }
          if (++q == C::kBChunks || last) {
            if (kPair) tc_commit_pair(&bempty_bar[sb], 3);
            else tc_commit(&bempty_bar[sb]);
            q = 0;
            if (++sb == C::kBStages) sb = 0;
          }
        }
        if (!ok) break;
        if (kPair) tc_commit_pair(&accfull_bar[ab], 3);
        else tc_commit(&accfull_bar[ab]);
        ++tl;
      }
      if (!ok) *abort_s = 1;
      // every MMA has completed before teardown frees TMEM (and, for a pair,
      // before either CTA exits)
      if (kPair) tc_commit_pair(drain_bar, 1);
      else tc_commit(drain_bar);
      mbar_wait(drain_bar, 0, p.err, kErrTimeoutOther);
    }
  } else if (warp < kDequantWarps) {
    // ------------------------------- dequant: this CTA's weight rows -> TMEM
    // The A stages of all tiles are numbered consecutively (gai); stage gai
    // (kAChunks chunks, both MXFP4 groups of each) is decoded by warpgroup
    // gai % 4 into TMEM slot gai % kASlots, so each slot has a single writer
    // and its empty/full phases advance in that warpgroup's program order.  A nibble
    // stage holds kAPerW A stages and is read (and released) by their
    // kAPerW warpgroups: all four for one-chunk A stages, else two, the
    // two pairs alternating stages so that one pair's barrier waits overlap
    // the other pair's decode.  In a pair both CTAs' warpgroups arrive on
    // rank 0's full barrier; rank 0's first wait for the stage's activations.
    const int wgi = warp >> 2;
    const int row = (warp & 3) * 32 + lane;     // weight row within the tile == TMEM lane
    const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
    const uint32_t swz = (uint32_t)(row & 7);   // 128-byte swizzle of the nibble rows
    const uint32_t full0 = kPair ? mapa_shared(smem_u32(full_bar), 0) : 0u;
    uint32_t ait = 0, wit = 0, bit = 0, tl = 0;
    for (int32_t t = unit; t < total_tiles; t += nunits) {
      TileInfo ti;
      if (!decode_tile<C::kMaxBN>(p, t, ftiles, ti, fstride, fofs)) continue;
      if (*abort_s) break;
      const uint32_t sb = tl & 1, sph = (tl >> 1) & 1;
      ++tl;
      const bool row_ok = ti.f0 + row < p.N;
      bool ok = mbar_wait(&scfull_bar[sb], sph, p.err, kErrTimeoutFull);
      const uint8_t* srow = sc_s + sb * kScaleBytes + row * G;
      for (int32_t j = 0; j < nstages && ok; ++j) {
        // this warpgroup's A stage in nibble stage j, if it reads the stage
        const int r = (wgi - (int)((ait + (uint32_t)(j * C::kAPerW)) & 3u)) & 3;
        if (r >= C::kAPerW) continue;
        const uint32_t wsi = wit + (uint32_t)j;
        const uint32_t ws = wsi % C::kWStages, wph = (wsi / C::kWStages) & 1;
        ok = mbar_wait(&wfull_bar[ws], wph, p.err, kErrTimeoutFull);
        if (!ok) break;
        // pieces 2q + g of the stage row, q = r * kAChunks + u (chunk), g = group
        const uint8_t* wrow = w_s + ws * kWStageBytes + row * kWRowBytes;
        uint4 nb[2 * C::kAChunks];
#pragma unroll
        for (int k = 0; k < 2 * C::kAChunks; ++k)
          nb[k] = *(const uint4*)(wrow + (((uint32_t)(2 * C::kAChunks * r + k) ^ swz) << 4));
        __syncwarp();
        if (lane == 0) mbar_arrive(&wempty_bar[ws]);
        const int32_t c0 = (j * C::kAPerW + r) * C::kAChunks;
        if (c0 >= nchunks) continue;            // no chunk here (short last stage)
        // decode the first chunk while the MMA may still be reading the slot
        uint32_t v0[16], v1[16];
        decode_group<kF16>(nb[0], srow[2 * c0], row_ok, v0);
        decode_group<kF16>(nb[1], srow[2 * c0 + 1], row_ok, v1);
        // wait until the MMA has consumed the slot's previous A stage
        const uint32_t gai = ait + (uint32_t)(j * C::kAPerW + r);
        const uint32_t slot = gai % C::kASlots, sph2 = (gai / C::kASlots) & 1u;
        ok = mbar_wait(&empty_bar[slot], sph2 ^ 1u, p.err, kErrTimeoutEmpty);
        if (!ok) break;
        const uint32_t ta = tmem_base + lane_base + C::kAColBase + slot * C::kASlotCols;
        __syncwarp();
        tc_fence_after();
        tmem_st_x16(ta, v0);
        tmem_st_x16(ta + 16, v1);
#pragma unroll
        for (int u = 1; u < C::kAChunks; ++u) {
          const int32_t c = c0 + u;
          if (c >= nchunks) break;
          decode_group<kF16>(nb[2 * u], srow[2 * c], row_ok, v0);
          decode_group<kF16>(nb[2 * u + 1], srow[2 * c + 1], row_ok, v1);
          tmem_st_x16(ta + u * 32, v0);
          tmem_st_x16(ta + u * 32 + 16, v1);
        }
        tmem_st_wait();
        tc_fence_before();
        if (rank == 0) {
          // the activation stage that holds chunks c0 .. c0 + kAChunks - 1
          // (for a pair: both CTAs' halves, counted on this barrier)
          const uint32_t bsi = bit + (uint32_t)(c0 / C::kBChunks);
          ok = mbar_wait(&bfull_bar[bsi % C::kBStages], (bsi / C::kBStages) & 1u, p.err, kErrTimeoutFull);
          if (!ok) break;
        }
        __syncwarp();
        if (lane == 0) {
          if (rank == 0) mbar_arrive(&full_bar[slot]);
          else mbar_arrive_cluster(full0 + slot * 8);
        }
      }
      ait += (uint32_t)nastages;
      wit += (uint32_t)nstages;
      bit += (uint32_t)nbstages;
      __syncwarp();
      if (lane == 0) mbar_arrive(&scempty_bar[sb]);
      if (!ok) { *abort_s = 1; break; }
    }
  } else {
    // ------------------------ epilogue: this CTA's rows, TMEM -> registers -> global
    const int q = warp - kEpiWarp0;               // TMEM lane quarter
    const int row = q * 32 + lane;
    const uint32_t lane_base = (uint32_t)(q * 32) << 16;
    const uint32_t accempty0 = kPair ? mapa_shared(smem_u32(accempty_bar), 0) : 0u;
    uint32_t tl = 0;
    for (int32_t t = unit; t < total_tiles; t += nunits) {
      TileInfo ti;
      if (!decode_tile<C::kMaxBN>(p, t, ftiles, ti, fstride, fofs)) continue;
      if (*abort_s) break;
      const uint32_t ab = tl & 1, aph = (tl >> 1) & 1;
      ++tl;
      const int32_t frow = ti.f0 + row;
      const bool row_ok = frow < p.N;
      const float bias = row_ok ? bf16_bits_to_f32(__ldg(p.bias + (size_t)ti.expert * p.N + frow)) : 0.0f;
      if (!mbar_wait(&accfull_bar[ab], aph, p.err, kErrTimeoutAccum)) { *abort_s = 1; break; }
      __syncwarp();
      tc_fence_after();
      const int32_t ncols = ti.f0 < p.N ? (ti.nrows + 31) & ~31 : 0;
      for (int32_t c0 = 0; c0 < ncols; c0 += 32) {
        uint32_t v[32];
        tmem_ld_x32(tmem_base + lane_base + ab * C::kAccCols + (uint32_t)c0, v);
        tmem_ld_wait();
        epilogue_block<kMode, kF16>(p, ti, v, c0, q, lane, bias, row_ok, frow,
                                    (uint16_t*)(smem + C::kEpi) + q * 1024);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (rank == 0) mbar_arrive(&accempty_bar[ab]);
        else mbar_arrive_cluster(accempty0 + ab * 8);
      }
    }
    // rows stored into other GPUs' memory are visible there before the
    // collective that follows the kernel
    if (kMode == 1 && p.row_dst != nullptr) __threadfence_system();
  }

  // ---- teardown: every role drains (the MMAs have completed), then the
  // allocating warp(s) free TMEM
  __syncwarp();
  tc_fence_before();
  if (kPair) cluster_sync_all();
  else __syncthreads();
  if (warp == kMmaWarp) {
    __syncwarp();
    tc_fence_after();
    if (kPair) tmem_dealloc_pair(tmem_base, kTmemCols);
    else tmem_dealloc(tmem_base, kTmemCols);
  }
}

// ------------------------------------------------------------------ host --
typedef CUresult (*PFN_encodeTiled)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                    const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                    CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static PFN_encodeTiled get_encode_fn() {
  static PFN_encodeTiled fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void* ptr = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = (PFN_encodeTiled)ptr;
  }
  return fn;
}

// 3-D tensor map: dims innermost first, byte strides of dims 1 and 2.
int make_tmap_3d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype, const uint64_t dims[3],
                 const uint64_t strides[2], const uint32_t box[3], CUtensorMapSwizzle swz) {
  PFN_encodeTiled enc = get_encode_fn();
  if (!enc) return -1;
  cuuint64_t d[3] = {dims[0], dims[1], dims[2]};
  cuuint64_t st[2] = {strides[0], strides[1]};
  cuuint32_t bx[3] = {box[0], box[1], box[2]};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(map, dtype, 3, const_cast<void*>(base), d, st, bx, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : -2;
}

// 2-D tensor map over a row-major matrix [rows, cols] of `esize`-byte elements.
int make_tmap_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype, int esize, uint64_t rows,
                 uint64_t cols, uint32_t box_cols, uint32_t box_rows, CUtensorMapSwizzle swz) {
  PFN_encodeTiled enc = get_encode_fn();
  if (!enc) return -1;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {cols * (uint64_t)esize};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, dtype, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : -2;
}



template <int kMode, bool kF16, int kVar>
static void launch_variant(const CUtensorMap& ta, const CUtensorMap& ta64, const CUtensorMap& tw, const GemmParams& p,
                           int grid, cudaStream_t stream) {
  const int smem = GemmCfg<kVar>::kAlloc;
  static FuncSmemAttr attr;
  ensure_dyn_smem(attr, (const void*)moe_gemm_tc_kernel<kMode, kF16, kVar>, (int)smem);
  moe_gemm_tc_kernel<kMode, kF16, kVar><<<grid, kGemmThreads, smem, stream>>>(ta, ta64, tw, p);
}

// Clusters of two CTAs, at most as many as fit at once (one CTA per SM);
// returns false when no cluster fits, so the caller can use the single-CTA form.
template <int kMode, bool kF16>
static bool launch_pair(const CUtensorMap& ta, const CUtensorMap& ta64, const CUtensorMap& tw, const GemmParams& p,
                        int grid, cudaStream_t stream) {
  auto kern = moe_gemm_tc_kernel<kMode, kF16, kVarPair>;
  const int smem = GemmCfg<kVarPair>::kAlloc;
  static FuncSmemAttr smem_attr;
  static std::atomic<int> fit[kMaxAttrDevices] = {};  // clusters that fit at once + 1 per device; 0 = unknown
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxAttrDevices) {
    (void)cudaGetLastError();
    return false;
  }
  ensure_dyn_smem(smem_attr, (const void*)kern, smem);
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.blockDim = dim3(kGemmThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int max_pairs = fit[dev].load(std::memory_order_acquire) - 1;
  if (max_pairs < 0) {
    cfg.gridDim = dim3((unsigned)(grid & ~1));
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess) {
      (void)cudaGetLastError();
      n = 0;
    }
    max_pairs = n;
    fit[dev].store(n + 1, std::memory_order_release);
  }
  const int pairs = grid / 2 < max_pairs ? grid / 2 : max_pairs;
  if (pairs <= 0) return false;
  cfg.gridDim = dim3((unsigned)(2 * pairs));
  return cudaLaunchKernelEx(&cfg, kern, ta, ta64, tw, p) == cudaSuccess;
}

// Prefill-sized tiles run on CTA pairs unless GPTOSS_MOE_PAIR=0 (the
// single-CTA form, kept for comparison and as the fallback).
static bool pair_enabled() {
  const char* e = getenv("GPTOSS_MOE_PAIR");
  return !(e && e[0] == '0');
}

// GPTOSS_MOE_GEMV=0 keeps decode-size GEMMs on the tensor-core kernel.
static bool gemv_enabled() {
  const char* e = getenv("GPTOSS_MOE_GEMV");
  return !(e && e[0] == '0');
}

bool moe_gemm_gathers(const GemmLaunch& L) {
  return moe_tile_rows_max(L.act_rows, L.E) <= kMoeTileRowsSmall && gemv_enabled() && moe_gemv_supported(L);
}

int launch_moe_gemm(int mode, const GemmLaunch& L, cudaStream_t stream) {
  // decode sizes (the same rule as the token-tile plan's small tiles): the
  // weights are streamed once through the MXFP4 GEMV kernel
  if (moe_gemm_gathers(L)) return launch_moe_gemv(mode, L, stream);
  if (L.act_gather) return -10;  // only the GEMV gathers
  if (L.K % kBK != 0 || L.K / 32 > kMaxGroups || L.K / 2 < kWRowBytes) return -10;
  {
    // every tile's scale block must be a whole number of 16-byte units
    const int32_t G = L.K / 32;
    const int32_t last = L.N % kBM ? L.N % kBM : kBM;
    if (((int64_t)kBM * G) % 16 || ((int64_t)last * G) % 16 || ((int64_t)L.N * G) % 16) return -11;
  }
  CUtensorMap tmap_act, tmap_act64, tmap_w;
  const CUtensorMapDataType adt = L.f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  int rc = make_tmap_2d(&tmap_act, L.act, adt, 2, (uint64_t)L.act_rows, (uint64_t)L.K, kBK, kBoxRows,
                        CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  // (with fewer rows than one big box no tile uses it; keep the encoding valid)
  rc = make_tmap_2d(&tmap_act64, L.act, adt, 2, (uint64_t)L.act_rows, (uint64_t)L.K, kBK,
                    L.act_rows < kBigBoxRows ? kBoxRows : kBigBoxRows, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  rc = make_tmap_2d(&tmap_w, L.blocks, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, (uint64_t)L.E * L.N, (uint64_t)L.K / 2,
                    kWRowBytes, kBM, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  GemmParams p;
  p.scales = L.scales;
  p.bias = L.bias;
  p.indptr = L.indptr;
  p.tile_ptr = L.tile_ptr;
  p.tile_rows = L.tile_rows;
  p.out = L.out;
  p.num_experts = L.E;
  p.N = L.N;
  p.K = L.K;
  p.ldo = L.ldo;
  p.alpha = L.alpha;
  p.limit = L.limit;
  p.err = L.err;
  p.row_dst = mode == 1 ? L.row_dst : nullptr;
  for (int i = 0; i < kMaxPeerRanks; ++i) p.peer_out[i] = L.peer_out[i];
  p.peer_out_rows = L.peer_out_rows;
  p.out_bf16 = L.out_bf16;
  // the token-tile plan used the same rule (moe_tile_rows_max) for these rows
  const bool small = moe_tile_rows_max(L.act_rows, L.E) <= kMoeTileRowsSmall;
  if (!small && pair_enabled()) {
    bool launched;
    if (mode == 0)
      launched = L.f16 ? launch_pair<0, true>(tmap_act, tmap_act64, tmap_w, p, L.grid, stream)
                       : launch_pair<0, false>(tmap_act, tmap_act64, tmap_w, p, L.grid, stream);
    else
      launched = L.f16 ? launch_pair<1, true>(tmap_act, tmap_act64, tmap_w, p, L.grid, stream)
                       : launch_pair<1, false>(tmap_act, tmap_act64, tmap_w, p, L.grid, stream);
    if (launched) return 0;
    (void)cudaGetLastError();
  }
  if (mode == 0) {
    if (small) {
      if (L.f16) launch_variant<0, true, kVarSmall>(tmap_act, tmap_act64, tmap_w, p, L.grid, stream);
      else launch_variant<0, false, kVarSmall>(tmap_act, tmap_act64, tmap_w, p, L.grid, stream);
    } else {
      if (L.f16) launch_variant<0, true, kVarLarge>(tmap_act, tmap_act64, tmap_w, p, L.grid, stream);
      else launch_variant<0, false, kVarLarge>(tmap_act, tmap_act64, tmap_w, p, L.grid, stream);
    }
  } else {
    if (small) {
      if (L.f16) launch_variant<1, true, kVarSmall>(tmap_act, tmap_act64, tmap_w, p, L.grid, stream);
      else launch_variant<1, false, kVarSmall>(tmap_act, tmap_act64, tmap_w, p, L.grid, stream);
    } else {
      if (L.f16) launch_variant<1, true, kVarLarge>(tmap_act, tmap_act64, tmap_w, p, L.grid, stream);
      else launch_variant<1, false, kVarLarge>(tmap_act, tmap_act64, tmap_w, p, L.grid, stream);
    }
  }
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

}  // namespace gptoss
