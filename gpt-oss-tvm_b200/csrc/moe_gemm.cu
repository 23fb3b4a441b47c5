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
// Design (sm_100a, one persistent CTA per SM):
//   * The weights are the MMA "A" operand and live in TMEM: dequant warps (one
//     TMEM lane = one weight row each) turn e2m1 nibbles into exact bf16 and
//     write them with tcgen05.st.  This keeps the shared-memory bandwidth for
//     the activation operand only.
//   * The activations (expert-major rows, bf16, K-major) are the "B" operand,
//     brought into 128-byte-swizzled shared memory by TMA.
//   * tcgen05.mma.cta_group::1.kind::f16 (M = 128 weight rows, N = up to 192
//     token rows, K = 16 per instruction) accumulates fp32 in TMEM.
//   * Nibbles are streamed by TMA (32-byte swizzle) through an 8-deep ring;
//     each tile's 128 x K/32 scale bytes arrive with one bulk copy.
// Warp roles: 0-15 dequant (four warpgroups: even / odd K chunks x the two
// 32-element MXFP4 groups of a 64-wide chunk), 16-19 epilogue (double-buffered
// TMEM accumulator, so the epilogue of tile i overlaps the main loop of tile
// i+1), 20 activation TMA, 21 MMA issuer (also owns TMEM), 22 weight TMA.
#include "common.cuh"
#include "launch.h"

namespace gptoss {

constexpr int kGemmThreads = 736;
constexpr int kBM = 128;            // weight rows per tile (MMA M)
constexpr int kMaxBN = kMoeTileMaxRows;  // token rows per tile (MMA N, max)
constexpr int kBoxRows = 16;        // activation TMA box height (up to 13 boxes per stage)
constexpr int kBK = 64;             // K per pipeline chunk (one 128 B swizzle row of bf16)
constexpr int kStages = 4;          // TMEM A stages (dequantised weights)
constexpr int kBStages = 6;         // shared-memory activation stages
constexpr int kWStages = 8;         // nibble ring depth
constexpr int kActStageBytes = kMaxBN * kBK * 2;   // 24 KB (192 rows of 128 B)
constexpr int kWStageBytes = kBM * (kBK / 2);      // 4 KB (128 rows x 32 nibble bytes)
constexpr int kMaxGroups = 96;                     // K/32 upper bound (K <= 3072)
constexpr int kScaleBytes = kBM * kMaxGroups;      // per-tile scale buffer (row stride = G)
constexpr int kAccCols = kMaxBN;                   // columns of one accumulator buffer
constexpr int kTmemCols = 512;
constexpr int kAColBase = 2 * kAccCols;            // A stage s at columns 384 + 32 s
static_assert(kAColBase + kStages * 32 <= kTmemCols, "TMEM budget");
constexpr int kDequantWarps = 16;  // 4 warpgroups: (chunk parity, MXFP4 group of the chunk)
constexpr int kDequantPerChunk = 8; // warps that fill one chunk's A stage
constexpr int kEpiWarp0 = 16;
constexpr int kActWarp = 20, kMmaWarp = 21, kWWarp = 22;

struct GemmParams {
  const uint8_t* scales;     // [E, N, G]
  const uint16_t* bias;      // [E, N] bf16
  const int32_t* indptr;     // [E + 1]  permuted rows of each expert
  const int32_t* tile_ptr;   // [E + 1]  prefix sum of token tiles per expert
  const int32_t* tile_rows;  // [E]      rows per token tile of each expert
  void* out;                 // mode 0: bf16 [R, N/2]; mode 1: f32 [R, N]
  int32_t num_experts;
  int32_t N;                 // weight rows per expert (output features)
  int32_t K;                 // reduction length (multiple of 64)
  int32_t ldo;               // output row stride in elements
  float alpha, limit;        // SwiGLU constants (mode 0)
  uint32_t* err;
};

struct GemmSmem {
  // offsets from the 1024-aligned base
  static constexpr int kAct = 0;
  static constexpr int kW = kAct + kBStages * kActStageBytes;
  static constexpr int kScale = kW + kWStages * kWStageBytes;
  static constexpr int kBar = kScale + 2 * kScaleBytes;
  static constexpr int kNumBars = 2 * kStages + 2 * kBStages + 2 * kWStages + 4 + 4;
  static constexpr int kMisc = kBar + kNumBars * 8;
  static constexpr int kTotal = kMisc + 64;
  static constexpr int kAlloc = kTotal + 1024;  // slack for manual 1024 B alignment
};

struct TileInfo {
  int32_t expert, row0, nrows, f0;
};

// Tile t -> (expert, first permuted row, rows, first feature row).
__device__ __forceinline__ bool decode_tile(const GemmParams& p, int32_t t, int32_t ftiles, TileInfo& ti) {
  const int32_t g = t / ftiles;
  const int32_t f = t - g * ftiles;
  int32_t lo = 0, hi = p.num_experts;  // find e with tile_ptr[e] <= g < tile_ptr[e+1]
  while (hi - lo > 1) {
    int32_t mid = (lo + hi) >> 1;
    if (__ldg(p.tile_ptr + mid) <= g) lo = mid; else hi = mid;
  }
  const int32_t e = lo;
  const int32_t tt = g - __ldg(p.tile_ptr + e);
  const int32_t per = __ldg(p.tile_rows + e);
  const int32_t base = __ldg(p.indptr + e);
  const int32_t cnt = __ldg(p.indptr + e + 1) - base;
  ti.expert = e;
  ti.row0 = base + tt * per;
  ti.nrows = min(per, cnt - tt * per);
  ti.f0 = f * kBM;
  return ti.nrows > 0;
}

__device__ __forceinline__ void tmem_st_x16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
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

// kF16: weights decoded to f16 by the hardware converter and activations in
// f16 (the fast path, valid when every scale code is in 104..140); otherwise
// exact bf16 decode and bf16 activations.
template <int kMode, bool kF16>
__global__ void __launch_bounds__(kGemmThreads, 1)
    moe_gemm_tc_kernel(const __grid_constant__ CUtensorMap tmap_act, const __grid_constant__ CUtensorMap tmap_w,
                       const GemmParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint8_t* act_s = smem + GemmSmem::kAct;
  uint8_t* w_s = smem + GemmSmem::kW;
  uint8_t* sc_s = smem + GemmSmem::kScale;
  uint64_t* bars = (uint64_t*)(smem + GemmSmem::kBar);
  uint64_t* full_bar = bars;                      // [kStages] TMEM A stage: 8 dequant warps
  uint64_t* empty_bar = full_bar + kStages;       // [kStages] MMA commit
  uint64_t* bfull_bar = empty_bar + kStages;      // [kBStages] activation TMA tx
  uint64_t* bempty_bar = bfull_bar + kBStages;    // [kBStages] MMA commit
  uint64_t* wfull_bar = bempty_bar + kBStages;    // [kWStages] nibble TMA tx
  uint64_t* wempty_bar = wfull_bar + kWStages;    // [kWStages] 8 dequant warps
  uint64_t* scfull_bar = wempty_bar + kWStages;   // [2] scale bulk copy tx
  uint64_t* scempty_bar = scfull_bar + 2;         // [2] all 16 dequant warps
  uint64_t* accfull_bar = scempty_bar + 2;        // [2] MMA commit
  uint64_t* accempty_bar = accfull_bar + 2;       // [2] 4 epilogue warps
  uint32_t* misc = (uint32_t*)(smem + GemmSmem::kMisc);
  volatile uint32_t* tmem_slot = misc;
  volatile uint32_t* abort_s = misc + 1;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int32_t G = p.K >> 5;
  const int32_t nchunks = p.K / kBK;
  const int32_t ftiles = (p.N + kBM - 1) / kBM;
  const int32_t total_tiles = __ldg(p.tile_ptr + p.num_experts) * ftiles;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full_bar[s], kDequantPerChunk);
      mbar_init(&empty_bar[s], 1);
    }
    for (int s = 0; s < kBStages; ++s) {
      mbar_init(&bfull_bar[s], 1);
      mbar_init(&bempty_bar[s], 1);
    }
    for (int s = 0; s < kWStages; ++s) {
      mbar_init(&wfull_bar[s], 1);
      mbar_init(&wempty_bar[s], kDequantPerChunk);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&scfull_bar[s], 1);
      mbar_init(&scempty_bar[s], kDequantWarps);
      mbar_init(&accfull_bar[s], 1);
      mbar_init(&accempty_bar[s], 4);
    }
    *abort_s = 0;
    fence_mbar_init();
  }
  if (warp == kMmaWarp) {
    tmem_alloc((uint32_t*)tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  if (warp == kActWarp && lane == 0) {
    tma_prefetch_desc(&tmap_act);
    tma_prefetch_desc(&tmap_w);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == kActWarp) {
    // ------------------------------------------------ activation producer
    if (elect_one()) {
      uint32_t it = 0;
      for (int32_t t = blockIdx.x; t < total_tiles && !*abort_s; t += gridDim.x) {
        TileInfo ti;
        if (!decode_tile(p, t, ftiles, ti)) continue;
        const int32_t nbox = (ti.nrows + kBoxRows - 1) / kBoxRows;
        for (int32_t c = 0; c < nchunks; ++c, ++it) {
          const uint32_t s = it % kBStages, ph = (it / kBStages) & 1;
          if (!mbar_wait(&bempty_bar[s], ph ^ 1, p.err, kErrTimeoutEmpty)) { *abort_s = 1; break; }
          mbar_arrive_expect_tx(&bfull_bar[s], (uint32_t)nbox * kBoxRows * 128);
          for (int32_t b = 0; b < nbox; ++b)
            tma_load_2d(act_s + s * kActStageBytes + b * kBoxRows * 128, &tmap_act, c * kBK, ti.row0 + b * kBoxRows,
                        &bfull_bar[s]);
        }
      }
    }
  } else if (warp == kWWarp) {
    // ---------------------------------------------------- weight producer
    if (elect_one()) {
      uint32_t wit = 0, tl = 0;
      for (int32_t t = blockIdx.x; t < total_tiles && !*abort_s; t += gridDim.x) {
        TileInfo ti;
        if (!decode_tile(p, t, ftiles, ti)) continue;
        const uint32_t sb = tl & 1, sph = (tl >> 1) & 1;
        ++tl;
        if (!mbar_wait(&scempty_bar[sb], sph ^ 1, p.err, kErrTimeoutEmpty)) { *abort_s = 1; break; }
        const int32_t frows = min(kBM, p.N - ti.f0);
        const uint32_t sbytes = (uint32_t)(frows * G);
        mbar_arrive_expect_tx(&scfull_bar[sb], sbytes);
        const uint8_t* src = p.scales + ((size_t)ti.expert * p.N + ti.f0) * G;
        asm volatile(
            "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                smem_u32(sc_s + sb * kScaleBytes)),
            "l"(src), "r"(sbytes), "r"(smem_u32(&scfull_bar[sb]))
            : "memory");
        const int32_t wrow = ti.expert * p.N + ti.f0;
        bool ok = true;
        for (int32_t c = 0; c < nchunks; ++c, ++wit) {
          const uint32_t s = wit % kWStages, ph = (wit / kWStages) & 1;
          if (!mbar_wait(&wempty_bar[s], ph ^ 1, p.err, kErrTimeoutEmpty)) { ok = false; break; }
          mbar_arrive_expect_tx(&wfull_bar[s], kWStageBytes);
          tma_load_2d(w_s + s * kWStageBytes, &tmap_w, c * (kBK / 2), wrow, &wfull_bar[s]);
        }
        if (!ok) { *abort_s = 1; break; }
      }
    }
  } else if (warp == kMmaWarp) {
    // --------------------------------------------------------- MMA issuer
    if (elect_one()) {
      uint32_t it = 0, tl = 0;
      for (int32_t t = blockIdx.x; t < total_tiles && !*abort_s; t += gridDim.x) {
        TileInfo ti;
        if (!decode_tile(p, t, ftiles, ti)) continue;
        const uint32_t n_mma = (uint32_t)((ti.nrows + 15) & ~15);
        const uint32_t idesc = kF16 ? make_idesc_f16(kBM, n_mma) : make_idesc_bf16(kBM, n_mma);
        const uint32_t ab = tl & 1, aph = (tl >> 1) & 1;
        if (!mbar_wait(&accempty_bar[ab], aph ^ 1, p.err, kErrTimeoutAccum)) { *abort_s = 1; break; }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + ab * kAccCols;
        bool ok = true;
        for (int32_t c = 0; c < nchunks; ++c, ++it) {
          const uint32_t s = it % kStages, ph = (it / kStages) & 1;
          const uint32_t sb = it % kBStages, phb = (it / kBStages) & 1;
          if (!mbar_wait(&bfull_bar[sb], phb, p.err, kErrTimeoutFull)) { ok = false; break; }
          if (!mbar_wait(&full_bar[s], ph, p.err, kErrTimeoutFull)) { ok = false; break; }
          tc_fence_after();
          const uint32_t b_base = smem_u32(act_s + sb * kActStageBytes);
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk) {
            tc_mma_ts(d_tmem, tmem_base + kAColBase + s * 32 + kk * 8, make_sdesc_sw128(b_base + kk * 32), idesc,
                      (c > 0 || kk > 0) ? 1u : 0u);
          }
          tc_commit(&empty_bar[s]);
          tc_commit(&bempty_bar[sb]);
        }
        if (!ok) { *abort_s = 1; break; }
        tc_commit(&accfull_bar[ab]);
        ++tl;
      }
    }
  } else if (warp < kDequantWarps) {
    // --------------------------------------------- dequant: weights -> TMEM
    const int wg = (warp >> 2) & 1;             // which MXFP4 group of the chunk
    const int parity = warp >> 3;               // even or odd chunks
    const int row = (warp & 3) * 32 + lane;     // weight row within the tile == TMEM lane
    const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
    uint32_t it = 0, wit = 0, tl = 0;
    for (int32_t t = blockIdx.x; t < total_tiles; t += gridDim.x) {
      TileInfo ti;
      if (!decode_tile(p, t, ftiles, ti)) continue;
      if (*abort_s) break;
      const uint32_t sb = tl & 1, sph = (tl >> 1) & 1;
      ++tl;
      const bool row_ok = ti.f0 + row < p.N;
      bool ok = mbar_wait(&scfull_bar[sb], sph, p.err, kErrTimeoutFull);
      const uint8_t* srow = sc_s + sb * kScaleBytes + row * G + wg;
      const uint32_t nib_off = (uint32_t)(wg ^ ((row >> 2) & 1)) << 4;  // 32-byte swizzle
      for (int32_t c = parity; c < nchunks && ok; c += 2) {
        const uint32_t witc = wit + (uint32_t)c, itc = it + (uint32_t)c;
        const uint32_t ws = witc % kWStages, wph = (witc / kWStages) & 1;
        const uint32_t s = itc % kStages, ph = (itc / kStages) & 1;
        ok = mbar_wait(&wfull_bar[ws], wph, p.err, kErrTimeoutFull);
        if (!ok) break;
        const uint4 nb = *(const uint4*)(w_s + ws * kWStageBytes + row * 32 + nib_off);
        const uint32_t sc = srow[2 * c];
        __syncwarp();
        if (lane == 0) mbar_arrive(&wempty_bar[ws]);
        uint32_t r[16];
        if (row_ok) {
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
        } else {
#pragma unroll
          for (int j = 0; j < 16; ++j) r[j] = 0u;
        }
        ok = mbar_wait(&empty_bar[s], ph ^ 1, p.err, kErrTimeoutEmpty);
        if (!ok) break;
        __syncwarp();
        tc_fence_after();
        tmem_st_x16(tmem_base + lane_base + kAColBase + s * 32 + wg * 16, r);
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&full_bar[s]);
      }
      it += (uint32_t)nchunks;
      wit += (uint32_t)nchunks;
      __syncwarp();
      if (lane == 0) mbar_arrive(&scempty_bar[sb]);
      if (!ok) { *abort_s = 1; break; }
    }
  } else {
    // ---------------------------------------- epilogue: TMEM -> registers -> global
    const int q = warp - kEpiWarp0;               // TMEM lane quarter
    const int row = q * 32 + lane;
    const uint32_t lane_base = (uint32_t)(q * 32) << 16;
    uint32_t tl = 0;
    for (int32_t t = blockIdx.x; t < total_tiles; t += gridDim.x) {
      TileInfo ti;
      if (!decode_tile(p, t, ftiles, ti)) continue;
      if (*abort_s) break;
      const uint32_t ab = tl & 1, aph = (tl >> 1) & 1;
      ++tl;
      const int32_t frow = ti.f0 + row;
      const bool row_ok = frow < p.N;
      const float bias = row_ok ? bf16_bits_to_f32(__ldg(p.bias + (size_t)ti.expert * p.N + frow)) : 0.0f;
      if (!mbar_wait(&accfull_bar[ab], aph, p.err, kErrTimeoutAccum)) { *abort_s = 1; break; }
      __syncwarp();
      tc_fence_after();
      const int32_t ncols = (ti.nrows + 31) & ~31;
      for (int32_t c0 = 0; c0 < ncols; c0 += 32) {
        uint32_t v[32];
        tmem_ld_x32(tmem_base + lane_base + ab * kAccCols + (uint32_t)c0, v);
        tmem_ld_wait();
        if (kMode == 0) {
          // lane pair (2j, 2j+1) holds the glu / linear rows of output column j:
          // the even lane finishes tokens c0..c0+15, the odd lane c0+16..c0+31
          const bool odd = lane & 1;
          uint16_t* out = (uint16_t*)p.out;
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const float mine_lo = __uint_as_float(v[i]) + bias;
            const float mine_hi = __uint_as_float(v[16 + i]) + bias;
            const float send = odd ? mine_lo : mine_hi;
            const float recv = __shfl_xor_sync(0xffffffffu, send, 1);
            const float gl = odd ? recv : mine_lo;
            const float li = odd ? mine_hi : recv;
            const int32_t col = c0 + i + (odd ? 16 : 0);
            const float g = fminf(gl, p.limit);
            const float l = fmaxf(fminf(li, p.limit), -p.limit);
            const float sg = 1.0f / (1.0f + expf(-(p.alpha * g)));
            const float y = (g * sg) * (l + 1.0f);
            if (row_ok && col < ti.nrows)
              out[(size_t)(ti.row0 + col) * p.ldo + (frow >> 1)] =
                  kF16 ? __half_as_ushort(__float2half_rn(y)) : f32_to_bf16_bits(y);
          }
        } else {
          float* out = (float*)p.out;
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const int32_t col = c0 + j;
            if (row_ok && col < ti.nrows)
              out[(size_t)(ti.row0 + col) * p.ldo + frow] = __uint_as_float(v[j]) + bias;
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&accempty_bar[ab]);
    }
  }

  // ---- teardown: everyone drains, then the allocating warp frees TMEM
  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
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



template <int kMode, bool kF16>
static void launch_variant(const CUtensorMap& ta, const CUtensorMap& tw, const GemmParams& p, int grid, int smem,
                           cudaStream_t stream) {
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(moe_gemm_tc_kernel<kMode, kF16>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    attr = true;
  }
  moe_gemm_tc_kernel<kMode, kF16><<<grid, kGemmThreads, smem, stream>>>(ta, tw, p);
}

int launch_moe_gemm(int mode, const GemmLaunch& L, cudaStream_t stream) {
  if (L.K % kBK != 0 || L.K / 32 > kMaxGroups) return -10;
  {
    // every tile's scale block must be a whole number of 16-byte units
    const int32_t G = L.K / 32;
    const int32_t last = L.N % kBM ? L.N % kBM : kBM;
    if (((int64_t)kBM * G) % 16 || ((int64_t)last * G) % 16 || ((int64_t)L.N * G) % 16) return -11;
  }
  CUtensorMap tmap_act, tmap_w;
  int rc = make_tmap_2d(&tmap_act, L.act, L.f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                        (uint64_t)L.act_rows, (uint64_t)L.K, kBK, kBoxRows, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  rc = make_tmap_2d(&tmap_w, L.blocks, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, (uint64_t)L.E * L.N, (uint64_t)L.K / 2,
                    kBK / 2, kBM, CU_TENSOR_MAP_SWIZZLE_32B);
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
  const int smem = GemmSmem::kAlloc;
  if (mode == 0) {
    if (L.f16) launch_variant<0, true>(tmap_act, tmap_w, p, L.grid, smem, stream);
    else launch_variant<0, false>(tmap_act, tmap_w, p, L.grid, smem, stream);
  } else {
    if (L.f16) launch_variant<1, true>(tmap_act, tmap_w, p, L.grid, smem, stream);
    else launch_variant<1, false>(tmap_act, tmap_w, p, L.grid, smem, stream);
  }
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

}  // namespace gptoss
