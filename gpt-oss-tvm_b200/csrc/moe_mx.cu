// moe_mx.cu -- decode-size grouped expert GEMMs on the block-scaled tensor cores
// (tcgen05.mma kind::mxf8f6f4.block_scale): the MXFP4 weights go to the MMA as
// they are stored, e2m1 codes with their E8M0 block-32 scales, and are never
// decoded by the SMs.
//
// Same maths as moe_gemm.cu (model/mlp.py:238-326 run_einsum, fused clamped
// SwiGLU for gate/up, fp32 output for down), same tile plan and epilogue; what
// changes is how the operands reach the tensor core:
//   * weights (MMA "A", 128 rows per tile): TMA with the 16U4_ALIGN16B element
//     type copies the checkpoint's packed e2m1 nibbles (blocks [E, N, K/32, 16])
//     into shared memory in the one-code-per-byte form the MMA reads, 128 K
//     elements (one 128-byte swizzled row) per stage.  That element type needs
//     a row length that is a multiple of 128 codes, so the TMA map covers the
//     first (K / 128) * 128 codes of each row and, when K % 128 == 64 (K = 2880:
//     22 stages + 64), one warp expands the last 32 bytes of each row itself;
//   * weight scales: the checkpoint's E8M0 bytes (scales [E, N, K/32]) for the
//     4 K-blocks of a stage are rearranged into the 512-byte scale-factor chunk
//     (row r of 128 at byte (r % 32) * 16 + (r / 32) * 4 + k) and moved into
//     tensor memory with tcgen05.cp (32 x 128 bit, copied to all four lane
//     quarters), where the MMA reads one byte per row and K-block;
//   * activations (MMA "B", the <= 32 token rows of the tile): each bf16/f16
//     value x is carried as two e4m3 codes, x = 2^e_hi * hi + 2^e_lo * lo with
//     one pair of E8M0 exponents per 32 values (quantize_mx_kernel below), and
//     every K-block runs two MMAs, one per term, into the same fp32 accumulator.
//     hi keeps 4 significant bits, lo the next 4 of the remainder: the sum
//     differs from x by at most 2^-8 of |x| (one extra bf16-sized rounding of
//     each activation), well inside the bf16 tolerance of the block, while the
//     weights stay exact.
// No warp decodes a weight: the roles are a weight TMA producer, two
// scale-factor builders (which also expand the 64-code row tails), an
// activation TMA producer, two MMA issuers (one owns TMEM) and four epilogue
// warps.
#include "common.cuh"
#include "launch.h"
#include "moe_tile.cuh"

namespace gptoss {

constexpr int kMxThreads = 320;                  // 10 warps
constexpr int kMxBK = 128;                       // K codes per stage (one 128-byte smem row)
constexpr int kMxStages = 6;
constexpr int kMxMaxN = kMoeTileRowsSmall;       // token rows per tile (32)
constexpr int kMxWBytes = kBM * kMxBK;           // 16 KB: 128 weight rows x 128 codes
constexpr int kMxActBytes = kMxMaxN * kMxBK;     // 4 KB: one activation term of one stage
constexpr int kMxActStage = 2 * kMxActBytes;     // a stage's two terms: the 32 hi rows, then the 32 lo rows
constexpr int kMxMmaN = 2 * kMxMaxN;             // MMA N: hi and lo rows in one MMA (64)
constexpr int kMxSfBytes = 512;                  // one scale-factor chunk: 128 rows x 4 K-blocks
constexpr int kMxMaxGroups = 96;                 // K / 32 <= 96 (K <= 3072)
constexpr int kMxScRow = 2 * kMxMaxGroups;       // bytes per row of the activation scales: hi, then lo
// Two scale-factor builders and two MMA issuers, each taking the stages of one
// parity (stage counter & 1): a single thread issuing 3 tcgen05.cp and 8
// tcgen05.mma per 128-code stage was the pace (measured: ~600 cycles of issue
// per stage, above the ~370 cycles the weights take to stream at HBM rate).
constexpr int kMxWarpW = 0, kMxWarpSf = 1, kMxWarpAct = 2, kMxWarpMma = 3, kMxWarpEpi0 = 4, kMxWarpSf1 = 8,
              kMxWarpMma1 = 9;
// TMEM columns: two accumulator buffers (tile i / i + 1), each a pair of
// 64-column accumulators (even / odd stages: one per MMA issuer; columns
// 0-31 the hi term, 32-63 the lo term of the tile's token rows; all four
// summed by the epilogue), then per pipeline stage its two scale-factor
// chunks (4 columns each), so that copying the chunks of one stage never
// writes columns the MMAs of another stage still read
constexpr int kMxAccCols = kMxMmaN;
constexpr int kMxSfCol0 = 4 * kMxAccCols, kMxSfStageCols = 8;
constexpr int kMxTmemCols = 512;
static_assert(kMxSfCol0 + kMxStages * kMxSfStageCols <= kMxTmemCols, "TMEM budget");

// shared memory layout (offsets from the 1024-aligned base)
constexpr int kMxOffW = 0;
constexpr int kMxOffA = kMxOffW + kMxStages * kMxWBytes;                 // [stage][hi rows | lo rows][128 B]
constexpr int kMxOffSf = kMxOffA + kMxStages * kMxActStage;              // [stage][2][512]
constexpr int kMxOffScW = kMxOffSf + kMxStages * 2 * kMxSfBytes;          // [2][128 x G] weight scales of a tile
constexpr int kMxOffScA = kMxOffScW + 2 * kBM * kMxMaxGroups;             // [2][32 x 192] activation scales
constexpr int kMxOffBar = kMxOffScA + 2 * kMxMaxN * kMxScRow;
constexpr int kMxNumBars = 2 * kMxStages + 2 + 2 + 2 + 2 + 1;
constexpr int kMxOffMisc = kMxOffBar + kMxNumBars * 8;
constexpr int kMxOffEpi = (kMxOffMisc + 64 + 15) & ~15;                  // 4 warps x 2 KB
constexpr int kMxSmem = kMxOffEpi + 4 * 2048 + 1024;
static_assert(kMxSmem <= 227 * 1024, "shared memory budget");
static_assert(kMxOffA % 1024 == 0 && kMxActBytes % 1024 == 0, "128-byte swizzle atoms stay 1024-aligned");

// ------------------------------------------------------------------ PTX --
// Instruction descriptor of kind::mxf8f6f4.block_scale: A e2m1 (K-major), B
// e4m3 (K-major), E8M0 scales, M = 128, N = n, the scale-factor byte of A and
// B (which of the 4 K-blocks of the chunk) in bits 29-30 and 4-5.
__host__ __device__ constexpr uint32_t make_idesc_mx(uint32_t n, uint32_t sf_id) {
  return (sf_id << 4)          // B scale-factor id
         | (5u << 7)           // A format: E2M1
         | (0u << 10)          // B format: E4M3
         | ((n >> 3) << 17)    // N / 8
         | (1u << 23)          // scale format: E8M0
         | ((128u >> 4) << 24) // M / 16
         | (sf_id << 29);      // A scale-factor id
}

// D[tmem] (+)= (A[smem] x SFA[tmem]) * (B[smem] x SFB[tmem])^T, K = 32.
__device__ __forceinline__ void tc_mma_mx(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                          uint32_t sfa_tmem, uint32_t sfb_tmem, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%5], [%6], p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(sfa_tmem), "r"(sfb_tmem)
      : "memory");
}

// 32 rows x 128 bits of shared memory into TMEM lanes 0-31 of four columns,
// repeated in the other three lane quarters.
__device__ __forceinline__ void tc_cp_sf(uint32_t taddr, uint64_t sdesc) {
  asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(sdesc) : "memory");
}

// Shared-memory descriptor of one scale-factor chunk for tcgen05.cp: K-major,
// no swizzle, 32 rows of 16 bytes = four 8-row core matrices 128 bytes apart.
__device__ __forceinline__ uint64_t make_sdesc_sf(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= (uint64_t)((smem_addr & 0x3FFFF) >> 4);
  d |= (uint64_t)(128 >> 4) << 16;  // leading byte offset (a single core matrix along K)
  d |= (uint64_t)(128 >> 4) << 32;  // stride byte offset: 8 rows x 16 B
  d |= (uint64_t)1 << 46;           // descriptor version (sm_100); layout type 0 = no swizzle
  return d;
}

// Generic-proxy shared-memory writes made visible to the tensor core's reads.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ uint32_t e4m3x2_from_f32(float lo, float hi) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
  return r;
}
__device__ __forceinline__ void f32x2_from_e4m3x2(uint32_t v, float& lo, float& hi) {
  uint32_t h;
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(h) : "h"((uint16_t)v));
  lo = __half2float(__ushort_as_half((uint16_t)(h & 0xFFFFu)));
  hi = __half2float(__ushort_as_half((uint16_t)(h >> 16)));
}

// ------------------------------------------------ activation quantizer --
// Row r of the output holds the activations of source row idx[r] (or r):
//   q [rows, 2K] bytes: hi codes (K), then lo codes (K), e4m3;
//   sc [rows, 192] bytes: E8M0 exponent of hi for each 32-value group (G <= 96
//   bytes), then at byte 96 the exponent of lo.
// Per group: e_hi = floor(log2 max|x|) - 7 (so |x| / 2^e_hi < 256, no e4m3
// overflow), hi = e4m3(x / 2^e_hi), e_lo = e_hi - 5, lo = e4m3((x / 2^e_hi -
// hi) * 32) -- the remainder is at most half an e4m3 step of hi (<= 8), so
// lo <= 256.  All scalings are exact powers of two; only the two e4m3
// roundings (to nearest even) lose bits.  One warp per row, one group per lane.
template <bool kSrcF16>
__global__ void quantize_mx_kernel(const uint16_t* __restrict__ src, const int32_t* __restrict__ idx, int64_t rows,
                                   int32_t K, uint8_t* __restrict__ q, uint8_t* __restrict__ sc) {
  const int64_t r = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (r >= rows) return;
  const int lane = threadIdx.x & 31;
  const int64_t sr = idx ? (int64_t)__ldg(idx + r) : r;
  const uint16_t* x = src + sr * K;
  uint8_t* qh = q + r * 2 * (int64_t)K;
  uint8_t* ql = qh + K;
  uint8_t* sh = sc + r * kMxScRow;
  const int32_t G = K >> 5;
  for (int32_t g = lane; g < G; g += 32) {
    uint4 raw[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) raw[i] = __ldg((const uint4*)(x + (size_t)g * 32) + i);
    const uint16_t* e = (const uint16_t*)raw;
    float f[32];
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      f[i] = kSrcF16 ? __half2float(__ushort_as_half(e[i])) : bf16_bits_to_f32(e[i]);
      amax = fmaxf(amax, fabsf(f[i]));
    }
    const int32_t E = (int32_t)((__float_as_uint(amax) >> 23) & 0xFFu) - 127;
    const int32_t e_hi = amax > 0.0f ? max(-127, min(120, E - 7)) : 0;
    const int32_t e_lo = max(-127, e_hi - 5);
    const float inv_hi = __uint_as_float((uint32_t)(127 - e_hi) << 23);
    const float lo_mul = __uint_as_float((uint32_t)(127 + e_hi - e_lo) << 23);
    uint32_t hw[8], lw[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      uint32_t h4 = 0, l4 = 0;
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const float a = f[4 * i + 2 * j] * inv_hi, b = f[4 * i + 2 * j + 1] * inv_hi;
        const uint32_t h = e4m3x2_from_f32(a, b);
        float ha, hb;
        f32x2_from_e4m3x2(h, ha, hb);
        const uint32_t l = e4m3x2_from_f32((a - ha) * lo_mul, (b - hb) * lo_mul);
        h4 |= h << (16 * j);
        l4 |= l << (16 * j);
      }
      hw[i] = h4;
      lw[i] = l4;
    }
    *(uint4*)(qh + (size_t)g * 32) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
    *(uint4*)(qh + (size_t)g * 32 + 16) = make_uint4(hw[4], hw[5], hw[6], hw[7]);
    *(uint4*)(ql + (size_t)g * 32) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
    *(uint4*)(ql + (size_t)g * 32 + 16) = make_uint4(lw[4], lw[5], lw[6], lw[7]);
    sh[g] = (uint8_t)(127 + e_hi);
    sh[kMxMaxGroups + g] = (uint8_t)(127 + e_lo);
  }
}

// ------------------------------------------------------ block-scaled GEMM --
struct MxParams {
  GemmParams g;           // tile plan, biases, outputs, error word (scales = the weight scales)
  const uint8_t* blocks;  // [E, N, K/32, 16] packed e2m1 (for the 64-code row tails)
  const uint8_t* act_sc;  // [act_rows, 192] E8M0 exponents of the two activation terms
};

// Persistent over tiles (expert, token tile <= 32 rows, 128 weight rows), one
// CTA per SM.  Per stage s (128 K codes): the weight TMA, the activation TMA
// (hi and lo terms) and the scale-factor builder each arrive on full[s]; the
// MMA thread copies the stage's three scale chunks into TMEM, issues two
// block-scaled MMAs per K-block of 32, and commits empty[s].
template <int kMode>
__global__ void __launch_bounds__(kMxThreads, 1)
    moe_gemm_mx_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_hi,
                       const __grid_constant__ CUtensorMap tmap_lo, const MxParams mp) {
  const GemmParams& p = mp.g;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint64_t* bars = (uint64_t*)(smem + kMxOffBar);
  uint64_t* full_bar = bars;                      // [stages] weights + activations + scale chunks
  uint64_t* empty_bar = full_bar + kMxStages;     // [stages] MMA commit
  uint64_t* scfull_bar = empty_bar + kMxStages;   // [2] the tile's scale rows (bulk copies)
  uint64_t* scempty_bar = scfull_bar + 2;         // [2] the scale-factor builder is done with them
  uint64_t* accfull_bar = scempty_bar + 2;        // [2] MMA commit
  uint64_t* accempty_bar = accfull_bar + 2;       // [2] the four epilogue warps
  uint64_t* drain_bar = accempty_bar + 2;         // [1] every MMA complete
  uint32_t* misc = (uint32_t*)(smem + kMxOffMisc);
  volatile uint32_t* tmem_slot = misc;
  volatile uint32_t* abort_s = misc + 1;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int32_t G = p.K >> 5;
  const int32_t nmain = p.K / kMxBK;                    // stages fed by the weight TMA
  const bool tail = (p.K % kMxBK) != 0;                 // one more stage of 64 codes
  const int32_t nst = nmain + (tail ? 1 : 0);
  const int32_t ftiles = (p.N + kBM - 1) / kBM;
  const int32_t total_tiles = __ldg(p.tile_ptr + p.num_experts) * ftiles;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kMxStages; ++s) {
      mbar_init(&full_bar[s], 3);
      mbar_init(&empty_bar[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&scfull_bar[s], 1);
      mbar_init(&scempty_bar[s], 2);   // both scale-factor builders
      mbar_init(&accfull_bar[s], 2);   // both MMA issuers
      mbar_init(&accempty_bar[s], 4);
    }
    mbar_init(drain_bar, 2);  // both MMA issuers commit once at the end
    *abort_s = 0;
    fence_mbar_init();
  }
  if (warp == kMxWarpMma) {
    tmem_alloc((uint32_t*)tmem_slot, kMxTmemCols);
    tmem_relinquish();
  }
  if (warp == kMxWarpW && lane == 0) {
    tma_prefetch_desc(&tmap_w);
    tma_prefetch_desc(&tmap_hi);
    tma_prefetch_desc(&tmap_lo);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == kMxWarpW) {
    // ------------------------------------ weights (TMA) + the tile's scale rows
    if (elect_one()) {
      uint32_t it = 0, tl = 0;
      for (int32_t t = blockIdx.x; t < total_tiles && !*abort_s; t += gridDim.x) {
        TileInfo ti;
        if (!decode_tile<kMxMaxN>(p, t, ftiles, ti)) continue;
        const uint32_t sb = tl & 1, sph = (tl >> 1) & 1;
        ++tl;
        if (!mbar_wait(&scempty_bar[sb], sph ^ 1, p.err, kErrTimeoutEmpty)) { *abort_s = 1; break; }
        const int32_t frows = min(kBM, p.N - ti.f0);
        const uint32_t wbytes = (uint32_t)(frows * G), abytes = (uint32_t)(ti.nrows * kMxScRow);
        mbar_arrive_expect_tx(&scfull_bar[sb], wbytes + abytes);
        asm volatile(
            "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                smem_u32(smem + kMxOffScW + sb * kBM * kMxMaxGroups)),
            "l"(p.scales + ((size_t)ti.expert * p.N + ti.f0) * G), "r"(wbytes), "r"(smem_u32(&scfull_bar[sb]))
            : "memory");
        asm volatile(
            "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                smem_u32(smem + kMxOffScA + sb * kMxMaxN * kMxScRow)),
            "l"(mp.act_sc + (size_t)ti.row0 * kMxScRow), "r"(abytes), "r"(smem_u32(&scfull_bar[sb]))
            : "memory");
        const int32_t wrow = ti.expert * p.N + ti.f0;
        bool ok = true;
        for (int32_t j = 0; j < nst; ++j, ++it) {
          const uint32_t s = it % kMxStages, ph = (it / kMxStages) & 1;
          if (!mbar_wait(&empty_bar[s], ph ^ 1, p.err, kErrTimeoutEmpty)) { ok = false; break; }
          if (j < nmain) {
            // the transaction counts the packed source bytes (4 bits per code), not the
            // padded bytes written to shared memory; rows past N are zero-filled and count too
            mbar_arrive_expect_tx(&full_bar[s], kMxWBytes / 2);
            tma_load_2d(smem + kMxOffW + s * kMxWBytes, &tmap_w, j * kMxBK, wrow, &full_bar[s]);
          } else {
            mbar_arrive(&full_bar[s]);  // the tail's weights come from the scale-factor builder
          }
        }
        if (!ok) { *abort_s = 1; break; }
      }
    }
  } else if (warp == kMxWarpAct) {
    // ------------------------------------------ activation terms (TMA)
    if (elect_one()) {
      uint32_t it = 0;
      for (int32_t t = blockIdx.x; t < total_tiles && !*abort_s; t += gridDim.x) {
        TileInfo ti;
        if (!decode_tile<kMxMaxN>(p, t, ftiles, ti)) continue;
        const int32_t nbox = (ti.nrows + 15) >> 4;
        bool ok = true;
        for (int32_t j = 0; j < nst; ++j, ++it) {
          const uint32_t s = it % kMxStages, ph = (it / kMxStages) & 1;
          if (!mbar_wait(&empty_bar[s], ph ^ 1, p.err, kErrTimeoutEmpty)) { ok = false; break; }
          mbar_arrive_expect_tx(&full_bar[s], (uint32_t)(2 * nbox * 16 * kMxBK));
          for (int32_t b = 0; b < nbox; ++b) {
            uint8_t* dst = smem + kMxOffA + s * kMxActStage + b * 16 * kMxBK;
            tma_load_2d(dst, &tmap_hi, j * kMxBK, ti.row0 + 16 * b, &full_bar[s]);
            tma_load_2d(dst + kMxActBytes, &tmap_lo, j * kMxBK, ti.row0 + 16 * b, &full_bar[s]);
          }
        }
        if (!ok) { *abort_s = 1; break; }
      }
    }
  } else if (warp == kMxWarpSf || warp == kMxWarpSf1) {
    // ------ scale-factor chunks of the stages of this warp's parity, and the 64-code tails
    const uint32_t par = warp == kMxWarpSf ? 0u : 1u;
    uint32_t it = 0, tl = 0;
    for (int32_t t = blockIdx.x; t < total_tiles; t += gridDim.x) {
      TileInfo ti;
      if (!decode_tile<kMxMaxN>(p, t, ftiles, ti)) continue;
      if (*abort_s) break;
      const uint32_t sb = tl & 1, sph = (tl >> 1) & 1;
      ++tl;
      bool ok = mbar_wait(&scfull_bar[sb], sph, p.err, kErrTimeoutFull);
      const uint8_t* scw = smem + kMxOffScW + sb * kBM * kMxMaxGroups;  // [128][G]
      const uint8_t* sca = smem + kMxOffScA + sb * kMxMaxN * kMxScRow;   // [32][192]
      const int32_t frows = min(kBM, p.N - ti.f0);
      for (int32_t j = 0; j < nst && ok; ++j, ++it) {
        if ((it & 1u) != par) continue;
        const uint32_t s = it % kMxStages, ph = (it / kMxStages) & 1;
        ok = mbar_wait(&empty_bar[s], ph ^ 1, p.err, kErrTimeoutEmpty);
        if (!ok) break;
        uint8_t* sf = smem + kMxOffSf + s * 2 * kMxSfBytes;
        // weights: line `lane` holds rows lane, lane + 32, lane + 64, lane + 96;
        // a row's 4 bytes are two 16-bit reads (rows are G bytes apart, G even)
        const int32_t g0 = 4 * j;
        const int32_t gvalid = min(4, G - g0);  // K-blocks of this stage (2 in a 64-code tail)
        const uint32_t keep = gvalid >= 4 ? 0xFFFFFFFFu : ((1u << (8 * gvalid)) - 1u);
        const uint32_t pad = 0x7F7F7F7Fu & ~keep;  // exponent 127 (x1) in the unused bytes
        uint32_t w4[4];
#pragma unroll
        for (int qq = 0; qq < 4; ++qq) {
          const int32_t row = lane + 32 * qq;
          uint32_t v = 0x7F7F7F7Fu;
          if (row < frows) {
            const uint16_t* src = (const uint16_t*)(scw + row * G + g0);
            v = ((uint32_t)src[0] | ((uint32_t)(gvalid > 2 ? src[1] : 0) << 16)) & keep;
            v |= pad;
          }
          w4[qq] = v;
        }
        *(uint4*)(sf + lane * 16) = make_uint4(w4[0], w4[1], w4[2], w4[3]);
        // activations: one 32-bit read per term (rows are 192 bytes apart); the
        // MMA's B rows are the 32 hi rows then the 32 lo rows, so lane r holds
        // B row r (hi of token row r) in word 0 and B row r + 32 (lo) in word 1,
        // the layout of the weights' rows r and r + 32.  Rows beyond the tile's
        // count get exponent 127 (their MMA columns are never stored)
        uint32_t vh = 0x7F7F7F7Fu, vl = 0x7F7F7F7Fu;
        if (lane < ti.nrows) {
          vh = (*(const uint32_t*)(sca + lane * kMxScRow + g0) & keep) | pad;
          vl = (*(const uint32_t*)(sca + lane * kMxScRow + kMxMaxGroups + g0) & keep) | pad;
        }
        *(uint4*)(sf + kMxSfBytes + lane * 16) = make_uint4(vh, vl, 0x7F7F7F7Fu, 0x7F7F7F7Fu);
        if (j == nmain) {
          // the row tails (codes nmain*128 .. K-1, 32 packed bytes per row) in
          // the form the TMA type writes: each 8 packed bytes (16 codes) then 8
          // bytes of zero, in the 128-byte swizzle of the stage's rows
          uint8_t* wst = smem + kMxOffW + s * kMxWBytes;
          const size_t row_bytes = (size_t)(p.K >> 1);
          for (int32_t row = lane; row < kBM; row += 32) {
            uint4 pk0 = make_uint4(0u, 0u, 0u, 0u), pk1 = pk0;
            if (row < frows) {
              const uint8_t* src = mp.blocks + ((size_t)ti.expert * p.N + ti.f0 + row) * row_bytes +
                                   (size_t)nmain * (kMxBK / 2);
              pk0 = ldg_nc_v4(src);
              pk1 = ldg_nc_v4(src + 16);
            }
            const uint32_t sw = (uint32_t)(row & 7);
            uint8_t* dst = wst + row * kMxBK;
            *(uint4*)(dst + ((0u ^ sw) << 4)) = make_uint4(pk0.x, pk0.y, 0u, 0u);
            *(uint4*)(dst + ((1u ^ sw) << 4)) = make_uint4(pk0.z, pk0.w, 0u, 0u);
            *(uint4*)(dst + ((2u ^ sw) << 4)) = make_uint4(pk1.x, pk1.y, 0u, 0u);
            *(uint4*)(dst + ((3u ^ sw) << 4)) = make_uint4(pk1.z, pk1.w, 0u, 0u);
          }
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&full_bar[s]);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&scempty_bar[sb]);
      if (!ok) { *abort_s = 1; break; }
    }
  } else if (warp == kMxWarpMma || warp == kMxWarpMma1) {
    // ---------------------------- MMA issuer of the stages of this warp's parity
    const uint32_t par = warp == kMxWarpMma ? 0u : 1u;
    if (elect_one()) {
      uint32_t it = 0, tl = 0;
      bool ok = true;
      const uint64_t wdesc0 = make_sdesc_sw128(smem_u32(smem + kMxOffW));
      const uint64_t bdesc0 = make_sdesc_sw128(smem_u32(smem + kMxOffA));
      for (int32_t t = blockIdx.x; t < total_tiles && !*abort_s; t += gridDim.x) {
        TileInfo ti;
        if (!decode_tile<kMxMaxN>(p, t, ftiles, ti)) continue;
        const uint32_t ab = tl & 1, aph = (tl >> 1) & 1;
        if (!mbar_wait(&accempty_bar[ab], aph ^ 1, p.err, kErrTimeoutAccum)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (2 * ab + par) * kMxAccCols;
        bool first = true;  // this issuer's first stage of the tile starts its accumulator
        for (int32_t j = 0; j < nst; ++j, ++it) {
          if ((it & 1u) != par) continue;
          const uint32_t s = it % kMxStages, ph = (it / kMxStages) & 1;
          if (!mbar_wait(&full_bar[s], ph, p.err, kErrTimeoutFull)) { ok = false; break; }
          tc_fence_after();
          const uint32_t sfs = smem_u32(smem + kMxOffSf + s * 2 * kMxSfBytes);
          const uint32_t sfa = tmem_base + kMxSfCol0 + s * kMxSfStageCols, sfb = sfa + 4;
          tc_cp_sf(sfa, make_sdesc_sf(sfs));
          tc_cp_sf(sfb, make_sdesc_sf(sfs + kMxSfBytes));
          const int32_t nkb = j < nmain ? kMxBK / 32 : (p.K - nmain * kMxBK) / 32;
          for (int32_t kb = 0; kb < nkb; ++kb) {
            // start-address field: (byte offset >> 4), 32 bytes (one K-block) per step
            const uint64_t adesc = wdesc0 + (uint64_t)((uint32_t)(s * kMxWBytes + kb * 32) >> 4);
            const uint64_t bdesc = bdesc0 + (uint64_t)((uint32_t)(s * kMxActStage + kb * 32) >> 4);
            const uint32_t idesc = make_idesc_mx((uint32_t)kMxMmaN, (uint32_t)kb);
            const uint32_t byte = (uint32_t)kb << 30;
            tc_mma_mx(d_tmem, adesc, bdesc, idesc, sfa | byte, sfb | byte, (!first || kb > 0) ? 1u : 0u);
          }
          tc_commit(&empty_bar[s]);
          first = false;
        }
        if (!ok) break;
        tc_commit(&accfull_bar[ab]);
        ++tl;
      }
      if (!ok) *abort_s = 1;
      tc_commit(drain_bar);
      mbar_wait(drain_bar, 0, p.err, kErrTimeoutOther);
    }
  } else {
    // ------------------------------ epilogue: TMEM -> registers -> global
    const int q = warp - kMxWarpEpi0;
    const int row = q * 32 + lane;
    const uint32_t lane_base = (uint32_t)(q * 32) << 16;
    uint32_t tl = 0;
    for (int32_t t = blockIdx.x; t < total_tiles; t += gridDim.x) {
      TileInfo ti;
      if (!decode_tile<kMxMaxN>(p, t, ftiles, ti)) continue;
      if (*abort_s) break;
      const uint32_t ab = tl & 1, aph = (tl >> 1) & 1;
      ++tl;
      const int32_t frow = ti.f0 + row;
      const bool row_ok = frow < p.N;
      const float bias = row_ok ? bf16_bits_to_f32(__ldg(p.bias + (size_t)ti.expert * p.N + frow)) : 0.0f;
      if (!mbar_wait(&accfull_bar[ab], aph, p.err, kErrTimeoutAccum)) { *abort_s = 1; break; }
      __syncwarp();
      tc_fence_after();
      // the four partial accumulators of each token row: even / odd stages x hi / lo term
      uint32_t v[32], v1[32];
      const uint32_t acc0 = tmem_base + lane_base + (2 * ab) * kMxAccCols;
      tmem_ld_x32(acc0, v);
#pragma unroll
      for (int part = 1; part < 4; ++part) {
        tmem_ld_x32(acc0 + (part >> 1) * kMxAccCols + (part & 1) * kMxMaxN, v1);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = __float_as_uint(__uint_as_float(v[i]) + __uint_as_float(v1[i]));
      }
      epilogue_block<kMode, true>(p, ti, v, 0, q, lane, bias, row_ok, frow, (uint16_t*)(smem + kMxOffEpi) + q * 1024);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&accempty_bar[ab]);
    }
  }

  // ---- teardown: every MMA has completed; the allocating warp frees TMEM
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == kMxWarpMma) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, kMxTmemCols);
  }
}

// ------------------------------------------------------------------ host --
int launch_quantize_mx(const uint16_t* src, int src_f16, const int32_t* idx, int64_t rows, int32_t K, uint8_t* q,
                       uint8_t* sc, cudaStream_t stream) {
  if (rows <= 0) return 0;
  if (K <= 0 || K % 32 || K / 32 > kMxMaxGroups || ((uintptr_t)src & 15) || ((uintptr_t)q & 15)) return -10;
  const unsigned blocks = (unsigned)((rows + 7) / 8);
  if (src_f16) quantize_mx_kernel<true><<<blocks, 256, 0, stream>>>(src, idx, rows, K, q, sc);
  else quantize_mx_kernel<false><<<blocks, 256, 0, stream>>>(src, idx, rows, K, q, sc);
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

typedef CUresult (*PFN_encodeTiledMx)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                      const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                      CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static PFN_encodeTiledMx mx_encode_fn() {
  static PFN_encodeTiledMx fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult qr;
    void* ptr = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &qr) == cudaSuccess &&
        qr == cudaDriverEntryPointSuccess)
      fn = (PFN_encodeTiledMx)ptr;
  }
  return fn;
}

// 2-D map, 128-byte swizzle: dims {inner, rows}, row stride in bytes, box {128, box_rows}.
static int mx_tmap(CUtensorMap* map, const void* base, CUtensorMapDataType dtype, uint64_t inner, uint64_t rows,
                   uint64_t stride_bytes, uint32_t box_rows) {
  PFN_encodeTiledMx enc = mx_encode_fn();
  if (!enc) return -1;
  cuuint64_t dims[2] = {inner, rows};
  cuuint64_t strides[1] = {stride_bytes};
  cuuint32_t box[2] = {(cuuint32_t)kMxBK, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, dtype, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : -2;
}

bool moe_mx_supported(int64_t act_rows, int32_t E, int32_t N, int32_t K, const void* blocks) {
  const int32_t G = K / 32;
  const int32_t last = N % kBM ? N % kBM : kBM;
  return act_rows > 0 && moe_tile_rows_max(act_rows, E) <= kMxMaxN && K >= 2 * kMxBK && K % 64 == 0 &&
         G <= kMxMaxGroups && ((uintptr_t)blocks & 31) == 0 && ((int64_t)kBM * G) % 16 == 0 &&
         ((int64_t)last * G) % 16 == 0 && ((int64_t)N * G) % 16 == 0;
}

int launch_moe_gemm_mx(int mode, const GemmLaunch& L, const uint8_t* q, const uint8_t* act_sc, cudaStream_t stream) {
  if (!moe_mx_supported(L.act_rows, L.E, L.N, L.K, L.blocks)) return -10;
  if (((uintptr_t)q & 15) || ((uintptr_t)act_sc & 15) || ((uintptr_t)L.scales & 15)) return -10;
  // weights: the first (K/128)*128 codes of every row, one code per byte in shared memory
  CUtensorMap tw, th, tlo;
  const int32_t kmain = (L.K / kMxBK) * kMxBK;
  int rc = mx_tmap(&tw, L.blocks, CU_TENSOR_MAP_DATA_TYPE_16U4_ALIGN16B, (uint64_t)kmain, (uint64_t)L.E * L.N,
                   (uint64_t)L.K / 2, kBM);
  if (rc) return rc;
  rc = mx_tmap(&th, q, CU_TENSOR_MAP_DATA_TYPE_UINT8, (uint64_t)L.K, (uint64_t)L.act_rows, 2 * (uint64_t)L.K, 16);
  if (rc) return rc;
  rc = mx_tmap(&tlo, q + L.K, CU_TENSOR_MAP_DATA_TYPE_UINT8, (uint64_t)L.K, (uint64_t)L.act_rows, 2 * (uint64_t)L.K,
               16);
  if (rc) return rc;
  MxParams mp;
  GemmParams& p = mp.g;
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
  p.row_dst = nullptr;
  for (int i = 0; i < kMaxPeerRanks; ++i) p.peer_out[i] = nullptr;
  p.peer_out_rows = 0;
  p.out_bf16 = 0;
  mp.blocks = L.blocks;
  mp.act_sc = act_sc;
  if (mode == 0) {
    static FuncSmemAttr attr;
    ensure_dyn_smem(attr, (const void*)moe_gemm_mx_kernel<0>, kMxSmem);
    moe_gemm_mx_kernel<0><<<L.grid, kMxThreads, kMxSmem, stream>>>(tw, th, tlo, mp);
  } else {
    static FuncSmemAttr attr;
    ensure_dyn_smem(attr, (const void*)moe_gemm_mx_kernel<1>, kMxSmem);
    moe_gemm_mx_kernel<1><<<L.grid, kMxThreads, kMxSmem, stream>>>(tw, th, tlo, mp);
  }
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

}  // namespace gptoss
