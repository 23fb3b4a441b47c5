// router_bf16.cu -- the router logits on the bf16 FMA pipe, bit-exact to the
// reference's serial bf16 accumulation.
//
// The reference step (nn.Linear with a bf16 accumulator, model/mlp.py:88-92,
// :376) is acc' = bf16(f32(acc + t*w)): t*w is exact in fp32, the sum is
// rounded to fp32 and then to bf16 (two roundings).  fma.rn.bf16x2 computes
// bf16(acc + t*w) with ONE rounding of the exact sum, at a quarter of the
// step latency of an fp32 FMA followed by a conversion.  The two roundings
// give a different result only when the fp32 rounding lands exactly on a
// bf16 midpoint that the exact sum is not on.  For a bf16 accumulator and a
// product of two bf16 values that requires
//   (a) t*w to be exactly a bf16 midpoint, and
//   (b) 0 < |acc| <= 2^(e - 24), e the binary exponent of t*w,
// i.e. an accumulator more than 2^23 times smaller than the product (the
// other cases are excluded by the grids the two addends live on: a
// difference from the midpoint of at most half an fp32 ulp cannot be formed
// from them).
//
// So every chain runs on fma.rn.bf16x2 (two chains per register) and tracks
// the smallest |accumulator| it fed into a step (min.xorsign.abs.bf16x2,
// off the dependent path).  At the end of each stage of k values that
// minimum is compared with a bound on 2^(e - 24) over the stage,
// 2^(E_t + E_w - 23) from the largest |t| and |w| of the stage; a stage that
// may have met (b) -- and one whose values are tiny enough that products
// could leave the fp32 normal range -- is recomputed from its starting
// accumulator with the reference's two roundings.  Exact zeros of the
// accumulator count as small (a harmless recompute); the first step of a
// chain starts from zero and is exact either way, so it runs before the
// tracked steps.
#include "common.cuh"
#include "launch.h"

namespace gptoss {

constexpr uint32_t kBf16InfPair = 0x7F807F80u;

// One step of a packed pair of chains: note |acc| in mn, then acc = bf16(acc + t*w).
__device__ __forceinline__ void rb_step(uint32_t& acc, uint32_t& mn, uint32_t t2, uint32_t w2) {
  asm("min.xorsign.abs.bf16x2 %0, %0, %1;" : "+r"(mn) : "r"(acc));
  asm("fma.rn.bf16x2 %0, %1, %2, %0;" : "+r"(acc) : "r"(t2), "r"(w2));
}

// The reference's step for a packed pair: fp32 FMA (exact product, one
// rounding to fp32), then round to bf16.
__device__ __forceinline__ uint32_t rb_step_exact(uint32_t acc, uint32_t t2, uint32_t w2) {
  const float lo = __fmaf_rn(__uint_as_float(t2 << 16), __uint_as_float(w2 << 16), __uint_as_float(acc << 16));
  const float hi = __fmaf_rn(__uint_as_float(t2 & 0xFFFF0000u), __uint_as_float(w2 & 0xFFFF0000u),
                             __uint_as_float(acc & 0xFFFF0000u));
  uint32_t d;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo));
  return d;
}

// The first step from a zero accumulator: bf16(t*w), exact on either path.
__device__ __forceinline__ uint32_t rb_first(uint32_t t2, uint32_t w2) {
  uint32_t acc = 0;
  asm("fma.rn.bf16x2 %0, %1, %2, %0;" : "+r"(acc) : "r"(t2), "r"(w2));
  return acc;
}

// Largest |value| of a bf16 pair word folded into m (bits of a
// non-negative bf16 in each half; the xorsign bit is cleared on use).
__device__ __forceinline__ void rb_absmax(uint32_t& m, uint32_t x) {
  asm("max.xorsign.abs.bf16x2 %0, %0, %1;" : "+r"(m) : "r"(x));
}

// Bound on 2^(e-24) for products of values up to |t| <= tmax, |w| <= wmax
// (bf16 bits, sign ignored), as bf16 bits: 0 when either side is all zero
// (no product can meet (b)), 0x7F80 (every accumulator counts as small, i.e.
// recompute) when the products may leave the fp32 normal range or a
// maximum is subnormal.
__device__ __forceinline__ uint32_t rb_bound(uint32_t tmax, uint32_t wmax) {
  tmax &= 0x7FFFu;
  wmax &= 0x7FFFu;
  if (tmax == 0 || wmax == 0) return 0u;
  const int et = (int)(tmax >> 7), ew = (int)(wmax >> 7);
  const int eb = et + ew - 150;  // biased exponent of 2^((et-127) + (ew-127) - 23)
  if (et == 0 || ew == 0 || eb < 8 || et + ew > 254 + 100) return 0x7F80u;
  return (uint32_t)eb << 7;
}

// Does a stage's minimum |accumulator| (pair mn) reach its bound (pair of bf16 bits)?
__device__ __forceinline__ bool rb_flag(uint32_t mn, uint32_t bound_lo, uint32_t bound_hi) {
  return (mn & 0x7FFFu) <= bound_lo || ((mn >> 16) & 0x7FFFu) <= bound_hi;
}

__device__ __forceinline__ uint32_t dup_lo(uint32_t x) { return prmt(x, x, 0x1010u); }
__device__ __forceinline__ uint32_t dup_hi(uint32_t x) { return prmt(x, x, 0x3232u); }

// =====================================================================
// Throughput form (many tokens).  A CTA covers kTok tokens x kBE experts;
// a thread owns kTT (1 or 2) tokens x 8 experts = 4 kTT packed chain pairs
// (adjacent experts share a register).  Per stage of kK k values the token
// values are staged duplicated ({t, t} words, k-major) and the expert values
// as pairs ({w_e, w_e+1} words, k-major), with the largest |t| and |w| of
// each 8-value piece of a row for the bounds.
//
// The stage's bound test runs first for the thread as a whole: one bound
// from the largest exponents of its tokens and experts, against the
// smallest |accumulator| of all its chains -- a superset of the per-chain
// tests, with the per-chain form (and the reruns) only behind it.

// 16-bit lane-wise max / min of non-negative bf16 bit patterns (the integer
// order is the numeric order there).
__device__ __forceinline__ uint32_t rb_max2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("max.u16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ uint32_t rb_min2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("min.u16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
// Zero halves raised to 0xFFFF (out of the way of a minimum over nonzeros).
__device__ __forceinline__ uint32_t rb_nz(uint32_t x) { return x | __vcmpeq2(x, 0u); }

// The thread-wide test.  tw: halves = stage maxima of the thread's tokens
// (kTT = 1: the high half is 0); w4: halves = stage maxima of its 8
// experts; mn_min: the smallest |accumulator| (bf16 bits) of its chains.
// True when some chain of the thread may need the rerun: a nonzero product
// whose bound rb_bound makes "always" (subnormal maxima, exponent sums
// below 158 or above 354) or an accumulator at or below the largest bound.
__device__ __forceinline__ bool rb_thread_flag(uint32_t tw, const uint32_t (&w4)[4], uint32_t mn_min) {
  const uint32_t wmx = rb_max2(rb_max2(w4[0], w4[1]), rb_max2(w4[2], w4[3]));
  const uint32_t tmax = max(tw & 0xFFFFu, tw >> 16), wmax = max(wmx & 0xFFFFu, wmx >> 16);
  if (tmax == 0 || wmax == 0) return false;  // every product of the stage is zero
  const uint32_t wn = rb_min2(rb_min2(rb_nz(w4[0]), rb_nz(w4[1])), rb_min2(rb_nz(w4[2]), rb_nz(w4[3])));
  const uint32_t tn2 = rb_nz(tw);
  const int etn = (int)(min(tn2 & 0xFFFFu, tn2 >> 16) >> 7), ewn = (int)(min(wn & 0xFFFFu, wn >> 16) >> 7);
  const int et = (int)(tmax >> 7), ew = (int)(wmax >> 7);
  if (etn == 0 || ewn == 0 || etn + ewn < 158 || et + ew > 254 + 100) return true;
  return mn_min <= (uint32_t)(et + ew - 150) << 7;
}

template <int kBE, int kTT, int kK>
struct RbCfg {
  static constexpr int kParts = kK / 8;                // 16-byte pieces per row per stage
  static constexpr int kEGroups = kBE / 8;             // expert groups of 8 per CTA
  static constexpr int kTGroups = 128 / kEGroups;      // token groups of kTT per CTA
  static constexpr int kTok = kTT * kTGroups;          // tokens per CTA
  static constexpr int kPairs = kBE / 2;
  static constexpr int kTPitch = kTok + 2;             // words per staged k row (8-byte aligned rows)
  static constexpr int kWPitch = kPairs + 4;           // words per staged k row (16-byte aligned rows)
  static constexpr int kTPieces = kTok * kParts / 128;  // token pieces per thread
  static constexpr int kWAll = kPairs * kParts;         // pair pieces per CTA
  static constexpr int kWPieces = (kWAll + 127) / 128;  // pair pieces per thread (the last may be partial)
  static_assert(kBE == 8 || kBE == 16 || kBE == 32 || kBE == 64, "experts per CTA");
  static_assert((kTT == 1 || kTT == 2) && kTPieces >= 1 && kTok * kParts % 128 == 0, "tokens per thread");
  static_assert(kK == 32 || kK == 64, "stage depth");
};

template <int kBE, int kTT, int kK>
__global__ void __launch_bounds__(128) router_bf16_kernel(const uint16_t* __restrict__ t,
                                                          const uint16_t* __restrict__ W,
                                                          const uint16_t* __restrict__ b, int64_t M, int32_t E,
                                                          int32_t H, uint16_t* __restrict__ logits) {
  using C = RbCfg<kBE, kTT, kK>;
  __shared__ __align__(16) uint32_t ts[kK][C::kTPitch];
  __shared__ __align__(16) uint32_t ws[kK][C::kWPitch];
  __shared__ __align__(16) uint16_t tmx[C::kParts][C::kTok];
  __shared__ __align__(16) uint16_t wmx[C::kParts][kBE];
  const int tid = threadIdx.x;
  const int tg = tid % C::kTGroups, eg = tid / C::kTGroups;
  const int64_t tok0 = (int64_t)blockIdx.x * C::kTok;
  const int32_t e0 = blockIdx.y * kBE;

  uint4 tq[C::kTPieces], wq0[C::kWPieces], wq1[C::kWPieces];
  auto load_stage = [&](int32_t k0) {
#pragma unroll
    for (int q = 0; q < C::kTPieces; ++q) {
      const int j = tid + 128 * q;
      const int tok = j % C::kTok, part = j / C::kTok;
      const int64_t m = tok0 + tok;
      tq[q] = make_uint4(0, 0, 0, 0);
      if (m < M && k0 + part * 8 < H) tq[q] = *(const uint4*)(t + m * H + k0 + part * 8);
    }
#pragma unroll
    for (int q = 0; q < C::kWPieces; ++q) {
      const int j = tid + 128 * q;
      const int pr = j % C::kPairs, part = j / C::kPairs;
      const int32_t e = e0 + 2 * pr;
      wq0[q] = wq1[q] = make_uint4(0, 0, 0, 0);
      if (j < C::kWAll && k0 + part * 8 < H) {
        wq0[q] = *(const uint4*)(W + (int64_t)e * H + k0 + part * 8);
        wq1[q] = *(const uint4*)(W + (int64_t)(e + 1) * H + k0 + part * 8);
      }
    }
  };
  auto store_stage = [&]() {
#pragma unroll
    for (int q = 0; q < C::kTPieces; ++q) {
      const int j = tid + 128 * q;
      const int tok = j % C::kTok, part = j / C::kTok;
      const uint32_t v[4] = {tq[q].x, tq[q].y, tq[q].z, tq[q].w};
      uint32_t mx = 0;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        ts[part * 8 + 2 * i][tok] = dup_lo(v[i]);
        ts[part * 8 + 2 * i + 1][tok] = dup_hi(v[i]);
        rb_absmax(mx, v[i]);
      }
      mx &= 0x7FFF7FFFu;
      tmx[part][tok] = (uint16_t)max(mx & 0xFFFFu, mx >> 16);
    }
#pragma unroll
    for (int q = 0; q < C::kWPieces; ++q) {
      const int j = tid + 128 * q;
      if (j < C::kWAll) {
        const int pr = j % C::kPairs, part = j / C::kPairs;
        const uint32_t a[4] = {wq0[q].x, wq0[q].y, wq0[q].z, wq0[q].w};
        const uint32_t c[4] = {wq1[q].x, wq1[q].y, wq1[q].z, wq1[q].w};
        uint32_t ma = 0, mc = 0;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          ws[part * 8 + 2 * i][pr] = prmt(a[i], c[i], 0x5410u);      // {w_e[k], w_e+1[k]}
          ws[part * 8 + 2 * i + 1][pr] = prmt(a[i], c[i], 0x7632u);  // {w_e[k+1], w_e+1[k+1]}
          rb_absmax(ma, a[i]);
          rb_absmax(mc, c[i]);
        }
        ma &= 0x7FFF7FFFu;
        mc &= 0x7FFF7FFFu;
        wmx[part][2 * pr] = (uint16_t)max(ma & 0xFFFFu, ma >> 16);
        wmx[part][2 * pr + 1] = (uint16_t)max(mc & 0xFFFFu, mc >> 16);
      }
    }
  };
  auto load_t = [&](int kk, uint32_t (&t2)[kTT]) {
    if constexpr (kTT == 2) {
      const uint2 tv = *(const uint2*)&ts[kk][2 * tg];
      t2[0] = tv.x;
      t2[1] = tv.y;
    } else {
      t2[0] = ts[kk][tg];
    }
  };

  uint32_t acc[kTT][4];
  load_stage(0);
  for (int32_t k0 = 0; k0 < H; k0 += kK) {
    __syncthreads();
    store_stage();
    __syncthreads();
    if (k0 + kK < H) load_stage(k0 + kK);  // the next stage's loads overlap this stage's chains
    const int32_t kn = min(kK, H - k0);
    int32_t kk0 = 0;
    if (k0 == 0) {
      uint32_t t2[kTT];
      load_t(0, t2);
      const uint4 wv = *(const uint4*)&ws[0][4 * eg];
      const uint32_t w2[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
      for (int i = 0; i < kTT; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = rb_first(t2[i], w2[j]);
      kk0 = 1;
    }
    uint32_t save[kTT][4], mn[kTT][4];
#pragma unroll
    for (int i = 0; i < kTT; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        save[i][j] = acc[i][j];
        mn[i][j] = kBf16InfPair;
      }
#pragma unroll 8
    for (int32_t kk = kk0; kk < kn; ++kk) {
      uint32_t t2[kTT];
      load_t(kk, t2);
      const uint4 wv = *(const uint4*)&ws[kk][4 * eg];
      const uint32_t w2[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
      for (int i = 0; i < kTT; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) rb_step(acc[i][j], mn[i][j], t2[i], w2[j]);
    }
    // the stage's bounds: the thread-wide test, then per chain pair; a chain
    // pair that may have met the double-rounding case reruns the stage with
    // the reference's two roundings
    uint32_t tw = 0, w4[4] = {0, 0, 0, 0}, mall = kBf16InfPair;
#pragma unroll
    for (int pp = 0; pp < C::kParts; ++pp) {
      if constexpr (kTT == 2) {
        tw = rb_max2(tw, *(const uint32_t*)&tmx[pp][2 * tg]);
      } else {
        tw = rb_max2(tw, (uint32_t)tmx[pp][tg]);
      }
      const uint4 wv = *(const uint4*)&wmx[pp][8 * eg];
      w4[0] = rb_max2(w4[0], wv.x);
      w4[1] = rb_max2(w4[1], wv.y);
      w4[2] = rb_max2(w4[2], wv.z);
      w4[3] = rb_max2(w4[3], wv.w);
    }
#pragma unroll
    for (int i = 0; i < kTT; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) asm("min.xorsign.abs.bf16x2 %0, %0, %1;" : "+r"(mall) : "r"(mn[i][j]));
    mall &= 0x7FFF7FFFu;
    if (rb_thread_flag(tw, w4, min(mall & 0xFFFFu, mall >> 16))) {
#pragma unroll
      for (int i = 0; i < kTT; ++i) {
        const int tok = kTT * tg + i;
        const uint32_t tm = kTT == 2 ? (i ? tw >> 16 : tw & 0xFFFFu) : tw;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const uint32_t wpair = w4[j];
          if (rb_flag(mn[i][j], rb_bound(tm, wpair & 0xFFFFu), rb_bound(tm, wpair >> 16))) {
            uint32_t a = save[i][j];
            for (int32_t kk = kk0; kk < kn; ++kk) a = rb_step_exact(a, ts[kk][tok], ws[kk][4 * eg + j]);
            acc[i][j] = a;
          }
        }
      }
    }
  }
#pragma unroll
  for (int i = 0; i < kTT; ++i) {
    const int64_t m = tok0 + kTT * tg + i;
    if (m >= M) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int32_t e = e0 + 8 * eg + 2 * j;
      const float a0 = __uint_as_float(acc[i][j] << 16), a1 = __uint_as_float(acc[i][j] & 0xFFFF0000u);
      logits[m * E + e] = f32_to_bf16_bits(__fadd_rn(a0, bf16_bits_to_f32(b[e])));
      logits[m * E + e + 1] = f32_to_bf16_bits(__fadd_rn(a1, bf16_bits_to_f32(b[e + 1])));
    }
  }
}

// =====================================================================
// Latency form (few tokens: decode).  One chain per thread: the step is a
// scalar fma.rn.bf16 (no operand permutes) and its latency, not issue,
// sets the pace.  A CTA covers 16 tokens x 16 experts: warps 0-7 run the
// chains, thread (tok, e) = (tid / 16, tid % 16); warps 8-11 bring in the
// whole rows -- lane r of warp 8 issues one bulk copy of row r (16 token
// rows, then 16 expert rows; few large copies keep the copy engine's
// per-request cost off the critical path), completing on the row's own
// mbarrier -- and then compute, chunk of 256 k by chunk, the per-row largest
// |value| for the bounds (an mbarrier per chunk).  A chain starts as soon
// as its two rows are in; the rows stay resident, so a flagged chunk is
// rerun from shared memory.
constexpr int kRcTok = 16, kRcExp = 16, kRcK = 256, kRcMaxChunks = 14;
constexpr int kRcMaxH = kRcMaxChunks * kRcK;  // 32 resident rows of 3584 + 8 values fit in 227 KB
constexpr int kRcThreads = 384;

__host__ __device__ constexpr int rc_pitch(int H) { return H + 8; }  // elements; rows shift by 4 banks
static size_t rc_smem_bytes(int H) { return (size_t)2 * 16 * rc_pitch(H) * 2 + (32 + kRcMaxChunks) * 8; }

__device__ __forceinline__ uint16_t rb_lo(uint32_t x) { return (uint16_t)(x & 0xFFFFu); }
__device__ __forceinline__ uint16_t rb_hi(uint32_t x) { return (uint16_t)(x >> 16); }

// One scalar step: note |acc| in mn, then acc = bf16(acc + t*w).
__device__ __forceinline__ void rb_step1(uint16_t& acc, uint16_t& mn, uint16_t t, uint16_t w) {
  asm("min.xorsign.abs.bf16 %0, %0, %1;" : "+h"(mn) : "h"(acc));
  asm("fma.rn.bf16 %0, %1, %2, %0;" : "+h"(acc) : "h"(t), "h"(w));
}
// Eight steps over 8 values of a token row and an expert row, in order.
__device__ __forceinline__ void rc_steps8(uint16_t& acc, uint16_t& mn, const uint4 tv, const uint4 wv) {
  const uint32_t tw[4] = {tv.x, tv.y, tv.z, tv.w}, ww[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    rb_step1(acc, mn, rb_lo(tw[i]), rb_lo(ww[i]));
    rb_step1(acc, mn, rb_hi(tw[i]), rb_hi(ww[i]));
  }
}
__device__ __forceinline__ uint16_t rb_step1_exact(uint16_t acc, uint16_t t, uint16_t w) {
  const float f = __fmaf_rn(__uint_as_float((uint32_t)t << 16), __uint_as_float((uint32_t)w << 16),
                            __uint_as_float((uint32_t)acc << 16));
  uint32_t d;
  asm("cvt.rn.bf16x2.f32 %0, %1, %1;" : "=r"(d) : "f"(f));
  return (uint16_t)d;
}

__global__ void __launch_bounds__(kRcThreads, 1) router_bf16_chain_kernel(const uint16_t* __restrict__ t,
                                                                       const uint16_t* __restrict__ W,
                                                                       const uint16_t* __restrict__ b, int64_t M,
                                                                       int32_t E, int32_t H,
                                                                       uint16_t* __restrict__ logits,
                                                                       uint32_t* err) {
  extern __shared__ __align__(16) uint8_t rc_smem[];
  const int pitch = rc_pitch(H);
  uint16_t* ts = (uint16_t*)rc_smem;                 // [16][pitch] token rows
  uint16_t* ws = ts + 16 * pitch;                    // [16][pitch] expert rows
  uint64_t* landed = (uint64_t*)(ws + 16 * pitch);   // [32] the row in shared memory
  uint64_t* bounded = landed + 32;                   // [chunks] the chunk's row maxima written
  __shared__ uint16_t tmx[kRcMaxChunks][kRcTok], wmx[kRcMaxChunks][kRcExp];
  const int tid = threadIdx.x;
  const int64_t m0 = (int64_t)blockIdx.y * kRcTok;
  const int32_t e0 = blockIdx.x * kRcExp;
  const int nch = (H + kRcK - 1) / kRcK;

  if (tid == 0) {
    for (int r = 0; r < 32; ++r) mbar_init(&landed[r], 1);
    for (int c = 0; c < nch; ++c) mbar_init(&bounded[c], 4);
    fence_mbar_init();
  }
  __syncthreads();

  if (tid >= 256) {
    const int j = tid - 256;
    if (j < 32) {
      // ---- lane r: the bulk copies of row r (a row past M or E copies nothing)
      const int r = j;
      const bool is_t = r < 16;
      const bool valid = is_t ? (m0 + r < M) : (e0 + r - 16 < E);
      const uint16_t* src = is_t ? t + (m0 + r) * H : W + (int64_t)(e0 + r - 16) * H;
      uint16_t* dst = is_t ? ts + r * pitch : ws + (r - 16) * pitch;
      if (valid) {
        const uint32_t bytes = (uint32_t)H * 2u;
        mbar_arrive_expect_tx(&landed[r], bytes);
        asm volatile(
            "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(dst)),
            "l"(src), "r"(bytes), "r"(smem_u32(&landed[r]))
            : "memory");
      } else {
        mbar_arrive(&landed[r]);
      }
    }
    // ---- row maxima of each chunk: 4 threads per row, 64 values each
    const int r = j >> 2, s = j & 3;
    const bool ok = mbar_wait(&landed[r], 0, err, kErrTimeoutOther);
    for (int c = 0; c < nch; ++c) {
      const int32_t k0 = c * kRcK, kn = min(kRcK, H - k0);
      uint32_t mx = 0;
      if (ok) {
        const uint16_t* row = (r < 16 ? ts + r * pitch : ws + (r - 16) * pitch) + k0;
        for (int32_t k = s * 8; k < kn; k += 32) {
          const uint4 v = *(const uint4*)(row + k);
          rb_absmax(mx, v.x);
          rb_absmax(mx, v.y);
          rb_absmax(mx, v.z);
          rb_absmax(mx, v.w);
        }
      }
      mx &= 0x7FFF7FFFu;
      mx = max(mx & 0xFFFFu, mx >> 16);
      mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      if (s == 0) {
        if (r < 16) tmx[c][r] = (uint16_t)(ok ? mx : 0x7F80u);
        else wmx[c][r - 16] = (uint16_t)(ok ? mx : 0x7F80u);
      }
      __syncwarp();
      if ((tid & 31) == 0) mbar_arrive(&bounded[c]);
    }
    return;
  }

  // ---- chain warps
  const int tok = tid >> 4, e = tid & 15;
  const int64_t m = m0 + tok;
  if (m >= M || e0 + e >= E) return;
  const uint16_t* trow = ts + tok * pitch;
  const uint16_t* wrow = ws + e * pitch;
  uint16_t acc = 0;
  if (!mbar_wait(&landed[tok], 0, err, kErrTimeoutOther) || !mbar_wait(&landed[16 + e], 0, err, kErrTimeoutOther))
    return;
  for (int c = 0; c < nch; ++c) {
    const int32_t k0 = c * kRcK, kend = k0 + min(kRcK, H - k0);
    int32_t kk = k0;
    if (c == 0) {
      asm("fma.rn.bf16 %0, %1, %2, %0;" : "+h"(acc) : "h"(trow[0]), "h"(wrow[0]));  // from zero: exact
      kk = 1;
    }
    const int32_t kbeg = kk;
    const uint16_t save = acc;
    uint16_t mn = 0x7F80u;
    for (; kk < kend && (kk & 7); ++kk) rb_step1(acc, mn, trow[kk], wrow[kk]);
    if (kk < kend) {
      // (kk and kend are multiples of 8 here) batches of 4 pieces of each
      // row in two register sets, the next batch's loads issued before this
      // one's steps: loads one piece ahead cost ~1.5 cycles a step
      const uint4* t4 = (const uint4*)(trow + kk);
      const uint4* w4 = (const uint4*)(wrow + kk);
      const int n8 = (kend - kk) >> 3;
      constexpr int kNb = 4;
      int i8 = 0;
      if (n8 >= 2 * kNb) {
        uint4 TA[kNb], WA[kNb], TB[kNb], WB[kNb];
#pragma unroll
        for (int j = 0; j < kNb; ++j) TA[j] = t4[j], WA[j] = w4[j];
        for (; i8 + 2 * kNb <= n8; i8 += 2 * kNb) {
#pragma unroll
          for (int j = 0; j < kNb; ++j) TB[j] = t4[i8 + kNb + j], WB[j] = w4[i8 + kNb + j];
#pragma unroll
          for (int j = 0; j < kNb; ++j) rc_steps8(acc, mn, TA[j], WA[j]);
          if (i8 + 3 * kNb <= n8) {
#pragma unroll
            for (int j = 0; j < kNb; ++j) TA[j] = t4[i8 + 2 * kNb + j], WA[j] = w4[i8 + 2 * kNb + j];
          }
#pragma unroll
          for (int j = 0; j < kNb; ++j) rc_steps8(acc, mn, TB[j], WB[j]);
        }
      }
      for (; i8 < n8; ++i8) rc_steps8(acc, mn, t4[i8], w4[i8]);
    }
    if (!mbar_wait(&bounded[c], 0, err, kErrTimeoutOther)) return;
    if (((uint32_t)mn & 0x7FFFu) <= rb_bound(tmx[c][tok], wmx[c][e])) {
      uint16_t a = save;
      for (int32_t k = kbeg; k < kend; ++k) a = rb_step1_exact(a, trow[k], wrow[k]);
      acc = a;
    }
  }
  const int32_t eg = e0 + e;
  logits[m * E + eg] = f32_to_bf16_bits(__fadd_rn(__uint_as_float((uint32_t)acc << 16), bf16_bits_to_f32(b[eg])));
}

// ------------------------------------------------------------------ host --

template <int kBE, int kTT, int kK>
static void launch_rb(const uint16_t* t, const uint16_t* W, const uint16_t* b, int64_t M, int32_t E, int32_t H,
                      uint16_t* logits, cudaStream_t s) {
  using C = RbCfg<kBE, kTT, kK>;
  dim3 grid((unsigned)((M + C::kTok - 1) / C::kTok), (unsigned)(E / kBE));
  router_bf16_kernel<kBE, kTT, kK><<<grid, 128, 0, s>>>(t, W, b, M, E, H, logits);
}

int launch_router_bf16(const uint16_t* t, const uint16_t* W, const uint16_t* b, int64_t M, int32_t E, int32_t H,
                       uint16_t* logits, uint32_t* err, cudaStream_t s) {
  if (M <= 0) return 0;
  if (E % 8 || E > 1024 || H % 8 || H <= 0 || ((uintptr_t)t & 15) || ((uintptr_t)W & 15)) return -12;
  // The latency form while its CTAs (one per SM) fit in two waves; past
  // that the throughput form, whose time grows more slowly with M.
  const int64_t sms = device_sm_count();
  const int64_t chain_ctas = ((E + kRcExp - 1) / kRcExp) * ((M + kRcTok - 1) / kRcTok);
  if (chain_ctas <= 2 * sms && H <= kRcMaxH) {
    static FuncSmemAttr attr;
    ensure_dyn_smem(attr, (const void*)router_bf16_chain_kernel, (int)rc_smem_bytes(kRcMaxH));
    dim3 grid((unsigned)((E + kRcExp - 1) / kRcExp), (unsigned)((M + kRcTok - 1) / kRcTok));
    router_bf16_chain_kernel<<<grid, kRcThreads, rc_smem_bytes(H), s>>>(t, W, b, M, E, H, logits, err);
  } else {
    // two tokens a thread (each staged value feeds more chains) once that
    // gives 1.5 CTAs per SM; one token a thread (twice the CTAs) below that
    auto ctas = [&](int be, int tt) { return ((M + tt * 1024 / be - 1) / (tt * 1024 / be)) * (E / be); };
    if (E % 64 == 0 && 2 * ctas(64, 2) >= 3 * sms) {
      launch_rb<64, 2, 64>(t, W, b, M, E, H, logits, s);
    } else if (E % 32 == 0 && 2 * ctas(32, 2) >= 3 * sms) {
      launch_rb<32, 2, 64>(t, W, b, M, E, H, logits, s);
    } else if (E % 32 == 0) {
      launch_rb<32, 1, 64>(t, W, b, M, E, H, logits, s);
    } else if (E % 16 == 0 && 2 * ctas(16, 2) >= 3 * sms) {
      launch_rb<16, 2, 64>(t, W, b, M, E, H, logits, s);
    } else if (E % 16 == 0) {
      launch_rb<16, 1, 64>(t, W, b, M, E, H, logits, s);
    } else {
      launch_rb<8, 1, 32>(t, W, b, M, E, H, logits, s);
    }
  }
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

}  // namespace gptoss
