// moe_route.cu -- the token side of the MoE block: RMSNorm, the router
// (bit-exact to the reference's serial bf16 accumulation), top-k + softmax,
// the expert-major permutation, the activation gather and the weighted
// combine with the residual.  All integer/index work is bit-exact; the
// floating-point steps reproduce the reference's operation order and
// rounding (no contraction: __fmul_rn/__fadd_rn where the reference has
// separate multiply and add).
#include <cstdlib>

#include "common.cuh"
#include "launch.h"

namespace gptoss {

// ------------------------------------------------------------ RMSNorm --
// nn.RMSNorm as lowered for model/mlp.py:81-87,375 (and attention.py:84,193):
// serial fp32 sum of squares in column order, r = 1/sqrtf(sum/H + eps),
// out = bf16((r*x)*w).  A block brings up to 16 whole token rows into shared
// memory with one bulk copy each; one thread per token runs the serial sum,
// then the whole block writes the normalised rows.
constexpr int kNormRows = 16;
__global__ void __launch_bounds__(128) rmsnorm_kernel(const uint16_t* __restrict__ x, const uint16_t* __restrict__ w,
                                                       int64_t M, int32_t H, int32_t rows_per_block, float eps,
                                                       uint16_t* __restrict__ out, uint32_t* err) {
  extern __shared__ __align__(16) uint8_t norm_smem[];
  __shared__ uint64_t bar;
  __shared__ float rs[kNormRows];
  uint16_t* rowbuf = (uint16_t*)norm_smem;
  const int32_t pitch = H + 8;  // padded row pitch (elements): rows start on different banks
  const int64_t m0 = (int64_t)blockIdx.x * rows_per_block;
  const int64_t left = M - m0;
  const int nrows = left < rows_per_block ? (int)left : rows_per_block;
  const uint32_t row_bytes = (uint32_t)H * 2;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    mbar_arrive_expect_tx(&bar, row_bytes * (uint32_t)nrows);
    for (int r = 0; r < nrows; ++r) {
      asm volatile(
          "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
              smem_u32(rowbuf + (size_t)r * pitch)),
          "l"(x + (m0 + r) * H), "r"(row_bytes), "r"(smem_u32(&bar))
          : "memory");
    }
  }
  const bool ok = mbar_wait(&bar, 0, err, kErrTimeoutOther);
  if (ok && threadIdx.x < nrows) {
    const uint4* row = (const uint4*)(rowbuf + (size_t)threadIdx.x * pitch);
    float ss = 0.0f;
    // the next 8 elements are read while the sum runs through these 8
    uint4 vn = row[0];
#pragma unroll 4
    for (int32_t k8 = 0; k8 < H / 8; ++k8) {
      const uint4 v = vn;
      if (k8 + 1 < H / 8) vn = row[k8 + 1];
      const uint32_t wv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float a = __uint_as_float(wv[q] << 16), b = __uint_as_float(wv[q] & 0xFFFF0000u);
        ss = __fadd_rn(ss, __fmul_rn(a, a));
        ss = __fadd_rn(ss, __fmul_rn(b, b));
      }
    }
    rs[threadIdx.x] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)H), eps)));
  }
  __syncthreads();
  if (!ok) return;
  const int32_t h2 = H / 2;
  for (int r = 0; r < nrows; ++r) {
    const float rr = rs[r];
    const uint32_t* src = (const uint32_t*)(rowbuf + (size_t)r * pitch);
    uint32_t* dst = (uint32_t*)(out + (m0 + r) * H);
    for (int32_t j = threadIdx.x; j < h2; j += blockDim.x) {
      const uint32_t v = src[j];
      const uint32_t wv = __ldg((const uint32_t*)w + j);
      const float a = __fmul_rn(__fmul_rn(rr, __uint_as_float(v << 16)), __uint_as_float(wv << 16));
      const float b = __fmul_rn(__fmul_rn(rr, __uint_as_float(v & 0xFFFF0000u)), __uint_as_float(wv & 0xFFFF0000u));
      dst[j] = (uint32_t)f32_to_bf16_bits(a) | ((uint32_t)f32_to_bf16_bits(b) << 16);
    }
  }
}

// Streaming form: every row's chain starts as soon as its first 256 values
// are in.  A CTA takes rows_per_cta (<= 32) rows; lane r of warp 0 runs row
// r's serial sum over `stages` chunk slots, each chunk of each row one bulk
// copy on the slot's mbarrier.  Few rows per CTA (decode): one slot per
// chunk, the rows stay resident and the block writes the normalised rows
// from shared memory.  Many rows: a ring of kNsStages slots, each refilled
// by the same warp once its lanes have read it, so up to 32 rows per CTA
// and three CTAs per SM run their chains at once (all 8192 rows of a
// prefill in one wave); the block then writes the normalised rows from a
// second, L2-resident read of x.
// ss += x*x over the 8 bf16 values of v, in order (fp32 products and sums,
// each rounded as the reference's serial loop rounds them).
__device__ __forceinline__ void ns_sq8(float& ss, const uint4 v) {
  const uint32_t wv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const float a = __uint_as_float(wv[q] << 16), b = __uint_as_float(wv[q] & 0xFFFF0000u);
    ss = __fadd_rn(ss, __fmul_rn(a, a));
    ss = __fadd_rn(ss, __fmul_rn(b, b));
  }
}

constexpr int kNsChunk = 256;                // values per row per stageconstexpr int kNsChunk = 256;                // values per row per stage
constexpr int kNsStages = 4;                 // ring slots
constexpr int kNsMaxSlots = 16;              // resident rows: H <= 4096
constexpr int kNsResidentBytes = 100 * 1024;
constexpr int kNsMaxRows = 32;
constexpr int kNsPitch = kNsChunk * 2 + 16;  // bytes per row slot: rows start 4 banks apart

__global__ void __launch_bounds__(256) rmsnorm_stream_kernel(const uint16_t* __restrict__ x,
                                                              const uint16_t* __restrict__ w, int64_t M, int32_t H,
                                                              int32_t rows_per_cta, int32_t stages, float eps,
                                                              uint16_t* __restrict__ out, uint32_t* err) {
  extern __shared__ __align__(128) uint8_t ns_smem[];  // [stages][rows_per_cta][kNsPitch]
  __shared__ uint64_t bar[kNsMaxSlots];
  __shared__ float rs[kNsMaxRows];
  __shared__ int all_ok;
  const int64_t m0 = (int64_t)blockIdx.x * rows_per_cta;
  const int nrows = (int)min64(rows_per_cta, M - m0);
  const int nch = (H + kNsChunk - 1) / kNsChunk;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x < stages) mbar_init(&bar[threadIdx.x], 1);
  if (threadIdx.x == 0) all_ok = 1;
  fence_mbar_init();
  __syncthreads();
  if (warp != 0) {
    // the other warps bring the norm weight into L2 while the chains run (its
    // loads come right after the chains; from HBM they would add their
    // latency to every decode-size call)
    for (int32_t i = threadIdx.x - 32; i < H / 64; i += blockDim.x - 32)
      asm volatile("prefetch.global.L2 [%0];" ::"l"(w + (size_t)i * 64));
  }
  if (warp == 0) {
    auto slot_row = [&](int c, int r) { return ns_smem + ((size_t)(c % stages) * rows_per_cta + r) * kNsPitch; };
    auto issue = [&](int c) {
      const int32_t k0 = c * kNsChunk;
      const uint32_t bytes = (uint32_t)min(kNsChunk, H - k0) * 2;
      uint64_t* b = &bar[c % stages];
      if (lane == 0) mbar_arrive_expect_tx(b, bytes * (uint32_t)nrows);
      if (lane < nrows)
        asm volatile(
            "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                smem_u32(slot_row(c, lane))),
            "l"(x + (m0 + lane) * H + k0), "r"(bytes), "r"(smem_u32(b))
            : "memory");
    };
    const int first = min(nch, stages);
    for (int c = 0; c < first; ++c) issue(c);
    int issued = first, c = 0;
    bool ok = true;
    float ss = 0.0f;
    for (; c < nch; ++c) {
      // (warp-uniform: every lane leaves the loop together)
      if (!__all_sync(0xffffffffu, mbar_wait(&bar[c % stages], (uint32_t)(c / stages) & 1u, err,
                                             kErrTimeoutOther))) {
        ok = false;
        break;
      }
      if (lane < nrows) {
        const uint4* row = (const uint4*)slot_row(c, lane);
        const int n8 = min(kNsChunk, H - c * kNsChunk) / 8;
        // batches of 8 pieces (64 values) in two register sets, the next
        // batch's loads issued before this one's adds (loads interleaved one
        // piece ahead cost ~1.2 extra cycles per value on the chain)
        constexpr int kNb = 8;
        int k8 = 0;
        if (n8 >= 2 * kNb) {
          uint4 A[kNb], B[kNb];
#pragma unroll
          for (int j = 0; j < kNb; ++j) A[j] = row[j];
          for (; k8 + 2 * kNb <= n8; k8 += 2 * kNb) {
#pragma unroll
            for (int j = 0; j < kNb; ++j) B[j] = row[k8 + kNb + j];
#pragma unroll
            for (int j = 0; j < kNb; ++j) ns_sq8(ss, A[j]);
            if (k8 + 3 * kNb <= n8) {
#pragma unroll
              for (int j = 0; j < kNb; ++j) A[j] = row[k8 + 2 * kNb + j];
            }
#pragma unroll
            for (int j = 0; j < kNb; ++j) ns_sq8(ss, B[j]);
          }
        }
        for (; k8 < n8; ++k8) ns_sq8(ss, row[k8]);
      }
      __syncwarp();
      if (c + stages < nch) {
        // the slot's reads (generic proxy) before the next bulk copy into it (async proxy)
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        issue(c + stages);
        ++issued;
      }
    }
    if (!ok) {
      // copies still in flight land before the CTA leaves (bounded waits)
      for (int d = c + 1; d < issued; ++d) mbar_wait(&bar[d % stages], (uint32_t)(d / stages) & 1u, err,
                                                     kErrTimeoutOther);
      if (lane == 0) all_ok = 0;
    }
    if (lane < nrows) rs[lane] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)H), eps)));
  }
  __syncthreads();
  if (!all_ok) return;
  if (stages >= nch)  // resident rows: every thread sees the copies' completion itself
    for (int c = 0; c < nch; ++c) mbar_wait(&bar[c], 0u, err, kErrTimeoutOther);
  // the CTA's rows are contiguous in x and out: one flat loop over their
  // 16-byte pieces, kNsUnroll loads in flight per thread; resident rows are
  // read back from their chunk slots
  constexpr int kNsUnroll = 8;
  const int32_t h8 = H / 8;
  const int32_t total = nrows * h8;
  const bool resident = stages >= nch;
  const uint4* src = (const uint4*)(x + m0 * H);
  uint4* dst = (uint4*)(out + m0 * H);
  for (int32_t i0 = threadIdx.x; i0 < total; i0 += blockDim.x * kNsUnroll) {
    uint4 v[kNsUnroll], wq[kNsUnroll];
#pragma unroll
    for (int u = 0; u < kNsUnroll; ++u) {
      const int32_t i = i0 + u * (int32_t)blockDim.x;
      if (i < total) {
        const int32_t r = i / h8, j = i - r * h8;
        v[u] = resident ? *(const uint4*)(ns_smem + ((size_t)(j / (kNsChunk / 8)) * rows_per_cta + r) * kNsPitch +
                                          (j % (kNsChunk / 8)) * 16)
                        : src[i];
        wq[u] = __ldg((const uint4*)w + j);
      }
    }
#pragma unroll
    for (int u = 0; u < kNsUnroll; ++u) {
      const int32_t i = i0 + u * (int32_t)blockDim.x;
      if (i < total) {
        const float rr = rs[i / h8];
        const uint32_t vv[4] = {v[u].x, v[u].y, v[u].z, v[u].w}, ww[4] = {wq[u].x, wq[u].y, wq[u].z, wq[u].w};
        uint32_t o[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float a = __fmul_rn(__fmul_rn(rr, __uint_as_float(vv[q] << 16)), __uint_as_float(ww[q] << 16));
          const float b = __fmul_rn(__fmul_rn(rr, __uint_as_float(vv[q] & 0xFFFF0000u)),
                                    __uint_as_float(ww[q] & 0xFFFF0000u));
          o[q] = (uint32_t)f32_to_bf16_bits(a) | ((uint32_t)f32_to_bf16_bits(b) << 16);
        }
        dst[i] = make_uint4(o[0], o[1], o[2], o[3]);
      }
    }
  }
}

// -------------------------------------------------------------- router --
// logits[m, e] = bf16(float(acc) + float(b[e])) where acc is a bf16 running
// sum: acc = bf16(float(acc) + t[m,k]*W[e,k]) for k = 0..H-1 in order
// (nn.Linear at model/mlp.py:88-92,376 lowered with a bf16 accumulator).
// t*W is exact in fp32, so fma(t, W, acc) == acc + t*W (one rounding to
// fp32, as in the reference), followed by the rounding to bf16.  Each
// thread owns a 4-token x 8-expert register tile of independent serial
// chains; two chains share one packed f32x2 FMA.
constexpr int kRTT = 2;   // tokens per thread
constexpr int kRTE = 8;   // experts per thread (a multiple of 4)
static_assert(kRTE % 4 == 0, "expert values load as 16-byte pairs");
constexpr int kRKT = 32;  // k per shared-memory stage (multiple of 8)

// bf16 rounding of two fp32 accumulators held as a packed pair: one cvt per
// value, whose zero low half leaves float(bf16(v)) in the register.
__device__ __forceinline__ unsigned long long round_pair_bf16(unsigned long long s) {
  uint32_t a, b;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(a) : "f"(__uint_as_float((uint32_t)s)), "f"(0.0f));
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(b) : "f"(__uint_as_float((uint32_t)(s >> 32))), "f"(0.0f));
  return ((unsigned long long)b << 32) | a;
}

// Above this many tokens the register-tiled kernel (throughput-bound) wins
// over one thread per chain pair (latency-bound).
constexpr int64_t kRouterChainMaxTokens = 512;

template <int kMaxTQ, int kMaxWQ>
__global__ void __launch_bounds__(128) router_kernel(const uint16_t* __restrict__ t, const uint16_t* __restrict__ W,
                                                      const uint16_t* __restrict__ b, int64_t M, int32_t E, int32_t H,
                                                      int32_t block_experts, uint16_t* __restrict__ logits) {
  extern __shared__ __align__(16) float rsm[];
  const int egroups = block_experts / kRTE;         // expert groups per block
  const int tgroups = 128 / egroups;                // token groups per block
  const int btok = tgroups * kRTT;                  // tokens per block
  float* ts = rsm;                                  // [kRKT][btok][2]  (each value twice)
  float* ws = ts + kRKT * btok * 2;                 // [kRKT][block_experts]
  const int tg = threadIdx.x % tgroups, eg = threadIdx.x / tgroups;
  const int64_t tok0 = (int64_t)blockIdx.x * btok;
  const int32_t e0 = blockIdx.y * block_experts;
  constexpr int kParts = kRKT / 8;                  // 16-byte pieces per row per stage
  const int ntq = (btok * kParts + 127) / 128, nwq = (block_experts * kParts + 127) / 128;
  uint4 tq[kMaxTQ], wq[kMaxWQ];
  auto load_stage = [&](int32_t k0) {
#pragma unroll
    for (int q = 0; q < kMaxTQ; ++q) {
      if (q >= ntq) break;
      const int j = threadIdx.x + 128 * q;
      const int tok = j / kParts, part = j % kParts;
      const int64_t m = tok0 + tok;
      tq[q] = make_uint4(0, 0, 0, 0);
      if (tok < btok && m < M && k0 + part * 8 < H) tq[q] = *(const uint4*)(t + m * H + k0 + part * 8);
    }
#pragma unroll
    for (int q = 0; q < kMaxWQ; ++q) {
      if (q >= nwq) break;
      const int j = threadIdx.x + 128 * q;
      const int e = j / kParts, part = j % kParts;
      wq[q] = make_uint4(0, 0, 0, 0);
      if (e < block_experts && e0 + e < E && k0 + part * 8 < H)
        wq[q] = *(const uint4*)(W + (int64_t)(e0 + e) * H + k0 + part * 8);
    }
  };
  auto store_stage = [&]() {
#pragma unroll
    for (int q = 0; q < kMaxTQ; ++q) {
      if (q >= ntq) break;
      const int j = threadIdx.x + 128 * q;
      const int tok = j / kParts, part = j % kParts;
      if (tok >= btok) continue;
      const uint32_t v[4] = {tq[q].x, tq[q].y, tq[q].z, tq[q].w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float lo = __uint_as_float(v[i] << 16), hi = __uint_as_float(v[i] & 0xFFFF0000u);
        *(float2*)(ts + ((part * 8 + 2 * i) * btok + tok) * 2) = make_float2(lo, lo);
        *(float2*)(ts + ((part * 8 + 2 * i + 1) * btok + tok) * 2) = make_float2(hi, hi);
      }
    }
#pragma unroll
    for (int q = 0; q < kMaxWQ; ++q) {
      if (q >= nwq) break;
      const int j = threadIdx.x + 128 * q;
      const int e = j / kParts, part = j % kParts;
      if (e >= block_experts) continue;
      const uint32_t v[4] = {wq[q].x, wq[q].y, wq[q].z, wq[q].w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        ws[(part * 8 + 2 * i) * block_experts + e] = __uint_as_float(v[i] << 16);
        ws[(part * 8 + 2 * i + 1) * block_experts + e] = __uint_as_float(v[i] & 0xFFFF0000u);
      }
    }
  };

  unsigned long long acc[kRTT][kRTE / 2];
#pragma unroll
  for (int i = 0; i < kRTT; ++i)
#pragma unroll
    for (int j = 0; j < kRTE / 2; ++j) acc[i][j] = 0ull;

  load_stage(0);
  for (int32_t k0 = 0; k0 < H; k0 += kRKT) {
    __syncthreads();
    store_stage();
    __syncthreads();
    if (k0 + kRKT < H) load_stage(k0 + kRKT);  // next stage's loads overlap this stage's chains
    const int32_t kn = min(kRKT, H - k0);
    for (int32_t kk = 0; kk < kn; ++kk) {
      // this thread's kRTT token values (each duplicated) and kRTE expert values
      unsigned long long tv[kRTT], wv[kRTE / 2];
      const unsigned long long* tp = (const unsigned long long*)(ts + (kk * btok + tg * kRTT) * 2);
#pragma unroll
      for (int i = 0; i < kRTT; i += 2) {
        if (i + 1 < kRTT) {
          const ulonglong2 v = *(const ulonglong2*)(tp + i);
          tv[i] = v.x;
          tv[i + 1] = v.y;
        } else {
          tv[i] = tp[i];
        }
      }
      const ulonglong2* wp = (const ulonglong2*)(ws + kk * block_experts + eg * kRTE);
#pragma unroll
      for (int q = 0; q < kRTE / 4; ++q) {
        const ulonglong2 v = wp[q];
        wv[2 * q] = v.x;
        wv[2 * q + 1] = v.y;
      }
#pragma unroll
      for (int i = 0; i < kRTT; ++i) {
#pragma unroll
        for (int j = 0; j < kRTE / 2; ++j) {
          unsigned long long sacc = acc[i][j];
          asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(sacc) : "l"(tv[i]), "l"(wv[j]));
          acc[i][j] = round_pair_bf16(sacc);
        }
      }
    }
  }
#pragma unroll
  for (int i = 0; i < kRTT; ++i) {
    const int64_t m = tok0 + tg * kRTT + i;
    if (m >= M) continue;
#pragma unroll
    for (int j = 0; j < kRTE / 2; ++j) {
      const int32_t e = e0 + eg * kRTE + 2 * j;
      if (e < E) {
        const float a0 = __uint_as_float((uint32_t)acc[i][j]);
        logits[m * E + e] = f32_to_bf16_bits(__fadd_rn(a0, bf16_bits_to_f32(b[e])));
      }
      if (e + 1 < E) {
        const float a1 = __uint_as_float((uint32_t)(acc[i][j] >> 32));
        logits[m * E + e + 1] = f32_to_bf16_bits(__fadd_rn(a1, bf16_bits_to_f32(b[e + 1])));
      }
    }
  }
}

// Few tokens (decode): the same serial chains, one per (token, expert), but
// spread over as many threads as there are chains -- the step latency of a
// chain (one packed FMA + one bf16 rounding), not ALU throughput, is the
// limit.  A block covers 16 tokens x 16 experts; thread (tok, p) runs the
// chains of experts p and p + 8 in one packed f32x2 accumulator.  Token and
// weight rows are staged through shared memory in k chunks with cp.async,
// double-buffered; the row pitch (kChainK + 8 elements) keeps the 16-byte
// reads of 8 different rows on distinct banks.
constexpr int kChainTok = 16, kChainExp = 16, kChainK = 256, kChainPitch = kChainK + 8;

__global__ void __launch_bounds__(128) router_chain_kernel(const uint16_t* __restrict__ t,
                                                            const uint16_t* __restrict__ W,
                                                            const uint16_t* __restrict__ b, int64_t M, int32_t E,
                                                            int32_t H, uint16_t* __restrict__ logits) {
  __shared__ __align__(16) uint16_t ts[2][kChainTok][kChainPitch];
  __shared__ __align__(16) uint16_t ws[2][kChainExp][kChainPitch];
  const int tok = threadIdx.x >> 3, p = threadIdx.x & 7;
  const int64_t m0 = (int64_t)blockIdx.y * kChainTok;
  const int32_t e0 = blockIdx.x * kChainExp;
  auto load = [&](int buf, int32_t k0) {
    const int32_t kn = min(kChainK, H - k0);
    const int parts = kn / 8;  // 16-byte pieces per row
    for (int j = threadIdx.x; j < 2 * 16 * parts; j += 128) {
      const int which = j / (16 * parts), rem = j % (16 * parts);
      const int r = rem / parts, q = rem % parts;
      const uint16_t* src = nullptr;
      uint16_t* dst;
      if (which == 0) {
        dst = &ts[buf][r][q * 8];
        if (m0 + r < M) src = t + (m0 + r) * H + k0 + q * 8;
      } else {
        dst = &ws[buf][r][q * 8];
        if (e0 + r < E) src = W + (int64_t)(e0 + r) * H + k0 + q * 8;
      }
      if (src)
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  unsigned long long acc = 0ull;
  load(0, 0);
  int buf = 0;
  for (int32_t k0 = 0; k0 < H; k0 += kChainK, buf ^= 1) {
    if (k0 + kChainK < H) {
      load(buf ^ 1, k0 + kChainK);
      asm volatile("cp.async.wait_group 1;" ::: "memory");
    } else {
      asm volatile("cp.async.wait_group 0;" ::: "memory");
    }
    __syncthreads();
    const int32_t kn = min(kChainK, H - k0);
    const uint16_t* trow = ts[buf][tok];
    const uint16_t* wa = ws[buf][p];
    const uint16_t* wb = ws[buf][p + 8];
    // the next 8 columns are read while the chain runs through these 8
    uint4 tn = *(const uint4*)trow, an = *(const uint4*)wa, bn = *(const uint4*)wb;
    for (int32_t kk = 0; kk < kn; kk += 8) {
      const uint4 tv = tn, av = an, bv = bn;
      if (kk + 8 < kn) {
        tn = *(const uint4*)(trow + kk + 8);
        an = *(const uint4*)(wa + kk + 8);
        bn = *(const uint4*)(wb + kk + 8);
      }
      const uint32_t tw[4] = {tv.x, tv.y, tv.z, tv.w};
      const uint32_t aw[4] = {av.x, av.y, av.z, av.w};
      const uint32_t bw[4] = {bv.x, bv.y, bv.z, bv.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const uint32_t tf = h ? (tw[i] & 0xFFFF0000u) : (tw[i] << 16);
          const uint32_t af = h ? (aw[i] & 0xFFFF0000u) : (aw[i] << 16);
          const uint32_t bf = h ? (bw[i] & 0xFFFF0000u) : (bw[i] << 16);
          const unsigned long long tp = ((unsigned long long)tf << 32) | tf;
          const unsigned long long wp = ((unsigned long long)bf << 32) | af;
          asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(acc) : "l"(tp), "l"(wp));
          acc = round_pair_bf16(acc);
        }
      }
    }
    __syncthreads();  // the buffer is refilled by the next iteration's load
  }
  const int64_t m = m0 + tok;
  if (m >= M) return;
  const int32_t ea = e0 + p, eb = e0 + p + 8;
  if (ea < E)
    logits[m * E + ea] = f32_to_bf16_bits(__fadd_rn(__uint_as_float((uint32_t)acc), bf16_bits_to_f32(b[ea])));
  if (eb < E)
    logits[m * E + eb] =
        f32_to_bf16_bits(__fadd_rn(__uint_as_float((uint32_t)(acc >> 32)), bf16_bits_to_f32(b[eb])));
}

// ------------------------------------------------------ top-k softmax --
// nn.op.topk(largest) + nn.op.softmax over the k values (model/mlp.py:381-382):
// value descending, ties to the lower expert index (+0 == -0); softmax with
// bf16 max, e_i = bf16(exp(v_i - max)), bf16 serial sum, w_i = bf16(e_i/sum).
// exp is evaluated in double and rounded once to float (the correctly
// rounded expf), matching a libm expf to the last bit in all but vanishingly
// rare cases.  One warp per token.
// One token's top-k + softmax by one warp (all lanes call; lane 0 writes
// weights[j], indices[j] for j < K and, when sidx is given, the indices to
// shared memory too).
__device__ __forceinline__ void topk_softmax_warp(const uint16_t* __restrict__ lg, int32_t E, int32_t K,
                                                  uint16_t* __restrict__ weights, int32_t* __restrict__ indices,
                                                  int32_t* sidx, uint32_t* err) {
  const int lane = threadIdx.x & 31;
  constexpr int kMaxPerLane = 8;  // E <= 256
  float v[kMaxPerLane];
  uint32_t taken = 0;
#pragma unroll
  for (int i = 0; i < kMaxPerLane; ++i) {
    const int32_t e = lane + 32 * i;
    v[i] = e < E ? bf16_bits_to_f32(lg[e]) : -INFINITY;
    if (e >= E) taken |= 1u << i;
  }
  float sel_v[8];
  int32_t sel_i[8];
  for (int j = 0; j < K; ++j) {
    float bv = 0.0f;
    int32_t bi = 0x7fffffff;
    bool have = false;
#pragma unroll
    for (int i = 0; i < kMaxPerLane; ++i) {
      if (taken & (1u << i)) continue;
      const int32_t e = lane + 32 * i;
      if (!have || v[i] > bv || (v[i] == bv && e < bi)) { bv = v[i]; bi = e; have = true; }
    }
    if (!have) { bv = -INFINITY; bi = 0x7fffffff; }
    for (int off = 16; off > 0; off >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
      const int32_t oi = __shfl_xor_sync(0xffffffffu, bi, off);
      if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
    }
    sel_v[j] = bv;
    sel_i[j] = bi;
    if ((bi & 31) == lane) taken |= 1u << (bi >> 5);
  }
  if (lane == 0) {
    float mx = round_bf16(-3.402823e+38f);
    for (int j = 0; j < K; ++j) mx = round_bf16(mx > sel_v[j] ? mx : sel_v[j]);
    float ex[8];
    for (int j = 0; j < K; ++j) ex[j] = round_bf16((float)exp((double)__fsub_rn(sel_v[j], mx)));
    float sum = 0.0f;
    for (int j = 0; j < K; ++j) sum = round_bf16(__fadd_rn(sum, ex[j]));
    for (int j = 0; j < K; ++j) {
      weights[j] = f32_to_bf16_bits(__fdiv_rn(ex[j], sum));
      indices[j] = sel_i[j];
      if (sidx) sidx[j] = sel_i[j];
      if (sel_i[j] < 0 || sel_i[j] >= E) raise_error(err, kErrBadRouting);
    }
  }
}

__global__ void topk_softmax_kernel(const uint16_t* __restrict__ logits, int64_t M, int32_t E, int32_t K,
                                    uint16_t* __restrict__ weights, int32_t* __restrict__ indices,
                                    uint32_t* err) {
  const int64_t m = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  if (m >= M) return;
  topk_softmax_warp(logits + m * E, E, K, weights + m * K, indices + m * K, nullptr, err);
}

// ------------------------------------------------------ permutation --
// Expert-major order of the (token, rank) pairs (the layout of the grouped
// kernels, model/mlp_optimized.py:118-170): rows of expert e occupy
// [indptr[e], indptr[e+1]) in ascending token order.  Also builds the token
// tiles the grouped GEMM walks: an expert with c rows gets ceil(c/T) tiles of
// roundup16(ceil(c/tiles)) rows, T = moe_tile_rows_max(all rows, experts).
// Stage 1 (one block): per-expert counts, exclusive scan, tile plan.
__global__ void __launch_bounds__(1024) moe_count_scan_kernel(const int32_t* __restrict__ idx, int64_t pairs, int32_t E,
                                                               int32_t* __restrict__ indptr,
                                                               int32_t* __restrict__ tile_ptr,
                                                               int32_t* __restrict__ tile_rows, uint32_t* err) {
  extern __shared__ int32_t cnt[];  // [E]
  for (int e = threadIdx.x; e < E; e += blockDim.x) cnt[e] = 0;
  __syncthreads();
  for (int64_t i = threadIdx.x; i < pairs; i += blockDim.x) {
    const int32_t e = idx[i];
    if (e >= 0 && e < E) atomicAdd(&cnt[e], 1);
    else raise_error(err, kErrBadRouting);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const int32_t tmax = moe_tile_rows_max(pairs, E);
    int32_t acc = 0, tacc = 0;
    for (int32_t e = 0; e < E; ++e) {
      const int32_t c = cnt[e];
      indptr[e] = acc;
      tile_ptr[e] = tacc;
      const int32_t nt = (c + tmax - 1) / tmax;
      const int32_t per = nt ? ((((c + nt - 1) / nt) + 15) & ~15) : 0;
      tile_rows[e] = per;
      acc += c;
      tacc += nt;
    }
    indptr[E] = acc;
    tile_ptr[E] = tacc;
  }
}

// Stage 2 (one block per expert): stable placement of the expert's pairs.
__global__ void __launch_bounds__(1024) moe_place_kernel(const int32_t* __restrict__ idx, int64_t pairs, int32_t K,
                                                          const int32_t* __restrict__ indptr,
                                                          int32_t* __restrict__ token_of_row,
                                                          int32_t* __restrict__ row_of_pair,
                                                          int32_t* __restrict__ expert_of_row) {
  __shared__ int32_t warp_tot[32];
  __shared__ int32_t running;
  const int32_t e = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) running = indptr[e];
  __syncthreads();
  for (int64_t base = 0; base < pairs; base += blockDim.x) {
    const int64_t i = base + threadIdx.x;
    const bool hit = i < pairs && idx[i] == e;
    const uint32_t bal = __ballot_sync(0xffffffffu, hit);
    if (lane == 0) warp_tot[warp] = __popc(bal);
    __syncthreads();
    int32_t before = 0;
    for (int w = 0; w < warp; ++w) before += warp_tot[w];
    const int32_t start = running;
    if (hit) {
      const int32_t row = start + before + __popc(bal & ((1u << lane) - 1u));
      token_of_row[row] = (int32_t)(i / K);
      row_of_pair[i] = row;
      expert_of_row[row] = e;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      int32_t tot = 0;
      for (int w = 0; w < (int)(blockDim.x >> 5); ++w) tot += warp_tot[w];
      running = start + tot;
    }
    __syncthreads();
  }
}

// ------------------------------------------------------------- gather --
// act[row] = t[token_of_row[row]]  (nn.op.take at model/mlp_optimized.py:150),
// optionally converted from bf16 to f16 for the f16 GEMM path (exact for
// |v| in the f16 normal range, which RMSNorm output stays in when the norm
// weights pass gptoss_moe_weights_prepare's check).
// Permutation by warp ranges (E <= 256).  The pairs are cut into contiguous
// ranges, one per warp.  Count: each warp counts its range per expert (lanes
// with one expert found by __match_any_sync, one add per expert and batch
// of 32 -- no atomics).  Scan: indptr, the tile plan, and each warp's
// starting row per expert (indptr[e] + the pairs of expert e in the ranges
// before it).  Place: each warp walks its range again in order, row = its
// running row of the expert + rank among the batch's lanes of that expert.
// Rows of one expert come out in pair order -- the stable order of
// moe_place_kernel -- without every expert's CTA reading every pair.
constexpr int kPermUnroll = 4;

// Pairs [lo, hi) counted per expert into cnt[0, E) (the warp's own row).
__device__ __forceinline__ void perm_warp_count(const int32_t* __restrict__ idx, int64_t lo, int64_t hi, int32_t E,
                                                int32_t* cnt, uint32_t* err) {
  const int lane = threadIdx.x & 31;
  const uint32_t lt = (1u << lane) - 1u;
  for (int e = lane; e < E; e += 32) cnt[e] = 0;
  __syncwarp();
  for (int64_t b0 = lo; b0 < hi; b0 += 32 * kPermUnroll) {
    int32_t ev[kPermUnroll];
#pragma unroll
    for (int u = 0; u < kPermUnroll; ++u) {
      const int64_t i = b0 + u * 32 + lane;
      ev[u] = i < hi ? idx[i] : INT32_MIN;
    }
#pragma unroll
    for (int u = 0; u < kPermUnroll; ++u) {
      int32_t e = ev[u];
      const bool ok = e >= 0 && e < E;
      if (!ok) {
        if (e != INT32_MIN) raise_error(err, kErrBadRouting);
        e = -1 - lane;  // a key that no valid pair shares
      }
      const uint32_t same = __match_any_sync(0xffffffffu, e);
      if (ok && (same & lt) == 0) cnt[e] += __popc(same);
      __syncwarp();
    }
  }
}

// Pairs [lo, hi) placed from base[0, E) (the warp's own running rows).
__device__ __forceinline__ void perm_warp_place(const int32_t* __restrict__ idx, int64_t lo, int64_t hi, int32_t K,
                                                int32_t E, int32_t* base, int32_t* __restrict__ token_of_row,
                                                int32_t* __restrict__ row_of_pair,
                                                int32_t* __restrict__ expert_of_row) {
  const int lane = threadIdx.x & 31;
  const uint32_t lt = (1u << lane) - 1u;
  for (int64_t b0 = lo; b0 < hi; b0 += 32 * kPermUnroll) {
    int32_t ev[kPermUnroll];
#pragma unroll
    for (int u = 0; u < kPermUnroll; ++u) {
      const int64_t i = b0 + u * 32 + lane;
      ev[u] = i < hi ? idx[i] : INT32_MIN;
    }
#pragma unroll
    for (int u = 0; u < kPermUnroll; ++u) {
      const int64_t i = b0 + u * 32 + lane;
      int32_t e = ev[u];
      const bool ok = e >= 0 && e < E;
      if (!ok) e = -1 - lane;
      const uint32_t same = __match_any_sync(0xffffffffu, e);
      if (ok) {
        const int32_t row = base[e] + __popc(same & lt);
        token_of_row[row] = (int32_t)(i / K);
        row_of_pair[i] = row;
        expert_of_row[row] = e;
      }
      __syncwarp();
      if (ok && (same & lt) == 0) base[e] += __popc(same);
      __syncwarp();
    }
  }
}

// The tile plan of an expert with c rows (moe_count_scan_kernel's rule).
__device__ __forceinline__ void perm_tiles(int32_t c, int32_t tmax, int32_t& nt, int32_t& per) {
  nt = (c + tmax - 1) / tmax;
  per = nt ? ((((c + nt - 1) / nt) + 15) & ~15) : 0;
}

// indptr / tile_ptr / tile_rows from the per-expert counts c (thread e of
// the first 256 threads; all threads of the block call it).  Returns
// indptr[e] for thread e < E.
__device__ __forceinline__ int32_t perm_scan_experts(int32_t c, int32_t E, int64_t pairs, int32_t* __restrict__ indptr,
                                                     int32_t* __restrict__ tile_ptr, int32_t* __restrict__ tile_rows,
                                                     int32_t (*wtot)[8]) {
  const int e = threadIdx.x, warp = e >> 5, lane = e & 31;
  int32_t nt = 0, per = 0;
  if (e < E) perm_tiles(c, moe_tile_rows_max(pairs, E), nt, per);
  int32_t sc = e < E ? c : 0, sn = nt;  // inclusive scans within the warp
  if (warp < 8) {
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const int32_t xc = __shfl_up_sync(0xffffffffu, sc, d), xn = __shfl_up_sync(0xffffffffu, sn, d);
      if (lane >= d) sc += xc, sn += xn;
    }
    if (lane == 31) wtot[0][warp] = sc, wtot[1][warp] = sn;
  }
  __syncthreads();
  int32_t start = 0;
  if (e < E) {
    for (int w = 0; w < warp; ++w) sc += wtot[0][w], sn += wtot[1][w];
    start = sc - c;
    indptr[e] = start;
    tile_ptr[e] = sn - nt;
    tile_rows[e] = per;
    if (e == E - 1) indptr[E] = sc, tile_ptr[E] = sn;
  }
  return start;
}

// Small pair counts: the three steps in one CTA of 32 warps.
constexpr int kPermWarps = 32;

__global__ void __launch_bounds__(kPermWarps * 32) moe_permute_onecta_kernel(
    const int32_t* __restrict__ idx, int64_t pairs, int32_t K, int32_t E, int32_t* __restrict__ indptr,
    int32_t* __restrict__ tile_ptr, int32_t* __restrict__ tile_rows, int32_t* __restrict__ token_of_row,
    int32_t* __restrict__ row_of_pair, int32_t* __restrict__ expert_of_row, uint32_t* err) {
  __shared__ int32_t wcnt[kPermWarps][256];  // counts, then running rows of each (warp, expert)
  __shared__ int32_t wtot[2][8];
  const int warp = threadIdx.x >> 5;
  const int64_t span = ((pairs + kPermWarps * 32 - 1) / (kPermWarps * 32)) * 32;
  const int64_t lo = (int64_t)warp * span, hi = min(pairs, lo + span);
  perm_warp_count(idx, lo, hi, E, wcnt[warp], err);
  __syncthreads();
  const int e = threadIdx.x;
  int32_t c = 0;
  if (e < E)
    for (int w = 0; w < kPermWarps; ++w) c += wcnt[w][e];
  const int32_t start = perm_scan_experts(c, E, pairs, indptr, tile_ptr, tile_rows, wtot);
  if (e < E) {
    int32_t run = start;
    for (int w = 0; w < kPermWarps; ++w) {
      const int32_t k = wcnt[w][e];
      wcnt[w][e] = run;
      run += k;
    }
  }
  __syncthreads();
  perm_warp_place(idx, lo, hi, K, E, wcnt[warp], token_of_row, row_of_pair, expert_of_row);
}

// Many pairs: the three steps as three launches over kPermRanges-ish warp
// ranges of 8-warp CTAs.  Range r = [r span, (r + 1) span), the last one
// running to the end; span >= E, so every range holds at least E pairs, and
// the range's counts, then its starting rows, live in row_of_pair[r span,
// r span + E) -- the range's own pairs, which only its own warp overwrites,
// after reading them.
constexpr int kPermRangeTarget = 256;
constexpr int64_t kPermOneCtaMaxPairs = 4096;
constexpr int kPermRangeWarps = 8;

__host__ __device__ __forceinline__ int64_t perm_span(int64_t pairs, int32_t E) {
  const int64_t s = (pairs + kPermRangeTarget - 1) / kPermRangeTarget;
  return ((max(s, (int64_t)E) + 31) / 32) * 32;
}

__global__ void __launch_bounds__(kPermRangeWarps * 32) moe_perm_count_kernel(const int32_t* __restrict__ idx,
                                                                              int64_t pairs, int32_t E,
                                                                              int32_t* __restrict__ row_of_pair,
                                                                              uint32_t* err) {
  __shared__ int32_t wcnt[kPermRangeWarps][256];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t span = perm_span(pairs, E), nr = pairs / span;
  const int64_t r = (int64_t)blockIdx.x * kPermRangeWarps + warp;
  if (r >= nr) return;
  const int64_t lo = r * span, hi = r == nr - 1 ? pairs : lo + span;
  perm_warp_count(idx, lo, hi, E, wcnt[warp], err);
  for (int e = lane; e < E; e += 32) row_of_pair[lo + e] = wcnt[warp][e];
}

// One CTA of 1024 threads: thread (p, e) = (tid / E, tid % E), p < 1024 / E,
// adds up the counts of expert e over the p-th part of the ranges (loads
// eight at a time), then writes that part's starting rows.
__global__ void __launch_bounds__(1024) moe_perm_scan_kernel(int64_t pairs, int32_t E, int32_t* __restrict__ indptr,
                                                             int32_t* __restrict__ tile_ptr,
                                                             int32_t* __restrict__ tile_rows,
                                                             int32_t* __restrict__ row_of_pair) {
  constexpr int kU = 8;
  __shared__ int32_t part[1024];  // [P][E]
  __shared__ int32_t wtot[2][8];
  __shared__ int32_t first[256];
  const int P = 1024 / E;
  const int e = threadIdx.x % E, p = threadIdx.x / E;
  const bool mine = p < P;
  const int64_t span = perm_span(pairs, E), nr = pairs / span;
  const int64_t r0 = mine ? nr * p / P : 0, r1 = mine ? nr * (p + 1) / P : 0;
  int32_t sum = 0;
  for (int64_t r = r0; r < r1; r += kU) {
    int32_t v[kU];
#pragma unroll
    for (int u = 0; u < kU; ++u) v[u] = r + u < r1 ? row_of_pair[(r + u) * span + e] : 0;
#pragma unroll
    for (int u = 0; u < kU; ++u) sum += v[u];
  }
  if (mine) part[p * E + e] = sum;
  __syncthreads();
  int32_t c = 0;
  if (threadIdx.x < E)
    for (int q = 0; q < P; ++q) c += part[q * E + threadIdx.x];
  const int32_t start = perm_scan_experts(c, E, pairs, indptr, tile_ptr, tile_rows, wtot);
  if (threadIdx.x < E) first[threadIdx.x] = start;
  __syncthreads();
  if (mine) {
    int32_t run = first[e];
    for (int q = 0; q < p; ++q) run += part[q * E + e];
    for (int64_t r = r0; r < r1; r += kU) {
      int32_t v[kU];
#pragma unroll
      for (int u = 0; u < kU; ++u) v[u] = r + u < r1 ? row_of_pair[(r + u) * span + e] : 0;
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        if (r + u < r1) row_of_pair[(r + u) * span + e] = run;
        run += v[u];
      }
    }
  }
}

__global__ void __launch_bounds__(kPermRangeWarps * 32) moe_perm_place_kernel(
    const int32_t* __restrict__ idx, int64_t pairs, int32_t K, int32_t E, int32_t* __restrict__ token_of_row,
    int32_t* __restrict__ row_of_pair, int32_t* __restrict__ expert_of_row) {
  __shared__ int32_t base[kPermRangeWarps][256];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t span = perm_span(pairs, E), nr = pairs / span;
  const int64_t r = (int64_t)blockIdx.x * kPermRangeWarps + warp;
  if (r >= nr) return;
  const int64_t lo = r * span, hi = r == nr - 1 ? pairs : lo + span;
  for (int e = lane; e < E; e += 32) base[warp][e] = row_of_pair[lo + e];
  __syncwarp();
  perm_warp_place(idx, lo, hi, K, E, base[warp], token_of_row, row_of_pair, expert_of_row);
}

// Decode sizes (M * K <= 1024 pairs, E <= 256): top-k + softmax, the
// expert counts and scan, the token-tile plan and the stable placement in
// one CTA -- the same results as topk_softmax_kernel, moe_count_scan_kernel
// and moe_place_kernel, without two launches between them.  A pair's row
// within its expert counts the earlier pairs with the same expert: within
// the warp by __match_any_sync, across warps from per-warp counts.
constexpr int kRouteSmallPairs = 1024;
__global__ void __launch_bounds__(1024) moe_route_small_kernel(const uint16_t* __restrict__ logits, int64_t M,
                                                                int32_t E, int32_t K, uint16_t* __restrict__ weights,
                                                                int32_t* __restrict__ indices,
                                                                int32_t* __restrict__ indptr,
                                                                int32_t* __restrict__ tile_ptr,
                                                                int32_t* __restrict__ tile_rows,
                                                                int32_t* __restrict__ token_of_row,
                                                                int32_t* __restrict__ row_of_pair,
                                                                int32_t* __restrict__ expert_of_row, uint32_t* err) {
  __shared__ int32_t sidx[kRouteSmallPairs];
  __shared__ int32_t wcnt[32][256];  // pairs of each expert per warp
  __shared__ int32_t sptr[257];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t pairs = M * K;
  for (int64_t m = warp; m < M; m += 32)
    topk_softmax_warp(logits + m * E, E, K, weights + m * K, indices + m * K, sidx + m * K, err);
  for (int e = lane; e < E; e += 32) wcnt[warp][e] = 0;
  __syncthreads();
  const int i = threadIdx.x;  // one pair per thread
  const bool live = i < pairs;
  int32_t e = live ? sidx[i] : -1;
  const bool ok = live && e >= 0 && e < E;
  if (!ok) e = -1 - lane;  // a key no valid pair shares
  const uint32_t same = __match_any_sync(0xffffffffu, e);
  const int rank_w = __popc(same & ((1u << lane) - 1u));
  if (ok && rank_w == 0) wcnt[warp][e] = __popc(same);
  __syncthreads();
  if ((int)threadIdx.x < E) {  // each expert's total, in parallel
    int32_t c = 0;
    for (int w = 0; w < 32; ++w) c += wcnt[w][threadIdx.x];
    sptr[threadIdx.x] = c;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const int32_t tmax = moe_tile_rows_max(pairs, E);
    int32_t acc = 0, tacc = 0;
    for (int32_t x = 0; x < E; ++x) {
      const int32_t c = sptr[x];
      sptr[x] = acc;
      indptr[x] = acc;
      tile_ptr[x] = tacc;
      const int32_t nt = (c + tmax - 1) / tmax;
      tile_rows[x] = nt ? ((((c + nt - 1) / nt) + 15) & ~15) : 0;
      acc += c;
      tacc += nt;
    }
    indptr[E] = acc;
    tile_ptr[E] = tacc;
  }
  __syncthreads();
  if (ok) {
    int32_t row = sptr[e] + rank_w;
    for (int w = 0; w < warp; ++w) row += wcnt[w][e];
    token_of_row[row] = i / K;
    row_of_pair[i] = row;
    expert_of_row[row] = e;
  }
}

template <bool kToF16>
__global__ void gather_rows_kernel(const uint16_t* __restrict__ t, const int32_t* __restrict__ token_of_row,
                                   int64_t rows, int32_t H, uint16_t* __restrict__ act) {
  const int64_t r = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (r >= rows) return;
  const int lane = threadIdx.x & 31;
  const int64_t src = token_of_row[r];
  const uint4* s = (const uint4*)(t + src * H);
  uint4* d = (uint4*)(act + r * H);
  for (int32_t i = lane; i < H / 8; i += 32) {
    uint4 v = s[i];
    if (kToF16) {
      uint32_t* w = (uint32_t*)&v;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const __half2 h = __floats2half2_rn(__uint_as_float(w[q] << 16), __uint_as_float(w[q] & 0xFFFF0000u));
        w[q] = *(const uint32_t*)&h;
      }
    }
    d[i] = v;
  }
}

// ------------------------------------------------------------ combine --
// out[m, c] = bf16(float(x[m,c]) + float(bf16(sum_r h2[row(m,r), c] * w[m,r])))
// with the serial fp32 sum over r of run_gating (model/mlp.py:328-369) and
// the residual of model/mlp.py:399-402.  One block per token, 4 columns per
// thread (16-byte loads of the fp32 expert rows).
// TIn = float: expert outputs in fp32 (the reference's arithmetic); uint16_t:
// expert outputs already rounded to bf16 (the expert-parallel return path).
template <typename TIn>
__global__ void __launch_bounds__(256) combine_kernel(const TIn* __restrict__ h2, const int32_t* __restrict__ row_of_pair,
                                                      const uint16_t* __restrict__ w, const uint16_t* __restrict__ x,
                                                      int64_t M, int32_t K, int32_t H, uint16_t* __restrict__ out) {
  const int64_t m = blockIdx.x;
  if (m >= M) return;
  const TIn* rows[8];
  float wr[8];
  for (int32_t r = 0; r < K; ++r) {
    rows[r] = h2 + (int64_t)__ldg(row_of_pair + m * K + r) * H;
    wr[r] = bf16_bits_to_f32(__ldg(w + m * K + r));
  }
  for (int32_t c4 = threadIdx.x; c4 < H / 4; c4 += blockDim.x) {
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    for (int32_t r = 0; r < K; ++r) {
      float4 v;
      if constexpr (sizeof(TIn) == 4) {
        v = __ldg((const float4*)rows[r] + c4);
      } else {
        const uint2 b = __ldg((const uint2*)rows[r] + c4);
        v = make_float4(__uint_as_float(b.x << 16), __uint_as_float(b.x & 0xFFFF0000u), __uint_as_float(b.y << 16),
                        __uint_as_float(b.y & 0xFFFF0000u));
      }
      acc[0] = __fadd_rn(acc[0], __fmul_rn(v.x, wr[r]));
      acc[1] = __fadd_rn(acc[1], __fmul_rn(v.y, wr[r]));
      acc[2] = __fadd_rn(acc[2], __fmul_rn(v.z, wr[r]));
      acc[3] = __fadd_rn(acc[3], __fmul_rn(v.w, wr[r]));
    }
    const uint2 xv = __ldg((const uint2*)(x + m * H) + c4);
    const float x0 = __uint_as_float(xv.x << 16), x1 = __uint_as_float(xv.x & 0xFFFF0000u);
    const float x2 = __uint_as_float(xv.y << 16), x3 = __uint_as_float(xv.y & 0xFFFF0000u);
    uint2 o;
    o.x = (uint32_t)f32_to_bf16_bits(__fadd_rn(x0, round_bf16(acc[0]))) |
          ((uint32_t)f32_to_bf16_bits(__fadd_rn(x1, round_bf16(acc[1]))) << 16);
    o.y = (uint32_t)f32_to_bf16_bits(__fadd_rn(x2, round_bf16(acc[2]))) |
          ((uint32_t)f32_to_bf16_bits(__fadd_rn(x3, round_bf16(acc[3]))) << 16);
    ((uint2*)(out + m * H))[c4] = o;
  }
}

// ------------------------------------------------------- MXFP4 decode --
// Standalone exact decode (model/mlp.py:146-236): out[r, 32g + j] =
// FP4_VALUES[nibble] * 2^(scale-127) as bf16.  Scale code 0 (2^-127) is
// applied as 2^-126 * 0.5 so that every code 0..254 decodes exactly.
__global__ void mxfp4_dequant_kernel(const uint8_t* __restrict__ blocks, const uint8_t* __restrict__ scales,
                                     int64_t groups_total, uint16_t* __restrict__ out) {
  const int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (g >= groups_total) return;
  const uint4 nb = *(const uint4*)(blocks + g * 16);
  const uint32_t s = scales[g];
  const uint32_t sc = s ? e8m0_scale_bf16x2(s) : 0x00800080u;
  const uint32_t fix = s ? 0x3F803F80u : 0x3F003F00u;
  uint32_t o[4];
  uint4* dst = (uint4*)(out + g * 32);
  const uint32_t words[4] = {nb.x, nb.y, nb.z, nb.w};
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    fp4x8_to_bf16x8(words[q], sc, o);
    dst[q] = make_uint4(bf16x2_mul(o[0], fix), bf16x2_mul(o[1], fix), bf16x2_mul(o[2], fix), bf16x2_mul(o[3], fix));
  }
}

// ------------------------------------------------------ weight ranges --
// min / max of the E8M0 scale codes of both projections and the largest
// |norm weight| (as fp32 bits), for choosing the f16 GEMM path.
// out4 = {min scale, max scale, max |norm weight| bits, unused}.
__global__ void weight_ranges_kernel(const uint8_t* __restrict__ s1, int64_t n1, const uint8_t* __restrict__ s2,
                                     int64_t n2, const uint16_t* __restrict__ norm_w, int32_t H,
                                     uint32_t* __restrict__ out4) {
  uint32_t lo = 255, hi = 0;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n1 + n2; i += stride) {
    const uint32_t v = i < n1 ? s1[i] : s2[i - n1];
    lo = min(lo, v);
    hi = max(hi, v);
  }
  for (int off = 16; off > 0; off >>= 1) {
    lo = min(lo, __shfl_xor_sync(0xffffffffu, lo, off));
    hi = max(hi, __shfl_xor_sync(0xffffffffu, hi, off));
  }
  if ((threadIdx.x & 31) == 0) {
    atomicMin(&out4[0], lo);
    atomicMax(&out4[1], hi);
  }
  if (blockIdx.x == 0) {
    uint32_t m = 0;
    for (int32_t k = threadIdx.x; k < H; k += blockDim.x) m = max(m, (uint32_t)(norm_w[k] & 0x7FFFu) << 16);
    for (int off = 16; off > 0; off >>= 1) m = max(m, __shfl_xor_sync(0xffffffffu, m, off));
    if ((threadIdx.x & 31) == 0) atomicMax(&out4[2], m);  // positive floats order like their bits
  }
}

// ------------------------------------------------ expert parallelism --
// Token tiles of the grouped GEMMs from an expert-row index (indptr): the
// same plan moe_count_scan_kernel builds, for rows that arrived from other
// ranks.
__global__ void moe_plan_tiles_kernel(const int32_t* __restrict__ indptr, int32_t E, int32_t* __restrict__ tile_ptr,
                                      int32_t* __restrict__ tile_rows) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  const int32_t tmax = moe_tile_rows_max(indptr[E], E);
  int32_t tacc = 0;
  for (int32_t e = 0; e < E; ++e) {
    const int32_t c = indptr[e + 1] - indptr[e];
    const int32_t nt = (c + tmax - 1) / tmax;
    tile_ptr[e] = tacc;
    tile_rows[e] = nt ? ((((c + nt - 1) / nt) + 15) & ~15) : 0;
    tacc += nt;
  }
  tile_ptr[E] = tacc;
}

// Rows exchanged between ranks arrive source-major: for each source rank s,
// the rows of local expert 0, 1, ... (counts[s][e] rows each).  The grouped
// GEMMs want them expert-major (for each expert, the rows of source 0, 1,
// ...).  One block per (s, e) segment moves its rows; dir 0 = source-major
// -> expert-major, dir 1 = back.  Block 0 also writes the expert-major
// indptr_local[E+1] when asked.
__global__ void segment_copy_kernel(const uint8_t* __restrict__ src, uint8_t* __restrict__ dst,
                                    const int32_t* __restrict__ counts, int32_t P, int32_t El, int64_t row_bytes,
                                    int32_t dir, int32_t* __restrict__ indptr_local) {
  const int32_t s = blockIdx.x / El, e = blockIdx.x % El;
  int64_t src_off = 0, dst_off = 0;
  for (int32_t i = 0; i < P * El; ++i) {
    const int32_t si = i / El, ei = i % El;
    const int32_t c = counts[i];
    if (si < s || (si == s && ei < e)) src_off += c;        // source-major position
    if (ei < e || (ei == e && si < s)) dst_off += c;        // expert-major position
  }
  if (blockIdx.x == 0 && indptr_local != nullptr && threadIdx.x <= El) {
    int32_t acc = 0;
    for (int32_t ei = 0; ei < (int32_t)threadIdx.x; ++ei)
      for (int32_t si = 0; si < P; ++si) acc += counts[si * El + ei];
    indptr_local[threadIdx.x] = acc;
  }
  const int64_t rows = counts[s * El + e];
  const int64_t a = dir == 0 ? src_off : dst_off;  // read position
  const int64_t b = dir == 0 ? dst_off : src_off;  // write position
  const int64_t vec = row_bytes / 16;
  const uint4* in = (const uint4*)(src + a * row_bytes);
  if (dir == 2) {
    // fp32 rows of row_bytes -> bf16 rows of row_bytes / 2 (round to nearest even)
    uint2* out = (uint2*)(dst + b * (row_bytes / 2));
    for (int64_t i = threadIdx.x; i < rows * vec; i += blockDim.x) {
      const uint4 v = in[i];
      uint2 o;
      o.x = (uint32_t)f32_to_bf16_bits(__uint_as_float(v.x)) | ((uint32_t)f32_to_bf16_bits(__uint_as_float(v.y)) << 16);
      o.y = (uint32_t)f32_to_bf16_bits(__uint_as_float(v.z)) | ((uint32_t)f32_to_bf16_bits(__uint_as_float(v.w)) << 16);
      out[i] = o;
    }
    return;
  }
  uint4* out = (uint4*)(dst + b * row_bytes);
  for (int64_t i = threadIdx.x; i < rows * vec; i += blockDim.x) out[i] = in[i];
}

// ------------------------------------------------------------- launch --
int launch_rmsnorm(const uint16_t* x, const uint16_t* w, int64_t M, int32_t H, float eps, uint16_t* out,
                   uint32_t* err, cudaStream_t s) {
  if (M <= 0) return 0;
  if (H % 8 || ((uintptr_t)x & 15)) return -12;
  if (!((uintptr_t)w & 15) && !((uintptr_t)out & 15)) {
    // rows per CTA: all rows in one wave of CTAs where they fit, <= 32
    const int64_t sms = device_sm_count();
    const int rows = (int)min64(kNsMaxRows, max64(1, (M + sms - 1) / sms));
    const int nch = (H + kNsChunk - 1) / kNsChunk;
    const bool resident = nch <= kNsMaxSlots && (size_t)nch * rows * kNsPitch <= (size_t)kNsResidentBytes;
    const int stages = resident ? nch : kNsStages;
    const size_t smem = (size_t)stages * rows * kNsPitch;
    static FuncSmemAttr attr_s;
    ensure_dyn_smem(attr_s, (const void*)rmsnorm_stream_kernel,
                    (int)max64(kNsStages * kNsMaxRows * kNsPitch, kNsResidentBytes));
    // (the ring form's second read of x and its stores want more loads in
    // flight: eight warps; the resident form four)
    rmsnorm_stream_kernel<<<(unsigned)((M + rows - 1) / rows), resident ? 128 : 256, smem, s>>>(x, w, M, H, rows,
                                                                                               stages, eps, out, err);
    return cudaGetLastError() == cudaSuccess ? 0 : -3;
  }
  const size_t row = (size_t)(H + 8) * 2;
  const size_t fit = (size_t)(100 * 1024) / row;
  int rows = fit < (size_t)kNormRows ? (int)fit : kNormRows;
  if (rows < 1) return -12;
  const size_t smem = row * rows;
  static FuncSmemAttr attr;
  ensure_dyn_smem(attr, (const void*)rmsnorm_kernel, 100 * 1024 + 1024);
  const int64_t blocks = (M + rows - 1) / rows;
  rmsnorm_kernel<<<(unsigned)blocks, 128, smem, s>>>(x, w, M, H, rows, eps, out, err);
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

template <int kTQ, int kWQ>
static void launch_router_variant(dim3 grid, size_t smem, cudaStream_t s, const uint16_t* t, const uint16_t* W,
                                  const uint16_t* b, int64_t M, int32_t E, int32_t H, int32_t be, uint16_t* logits) {
  static FuncSmemAttr attr;
  ensure_dyn_smem(attr, (const void*)router_kernel<kTQ, kWQ>, 200 * 1024);
  router_kernel<kTQ, kWQ><<<grid, 128, smem, s>>>(t, W, b, M, E, H, be, logits);
}

static int launch_router_tiles(int egroups, dim3 grid, size_t smem, cudaStream_t s, const uint16_t* t,
                               const uint16_t* W, const uint16_t* b, int64_t M, int32_t E, int32_t H, int32_t be,
                               uint16_t* logits) {
  // prefetch registers per thread: token tile (btok rows x 4 pieces) and expert tile (be rows x 4 pieces)
  switch (egroups) {
    case 16: launch_router_variant<1, 2>(grid, smem, s, t, W, b, M, E, H, be, logits); break;
    case 8: launch_router_variant<1, 2>(grid, smem, s, t, W, b, M, E, H, be, logits); break;
    case 4: launch_router_variant<2, 1>(grid, smem, s, t, W, b, M, E, H, be, logits); break;
    case 2: launch_router_variant<4, 1>(grid, smem, s, t, W, b, M, E, H, be, logits); break;
    case 1: launch_router_variant<8, 1>(grid, smem, s, t, W, b, M, E, H, be, logits); break;
    default: return -12;
  }
  return 0;
}

// GPTOSS_ROUTER_BF16=0 keeps the router on the fp32-FMA chain kernels below
// (same bits, slower); otherwise router_bf16.cu's kernels run.
static bool router_bf16_enabled() {
  const char* e = getenv("GPTOSS_ROUTER_BF16");
  return !(e && e[0] == '0');
}

int launch_router(const uint16_t* t, const uint16_t* W, const uint16_t* b, int64_t M, int32_t E, int32_t H,
                  uint16_t* logits, uint32_t* err, cudaStream_t s) {
  if (M <= 0) return 0;
  if (router_bf16_enabled()) return launch_router_bf16(t, W, b, M, E, H, logits, err, s);
  if (E % kRTE != 0 || E > 1024 || H % 8 || ((uintptr_t)t & 15) || ((uintptr_t)W & 15)) return -12;
  if (M <= kRouterChainMaxTokens) {
    dim3 grid((unsigned)((E + kChainExp - 1) / kChainExp), (unsigned)((M + kChainTok - 1) / kChainTok));
    router_chain_kernel<<<grid, 128, 0, s>>>(t, W, b, M, E, H, logits);
    return cudaGetLastError() == cudaSuccess ? 0 : -3;
  }
  const int block_experts = E >= 64 ? 64 : E;
  if (E % block_experts) return -12;
  const int egroups = block_experts / kRTE;
  if (128 % egroups) return -12;
  const int btok = (128 / egroups) * kRTT;
  const size_t smem = (size_t)kRKT * btok * 2 * 4 + (size_t)kRKT * block_experts * 4;
  if (smem > 200 * 1024) return -12;
  dim3 grid((unsigned)((M + btok - 1) / btok), (unsigned)(E / block_experts));
  const int rc = launch_router_tiles(egroups, grid, smem, s, t, W, b, M, E, H, block_experts, logits);
  if (rc) return rc;
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

int launch_topk_softmax(const uint16_t* logits, int64_t M, int32_t E, int32_t K, uint16_t* weights,
                        int32_t* indices, uint32_t* err, cudaStream_t s) {
  if (M <= 0) return 0;
  if (E > 256 || K > 8 || K < 1 || K > E) return -12;
  const unsigned blocks = (unsigned)((M * 32 + 255) / 256);
  topk_softmax_kernel<<<blocks, 256, 0, s>>>(logits, M, E, K, weights, indices, err);
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

int launch_permute(const int32_t* idx, int64_t M, int32_t K, int32_t E, int32_t* indptr, int32_t* tile_ptr,
                   int32_t* tile_rows, int32_t* token_of_row, int32_t* row_of_pair, int32_t* expert_of_row,
                   uint32_t* err, cudaStream_t s) {
  const int64_t pairs = M * K;
  if (E <= 256 && pairs > kPermOneCtaMaxPairs) {
    const int64_t nr = pairs / perm_span(pairs, E);
    const unsigned grid = (unsigned)((nr + kPermRangeWarps - 1) / kPermRangeWarps);
    moe_perm_count_kernel<<<grid, kPermRangeWarps * 32, 0, s>>>(idx, pairs, E, row_of_pair, err);
    moe_perm_scan_kernel<<<1, 1024, 0, s>>>(pairs, E, indptr, tile_ptr, tile_rows, row_of_pair);
    moe_perm_place_kernel<<<grid, kPermRangeWarps * 32, 0, s>>>(idx, pairs, K, E, token_of_row, row_of_pair,
                                                                 expert_of_row);
    return cudaGetLastError() == cudaSuccess ? 0 : -3;
  }
  if (E <= 256) {
    moe_permute_onecta_kernel<<<1, kPermWarps * 32, 0, s>>>(idx, pairs, K, E, indptr, tile_ptr, tile_rows, token_of_row,
                                                 row_of_pair, expert_of_row, err);
    return cudaGetLastError() == cudaSuccess ? 0 : -3;
  }
  moe_count_scan_kernel<<<1, 1024, (size_t)E * 4, s>>>(idx, pairs, E, indptr, tile_ptr, tile_rows, err);
  if (pairs > 0) moe_place_kernel<<<E, 1024, 0, s>>>(idx, pairs, K, indptr, token_of_row, row_of_pair, expert_of_row);
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

int launch_route_small(const uint16_t* logits, int64_t M, int32_t E, int32_t K, uint16_t* weights,
                       int32_t* indices, int32_t* indptr, int32_t* tile_ptr, int32_t* tile_rows,
                       int32_t* token_of_row, int32_t* row_of_pair, int32_t* expert_of_row, uint32_t* err,
                       cudaStream_t s) {
  if (M <= 0) return 0;
  if (M * K > kRouteSmallPairs || E > 256 || K > 8 || K < 1 || K > E) return -12;
  moe_route_small_kernel<<<1, 1024, 0, s>>>(logits, M, E, K, weights, indices, indptr, tile_ptr, tile_rows,
                                            token_of_row, row_of_pair, expert_of_row, err);
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}
int route_small_max_pairs() { return kRouteSmallPairs; }

int launch_gather(const uint16_t* t, const int32_t* token_of_row, int64_t rows, int32_t H, uint16_t* act,
                  int32_t to_f16, cudaStream_t s) {
  if (rows <= 0) return 0;
  if (H % 8) return -12;
  if (to_f16) gather_rows_kernel<true><<<(unsigned)((rows + 7) / 8), 256, 0, s>>>(t, token_of_row, rows, H, act);
  else gather_rows_kernel<false><<<(unsigned)((rows + 7) / 8), 256, 0, s>>>(t, token_of_row, rows, H, act);
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

int launch_combine(const float* h2, const int32_t* row_of_pair, const uint16_t* w, const uint16_t* x, int64_t M,
                   int32_t K, int32_t H, uint16_t* out, cudaStream_t s) {
  if (M <= 0) return 0;
  if (H % 4 || K > 8) return -12;
  const int64_t blocks = M;
  combine_kernel<float><<<(unsigned)blocks, 256, 0, s>>>(h2, row_of_pair, w, x, M, K, H, out);
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

int launch_combine_bf16(const uint16_t* h2, const int32_t* row_of_pair, const uint16_t* w, const uint16_t* x,
                        int64_t M, int32_t K, int32_t H, uint16_t* out, cudaStream_t s) {
  if (M <= 0) return 0;
  if (H % 4 || K > 8) return -12;
  combine_kernel<uint16_t><<<(unsigned)M, 256, 0, s>>>(h2, row_of_pair, w, x, M, K, H, out);
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

int launch_mxfp4_dequant(const uint8_t* blocks, const uint8_t* scales, int64_t groups_total, uint16_t* out,
                         cudaStream_t s) {
  if (groups_total <= 0) return 0;
  mxfp4_dequant_kernel<<<(unsigned)((groups_total + 255) / 256), 256, 0, s>>>(blocks, scales, groups_total, out);
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

}  // namespace gptoss

namespace gptoss {
int launch_weight_ranges(const uint8_t* s1, int64_t n1, const uint8_t* s2, int64_t n2, const uint16_t* norm_w,
                         int32_t H, uint32_t* out4, cudaStream_t s) {
  weight_ranges_kernel<<<592, 256, 0, s>>>(s1, n1, s2, n2, norm_w, H, out4);
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}
int launch_plan_tiles(const int32_t* indptr, int32_t E, int32_t* tile_ptr, int32_t* tile_rows, cudaStream_t s) {
  moe_plan_tiles_kernel<<<1, 32, 0, s>>>(indptr, E, tile_ptr, tile_rows);
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}
int launch_segment_copy(const void* src, void* dst, const int32_t* counts, int32_t P, int32_t El, int64_t row_bytes,
                        int32_t dir, int32_t* indptr_local, cudaStream_t s) {
  if (P <= 0 || El <= 0 || row_bytes % 16) return -12;
  segment_copy_kernel<<<(unsigned)(P * El), 256, 0, s>>>((const uint8_t*)src, (uint8_t*)dst, counts, P, El, row_bytes,
                                                          dir, indptr_local);
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}
}  // namespace gptoss
