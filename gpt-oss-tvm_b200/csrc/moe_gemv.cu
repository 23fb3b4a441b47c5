// moe_gemv.cu -- decode-size grouped expert GEMMs as bandwidth-bound MXFP4 GEMVs.
//
// With few token rows per expert (decode: a handful per expert) the expert
// GEMMs are weight streams: every byte of the chosen experts' packed e2m1
// nibbles is read once and multiplied by a few activation rows.  This
// kernel streams the nibbles straight from HBM into registers with 16-byte
// loads (one whole 32-element MXFP4 group per lane), decodes them in
// registers with the hardware e2m1 -> f16 converter, multiplies by the group's
// E8M0 scale as packed f16 (exact for scale codes 104..140, the f16 path),
// and feeds them to mma.sync m16n8k16 (f16 x f16 -> fp32) as the M operand;
// the token rows (at most 16 per pass, two n8 tiles) sit in shared memory as
// the N operand.  No shared-memory round trip for the weights, no TMEM.
//
// A CTA covers 32 weight rows (two m16 tiles) of one expert; its four warps
// split K (warp w takes rounds w, w + 4, ...) so that four times as many
// warps stream weights as with one warp per row tile -- with one or two
// tokens per expert the kernel is bound by the bytes each SM has in flight --
// and add their partial sums through shared memory before the epilogue.
// Lane (g, q) of a warp owns weight rows g and g + 8 of each m16 tile and, in
// round r, the MXFP4 group 4r + q of those rows.  The MMA's
// k index is therefore a permutation of the physical columns (lane q's k
// values come from group 4r + q); the token fragments are read with the same
// permutation from shared memory, so the dot products are unchanged.
//
// Results equal the tensor-core GEMM's within fp32 accumulation order; the
// epilogues (bias, clamped SwiGLU, f16 / fp32 stores) are the same math.
#include "common.cuh"
#include "launch.h"

namespace gptoss {

constexpr int kGvWarps = 4;     // warps per CTA, each a quarter of the K rounds
constexpr int kGvRowsCta = 32;  // weight rows per CTA: two m16 MMA tiles
constexpr int kGvTok = 16;      // token rows per pass at most: two n8 MMA tiles
constexpr int kGvTokDecode = 8;  // token rows staged per pass by the launcher
constexpr int kGvMaxK = 4096;
constexpr int kGvMaxRows = 64;  // routed rows up to which the GEMV replaces the tensor-core kernel
constexpr int kGvRedBytes = kGvWarps * 32 * 16 * 4;  // partial sums of the four warps

struct GemvParams {
  const uint16_t* act;  // [act_rows, K] f16, expert-major rows
  int64_t act_rows;
  const uint8_t* blocks;  // [E, N, K/32, 16]
  const uint8_t* scales;  // [E, N, K/32]
  const uint16_t* bias;   // [E, N] bf16
  const int32_t* indptr;  // [E + 1]
  void* out;              // mode 0: [act_rows, N/2] f16; mode 1: [act_rows, N] f32
  int32_t E, N, K, ldo;
  float alpha, limit;
  int32_t tok_cap;  // token rows staged per pass (<= kGvTok)
  uint32_t* err;
  const int32_t* gather;  // optional: act holds bf16 token rows, row r = f16(act[gather[r]])
};

__device__ __forceinline__ void mma_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                          uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Shared-memory position of 16-byte chunk c (columns 8c .. 8c + 7) of group
// gi in a token row: the four chunks of a group are rotated by gi / 2, so
// the lanes q = 0..3 of a quad, reading chunk c of groups 4r + q, hit four
// different bank groups (with the 32-byte row padding, rows n and n + 1 too).
__device__ __forceinline__ uint32_t gv_chunk_ofs(int32_t gi, int32_t c) {
  return (uint32_t)gi * 64u + ((uint32_t)((c + (gi >> 1)) & 3) << 4);
}

struct GvLoad {
  uint4 nb[2][2];     // [m tile][row g / g + 8]: the lane's group of nibbles
  uint32_t sc[2][2];  // its E8M0 scale codes
};

__device__ __forceinline__ void gv_load(GvLoad& L, const uint8_t* const (&wrow)[2][2],
                                        const uint8_t* const (&srow)[2][2], int32_t gi, int32_t G) {
  if (gi < G) {
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
      for (int rr = 0; rr < 2; ++rr) {
        L.nb[mt][rr] = __ldg((const uint4*)(wrow[mt][rr] + (size_t)gi * 16));
        L.sc[mt][rr] = __ldg(srow[mt][rr] + gi);
      }
  } else {
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
      for (int rr = 0; rr < 2; ++rr) {
        L.nb[mt][rr] = make_uint4(0u, 0u, 0u, 0u);
        L.sc[mt][rr] = 127u;
      }
  }
}

__device__ __forceinline__ uint32_t word_of(const uint4& v, int i) {
  return i == 0 ? v.x : (i == 1 ? v.y : (i == 2 ? v.z : v.w));
}

// One round: group gi = 4r + q of the lane's four rows against the staged
// token rows (n = g and, with two n tiles, n = 8 + g).
template <bool kTwoN>
__device__ __forceinline__ void gv_round(const GvLoad& L, float (&acc)[2][2][4], const uint8_t* act_s, uint32_t S,
                                         int32_t gi, int32_t G, int g, int nv) {
  uint4 b[2][4];
#pragma unroll
  for (int nt = 0; nt < (kTwoN ? 2 : 1); ++nt) {
    const int n = nt * 8 + g;
    if (gi < G && n < nv) {
      const uint8_t* base = act_s + (size_t)n * S;
#pragma unroll
      for (int c = 0; c < 4; ++c) b[nt][c] = *(const uint4*)(base + gv_chunk_ofs(gi, c));
    } else {
#pragma unroll
      for (int c = 0; c < 4; ++c) b[nt][c] = make_uint4(0u, 0u, 0u, 0u);
    }
  }
  uint32_t sc2[2][2];
#pragma unroll
  for (int mt = 0; mt < 2; ++mt)
#pragma unroll
    for (int rr = 0; rr < 2; ++rr) sc2[mt][rr] = e8m0_scale_f16x2(L.sc[mt][rr]);
#pragma unroll
  for (int i = 0; i < 4; ++i) {  // word i: columns 8i .. 8i + 7 of the group
    uint32_t a[2][2][4];
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
      for (int rr = 0; rr < 2; ++rr)
        fp4x8_to_f16x8(word_of(L.nb[mt][rr], i), sc2[mt][rr], a[mt][rr][0], a[mt][rr][1], a[mt][rr][2],
                       a[mt][rr][3]);
#pragma unroll
    for (int h = 0; h < 2; ++h) {  // k step: columns 8i + 4h .. 8i + 4h + 3
#pragma unroll
      for (int mt = 0; mt < 2; ++mt) {
#pragma unroll
        for (int nt = 0; nt < (kTwoN ? 2 : 1); ++nt) {
          const uint32_t b0 = h ? b[nt][i].z : b[nt][i].x;
          const uint32_t b1 = h ? b[nt][i].w : b[nt][i].y;
          mma_16816(acc[mt][nt], a[mt][0][2 * h], a[mt][1][2 * h], a[mt][0][2 * h + 1], a[mt][1][2 * h + 1], b0,
                    b1);
        }
      }
    }
  }
}

// The y-th expert (in expert order) that has routed rows, or -1: each warp
// scans indptr 32 experts at a time with a ballot.
__device__ __forceinline__ int32_t gv_routed_expert(const int32_t* __restrict__ indptr, int32_t E, int32_t y) {
  const int lane = threadIdx.x & 31;
  int32_t seen = 0;
  for (int32_t base = 0; base < E; base += 32) {
    const int32_t e = base + lane;
    const bool has = e < E && __ldg(indptr + e + 1) > __ldg(indptr + e);
    const uint32_t m = __ballot_sync(0xffffffffu, has);
    const int32_t n = __popc(m);
    if (y < seen + n) {
      uint32_t mm = m;
      for (int32_t k = 0; k < y - seen; ++k) mm &= mm - 1;  // drop the lower set bits
      return base + __ffs(mm) - 1;
    }
    seen += n;
  }
  return -1;
}

template <int kMode>
__global__ void __launch_bounds__(kGvWarps * 32) moe_gemv_kernel(const GemvParams p) {
  extern __shared__ __align__(16) uint8_t gv_smem[];
  const int32_t e = gv_routed_expert(p.indptr, p.E, blockIdx.y);  // grid.y covers the routed experts at most
  if (e < 0) return;
  const int64_t r0 = __ldg(p.indptr + e), r1 = __ldg(p.indptr + e + 1);
  const int64_t nrows = r1 - r0;
  if (nrows <= 0) return;
  if (r0 < 0 || r1 > p.act_rows) {
    if (threadIdx.x == 0) raise_error(p.err, kErrBadRouting);
    return;
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, q = lane & 3;
  const bool odd = g & 1;
  const int32_t wrow0 = blockIdx.x * kGvRowsCta;  // N % 32 == 0: the CTA's 32 rows all exist
  const int32_t G = p.K >> 5;
  const int32_t rounds = (G + 3) >> 2;
  const size_t row_bytes = (size_t)(p.K >> 1);
  const uint32_t S = 2u * (uint32_t)p.K + 32u;  // staged token row stride, bytes
  const uint8_t* wrow[2][2];
  const uint8_t* srow[2][2];
#pragma unroll
  for (int mt = 0; mt < 2; ++mt)
#pragma unroll
    for (int rr = 0; rr < 2; ++rr) {
      const int32_t row = wrow0 + mt * 16 + rr * 8 + g;
      wrow[mt][rr] = p.blocks + ((size_t)e * p.N + row) * row_bytes;
      srow[mt][rr] = p.scales + ((size_t)e * p.N + row) * G;
    }
  const int32_t chunks_row = p.K >> 3;
  float* red = (float*)(gv_smem + (size_t)p.tok_cap * S);  // [warp][lane][16]
  constexpr int kStep = kGvWarps;
  for (int64_t c0 = 0; c0 < nrows; c0 += p.tok_cap) {
    const int nv = (int)min64(p.tok_cap, nrows - c0);
    if (c0 > 0) __syncthreads();  // the previous pass is done with the staged rows
    // the first round of weights is requested before the token rows are
    // staged (they do not depend on each other)
    GvLoad A, B;
    if (warp < rounds) gv_load(A, wrow, srow, 4 * warp + q, G);
    for (int i = threadIdx.x; i < nv * chunks_row; i += blockDim.x) {
      const int n = i / chunks_row, ch = i - n * chunks_row;
      const int64_t src = p.gather ? (int64_t)__ldg(p.gather + r0 + c0 + n) : r0 + c0 + n;
      uint4 v = __ldg((const uint4*)(p.act + (size_t)src * p.K) + ch);
      if (p.gather) {  // bf16 token row -> f16 (exact in the f16 path's range)
        uint32_t* w = (uint32_t*)&v;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const __half2 h = __floats2half2_rn(__uint_as_float(w[q] << 16), __uint_as_float(w[q] & 0xFFFF0000u));
          w[q] = *(const uint32_t*)&h;
        }
      }
      *(uint4*)(gv_smem + (size_t)n * S + gv_chunk_ofs(ch >> 2, ch & 3)) = v;
    }
    __syncthreads();
    float acc[2][2][4];
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[mt][nt][j] = 0.f;
    const bool two_n = nv > 8;
    for (int32_t r = warp; r < rounds; r += 2 * kStep) {
      const int32_t r1 = r + kStep, r2 = r + 2 * kStep;
      if (r1 < rounds) gv_load(B, wrow, srow, 4 * r1 + q, G);
      if (two_n) gv_round<true>(A, acc, gv_smem, S, 4 * r + q, G, g, nv);
      else gv_round<false>(A, acc, gv_smem, S, 4 * r + q, G, g, nv);
      if (r1 < rounds) {
        if (r2 < rounds) gv_load(A, wrow, srow, 4 * r2 + q, G);
        if (two_n) gv_round<true>(B, acc, gv_smem, S, 4 * r1 + q, G, g, nv);
        else gv_round<false>(B, acc, gv_smem, S, 4 * r1 + q, G, g, nv);
      }
    }
    // the four warps' partial sums -> warp 0
    {
      float4* mine = (float4*)(red + ((size_t)warp * 32 + lane) * 16);
#pragma unroll
      for (int mt = 0; mt < 2; ++mt)
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) mine[mt * 2 + nt] = make_float4(acc[mt][nt][0], acc[mt][nt][1], acc[mt][nt][2],
                                                                       acc[mt][nt][3]);
    }
    __syncthreads();
    if (warp != 0) continue;
#pragma unroll
    for (int w = 1; w < kGvWarps; ++w) {
      const float4* other = (const float4*)(red + ((size_t)w * 32 + lane) * 16);
#pragma unroll
      for (int mt = 0; mt < 2; ++mt)
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) {
          const float4 o = other[mt * 2 + nt];
          acc[mt][nt][0] += o.x;
          acc[mt][nt][1] += o.y;
          acc[mt][nt][2] += o.z;
          acc[mt][nt][3] += o.w;
        }
    }
    // epilogue: lane (g, q) holds weight rows wrow0 + mt * 16 + {g, g + 8}
    // for tokens nt * 8 + 2q + {0, 1} (d0, d1: row g; d2, d3: row g + 8)
    const uint16_t* bias = p.bias + (size_t)e * p.N;
#pragma unroll
    for (int mt = 0; mt < 2; ++mt) {
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
        if (nt == 1 && !two_n) break;
        const float* d = acc[mt][nt];
        if (kMode == 0) {
          // (glu, linear) = rows (2j, 2j + 1): the even-g lane finishes the pair
          // (g, g + 1), the odd-g lane the pair (g + 7, g + 8)
          const float s0 = odd ? d[0] : d[2], s1 = odd ? d[1] : d[3];
          const float x0 = __shfl_xor_sync(0xffffffffu, s0, 4), x1 = __shfl_xor_sync(0xffffffffu, s1, 4);
          const int32_t grow = wrow0 + mt * 16 + (odd ? g + 7 : g);
          const float bg = bf16_bits_to_f32(__ldg(bias + grow)), bl = bf16_bits_to_f32(__ldg(bias + grow + 1));
          const float glu[2] = {odd ? x0 : d[0], odd ? x1 : d[1]};
          const float lin[2] = {odd ? d[2] : x0, odd ? d[3] : x1};
          uint16_t* out = (uint16_t*)p.out;
#pragma unroll
          for (int t = 0; t < 2; ++t) {
            const int n = nt * 8 + 2 * q + t;
            if (n < nv) {
              const float y = swiglu_f32(glu[t] + bg, lin[t] + bl, p.alpha, p.limit);
              out[(size_t)(r0 + c0 + n) * p.ldo + (grow >> 1)] = __half_as_ushort(__float2half_rn(y));
            }
          }
        } else {
          float* out = (float*)p.out;
#pragma unroll
          for (int rr = 0; rr < 2; ++rr) {
            const int32_t row = wrow0 + mt * 16 + rr * 8 + g;
            const float b = bf16_bits_to_f32(__ldg(bias + row));
#pragma unroll
            for (int t = 0; t < 2; ++t) {
              const int n = nt * 8 + 2 * q + t;
              if (n < nv) out[(size_t)(r0 + c0 + n) * p.ldo + row] = d[rr * 2 + t] + b;
            }
          }
        }
      }
    }
  }
}

bool moe_gemv_supported(const GemmLaunch& L) {
  return L.f16 && L.row_dst == nullptr && L.act_rows <= kGvMaxRows && L.K % 64 == 0 && L.K <= kGvMaxK &&
         L.N % 32 == 0 && ((uintptr_t)L.act & 15) == 0 && ((uintptr_t)L.blocks & 15) == 0;
}

int launch_moe_gemv(int mode, const GemmLaunch& L, cudaStream_t stream) {
  if (!moe_gemv_supported(L)) return -10;
  GemvParams p;
  p.act = L.act;
  p.act_rows = L.act_rows;
  p.blocks = L.blocks;
  p.scales = L.scales;
  p.bias = L.bias;
  p.indptr = L.indptr;
  p.out = L.out;
  p.E = L.E;
  p.N = L.N;
  p.K = L.K;
  p.ldo = L.ldo;
  p.alpha = L.alpha;
  p.limit = L.limit;
  p.tok_cap = (int32_t)min64(kGvTokDecode, L.act_rows);
  p.err = L.err;
  p.gather = L.act_gather;
  const size_t smem = (size_t)p.tok_cap * (2 * (size_t)L.K + 32) + kGvRedBytes;
  // at most act_rows experts have rows: CTAs for the routed experts only
  const dim3 grid((unsigned)((L.N + kGvRowsCta - 1) / kGvRowsCta), (unsigned)min64(L.E, L.act_rows));
  if (mode == 0) {
    static FuncSmemAttr attr;
    ensure_dyn_smem(attr, (const void*)moe_gemv_kernel<0>, kGvTok * (2 * kGvMaxK + 32) + kGvRedBytes);
    moe_gemv_kernel<0><<<grid, kGvWarps * 32, smem, stream>>>(p);
  } else {
    static FuncSmemAttr attr;
    ensure_dyn_smem(attr, (const void*)moe_gemv_kernel<1>, kGvTok * (2 * kGvMaxK + 32) + kGvRedBytes);
    moe_gemv_kernel<1><<<grid, kGvWarps * 32, smem, stream>>>(p);
  }
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

}  // namespace gptoss
