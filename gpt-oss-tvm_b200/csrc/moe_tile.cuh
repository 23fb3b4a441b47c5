// moe_tile.cuh -- pieces shared by the grouped expert GEMM kernels
// (moe_gemm.cu: tcgen05 kind::f16 with on-chip MXFP4 decode; moe_mx.cu:
// tcgen05 block-scaled kind::mxf8f6f4): the launch parameters, the decoding
// of a persistent tile index into (expert, token rows, weight rows), and the
// epilogue that turns one 32-token block of a finished fp32 accumulator into
// the GEMM's output (clamped SwiGLU for gate/up, fp32 or peer stores for down).
#pragma once

#include "common.cuh"
#include "launch.h"

namespace gptoss {

constexpr int kBM = 128;  // weight rows per tile (MMA M)

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
  // mode 1, optional: row r of the output goes to row (row_dst[r] & 0xFFFFFF)
  // of peer_out[row_dst[r] >> 24] (another GPU's memory), bf16 if out_bf16
  const int32_t* row_dst;
  void* peer_out[kMaxPeerRanks];
  int64_t peer_out_rows;
  int32_t out_bf16;
};

struct TileInfo {
  int32_t expert, row0, nrows, f0;
};

// Tile t -> (expert, first permuted row, rows, first feature row).  A tile
// plan made for larger tiles than this variant holds is reported and skipped
// by every role alike.
// Token-tile-major order: the CTAs running at the same time share one token
// tile's activations (L2 hits) and an expert's weight tiles are reused by its
// token tiles within a short window (DRAM reads close to the algorithmic ones).
// The feature rows of tile t start at f * fstride + fofs (the CTA-pair kernel
// covers 2 x 128 rows per tile, its CTA of rank r the rows from r * 128).
template <int kMaxBN>
__device__ __forceinline__ bool decode_tile(const GemmParams& p, int32_t t, int32_t ftiles, TileInfo& ti,
                                            int32_t fstride = kBM, int32_t fofs = 0) {
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
  ti.f0 = f * fstride + fofs;
  if (per > kMaxBN) {
    if (f == 0 && threadIdx.x == 0) raise_error(p.err, kErrBadTilePlan);
    return false;
  }
  return ti.nrows > 0;
}

// Epilogue of one 32-token column block of a finished accumulator: this
// thread holds weight row `frow` (TMEM lane q * 32 + lane) for tokens
// c0 .. c0 + 31 of the tile in v[].  Mode 0 applies the clamped SwiGLU to
// (glu, linear) lane pairs and stores bf16 (f16) outputs through the warp's
// shared tile; mode 1 stores fp32, or scatters the rows to other GPUs'
// return buffers (bf16 through the shared tile, or fp32).  `tile`: the warp's
// 2 KB of shared memory.
template <int kMode, bool kF16>
__device__ __forceinline__ void epilogue_block(const GemmParams& p, const TileInfo& ti, const uint32_t (&v)[32],
                                               int32_t c0, int q, int lane, float bias, bool row_ok, int32_t frow,
                                               uint16_t* tile) {
  if (kMode == 0) {
    // lane pair (2j, 2j+1) holds the glu / linear rows of output feature
    // j: the even lane finishes tokens c0..c0+15, the odd lane c0+16..31.
    // The 32 x 16 outputs go through this warp's shared tile
    // [token][feature] and leave as 16-byte rows of 8 features.
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
      const float y = swiglu_f32(gl, li, p.alpha, p.limit);
      const int tok = i + (odd ? 16 : 0);
      tile[tok * 16 + (lane >> 1)] = kF16 ? __half_as_ushort(__float2half_rn(y)) : f32_to_bf16_bits(y);
    }
    __syncwarp();
    const bool warp_rows_ok = ti.f0 + q * 32 + 32 <= p.N;
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const int tok = lane, h = k ^ ((lane >> 2) & 1);  // alternate halves: no bank conflicts
      const int32_t col = c0 + tok;
      const uint4 val = *(const uint4*)(tile + tok * 16 + h * 8);
      const int32_t f = (ti.f0 >> 1) + q * 16 + h * 8;  // first output feature of the 8
      if (col < ti.nrows) {
        uint16_t* dst = out + (size_t)(ti.row0 + col) * p.ldo + f;
        if (warp_rows_ok) {
          *(uint4*)dst = val;
        } else {
          const uint16_t* e = (const uint16_t*)&val;
          for (int u = 0; u < 8; ++u)
            if (2 * (f + u) < p.N) dst[u] = e[u];
        }
      }
    }
    __syncwarp();
  } else if (p.row_dst != nullptr && p.out_bf16) {
    // each token row to its owner's return buffer, bf16: the warp's 32
    // features x 32 tokens go through its shared tile [token][feature] and
    // leave as 16-byte pieces (8 features of one token per lane, 8 tokens per
    // instruction) instead of 2-byte stores
    const int32_t mine = c0 + lane < ti.nrows ? __ldg(p.row_dst + ti.row0 + c0 + lane) : 0;
#pragma unroll
    for (int j = 0; j < 32; ++j)
      tile[j * 32 + lane] = row_ok ? f32_to_bf16_bits(__uint_as_float(v[j]) + bias) : (uint16_t)0;
    __syncwarp();
    const int32_t fq = lane & 3;                        // 8-feature piece of the warp's 32 features
    const int32_t f = ti.f0 + q * 32 + fq * 8;          // its first feature
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int32_t tok = (lane >> 2) + 8 * k;
      const uint32_t o = (uint32_t)__shfl_sync(0xffffffffu, mine, tok);
      const uint32_t peer = o >> 24, orow = o & 0xFFFFFFu;
      void* base = peer < (uint32_t)kMaxPeerRanks ? p.peer_out[peer] : nullptr;
      if (c0 + tok < ti.nrows && base != nullptr && (int64_t)orow < p.peer_out_rows && f < p.N) {
        const uint4 val = *(const uint4*)(tile + tok * 32 + fq * 8);
        uint16_t* dst = (uint16_t*)base + (size_t)orow * p.ldo + f;
        if (f + 8 <= p.N) {
          *(uint4*)dst = val;
        } else {
          const uint16_t* e = (const uint16_t*)&val;
          for (int u = 0; u < 8 && f + u < p.N; ++u) dst[u] = e[u];
        }
      }
    }
    __syncwarp();
  } else if (p.row_dst != nullptr) {
    // fp32 rows to their owners' return buffers: the 32 lanes store 32
    // consecutive features of one row per instruction
    const int32_t mine = c0 + lane < ti.nrows ? __ldg(p.row_dst + ti.row0 + c0 + lane) : 0;
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const int32_t col = c0 + j;
      const uint32_t o = (uint32_t)__shfl_sync(0xffffffffu, mine, j);
      const uint32_t peer = o >> 24, orow = o & 0xFFFFFFu;
      void* base = peer < (uint32_t)kMaxPeerRanks ? p.peer_out[peer] : nullptr;
      if (row_ok && col < ti.nrows && base != nullptr && (int64_t)orow < p.peer_out_rows) {
        const size_t at = (size_t)orow * p.ldo + frow;
        const float y = __uint_as_float(v[j]) + bias;
        if (p.out_bf16) ((uint16_t*)base)[at] = f32_to_bf16_bits(y);
        else ((float*)base)[at] = y;
      }
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

}  // namespace gptoss
