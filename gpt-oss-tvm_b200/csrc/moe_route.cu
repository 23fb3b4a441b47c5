// moe_route.cu -- the token side of the MoE block: RMSNorm, the router
// (bit-exact to the reference's serial bf16 accumulation), top-k + softmax,
// the expert-major permutation, the activation gather and the weighted
// combine with the residual.  All integer/index work is bit-exact; the
// floating-point steps reproduce the reference's operation order and
// rounding (no contraction: __fmul_rn/__fadd_rn where the reference has
// separate multiply and add).
#include "common.cuh"

namespace gptoss {

// ------------------------------------------------------------ RMSNorm --
// nn.RMSNorm as lowered for model/mlp.py:81-87,375 (and attention.py:84,193):
// serial fp32 sum of squares in column order, r = 1/sqrtf(sum/H + eps),
// out = bf16((r*x)*w).  One lane owns one token's serial sum; a warp stages
// 32 tokens x 64 columns through shared memory so global reads coalesce.
constexpr int kNormTok = 32;
__global__ void __launch_bounds__(256) rmsnorm_kernel(const uint16_t* __restrict__ x, const uint16_t* __restrict__ w,
                                                       int64_t M, int32_t H, float eps, uint16_t* __restrict__ out) {
  __shared__ uint16_t tile[8][kNormTok][66];
  __shared__ float rs[8][kNormTok];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t tok0 = ((int64_t)blockIdx.x * 8 + warp) * kNormTok;
  if (tok0 >= M) return;
  float ss = 0.0f;
  for (int32_t k0 = 0; k0 < H; k0 += 64) {
    // load 32 tokens x 64 columns (2 columns per lane per token)
    for (int t = 0; t < kNormTok; ++t) {
      const int64_t m = tok0 + t;
      uint32_t v = 0;
      const int32_t k = k0 + 2 * lane;
      if (m < M && k + 1 < H) v = *(const uint32_t*)(x + m * H + k);
      else if (m < M && k < H) v = x[m * H + k];
      tile[warp][t][2 * lane] = (uint16_t)(v & 0xFFFF);
      tile[warp][t][2 * lane + 1] = (uint16_t)(v >> 16);
    }
    __syncwarp();
    const int32_t kn = min(64, H - k0);
    for (int32_t j = 0; j < kn; ++j) {
      const float v = bf16_bits_to_f32(tile[warp][lane][j]);
      ss = __fadd_rn(ss, __fmul_rn(v, v));
    }
    __syncwarp();
  }
  rs[warp][lane] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)H), eps)));
  __syncwarp();
  for (int t = 0; t < kNormTok; ++t) {
    const int64_t m = tok0 + t;
    if (m >= M) break;
    const float r = rs[warp][t];
    for (int32_t k = lane; k < H; k += 32) {
      const float v = __fmul_rn(__fmul_rn(r, bf16_bits_to_f32(x[m * H + k])), bf16_bits_to_f32(w[k]));
      out[m * H + k] = f32_to_bf16_bits(v);
    }
  }
}

// -------------------------------------------------------------- router --
// logits[m, e] = bf16(float(acc) + float(b[e])) where acc is a bf16 running
// sum: acc = bf16(float(acc) + t[m,k]*W[e,k]) for k = 0..H-1 in order
// (nn.Linear at model/mlp.py:88-92,376 lowered with a bf16 accumulator).
// t*W is exact in fp32, so fma(t, W, acc) == acc + t*W; the bf16 rounding is
// a cvt.rn.bf16x2 whose other half is zero, which leaves float(bf16(s)) in
// the register.  Two chains share one packed f32x2 FMA.
constexpr int kRouterTok = 16;   // tokens per block
constexpr int kRouterKT = 32;    // k per shared-memory tile
template <int EPT>  // experts per thread (even)
__global__ void __launch_bounds__(128) router_kernel(const uint16_t* __restrict__ t, const uint16_t* __restrict__ W,
                                                      const uint16_t* __restrict__ b, int64_t M, int32_t E, int32_t H,
                                                      uint16_t* __restrict__ logits) {
  // thread = (token slot 0..15, expert group 0..7); expert group g owns
  // experts [g*EPT, (g+1)*EPT)
  extern __shared__ float rsm[];
  constexpr int kTS = kRouterKT + 2;               // padded row: 16 token rows hit distinct banks
  float* ts = rsm;                                  // [kRouterTok][kTS]
  float2* ws = (float2*)(ts + kRouterTok * kTS);    // [kRouterKT][E/2] pairs (e, e+1)
  const int tid = threadIdx.x;
  const int slot = tid & 15, grp = tid >> 4;
  const int64_t m = (int64_t)blockIdx.x * kRouterTok + slot;
  constexpr int P = EPT / 2;
  unsigned long long acc[P];
#pragma unroll
  for (int i = 0; i < P; ++i) acc[i] = 0ull;
  const int32_t pairs = E / 2;
  for (int32_t k0 = 0; k0 < H; k0 += kRouterKT) {
    __syncthreads();
    for (int i = tid; i < kRouterTok * kRouterKT; i += 128) {
      const int s = i / kRouterKT, kk = i % kRouterKT;
      const int64_t mm = (int64_t)blockIdx.x * kRouterTok + s;
      ts[s * kTS + kk] = (mm < M && k0 + kk < H) ? bf16_bits_to_f32(t[mm * H + k0 + kk]) : 0.0f;
    }
    for (int i = tid; i < kRouterKT * pairs; i += 128) {
      const int kk = i / pairs, pr = i % pairs;
      float2 v = make_float2(0.0f, 0.0f);
      if (k0 + kk < H) {
        v.x = bf16_bits_to_f32(W[(int64_t)(2 * pr) * H + k0 + kk]);
        v.y = bf16_bits_to_f32(W[(int64_t)(2 * pr + 1) * H + k0 + kk]);
      }
      ws[kk * pairs + pr] = v;
    }
    __syncthreads();
    const int32_t kn = min(kRouterKT, H - k0);
    for (int32_t kk = 0; kk < kn; ++kk) {
      const float tv = ts[slot * kTS + kk];
      const unsigned long long tt = ((unsigned long long)__float_as_uint(tv) << 32) | __float_as_uint(tv);
#pragma unroll
      for (int i = 0; i < P; ++i) {
        const float2 wv = ws[kk * pairs + grp * P + i];
        const unsigned long long ww = ((unsigned long long)__float_as_uint(wv.y) << 32) | __float_as_uint(wv.x);
        unsigned long long s = acc[i];
        asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(s) : "l"(tt), "l"(ww));
        uint32_t lo, hi;
        asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(lo) : "f"(__uint_as_float((uint32_t)s)), "f"(0.0f));
        asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(hi) : "f"(__uint_as_float((uint32_t)(s >> 32))), "f"(0.0f));
        acc[i] = ((unsigned long long)hi << 32) | lo;
      }
    }
  }
  if (m < M) {
#pragma unroll
    for (int i = 0; i < P; ++i) {
      const int32_t e0 = 2 * (grp * P + i);
      if (e0 < E) {
        const float a0 = __uint_as_float((uint32_t)acc[i]), a1 = __uint_as_float((uint32_t)(acc[i] >> 32));
        logits[m * E + e0] = f32_to_bf16_bits(__fadd_rn(a0, bf16_bits_to_f32(b[e0])));
        logits[m * E + e0 + 1] = f32_to_bf16_bits(__fadd_rn(a1, bf16_bits_to_f32(b[e0 + 1])));
      }
    }
  }
}

// ------------------------------------------------------ top-k softmax --
// nn.op.topk(largest) + nn.op.softmax over the k values (model/mlp.py:381-382):
// value descending, ties to the lower expert index (+0 == -0); softmax with
// bf16 max, e_i = bf16(exp(v_i - max)), bf16 serial sum, w_i = bf16(e_i/sum).
// exp is evaluated in double and rounded once to float (the correctly
// rounded expf), matching a libm expf to the last bit in all but vanishingly
// rare cases.  One warp per token.
__global__ void topk_softmax_kernel(const uint16_t* __restrict__ logits, int64_t M, int32_t E, int32_t K,
                                    uint16_t* __restrict__ weights, int32_t* __restrict__ indices,
                                    uint32_t* err) {
  const int64_t m = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (m >= M) return;
  constexpr int kMaxPerLane = 8;  // E <= 256
  float v[kMaxPerLane];
  uint32_t taken = 0;
#pragma unroll
  for (int i = 0; i < kMaxPerLane; ++i) {
    const int32_t e = lane + 32 * i;
    v[i] = e < E ? bf16_bits_to_f32(logits[m * E + e]) : -INFINITY;
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
      weights[m * K + j] = f32_to_bf16_bits(__fdiv_rn(ex[j], sum));
      indices[m * K + j] = sel_i[j];
      if (sel_i[j] < 0 || sel_i[j] >= E) raise_error(err, kErrBadRouting);
    }
  }
}

// ------------------------------------------------------ permutation --
// Expert-major order of the (token, rank) pairs (the layout of the grouped
// kernels, model/mlp_optimized.py:118-170): rows of expert e occupy
// [indptr[e], indptr[e+1]) in ascending token order.  Also builds the token
// tiles the grouped GEMM walks: an expert with c rows gets ceil(c/256)
// tiles of roundup16(ceil(c/tiles)) rows.
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
    int32_t acc = 0, tacc = 0;
    for (int32_t e = 0; e < E; ++e) {
      const int32_t c = cnt[e];
      indptr[e] = acc;
      tile_ptr[e] = tacc;
      const int32_t nt = (c + 255) / 256;
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
// act[row] = t[token_of_row[row]]  (nn.op.take at model/mlp_optimized.py:150)
__global__ void gather_rows_kernel(const uint16_t* __restrict__ t, const int32_t* __restrict__ token_of_row,
                                   int64_t rows, int32_t H, uint16_t* __restrict__ act) {
  const int64_t r = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (r >= rows) return;
  const int lane = threadIdx.x & 31;
  const int64_t src = token_of_row[r];
  const uint4* s = (const uint4*)(t + src * H);
  uint4* d = (uint4*)(act + r * H);
  for (int32_t i = lane; i < H / 8; i += 32) d[i] = s[i];
}

// ------------------------------------------------------------ combine --
// out[m, c] = bf16(float(x[m,c]) + float(bf16(sum_r h2[row(m,r), c] * w[m,r])))
// with the serial fp32 sum over r of run_gating (model/mlp.py:328-369) and
// the residual of model/mlp.py:399-402.
__global__ void combine_kernel(const float* __restrict__ h2, const int32_t* __restrict__ row_of_pair,
                               const uint16_t* __restrict__ w, const uint16_t* __restrict__ x, int64_t M, int32_t K,
                               int32_t H, uint16_t* __restrict__ out) {
  const int32_t cblocks = (H + blockDim.x - 1) / blockDim.x;
  const int64_t m = blockIdx.x / cblocks;
  const int32_t c = (int32_t)(blockIdx.x % cblocks) * blockDim.x + threadIdx.x;
  if (m >= M || c >= H) return;
  float acc = 0.0f;
  for (int32_t r = 0; r < K; ++r) {
    const int32_t row = row_of_pair[m * K + r];
    acc = __fadd_rn(acc, __fmul_rn(h2[(int64_t)row * H + c], bf16_bits_to_f32(w[m * K + r])));
  }
  const float o = round_bf16(acc);
  out[m * H + c] = f32_to_bf16_bits(__fadd_rn(bf16_bits_to_f32(x[m * H + c]), o));
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

// ------------------------------------------------------------- launch --
int launch_rmsnorm(const uint16_t* x, const uint16_t* w, int64_t M, int32_t H, float eps, uint16_t* out,
                   cudaStream_t s) {
  if (M <= 0) return 0;
  const int64_t blocks = (M + 8 * kNormTok - 1) / (8 * kNormTok);
  rmsnorm_kernel<<<(unsigned)blocks, 256, 0, s>>>(x, w, M, H, eps, out);
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

int launch_router(const uint16_t* t, const uint16_t* W, const uint16_t* b, int64_t M, int32_t E, int32_t H,
                  uint16_t* logits, cudaStream_t s) {
  if (M <= 0) return 0;
  if (E % 16 != 0 || E > 256) return -12;
  const unsigned blocks = (unsigned)((M + kRouterTok - 1) / kRouterTok);
  const size_t smem = (size_t)kRouterTok * (kRouterKT + 2) * 4 + (size_t)kRouterKT * E * 4;
  const int ept = E / 8;
  switch (ept) {
    case 2: router_kernel<2><<<blocks, 128, smem, s>>>(t, W, b, M, E, H, logits); break;
    case 4: router_kernel<4><<<blocks, 128, smem, s>>>(t, W, b, M, E, H, logits); break;
    case 6: router_kernel<6><<<blocks, 128, smem, s>>>(t, W, b, M, E, H, logits); break;
    case 8: router_kernel<8><<<blocks, 128, smem, s>>>(t, W, b, M, E, H, logits); break;
    case 12: router_kernel<12><<<blocks, 128, smem, s>>>(t, W, b, M, E, H, logits); break;
    case 16: router_kernel<16><<<blocks, 128, smem, s>>>(t, W, b, M, E, H, logits); break;
    case 24: router_kernel<24><<<blocks, 128, smem, s>>>(t, W, b, M, E, H, logits); break;
    case 32: router_kernel<32><<<blocks, 128, smem, s>>>(t, W, b, M, E, H, logits); break;
    default: return -12;
  }
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
  moe_count_scan_kernel<<<1, 1024, (size_t)E * 4, s>>>(idx, pairs, E, indptr, tile_ptr, tile_rows, err);
  if (pairs > 0) moe_place_kernel<<<E, 1024, 0, s>>>(idx, pairs, K, indptr, token_of_row, row_of_pair, expert_of_row);
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

int launch_gather(const uint16_t* t, const int32_t* token_of_row, int64_t rows, int32_t H, uint16_t* act,
                  cudaStream_t s) {
  if (rows <= 0) return 0;
  if (H % 8) return -12;
  gather_rows_kernel<<<(unsigned)((rows + 7) / 8), 256, 0, s>>>(t, token_of_row, rows, H, act);
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

int launch_combine(const float* h2, const int32_t* row_of_pair, const uint16_t* w, const uint16_t* x, int64_t M,
                   int32_t K, int32_t H, uint16_t* out, cudaStream_t s) {
  if (M <= 0) return 0;
  const int64_t blocks = (int64_t)((H + 255) / 256) * M;
  combine_kernel<<<(unsigned)blocks, 256, 0, s>>>(h2, row_of_pair, w, x, M, K, H, out);
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

int launch_mxfp4_dequant(const uint8_t* blocks, const uint8_t* scales, int64_t groups_total, uint16_t* out,
                         cudaStream_t s) {
  if (groups_total <= 0) return 0;
  mxfp4_dequant_kernel<<<(unsigned)((groups_total + 255) / 256), 256, 0, s>>>(blocks, scales, groups_total, out);
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

}  // namespace gptoss
