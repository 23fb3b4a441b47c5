// dense.cu -- the attention block's dense bf16 projections at decode sizes.
//
// With at most a few tokens, y = x W^T + b (W [N, K] bf16, row-major, the
// nn.Linear weight) is a weight stream: every byte of W is read once and
// multiplied by a few activation rows.  One warp per output row: its lanes
// read the row in 16-byte pieces (8 bf16), straight from HBM into registers,
// against the token rows held in shared memory as fp32, accumulate in fp32,
// add across the warp with shuffles, add the bias in fp32 and round once to
// bf16.  The token rows are staged once per CTA (8 warps = 8 output rows).
#include "common.cuh"
#include "launch.h"

namespace gptoss {

constexpr int kDenseWarps = 8;
constexpr int kDenseMaxT = 4;
constexpr int kDenseMaxK = 8192;

template <int kT>
__global__ void __launch_bounds__(kDenseWarps * 32) dense_gemv_kernel(const uint16_t* __restrict__ x,
                                                                      const uint16_t* __restrict__ W,
                                                                      const uint16_t* __restrict__ bias, int32_t N,
                                                                      int32_t K, uint16_t* __restrict__ out) {
  extern __shared__ __align__(16) float xs[];  // [kT][K] fp32
  for (int i = threadIdx.x; i < kT * K; i += blockDim.x) xs[i] = bf16_bits_to_f32(__ldg(x + i));
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int32_t n = blockIdx.x * kDenseWarps + warp;
  if (n >= N) return;
  const uint4* wr = (const uint4*)(W + (size_t)n * K);
  const int32_t chunks = K >> 3;
  float acc[kT];
#pragma unroll
  for (int t = 0; t < kT; ++t) acc[t] = 0.f;
#pragma unroll 4
  for (int32_t c = lane; c < chunks; c += 32) {
    const uint4 v = __ldg(wr + c);
    const uint32_t wv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int t = 0; t < kT; ++t) {
      const float4* xp = (const float4*)(xs + (size_t)t * K + (size_t)c * 8);
      const float4 a = xp[0], b = xp[1];
      const float xa[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        acc[t] = fmaf(__uint_as_float(wv[j] << 16), xa[2 * j], acc[t]);
        acc[t] = fmaf(__uint_as_float(wv[j] & 0xFFFF0000u), xa[2 * j + 1], acc[t]);
      }
    }
  }
#pragma unroll
  for (int t = 0; t < kT; ++t) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc[t] += __shfl_xor_sync(0xffffffffu, acc[t], o);
  }
  if (lane == 0) {
    const float b = bias ? bf16_bits_to_f32(__ldg(bias + n)) : 0.f;
#pragma unroll
    for (int t = 0; t < kT; ++t) out[(size_t)t * N + n] = f32_to_bf16_bits(acc[t] + b);
  }
}

int dense_gemv_max_tokens() { return kDenseMaxT; }

int launch_dense_gemv(const uint16_t* x, int64_t T, const uint16_t* W, const uint16_t* bias, int32_t N, int32_t K,
                      uint16_t* out, cudaStream_t s) {
  if (T <= 0) return 0;
  if (T > kDenseMaxT || N <= 0 || K <= 0 || K % 8 || K > kDenseMaxK || ((uintptr_t)W & 15)) return -12;
  const size_t smem = (size_t)T * K * sizeof(float);
  const unsigned grid = (unsigned)((N + kDenseWarps - 1) / kDenseWarps);
  static FuncSmemAttr attr1, attr2, attr3, attr4;
  {
    const int mx = kDenseMaxT * kDenseMaxK * (int)sizeof(float);
    ensure_dyn_smem(attr1, (const void*)dense_gemv_kernel<1>, mx);
    ensure_dyn_smem(attr2, (const void*)dense_gemv_kernel<2>, mx);
    ensure_dyn_smem(attr3, (const void*)dense_gemv_kernel<3>, mx);
    ensure_dyn_smem(attr4, (const void*)dense_gemv_kernel<4>, mx);
  }
  switch (T) {
    case 1: dense_gemv_kernel<1><<<grid, kDenseWarps * 32, smem, s>>>(x, W, bias, N, K, out); break;
    case 2: dense_gemv_kernel<2><<<grid, kDenseWarps * 32, smem, s>>>(x, W, bias, N, K, out); break;
    case 3: dense_gemv_kernel<3><<<grid, kDenseWarps * 32, smem, s>>>(x, W, bias, N, K, out); break;
    default: dense_gemv_kernel<4><<<grid, kDenseWarps * 32, smem, s>>>(x, W, bias, N, K, out); break;
  }
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

}  // namespace gptoss
