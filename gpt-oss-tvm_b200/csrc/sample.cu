// sample.cu -- top-p sampling from logits on the GPU, the reference's
// sampler (engine.py:38-39, :172-174: TVM's vm.builtin.sample_top_p_from_logits,
// src/runtime/vm/lm_support.cc SampleTopPFromLogits) without the host copy.
//
// The reference sorts (logit, index) by descending logit, returns the first
// when temperature < 1e-6, otherwise takes e = expf((l - max) * (1/T)) and
// their sum S -- a float running sum in sorted order --, then a second float
// running sum of e / S in that order: top_p_sum collects the probabilities
// added while the running sum was below top_p, and the token is the first
// whose running sum / top_p_sum exceeds the uniform draw u.  Both running sums
// round at every step, and over thousands of small terms that rounding moves
// the chosen token by many positions, so this kernel runs the same loops in
// the same order (one thread) rather than another summation.  Only the order
// is computed differently:
//
//   * an element with e < S / 2^27 cannot change either running sum (it is
//     below half an ulp of the sum it is added to, and everything after it is
//     smaller), so only the set C of larger elements is sorted;
//   * C is sorted by (logit descending, index ascending) in shared memory when
//     it has at most 2048 elements, otherwise by a stable radix sort in the
//     caller's scratch (4-bit digits, eight passes, one CTA per row).
//
// One CTA per row.  Ties among logits go to the lower index (std::sort leaves
// their order unspecified).  expf is CUDA's (within 2 ulp); glibc's may differ
// in the last bit, which moves a draw only within ~1e-7 of a boundary.
#include "common.cuh"
#include "launch.h"

namespace gptoss {

constexpr int kSmpThreads = 1024;
constexpr int kSmpCand = 2048;
constexpr int kSmpDigits = 16;  // radix-sort buckets (4-bit digits)

struct SmpShared {
  unsigned long long key[kSmpCand];          // (sortable logit) << 32 | index
  unsigned int cnt[kSmpDigits][kSmpThreads];  // radix-sort counts / offsets per digit and thread
  float redf[32];
  int redi[32];
  unsigned int redu[32];
  int result;
};

// Orders floats: a > b exactly when key(a) < key(b) (descending logits first).
__device__ __forceinline__ uint32_t smp_desc_key(float f) {
  const uint32_t b = __float_as_uint(f);
  const uint32_t asc = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
  return ~asc;
}
__device__ __forceinline__ float smp_key_value(uint32_t k) {
  const uint32_t asc = ~k;
  return __uint_as_float((asc & 0x80000000u) ? (asc & 0x7FFFFFFFu) : ~asc);
}

__device__ __forceinline__ float smp_block_sum(float v, SmpShared& sh) {
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) sh.redf[w] = v;
  __syncthreads();
  v = sh.redf[l];
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Exclusive prefix of v over the block in thread order; the total in `total`.
__device__ __forceinline__ unsigned smp_block_scan(unsigned v, SmpShared& sh, unsigned& total) {
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  unsigned incl = v;
  for (int o = 1; o < 32; o <<= 1) {
    const unsigned t = __shfl_up_sync(0xffffffffu, incl, o);
    if (l >= o) incl += t;
  }
  __syncthreads();
  if (l == 31) sh.redu[w] = incl;
  __syncthreads();
  unsigned wsum = sh.redu[l];
  unsigned wincl = wsum;
  for (int o = 1; o < 32; o <<= 1) {
    const unsigned t = __shfl_up_sync(0xffffffffu, wincl, o);
    if (l >= o) wincl += t;
  }
  total = __shfl_sync(0xffffffffu, wincl, 31);
  const unsigned wbase = __shfl_sync(0xffffffffu, wincl - wsum, w);
  return wbase + incl - v;
}

// Largest value, and the lowest index holding it.
__device__ __forceinline__ void smp_block_argmax(float& v, int& i, SmpShared& sh) {
  for (int o = 16; o > 0; o >>= 1) {
    const float v2 = __shfl_xor_sync(0xffffffffu, v, o);
    const int i2 = __shfl_xor_sync(0xffffffffu, i, o);
    if (v2 > v || (v2 == v && i2 < i)) {
      v = v2;
      i = i2;
    }
  }
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) {
    sh.redf[w] = v;
    sh.redi[w] = i;
  }
  __syncthreads();
  v = sh.redf[l];
  i = sh.redi[l];
  for (int o = 16; o > 0; o >>= 1) {
    const float v2 = __shfl_xor_sync(0xffffffffu, v, o);
    const int i2 = __shfl_xor_sync(0xffffffffu, i, o);
    if (v2 > v || (v2 == v && i2 < i)) {
      v = v2;
      i = i2;
    }
  }
}

// The reference's two loops over n elements in order (one thread):
// element j has logit value(j) and index index(j).
template <typename ValueAt, typename IndexAt>
__device__ int smp_reference_loops(int64_t n, float mx, float scale, double top_p, double u, ValueAt value,
                                   IndexAt index) {
  float S = 0.0f;
  for (int64_t j = 0; j < n; ++j) S += expf((value(j) - mx) * scale);
  // running sum of probabilities; top_p_sum while it is below top_p
  float cum = 0.0f, tps = 0.0f;
  int64_t kept = n - 1;
  for (int64_t j = 0; j < n; ++j) {
    const float prob = __fdiv_rn(expf((value(j) - mx) * scale), S);
    if ((double)cum < top_p) tps += prob;
    cum += prob;
    if ((double)cum >= top_p) {  // every later probability adds nothing to tps
      kept = j;
      break;
    }
  }
  cum = 0.0f;
  for (int64_t j = 0; j <= kept; ++j) {
    cum += __fdiv_rn(expf((value(j) - mx) * scale), S);
    if (u < (double)__fdiv_rn(cum, tps)) return index(j);
  }
  // past the kept prefix the reference keeps scanning; u < 1 is always hit by then
  for (int64_t j = kept + 1; j < n; ++j) {
    cum += __fdiv_rn(expf((value(j) - mx) * scale), S);
    if (u < (double)__fdiv_rn(cum, tps)) return index(j);
  }
  return index(0);
}

__global__ void __launch_bounds__(kSmpThreads) sample_top_p_kernel(const float* __restrict__ logits, int64_t V,
                                                                   int64_t row0, int32_t greedy, float scale,
                                                                   double top_p, const double* __restrict__ uniform,
                                                                   double uniform0, uint32_t* __restrict__ scratch,
                                                                   int32_t* __restrict__ out) {
  extern __shared__ __align__(16) uint8_t smp_raw[];
  SmpShared& sh = *reinterpret_cast<SmpShared*>(smp_raw);
  const int64_t r = row0 + blockIdx.x;
  const float* row = logits + r * V;
  const double u = uniform ? uniform[r] : uniform0;
  const int tid = threadIdx.x;

  // 1. max and argmax
  float mx = -INFINITY;
  int am = 0x7FFFFFFF;
  for (int64_t i = tid; i < V; i += blockDim.x) {
    const float l = row[i];
    if (l > mx) {
      mx = l;
      am = (int)i;
    }
  }
  smp_block_argmax(mx, am, sh);
  if (greedy) {
    if (tid == 0) out[r] = am;
    return;
  }
  // 2. the set C: e >= S / 2^27 (S from a tree sum, only to draw the line)
  float part = 0.0f;
  for (int64_t i = tid; i < V; i += blockDim.x) part += expf((row[i] - mx) * scale);
  const float thr = smp_block_sum(part, sh) * (1.0f / 134217728.0f);
  // contiguous index ranges per thread keep C in index order (stable)
  const int64_t per = (V + blockDim.x - 1) / blockDim.x;
  const int64_t lo = min64(V, (int64_t)tid * per), hi = min64(V, lo + per);
  unsigned c = 0;
  for (int64_t i = lo; i < hi; ++i) c += expf((row[i] - mx) * scale) >= thr ? 1u : 0u;
  unsigned n;
  unsigned pos = smp_block_scan(c, sh, n);

  if (n <= (unsigned)kSmpCand) {
    // 3a. shared memory: bitonic sort of (key, index)
    for (int64_t i = lo; i < hi; ++i)
      if (expf((row[i] - mx) * scale) >= thr)
        sh.key[pos++] = ((unsigned long long)smp_desc_key(row[i]) << 32) | (uint32_t)i;
    for (int j = n + tid; j < kSmpCand; j += blockDim.x) sh.key[j] = ~0ull;
    for (int k = 2; k <= kSmpCand; k <<= 1) {
      for (int j = k >> 1; j > 0; j >>= 1) {
        __syncthreads();
        for (int i = tid; i < kSmpCand; i += blockDim.x) {
          const int p = i ^ j;
          if (p > i) {
            const unsigned long long a = sh.key[i], b = sh.key[p];
            if (((i & k) == 0) ? (a > b) : (a < b)) {
              sh.key[i] = b;
              sh.key[p] = a;
            }
          }
        }
      }
    }
    __syncthreads();
    if (tid == 0) {
      out[r] = smp_reference_loops(
          (int64_t)n, mx, scale, top_p, u, [&](int64_t j) { return smp_key_value((uint32_t)(sh.key[j] >> 32)); },
          [&](int64_t j) { return (int)(uint32_t)sh.key[j]; });
    }
    return;
  }

  // 3b. scratch: stable radix sort of (key, index) over C, 4 bits per pass
  uint32_t* ka = scratch + (size_t)blockIdx.x * 4 * (size_t)V;
  uint32_t* ia = ka + V;
  uint32_t* kb = ia + V;
  uint32_t* ib = kb + V;
  for (int64_t i = lo; i < hi; ++i) {
    if (expf((row[i] - mx) * scale) >= thr) {
      ka[pos] = smp_desc_key(row[i]);
      ia[pos] = (uint32_t)i;
      ++pos;
    }
  }
  const int64_t cper = ((int64_t)n + blockDim.x - 1) / blockDim.x;
  const int64_t clo = min64((int64_t)n, (int64_t)tid * cper), chi = min64((int64_t)n, clo + cper);
  for (int pass = 0; pass < 8; ++pass) {
    const int sft = 4 * pass;
    __syncthreads();  // the previous pass's scatter is complete
    for (int d = 0; d < kSmpDigits; ++d) sh.cnt[d][tid] = 0;
    for (int64_t i = clo; i < chi; ++i) ++sh.cnt[(ka[i] >> sft) & 15][tid];
    __syncthreads();
    // exclusive scan over (digit, thread) in that order: thread j owns the 16
    // consecutive entries j*16 .. j*16+15 of the flattened array
    unsigned* flat = &sh.cnt[0][0];
    unsigned run = 0, loc[kSmpDigits];
#pragma unroll
    for (int q = 0; q < kSmpDigits; ++q) {
      loc[q] = run;
      run += flat[tid * kSmpDigits + q];
    }
    unsigned tot;
    const unsigned base = smp_block_scan(run, sh, tot);
    __syncthreads();
#pragma unroll
    for (int q = 0; q < kSmpDigits; ++q) flat[tid * kSmpDigits + q] = base + loc[q];
    __syncthreads();
    for (int64_t i = clo; i < chi; ++i) {
      const uint32_t k = ka[i];
      const unsigned dst = sh.cnt[(k >> sft) & 15][tid]++;
      kb[dst] = k;
      ib[dst] = ia[i];
    }
    uint32_t* t = ka;
    ka = kb;
    kb = t;
    t = ia;
    ia = ib;
    ib = t;
  }
  __syncthreads();
  if (tid == 0) {
    out[r] = smp_reference_loops((int64_t)n, mx, scale, top_p, u, [&](int64_t j) { return smp_key_value(ka[j]); },
                                 [&](int64_t j) { return (int)ia[j]; });
  }
}

int64_t sample_top_p_scratch_bytes_per_row(int64_t V) { return 16 * V; }

int launch_sample_top_p(const float* logits, int64_t B, int64_t V, double temperature, double top_p,
                        const double* uniform, double uniform0, void* scratch, int64_t scratch_bytes, int32_t* out,
                        cudaStream_t s) {
  if (B <= 0) return 0;
  if (V <= 0 || V > 0x7FFFFFFF) return -12;
  const int greedy = temperature < 1e-6 ? 1 : 0;
  const float scale = greedy ? 1.0f : (float)(1.0 / temperature);  // the reference's 1.0f / temperature
  const int64_t per_row = sample_top_p_scratch_bytes_per_row(V);
  const int64_t rows = greedy ? B : (scratch ? scratch_bytes / per_row : 0);
  if (rows < 1) return -13;
  static FuncSmemAttr attr;
  ensure_dyn_smem(attr, (const void*)sample_top_p_kernel, (int)sizeof(SmpShared));
  // rows in groups that the scratch holds
  for (int64_t r0 = 0; r0 < B; r0 += rows) {
    const int64_t nb = min64(rows, B - r0);
    sample_top_p_kernel<<<(unsigned)nb, kSmpThreads, sizeof(SmpShared), s>>>(
        logits, V, r0, greedy, scale, top_p, uniform, uniform0, (uint32_t*)scratch, out);
  }
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

}  // namespace gptoss
