// dense_tc.cu -- the dense bf16 projections (QKV, attention output,
// unembedding) on the sm_100a tensor cores.
//
// y[t, n] = sum_k x[t, k] W[n, k] (+ b[n]), x [T, K] and W [N, K] bf16
// row-major (nn.Linear), fp32 accumulation in TMEM, one rounding to bf16.
// One kernel serves both shapes the model has:
//
// * decode / few tokens (T <= 256): the weight rows are the MMA's M side
//   (128 rows per tile, A operand) and the tokens its N side (B operand,
//   16..256 columns), so a tile streams 128 weight rows once.  When the
//   weight tiles are fewer than the CTA slots, a cluster of S CTAs splits
//   K; each CTA leaves its fp32 partial in shared memory and, after a
//   cluster barrier, every CTA sums a slice of the rows over the S partials
//   through distributed shared memory (fixed order: deterministic) and
//   writes it.
// * prefill (T > 256): tokens on M (128 per tile), weight rows on N (256
//   per tile); persistent CTAs walk the tiles with double-buffered TMEM
//   accumulators so the epilogue of one tile overlaps the MMAs of the next.
//
// Both operands arrive by TMA (128-byte swizzle, 64 bf16 of K per row and
// stage); one thread issues tcgen05.mma kind::f16 (bf16 x bf16 -> fp32)
// from shared-memory descriptors; four epilogue warps read TMEM with
// tcgen05.ld.  Every wait is bounded (kWaitPolls) and reports through the
// caller's error word.
#include "common.cuh"
#include "launch.h"

namespace gptoss {

constexpr int kDnThreads = 192;          // warp 0 TMA, warp 1 MMA + TMEM, warps 2-5 epilogue
constexpr int kDnBK = 64;                // K elements per stage (one 128-byte swizzled row)
constexpr int kDnABytes = 128 * 128;     // A stage: 128 rows x 128 bytes
constexpr int kDnMaxSplit = 8;

struct DenseParams {
  uint16_t* out;
  const uint16_t* bias;   // indexed by the output feature, or null
  int64_t ld_a;           // output element stride of an A row
  int64_t ld_b;           // output element stride of a B row
  int32_t rows_a, rows_b, K;
  int32_t tiles_a, tiles_b;
  int32_t bias_on_a;      // 1: bias[a_row], 0: bias[b_row]
  uint32_t* err;
};

template <int kBN>
struct DenseCfg {
  static constexpr int kBBytes = kBN * 128;
  static constexpr int kStageBytes = kDnABytes + kBBytes;
  static constexpr int kStages = kBN <= 32 ? 5 : (kBN == 64 ? 4 : (kBN == 128 ? 6 : 4));
  static constexpr int kBarOff = kStages * kStageBytes;
  static constexpr int kAlloc = kBarOff + 256 + 1024;  // + barriers/misc + alignment slack
  static constexpr uint32_t kTmemCols = 2 * kBN < 32 ? 32 : 2 * kBN;
  static_assert(kBN % 16 == 0 && kBN >= 16 && kBN <= 256, "MMA N for M = 128");
  static_assert(kStages * kStageBytes >= 129 * kBN * 4, "the split-K partial reuses the stage buffers");
};

// 32 columns of this warp's TMEM lane quarter into r[0..31], or 16 into
// r[0..15] when only 16 are left (kBN = 16).
__device__ __forceinline__ void dense_tmem_ld(uint32_t taddr, int ncols, uint32_t (&r)[32]) {
  if (ncols >= 32) {
    tmem_ld_x32(taddr, r);
  } else {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr)
        : "memory");
  }
  tmem_ld_wait();
}

// One output element: fp32 sum + bias, rounded once.
__device__ __forceinline__ void dense_store(const DenseParams& p, int32_t a, int32_t b, float v) {
  if (p.bias) v += bf16_bits_to_f32(__ldg(p.bias + (p.bias_on_a ? a : b)));
  p.out[(int64_t)a * p.ld_a + (int64_t)b * p.ld_b] = f32_to_bf16_bits(v);
}

template <int kBN>
__global__ void __launch_bounds__(kDnThreads, 1)
    dense_gemm_tc_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                         const DenseParams p) {
  using C = DenseCfg<kBN>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint64_t* bars = (uint64_t*)(smem + C::kBarOff);
  uint64_t* full_bar = bars;                   // [kStages] TMA tx
  uint64_t* empty_bar = full_bar + C::kStages;  // [kStages] MMA commit
  uint64_t* accfull_bar = empty_bar + C::kStages;  // [2] MMA commit at the end of a tile
  uint64_t* accempty_bar = accfull_bar + 2;        // [2] the four epilogue warps
  uint32_t* misc = (uint32_t*)(accempty_bar + 2);
  volatile uint32_t* tmem_slot = misc;
  volatile uint32_t* abort_s = misc + 1;

  const int warp = threadIdx.x >> 5;
  const uint32_t S = gridDim.y;                   // CTAs of a cluster splitting K
  const uint32_t srank = blockIdx.y;              // this CTA's K slice
  const int32_t nch = (p.K + kDnBK - 1) / kDnBK;  // K chunks of the whole product
  const int32_t c_lo = (int32_t)(((int64_t)nch * srank) / S), c_hi = (int32_t)(((int64_t)nch * (srank + 1)) / S);
  const int32_t total = p.tiles_a * p.tiles_b;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&accfull_bar[s], 1);
      mbar_init(&accempty_bar[s], 4);
    }
    *abort_s = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc((uint32_t*)tmem_slot, C::kTmemCols);
    tmem_relinquish();
  }
  if (warp == 0 && (threadIdx.x & 31) == 0) {
    tma_prefetch_desc(&tmap_a);
    tma_prefetch_desc(&tmap_b);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------- TMA producer
    if (elect_one()) {
      uint32_t it = 0;
      for (int32_t t = blockIdx.x; t < total && !*abort_s; t += gridDim.x) {
        const int32_t ta = t % p.tiles_a, tb = t / p.tiles_a;
        for (int32_t c = c_lo; c < c_hi; ++c, ++it) {
          const uint32_t s = it % C::kStages, ph = (it / C::kStages) & 1;
          if (!mbar_wait(&empty_bar[s], ph ^ 1, p.err, kErrTimeoutEmpty)) { *abort_s = 1; break; }
          uint8_t* st = smem + s * C::kStageBytes;
          // out-of-range rows and K columns land as zeros and still count
          mbar_arrive_expect_tx(&full_bar[s], C::kStageBytes);
          tma_load_2d(st, &tmap_a, c * kDnBK, ta * 128, &full_bar[s]);
          tma_load_2d(st + kDnABytes, &tmap_b, c * kDnBK, tb * kBN, &full_bar[s]);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------- MMA issuer
    if (elect_one()) {
      const uint32_t idesc = make_idesc_bf16(128, kBN);
      uint32_t it = 0, tl = 0;
      for (int32_t t = blockIdx.x; t < total && !*abort_s; t += gridDim.x, ++tl) {
        const uint32_t ab = tl & 1, aph = (tl >> 1) & 1;
        if (!mbar_wait(&accempty_bar[ab], aph ^ 1, p.err, kErrTimeoutAccum)) { *abort_s = 1; break; }
        tc_fence_after();
        const uint32_t d = tmem_base + ab * kBN;
        bool ok = true;
        for (int32_t c = c_lo; c < c_hi; ++c, ++it) {
          const uint32_t s = it % C::kStages, ph = (it / C::kStages) & 1;
          if (!mbar_wait(&full_bar[s], ph, p.err, kErrTimeoutFull)) { ok = false; break; }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + s * C::kStageBytes);
          const uint64_t da = make_sdesc_sw128(sa), db = make_sdesc_sw128(sa + kDnABytes);
#pragma unroll
          for (int k = 0; k < 4; ++k) tc_mma_ss(d, da + 2 * k, db + 2 * k, idesc, (c > c_lo || k > 0) ? 1u : 0u);
          tc_commit(&empty_bar[s]);
        }
        if (!ok) { *abort_s = 1; break; }
        tc_commit(&accfull_bar[ab]);
      }
    }
  } else {
    // ------------------------------------------------ epilogue (warps 2-5)
    const int q = warp & 3;                 // TMEM lane quarter this warp may read
    const int lane = threadIdx.x & 31;
    const int row = q * 32 + lane;          // accumulator row = A row within the tile
    uint32_t tl = 0;
    for (int32_t t = blockIdx.x; t < total; t += gridDim.x, ++tl) {
      const uint32_t ab = tl & 1, aph = (tl >> 1) & 1;
      if (*abort_s) break;
      if (!mbar_wait(&accfull_bar[ab], aph, p.err, kErrTimeoutAccum)) { *abort_s = 1; break; }
      tc_fence_after();
      const int32_t ta = t % p.tiles_a, tb = t / p.tiles_a;
      const int32_t a = ta * 128 + row;
      const uint32_t tq = tmem_base + ((uint32_t)(q * 32) << 16) + ab * kBN;
      if (S == 1) {
        for (int j0 = 0; j0 < kBN; j0 += 32) {
          uint32_t r[32];
          const int ncol = kBN - j0 < 32 ? kBN - j0 : 32;
          dense_tmem_ld(tq + j0, ncol, r);
          if (a < p.rows_a) {
            if (p.ld_b == 1 && (tb * kBN + j0 + 32 <= p.rows_b) && ncol == 32 && ((p.ld_a & 7) == 0)) {
              // 32 consecutive outputs of one row: four 16-byte stores
              uint32_t w[16];
#pragma unroll
              for (int i = 0; i < 16; ++i) {
                const int32_t b0 = tb * kBN + j0 + 2 * i;
                float v0 = __uint_as_float(r[2 * i]), v1 = __uint_as_float(r[2 * i + 1]);
                if (p.bias) {
                  v0 += bf16_bits_to_f32(__ldg(p.bias + (p.bias_on_a ? a : b0)));
                  v1 += bf16_bits_to_f32(__ldg(p.bias + (p.bias_on_a ? a : b0 + 1)));
                }
                w[i] = (uint32_t)f32_to_bf16_bits(v0) | ((uint32_t)f32_to_bf16_bits(v1) << 16);
              }
              uint4* dst = (uint4*)(p.out + (int64_t)a * p.ld_a + tb * kBN + j0);
#pragma unroll
              for (int i = 0; i < 4; ++i) dst[i] = make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
            } else {
#pragma unroll
              for (int i = 0; i < 32; ++i) {
                const int32_t b = tb * kBN + j0 + i;
                if (i < ncol && b < p.rows_b) dense_store(p, a, b, __uint_as_float(r[i]));
              }
            }
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&accempty_bar[ab]);
      } else {
        // split K: this CTA's partial -> shared memory, column-major with a
        // 129-float pitch (conflict-free both along rows and along columns)
        float* part = (float*)smem;
        const int32_t nvalid = min(kBN, p.rows_b - tb * kBN);  // token columns that exist
        for (int j0 = 0; j0 < kBN && j0 < nvalid; j0 += 32) {
          uint32_t r[32];
          const int ncol = kBN - j0 < 32 ? kBN - j0 : 32;
          dense_tmem_ld(tq + j0, ncol, r);
#pragma unroll
          for (int i = 0; i < 32; ++i)
            if (i < ncol && j0 + i < nvalid) part[(j0 + i) * 129 + row] = __uint_as_float(r[i]);
        }
        break;  // one tile per cluster in split mode
      }
    }
  }

  if (S > 1) {
    // every CTA of the cluster has its partial in shared memory (or gave up)
    __syncwarp();
    cluster_sync_all();
    if (warp >= 2 && !*abort_s) {
      const int32_t t = blockIdx.x;
      const int32_t ta = t % p.tiles_a, tb = t / p.tiles_a;
      // this CTA's slice of the tile's rows, summed over the S partials
      const int32_t r_lo = (int32_t)((128u * srank) / S), r_hi = (int32_t)((128u * (srank + 1)) / S);
      const int32_t nr = r_hi - r_lo;
      const uint32_t part0 = smem_u32(smem);
      const int32_t nvalid = min(kBN, p.rows_b - tb * kBN);
      const int et = threadIdx.x - 64;
      const bool rows_fast = p.ld_a == 1;  // consecutive threads on consecutive output addresses
      for (int32_t e = et; e < nr * nvalid; e += 128) {
        const int32_t rr = rows_fast ? r_lo + e % nr : r_lo + e / nvalid;
        const int32_t jj = rows_fast ? e / nr : e % nvalid;
        const int32_t a = ta * 128 + rr, b = tb * kBN + jj;
        // the S partials are read independently, then added in rank order
        float x[kDnMaxSplit];
#pragma unroll
        for (int s = 0; s < kDnMaxSplit; ++s) {
          x[s] = 0.0f;
          if ((uint32_t)s < S) {
            const uint32_t addr = mapa_shared(part0 + (uint32_t)((jj * 129 + rr) * 4), (uint32_t)s);
            asm("ld.shared::cluster.f32 %0, [%1];" : "=f"(x[s]) : "r"(addr));
          }
        }
        float v = x[0];
#pragma unroll
        for (int s = 1; s < kDnMaxSplit; ++s)
          if ((uint32_t)s < S) v += x[s];
        if (a < p.rows_a && b < p.rows_b) dense_store(p, a, b, v);
      }
    }
    // no CTA leaves while another still reads its shared memory
    cluster_sync_all();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::kTmemCols);
  }
}

// ------------------------------------------------------------------ host --
int make_tmap_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype, int esize, uint64_t rows,
                 uint64_t cols, uint32_t box_cols, uint32_t box_rows, CUtensorMapSwizzle swz);

static int dense_slots_per_sm(int bn) { return bn <= 64 ? 2 : 1; }

// Clusters of `split` CTAs of this configuration that can be resident at
// once (cached per device, configuration and split; 0 when none fits).
template <int kBN>
static int dense_max_clusters(int split) {
  constexpr int kMaxDev = 16;
  static std::atomic<int> cache[kMaxDev][kDnMaxSplit + 1] = {};  // clusters + 1; 0 = not measured yet
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDev) {
    (void)cudaGetLastError();
    return 0;
  }
  int c = cache[dev][split].load(std::memory_order_acquire);
  if (c == 0) {
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attrs[1];
    attrs[0].id = cudaLaunchAttributeClusterDimension;
    attrs[0].val.clusterDim.x = 1;
    attrs[0].val.clusterDim.y = split;
    attrs[0].val.clusterDim.z = 1;
    cfg.blockDim = dim3(kDnThreads);
    cfg.dynamicSmemBytes = DenseCfg<kBN>::kAlloc;
    cfg.gridDim = dim3(1, split);
    cfg.attrs = attrs;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, dense_gemm_tc_kernel<kBN>, &cfg) != cudaSuccess) {
      (void)cudaGetLastError();
      n = 0;
    }
    c = n + 1;
    cache[dev][split].store(c, std::memory_order_release);
  }
  return c - 1;
}

template <int kBN>
static int launch_dense_bn(const CUtensorMap& ta, const CUtensorMap& tb, const DenseParams& p, cudaStream_t s) {
  using C = DenseCfg<kBN>;
  auto kern = dense_gemm_tc_kernel<kBN>;
  static FuncSmemAttr attr;
  // (all of the SM's unified memory as shared memory: two decode-size CTAs per SM)
  ensure_dyn_smem(attr, (const void*)kern, C::kAlloc, 100);
  const int slots = device_sm_count() * dense_slots_per_sm(kBN);
  const int32_t tiles = p.tiles_a * p.tiles_b;
  const int32_t nch = (p.K + kDnBK - 1) / kDnBK;
  int split = 1;
  if (tiles < slots) {
    // the largest split whose clusters all fit at once, at least four K chunks per CTA
    for (int c = kDnMaxSplit; c >= 2; --c) {
      if (tiles * c > slots || nch / c < 4) continue;
      if (tiles <= dense_max_clusters<kBN>(c)) {
        split = c;
        break;
      }
    }
  }
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attrs[1];
  cfg.blockDim = dim3(kDnThreads);
  cfg.dynamicSmemBytes = C::kAlloc;
  cfg.stream = s;
  if (split > 1) {
    attrs[0].id = cudaLaunchAttributeClusterDimension;
    attrs[0].val.clusterDim.x = 1;
    attrs[0].val.clusterDim.y = split;
    attrs[0].val.clusterDim.z = 1;
    cfg.attrs = attrs;
    cfg.numAttrs = 1;
    cfg.gridDim = dim3((unsigned)tiles, (unsigned)split);
  } else {
    cfg.gridDim = dim3((unsigned)(tiles < slots ? tiles : slots), 1);
  }
  return cudaLaunchKernelEx(&cfg, kern, ta, tb, p) == cudaSuccess ? 0 : -3;
}

int launch_dense_gemm(const uint16_t* x, int64_t T, const uint16_t* W, const uint16_t* bias, int32_t N, int32_t K,
                      uint16_t* out, uint32_t* err, cudaStream_t s) {
  if (T <= 0) return 0;
  if (N <= 0 || K <= 0 || K % 8 || ((uintptr_t)x & 15) || ((uintptr_t)W & 15) || ((uintptr_t)out & 15)) return -12;
  if (T > 0x7FFFFFFF) return -12;
  DenseParams p;
  p.out = out;
  p.bias = bias;
  p.K = K;
  p.err = err;
  CUtensorMap ta, tb;
  int rc;
  if (T <= 256) {
    // weights on the MMA's M side, tokens on N
    const int bn = T <= 16 ? 16 : T <= 32 ? 32 : T <= 64 ? 64 : T <= 128 ? 128 : 256;
    p.rows_a = N;
    p.rows_b = (int32_t)T;
    p.tiles_a = (N + 127) / 128;
    p.tiles_b = 1;
    p.ld_a = 1;
    p.ld_b = N;
    p.bias_on_a = 1;
    rc = make_tmap_2d(&ta, W, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, (uint64_t)N, (uint64_t)K, kDnBK, 128,
                      CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    rc = make_tmap_2d(&tb, x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, (uint64_t)T, (uint64_t)K, kDnBK, (uint32_t)bn,
                      CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    switch (bn) {
      case 16: return launch_dense_bn<16>(ta, tb, p, s);
      case 32: return launch_dense_bn<32>(ta, tb, p, s);
      case 64: return launch_dense_bn<64>(ta, tb, p, s);
      case 128: return launch_dense_bn<128>(ta, tb, p, s);
      default: return launch_dense_bn<256>(ta, tb, p, s);
    }
  }
  // tokens on M, weight rows on N
  p.rows_a = (int32_t)T;
  p.rows_b = N;
  p.tiles_a = (int32_t)((T + 127) / 128);
  p.tiles_b = (N + 255) / 256;
  p.ld_a = N;
  p.ld_b = 1;
  p.bias_on_a = 0;
  rc = make_tmap_2d(&ta, x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, (uint64_t)T, (uint64_t)K, kDnBK, 128,
                    CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  rc = make_tmap_2d(&tb, W, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, (uint64_t)N, (uint64_t)K, kDnBK, 256,
                    CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  return launch_dense_bn<256>(ta, tb, p, s);
}

}  // namespace gptoss
