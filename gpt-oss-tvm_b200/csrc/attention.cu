// attention.cu -- gpt-oss attention with learned sinks, sliding-window / full
// causal masks, GQA and YaRN RoPE (model/attention.py:15-256).
//
//   qkv_rope_kernel      split of the fused QKV projection, YaRN RoPE on q and
//                        k (attention.py:96-180), k/v written to cache slots
//                        (the append_mha_kv step, attention.py:214)
//   attn_prefill_tc_kernel  tcgen05 attention for long key ranges (full-causal
//                        layers): two 128-query tiles ping-pong on one SM,
//                        scores and outputs in TMEM (see below)
//   attn_prefill_kernel  FlashAttention-style causal attention of a chunk of
//                        queries over its keys, optional sliding window,
//                        base-2 online softmax, lse, sink rescale fused
//   attn_decode_kernel   one query per sequence over its cache, split along
//                        the keys (each split keeps its own softmax state)
//   attn_decode_merge    merges the splits, applies the sink
//   attn_merge_kernel    merge of two (o, lse) states (extend mode,
//                        attention.py:225-233)
//   sink_rescale_kernel  o *= bf16(sigmoid(ln2*lse - sink)) (attention.py:240-247)
//
// Score convention (the reference's TVM kernels): s = q.k * sm_scale * log2(e),
// lse = m + log2(sum exp2(s - m)) (base 2).  The sink rescale folds exp(sink)
// into the softmax denominator: sigmoid(ln2*lse - sink) = Z / (Z + e^sink).
#include "common.cuh"
#include "launch.h"

namespace gptoss {

constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

// ------------------------------------------------------------ mma.sync --
__device__ __forceinline__ void mma_16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
// 16-byte async copy with zero fill when !valid.
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
  const int n = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(n) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}
// Byte offset of 16-byte chunk `c` of row `r` in a tile of 128-byte rows,
// XOR-swizzled so that ldmatrix row reads are bank-conflict free.
__device__ __forceinline__ uint32_t swz(int r, int c) { return (uint32_t)(r * 128 + ((c ^ (r & 7)) << 4)); }

// ----------------------------------------------------------- QKV + RoPE --
// qkv [S, (Hq + 2 Hkv) * D] bf16 (the fused projection, attention.py:206-211)
// -> q [S, Hq, D] rotated; k rotated and v copied into cache rows slot[s]
// (k_cache / v_cache [num_slots, Hkv, D]).  inv_freq [D/2] is the YaRN
// inverse frequency table (computed on the host in fp32 with the reference's
// formula); angle = float(pos) * inv_freq; the rotation is
//   d <  D/2 : x[d]*(cos*conc) - x[d+D/2]*(sin*conc)
//   d >= D/2 : x[d-D/2]*(sin*conc) + x[d]*(cos*conc)
// with one rounding to bf16 at the end (attention.py:126-167).
struct RopeTable {
  float inv_freq[128];
};

// One block per (token, group of kRopeHeads heads): the block computes the
// D/2 rotation factors of its token once (sincosf of pos * inv_freq[f],
// times the concentration) and applies them to its heads.
constexpr int kRopeHeads = 8;

__global__ void qkv_rope_kernel(const uint16_t* __restrict__ qkv, const int32_t* __restrict__ pos,
                                const int32_t* __restrict__ slot, int64_t S, int32_t Hq, int32_t Hkv, int32_t D,
                                const RopeTable tab, float conc, uint16_t* __restrict__ q_out,
                                uint16_t* __restrict__ k_cache, uint16_t* __restrict__ v_cache) {
  __shared__ float cos_s[128], sin_s[128];
  const int64_t s = blockIdx.x;
  if (s >= S) return;
  const int32_t Ht = Hq + 2 * Hkv;
  const int32_t h0 = blockIdx.y * kRopeHeads;
  const int32_t nh = min(kRopeHeads, Ht - h0);
  const uint16_t* row = qkv + s * (int64_t)Ht * D;
  const int32_t half = D / 2;
  const float p = (float)pos[s];
  const int64_t dst_slot = slot ? slot[s] : s;
  for (int32_t f = threadIdx.x; f < half; f += blockDim.x) {
    const float ang = __fmul_rn(p, tab.inv_freq[f]);
    float sn, cs;
    sincosf(ang, &sn, &cs);
    cos_s[f] = __fmul_rn(cs, conc);
    sin_s[f] = __fmul_rn(sn, conc);
  }
  __syncthreads();
  for (int32_t i = threadIdx.x; i < nh * D; i += blockDim.x) {
    const int32_t h = h0 + i / D, d = i % D;
    const uint16_t* xr = row + (int64_t)h * D;
    if (h >= Hq + Hkv) {  // v: copy
      v_cache[(dst_slot * Hkv + (h - Hq - Hkv)) * D + d] = xr[d];
      continue;
    }
    const int32_t f = d & (half - 1);
    const float c = cos_s[f], sv = sin_s[f];
    float o;
    if (d >= half) o = __fadd_rn(__fmul_rn(bf16_bits_to_f32(xr[d - half]), sv), __fmul_rn(bf16_bits_to_f32(xr[d]), c));
    else o = __fsub_rn(__fmul_rn(bf16_bits_to_f32(xr[d]), c), __fmul_rn(bf16_bits_to_f32(xr[d + half]), sv));
    const uint16_t ob = f32_to_bf16_bits(o);
    if (h < Hq) q_out[(s * Hq + h) * D + d] = ob;
    else k_cache[(dst_slot * Hkv + (h - Hq)) * D + d] = ob;
  }
}

// Standalone YaRN RoPE: x [S, Hh, D] -> out (same layout).
__global__ void rope_kernel(const uint16_t* __restrict__ x, const int32_t* __restrict__ pos, int64_t S, int32_t Hh,
                            int32_t D, const RopeTable tab, float conc, uint16_t* __restrict__ out) {
  const int64_t s = blockIdx.x;
  if (s >= S) return;
  const int32_t half = D / 2;
  const float p = (float)pos[s];
  for (int32_t i = threadIdx.x; i < Hh * D; i += blockDim.x) {
    const int32_t h = i / D, d = i % D;
    const uint16_t* xr = x + (s * Hh + h) * (int64_t)D;
    const int32_t f = d & (half - 1);
    const float ang = __fmul_rn(p, tab.inv_freq[f]);
    float sn, cs;
    sincosf(ang, &sn, &cs);
    const float c = __fmul_rn(cs, conc), sv = __fmul_rn(sn, conc);
    float o;
    if (d >= half) o = __fadd_rn(__fmul_rn(bf16_bits_to_f32(xr[d - half]), sv), __fmul_rn(bf16_bits_to_f32(xr[d]), c));
    else o = __fsub_rn(__fmul_rn(bf16_bits_to_f32(xr[d]), c), __fmul_rn(bf16_bits_to_f32(xr[d + half]), sv));
    out[(s * Hh + h) * (int64_t)D + d] = f32_to_bf16_bits(o);
  }
}

// ----------------------------------------------------------- sink fold --
// o_bf16 * bf16(sigmoid(ln2*lse2 - sink)) rounded to bf16 (attention.py:240-247).
__device__ __forceinline__ float sink_scale(float lse2, float sink) {
  const float z = __fsub_rn(__fmul_rn(kLn2, lse2), sink);
  return round_bf16(1.0f / (1.0f + expf(-z)));
}

// -------------------------------------------------------------- prefill --
// One CTA = 64 queries x one q head; 4 warps x 16 query rows.  K/V tiles of
// 64 keys stream through double-buffered, swizzled shared memory (cp.async).
// q [S_q, Hq, 64], k/v [S_kv, Hkv, 64]; query i sits at key position
// S_kv - S_q + i.  Key j is visible to query i iff j <= pos_i and, with a
// window W > 0, j >= pos_i - W + 1 (tvm_fix.patch:35-47).
constexpr int kAttD = 64;
constexpr int kAttBQ = 64;
constexpr int kAttBK = 64;

__global__ void __launch_bounds__(128) attn_prefill_kernel(const uint16_t* __restrict__ q, const uint16_t* __restrict__ k,
                                                            const uint16_t* __restrict__ v,
                                                            const uint16_t* __restrict__ sinks, int64_t Sq, int64_t Skv,
                                                            int32_t Hq, int32_t Hkv, int32_t window, float sm_scale,
                                                            uint16_t* __restrict__ o, float* __restrict__ lse) {
  __shared__ __align__(128) uint8_t sq[kAttBQ * 128];
  __shared__ __align__(128) uint8_t sk[2][kAttBK * 128];
  __shared__ __align__(128) uint8_t sv[2][kAttBK * 128];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h = blockIdx.y;
  const int hk = h / (Hq / Hkv);
  const int64_t i0 = (int64_t)blockIdx.x * kAttBQ;
  const int64_t off = Skv - Sq;
  const float scale2 = sm_scale * kLog2e;

  // key range of this query tile
  const int64_t last_q = min64(i0 + kAttBQ - 1, Sq - 1);
  const int64_t j_end = min64(Skv, off + last_q + 1);
  int64_t j_beg = 0;
  if (window > 0) j_beg = max64(0, off + i0 - window + 1);
  j_beg = (j_beg / kAttBK) * kAttBK;
  const int ntiles = (int)((j_end - j_beg + kAttBK - 1) / kAttBK);

  // Q tile
  for (int c = threadIdx.x; c < kAttBQ * 8; c += 128) {
    const int r = c >> 3, ch = c & 7;
    const int64_t qi = i0 + r;
    cp_async16(smem_u32(sq) + swz(r, ch), q + ((qi < Sq ? qi : 0) * Hq + h) * kAttD + ch * 8, qi < Sq);
  }
  auto load_kv = [&](int buf, int64_t j0) {
    for (int c = threadIdx.x; c < kAttBK * 8; c += 128) {
      const int r = c >> 3, ch = c & 7;
      const int64_t kj = j0 + r;
      const bool ok = kj < Skv;
      const int64_t src = ((ok ? kj : 0) * Hkv + hk) * kAttD + ch * 8;
      cp_async16(smem_u32(sk[buf]) + swz(r, ch), k + src, ok);
      cp_async16(smem_u32(sv[buf]) + swz(r, ch), v + src, ok);
    }
  };
  if (ntiles > 0) load_kv(0, j_beg);
  cp_async_commit();

  float m_r[2] = {-1e30f, -1e30f}, l_r[2] = {0.f, 0.f};
  float acc[8][4];
#pragma unroll
  for (int i = 0; i < 8; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
  uint32_t qf[4][4];
  const int g = lane >> 2, t4 = lane & 3;
  const int64_t row_q[2] = {i0 + warp * 16 + g, i0 + warp * 16 + g + 8};
  const int64_t pos_q[2] = {off + row_q[0], off + row_q[1]};

  for (int it = 0; it < ntiles; ++it) {
    const int buf = it & 1;
    const int64_t j0 = j_beg + (int64_t)it * kAttBK;
    if (it + 1 < ntiles) load_kv(buf ^ 1, j0 + kAttBK);
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    if (it == 0) {
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        const int r = warp * 16 + (lane & 15), ch = 2 * kk + (lane >> 4);
        ldsm_x4(qf[kk], smem_u32(sq) + swz(r, ch));
      }
    }
    // S = Q K^T for this warp's 16 rows x 64 keys
    float sc[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i) sc[i][0] = sc[i][1] = sc[i][2] = sc[i][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
      for (int kg = 0; kg < 4; ++kg) {
        uint32_t b[4];
        const int r = kg * 16 + (lane & 7) + ((lane >> 4) << 3), ch = 2 * kk + ((lane >> 3) & 1);
        ldsm_x4(b, smem_u32(sk[buf]) + swz(r, ch));
        mma_16816(sc[2 * kg], qf[kk], b[0], b[1]);
        mma_16816(sc[2 * kg + 1], qf[kk], b[2], b[3]);
      }
    }
    // scale, mask, online softmax (base 2)
    const bool full_tile = (j0 + kAttBK - 1 <= off + i0) && (j0 + kAttBK <= Skv) &&
                           (window <= 0 || j0 >= off + last_q - window + 1);
    float mx[2] = {-1e30f, -1e30f};
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int rr = e >> 1;
        const int64_t kj = j0 + nt * 8 + 2 * t4 + (e & 1);
        float sv_ = sc[nt][e] * scale2;
        if (!full_tile) {
          bool vis = kj <= pos_q[rr] && kj < Skv && row_q[rr] < Sq;
          if (window > 0) vis = vis && kj >= pos_q[rr] - window + 1;
          if (!vis) sv_ = -1e30f;
        }
        sc[nt][e] = sv_;
        mx[rr] = fmaxf(mx[rr], sv_);
      }
    }
#pragma unroll
    for (int rr = 0; rr < 2; ++rr) {
      mx[rr] = fmaxf(mx[rr], __shfl_xor_sync(0xffffffffu, mx[rr], 1));
      mx[rr] = fmaxf(mx[rr], __shfl_xor_sync(0xffffffffu, mx[rr], 2));
    }
    float corr[2], rs[2] = {0.f, 0.f};
#pragma unroll
    for (int rr = 0; rr < 2; ++rr) {
      const float mn = fmaxf(m_r[rr], mx[rr]);
      corr[rr] = exp2f(m_r[rr] - mn);
      m_r[rr] = mn;
    }
    uint32_t pf[4][4];
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      float pv[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int rr = e >> 1;
        pv[e] = sc[nt][e] <= -1e29f ? 0.f : exp2f(sc[nt][e] - m_r[rr]);
        rs[rr] += pv[e];
      }
      pf[nt >> 1][(nt & 1) * 2 + 0] = pack_bf16x2(pv[0], pv[1]);
      pf[nt >> 1][(nt & 1) * 2 + 1] = pack_bf16x2(pv[2], pv[3]);
    }
#pragma unroll
    for (int rr = 0; rr < 2; ++rr) {
      rs[rr] += __shfl_xor_sync(0xffffffffu, rs[rr], 1);
      rs[rr] += __shfl_xor_sync(0xffffffffu, rs[rr], 2);
      l_r[rr] = l_r[rr] * corr[rr] + rs[rr];
    }
#pragma unroll
    for (int dt = 0; dt < 8; ++dt) {
      acc[dt][0] *= corr[0];
      acc[dt][1] *= corr[0];
      acc[dt][2] *= corr[1];
      acc[dt][3] *= corr[1];
    }
    // O += P V
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      // A fragment regs: (row g, keys lo), (row g+8, keys lo), (row g, keys hi), (row g+8, keys hi)
      const uint32_t a[4] = {pf[kk][0], pf[kk][1], pf[kk][2], pf[kk][3]};
#pragma unroll
      for (int dg = 0; dg < 4; ++dg) {
        uint32_t b[4];
        const int r = kk * 16 + (lane & 7) + (((lane >> 3) & 1) << 3), ch = 2 * dg + (lane >> 4);
        ldsm_x4_t(b, smem_u32(sv[buf]) + swz(r, ch));
        mma_16816(acc[2 * dg], a, b[0], b[1]);
        mma_16816(acc[2 * dg + 1], a, b[2], b[3]);
      }
    }
    __syncthreads();
  }
  cp_async_wait<0>();

  // epilogue: normalise, lse, sink rescale, store
#pragma unroll
  for (int rr = 0; rr < 2; ++rr) {
    const int64_t qi = row_q[rr];
    if (qi >= Sq) continue;
    const float inv_l = l_r[rr] > 0.f ? 1.0f / l_r[rr] : 0.f;
    const float lse2 = m_r[rr] + log2f(l_r[rr]);
    if (lse && t4 == 0) lse[qi * Hq + h] = lse2;
    const float ss = sinks ? sink_scale(lse2, bf16_bits_to_f32(sinks[h])) : 1.0f;
    uint32_t* orow = (uint32_t*)(o + (qi * Hq + h) * kAttD);
#pragma unroll
    for (int dt = 0; dt < 8; ++dt) {
      float v0 = round_bf16(acc[dt][2 * rr] * inv_l), v1 = round_bf16(acc[dt][2 * rr + 1] * inv_l);
      if (sinks) {
        v0 = __fmul_rn(v0, ss);
        v1 = __fmul_rn(v1, ss);
      }
      orow[dt * 4 + t4] = (uint32_t)f32_to_bf16_bits(v0) | ((uint32_t)f32_to_bf16_bits(v1) << 16);
    }
  }
}

// ------------------------------------------------------ prefill, tcgen05 --
// One CTA = two tiles of 128 queries (tile t = 0, 1: rows i0 + 128 t ..) of one
// q head, 10 warps:
//   warps 0-3 / 4-7  softmax of tile 0 / tile 1: thread = query row = TMEM
//              lane.  Per key block it reads the score tile S (fp32, 128 keys)
//              from TMEM in one go, masks, runs the base-2 online softmax and
//              writes P (bf16) to TMEM as the A operand of O += P V;
//   warp 8     TMA: the two Q tiles once, then K and V tiles of 128 keys;
//   warp 9     MMA issuer (owns TMEM): S_t = Q_t K_j^T (A = Q_t, B = K_j in
//              shared memory, M = N = 128, K = 64) and O_t += P_t V_j (A = P_t
//              in TMEM, B = V_j read MN-major, N = 64, K = 128), O_t staying in
//              TMEM for the whole key loop.
// The two tiles ping-pong: while one tile's softmax runs, the tensor core
// works on the other tile.  The output is rescaled lazily: P uses the row's
// reference maximum m_ref, which only moves (and O_t, l are rescaled, a
// TMEM read-modify-write of O_t) when the running maximum exceeds it by more
// than 8 (P <= 2^8 stays exact enough in bf16 and fp32).  TMEM columns:
// S_0 [0,128), S_1 [128,256), O_0 [256,320), O_1 [320,384), P_0 [384,448),
// P_1 [448,512).
constexpr int kTcBQ = 128, kTcBK = 128, kTcStages = 3, kTcThreads = 320;
constexpr int kAttShortWindow = 512;  // windows up to this many keys take the mma.sync kernel
constexpr uint32_t kTcColO = 256, kTcColP = 384;
constexpr float kTcRescale = 8.0f;
constexpr int kTcQBytes = kTcBQ * 128, kTcKVBytes = kTcBK * 128;
constexpr int kTcSmemKV = 2 * kTcQBytes;
constexpr int kTcSmemBar = kTcSmemKV + kTcStages * 2 * kTcKVBytes;
constexpr int kTcSmemAlloc = kTcSmemBar + 256 + 1024;  // > 114 KB: one CTA (and its 512 TMEM columns) per SM

__device__ __forceinline__ void tmem_st_x16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}
// 32 lanes x 32 bit, 32 consecutive columns per thread, no wait.
__device__ __forceinline__ void tmem_ld_x32_nowait(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
}

__device__ __forceinline__ unsigned long long pack_f32x2(float lo, float hi) {
  return ((unsigned long long)__float_as_uint(hi) << 32) | __float_as_uint(lo);
}

__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__global__ void __launch_bounds__(kTcThreads, 1)
    attn_prefill_tc_kernel(const __grid_constant__ CUtensorMap tmap_q, const __grid_constant__ CUtensorMap tmap_k,
                           const __grid_constant__ CUtensorMap tmap_v, const uint16_t* __restrict__ sinks, int64_t Sq,
                           int64_t Skv, int32_t Hq, int32_t Hkv, int32_t window, float sm_scale,
                           uint16_t* __restrict__ o, float* __restrict__ lse) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint64_t* bars = (uint64_t*)(smem + kTcSmemBar);
  uint64_t* qfull = bars;
  uint64_t* kvfull = bars + 1;             // [kTcStages]
  uint64_t* kvempty = kvfull + kTcStages;  // [kTcStages] MMA commit after both tiles' P V
  uint64_t* sfull = kvempty + kTcStages;   // [2] per tile: MMA commit after Q K^T
  uint64_t* sfree = sfull + 2;             // [2] per tile: its 4 softmax warps read S
  uint64_t* pfull = sfree + 2;             // [2] per tile: its 4 softmax warps wrote P (and rescaled O)
  uint64_t* ofull = pfull + 2;             // [2] per tile: MMA commit after P V
  volatile uint32_t* tmem_slot = (volatile uint32_t*)(ofull + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h = blockIdx.y;
  const int hk = h / (Hq / Hkv);
  const int64_t qt = (int64_t)gridDim.x - 1 - blockIdx.x;  // the longest key ranges first
  const int64_t i0 = qt * 2 * kTcBQ;
  const int64_t off = Skv - Sq;
  const int64_t last_q = min64(i0 + 2 * kTcBQ - 1, Sq - 1);
  const int64_t j_end = min64(Skv, off + last_q + 1);
  int64_t j_beg = 0;
  if (window > 0) j_beg = max64(0, off + i0 - window + 1);
  j_beg = (j_beg / kTcBK) * kTcBK;
  const int n = (int)((j_end - j_beg + kTcBK - 1) / kTcBK);

  if (threadIdx.x == 0) {
    mbar_init(qfull, 1);
    for (int s = 0; s < kTcStages; ++s) {
      mbar_init(&kvfull[s], 1);
      mbar_init(&kvempty[s], 1);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(&sfull[t], 1);
      mbar_init(&sfree[t], 4);
      mbar_init(&pfull[t], 4);
      mbar_init(&ofull[t], 1);
    }
    fence_mbar_init();
  }
  if (warp == 9) {
    tmem_alloc((uint32_t*)tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 8) {
    // ------------------------------------------------------------ loads
    if (elect_one()) {
      mbar_arrive_expect_tx(qfull, 2 * kTcQBytes);
      tma_load_3d(smem, &tmap_q, 0, h, (int32_t)i0, qfull);
      tma_load_3d(smem + kTcQBytes, &tmap_q, 0, h, (int32_t)(i0 + kTcBQ), qfull);
      for (int j = 0; j < n; ++j) {
        const int s = j % kTcStages;
        const uint32_t ph = (uint32_t)(j / kTcStages) & 1u;
        if (!mbar_wait(&kvempty[s], ph ^ 1u, nullptr, 0)) break;
        uint8_t* kv = smem + kTcSmemKV + s * 2 * kTcKVBytes;
        mbar_arrive_expect_tx(&kvfull[s], 2 * kTcKVBytes);
        const int32_t kz = (int32_t)(j_beg + (int64_t)j * kTcBK);
        tma_load_3d(kv, &tmap_k, 0, hk, kz, &kvfull[s]);
        tma_load_3d(kv + kTcKVBytes, &tmap_v, 0, hk, kz, &kvfull[s]);
      }
    }
  } else if (warp == 9) {
    // --------------------------------------------------------------- MMA
    if (elect_one()) {
      const uint32_t idesc_s = make_idesc_bf16(kTcBQ, kTcBK);
      const uint32_t idesc_pv = make_idesc_bf16(kTcBQ, 64) | (1u << 16);  // B (V) read MN-major
      bool ok = mbar_wait(qfull, 0, nullptr, 0);
      auto issue_s = [&](int t, int j) {
        const int s = j % kTcStages;
        const uint64_t qdesc = make_sdesc_sw128(smem_u32(smem + t * kTcQBytes));
        const uint64_t kdesc = make_sdesc_sw128(smem_u32(smem + kTcSmemKV + s * 2 * kTcKVBytes));
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          tc_mma_ss(tmem + (uint32_t)t * kTcBK, qdesc + 2 * kk, kdesc + 2 * kk, idesc_s, kk > 0 ? 1u : 0u);
        tc_commit(&sfull[t]);
      };
      auto issue_pv = [&](int t, int j) {
        const int s = j % kTcStages;
        // V tile: 128 key rows of 128 B, 128-byte swizzle; MN-major B with
        // 8-row groups 1024 B apart; 16 keys (2048 B) per K step
        const uint64_t vdesc = make_sdesc_sw128(smem_u32(smem + kTcSmemKV + s * 2 * kTcKVBytes + kTcKVBytes));
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          tc_mma_ts(tmem + kTcColO + 64 * t, tmem + kTcColP + 64 * t + kk * 8, vdesc + 128 * kk, idesc_pv,
                    (j > 0 || kk > 0) ? 1u : 0u);
        tc_commit(&ofull[t]);
      };
      if (ok && n > 0) {
        ok = mbar_wait(&kvfull[0], 0, nullptr, 0);
        if (ok) {
          tc_fence_after();
          issue_s(0, 0);
          issue_s(1, 0);
        }
      }
      for (int j = 0; j < n && ok; ++j) {
        const bool more = j + 1 < n;
        if (more) {
          ok = mbar_wait(&kvfull[(j + 1) % kTcStages], (uint32_t)((j + 1) / kTcStages) & 1u, nullptr, 0);
          if (!ok) break;
        }
        for (int t = 0; t < 2 && ok; ++t) {
          if (more) {
            ok = mbar_wait(&sfree[t], (uint32_t)j & 1u, nullptr, 0);  // the softmax has read S_t(j)
            if (!ok) break;
            tc_fence_after();
            issue_s(t, j + 1);
          }
          ok = mbar_wait(&pfull[t], (uint32_t)j & 1u, nullptr, 0);
          if (!ok) break;
          tc_fence_after();
          issue_pv(t, j);
        }
        tc_commit(&kvempty[j % kTcStages]);
      }
    }
  } else {
    // ----------------------------------------------------------- softmax
    const int t = warp >> 2;                       // tile
    const int row = (warp & 3) * 32 + lane;        // TMEM lane
    const int64_t qi = i0 + t * kTcBQ + row;
    const int64_t pos = off + qi;
    const bool row_ok = qi < Sq;
    const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
    const uint32_t s_col = tmem + lane_base + (uint32_t)t * kTcBK;
    const uint32_t o_col = tmem + lane_base + kTcColO + 64 * t;
    const uint32_t p_col = tmem + lane_base + kTcColP + 64 * t;
    const float scale2 = sm_scale * kLog2e;
    const int64_t tile_last = min64(i0 + t * kTcBQ + kTcBQ - 1, Sq - 1);
    float m_ref = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < n && ok; ++j) {
      if (!mbar_wait(&sfull[t], (uint32_t)j & 1u, nullptr, 0)) { ok = false; break; }
      tc_fence_after();
      const int64_t j0 = j_beg + (int64_t)j * kTcBK;
      const bool full_tile = (j0 + kTcBK - 1 <= off + i0 + t * kTcBQ) && (j0 + kTcBK <= Skv) &&
                             (window <= 0 || j0 >= off + tile_last - window + 1);
      // raw score of key j0 + e with the mask applied (-inf when not visible)
      auto masked = [&](uint32_t bits, int e) -> uint32_t {
        const int64_t kj = j0 + e;
        bool vis = kj <= pos && kj < Skv && row_ok;
        if (window > 0) vis = vis && kj >= pos - window + 1;
        return vis ? bits : __float_as_uint(-INFINITY);
      };
      // pass 1: row max of the raw scores (sm_scale * log2(e) > 0)
      float mx = -INFINITY;
#pragma unroll
      for (int hb = 0; hb < 2; ++hb) {
        uint32_t r[64];
        tmem_ld_x32_nowait(s_col + 64 * hb, r);
        tmem_ld_x32_nowait(s_col + 64 * hb + 32, r + 32);
        tmem_ld_wait();
        if (full_tile) {
#pragma unroll
          for (int e = 0; e < 64; ++e) mx = fmaxf(mx, __uint_as_float(r[e]));
        } else {
#pragma unroll
          for (int e = 0; e < 64; ++e) mx = fmaxf(mx, __uint_as_float(masked(r[e], 64 * hb + e)));
        }
      }
      const float mxs = mx * scale2;  // base-2 row max of this block
      // lazy rescale: move the reference maximum only when P would exceed 2^8
      const bool move = mxs > m_ref + kTcRescale;
      const float m_new = move ? mxs : m_ref;
      const float c = move ? fast_exp2(m_ref - m_new) : 1.0f;
      const float m_eff = m_new == -INFINITY ? 0.f : m_new;  // fully masked so far: every p is 0
      // P_t and O_t are free once P_t(j-1) V(j-1) is done
      if (j > 0) {
        if (!mbar_wait(&ofull[t], (uint32_t)(j - 1) & 1u, nullptr, 0)) { ok = false; break; }
        tc_fence_after();
      }
      // pass 2: p = 2^(s * scale2 - m) two at a time (packed f32x2 FMA / add),
      // stored to TMEM as bf16 32 keys at a time; the row sum stays fp32
      const unsigned long long sc2 = pack_f32x2(scale2, scale2), negm = pack_f32x2(-m_eff, -m_eff);
      unsigned long long acc2 = 0ull;
#pragma unroll
      for (int q4 = 0; q4 < 4; ++q4) {
        uint32_t r[32], pk[16];
        tmem_ld_x32_nowait(s_col + 32 * q4, r);
        tmem_ld_wait();
        if (!full_tile) {
#pragma unroll
          for (int e = 0; e < 32; ++e) r[e] = masked(r[e], 32 * q4 + e);
        }
#pragma unroll
        for (int e2 = 0; e2 < 16; ++e2) {
          const int e = 2 * e2;
          unsigned long long x = ((unsigned long long)r[e + 1] << 32) | r[e];
          asm("fma.rn.f32x2 %0, %0, %1, %2;" : "+l"(x) : "l"(sc2), "l"(negm));
          const float p0 = fast_exp2(__uint_as_float((uint32_t)x));
          const float p1 = fast_exp2(__uint_as_float((uint32_t)(x >> 32)));
          const unsigned long long pp = pack_f32x2(p0, p1);
          asm("add.rn.f32x2 %0, %0, %1;" : "+l"(acc2) : "l"(pp));
          pk[e2] = pack_bf16x2(p0, p1);
        }
        tmem_st_x16(p_col + 16 * q4, pk);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sfree[t]);  // S_t read: the next Q K^T may overwrite it
      const float rs = __uint_as_float((uint32_t)acc2) + __uint_as_float((uint32_t)(acc2 >> 32));
      l = l * c + rs;
      m_ref = m_new;
      if (j > 0 && __any_sync(0xffffffffu, move)) {
        // the reference maximum moved: O_t (blocks < j) by c, before P_t V(j) adds to it
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
          uint32_t ov[32];
          tmem_ld_x32(o_col + 32 * hf, ov);
          tmem_ld_wait();
#pragma unroll
          for (int d = 0; d < 32; ++d) ov[d] = __float_as_uint(__uint_as_float(ov[d]) * c);
          tmem_st_x32(o_col + 32 * hf, ov);
        }
      }
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&pfull[t]);
    }
    // normalise, lse, sink rescale, store (attention.py:240-247)
    if (ok && n > 0 && mbar_wait(&ofull[t], (uint32_t)(n - 1) & 1u, nullptr, 0)) {
      tc_fence_after();
      uint32_t ov[64];
      tmem_ld_x32_nowait(o_col, ov);
      tmem_ld_x32_nowait(o_col + 32, ov + 32);
      tmem_ld_wait();
      if (row_ok) {
        const float inv_l = l > 0.f ? 1.0f / l : 0.f;
        const float lse2 = m_ref + log2f(l);
        if (lse) lse[qi * Hq + h] = lse2;
        const float ss = sinks ? sink_scale(lse2, bf16_bits_to_f32(sinks[h])) : 1.0f;
        uint4* orow = (uint4*)(o + (qi * Hq + h) * kAttD);
#pragma unroll
        for (int d8 = 0; d8 < 8; ++d8) {
          uint32_t w4[4];
#pragma unroll
          for (int q2 = 0; q2 < 4; ++q2) {
            float v0 = round_bf16(__uint_as_float(ov[8 * d8 + 2 * q2]) * inv_l);
            float v1 = round_bf16(__uint_as_float(ov[8 * d8 + 2 * q2 + 1]) * inv_l);
            if (sinks) {
              v0 = __fmul_rn(v0, ss);
              v1 = __fmul_rn(v1, ss);
            }
            w4[q2] = (uint32_t)f32_to_bf16_bits(v0) | ((uint32_t)f32_to_bf16_bits(v1) << 16);
          }
          orow[d8] = make_uint4(w4[0], w4[1], w4[2], w4[3]);
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// --------------------------------------------------------------- decode --
// One CTA = (sequence b, kv head g, key split).  The 8 query heads of the
// group (GQA) are rows 0..7 of a 16-row MMA tile (rows 8..15 are zero).
// Each of the 4 warps walks 64-key tiles of the split with its own
// double-buffered shared-memory tiles and softmax state; the warps merge at
// the end and the CTA writes an unnormalised partial (o, m, l) per head.
// q [B, Hq, 64]; caches [B, max_len, Hkv, 64]; kv_len [B].
constexpr int kDecWarps = 4;
// Keys per split with many sequences: a CTA's set-up, warp merge and partial
// store are paid once per split (B = 32 x 8192 keys: 1024-key splits 0.144 ms,
// 2048 0.128, 4096 0.130, 512 0.177)
constexpr int kDecSplitKeys = 2048;

// Cache row of key j of sequence b: contiguous caches hold it at row
// b * max_len + j; a paged cache (table != NULL) at row
// table[b * tstride + (j / 16) % tstride] * 16 + j % 16 of its page pool (a
// ring of tstride pages when tstride pages do not cover the sequence).
__device__ __forceinline__ int64_t kv_row(const int32_t* __restrict__ table, int32_t tstride, int64_t max_len, int b,
                                          int64_t j) {
  if (table == nullptr) return (int64_t)b * max_len + j;
  const int64_t lp = (j >> 4) % tstride;
  return (int64_t)__ldg(table + (int64_t)b * tstride + lp) * 16 + (j & 15);
}

__global__ void __launch_bounds__(128) attn_decode_kernel(const uint16_t* __restrict__ q,
                                                           const uint16_t* __restrict__ kc,
                                                           const uint16_t* __restrict__ vc,
                                                           const int32_t* __restrict__ kv_len, int64_t max_len,
                                                           int32_t Hq, int32_t Hkv, int32_t window, float sm_scale,
                                                           int32_t splits, float* __restrict__ part_o,
                                                           float* __restrict__ part_ml,
                                                           const int32_t* __restrict__ table, int32_t tstride) {
  extern __shared__ __align__(128) uint8_t dsm[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int bg = blockIdx.x;  // b * Hkv + g
  const int split = blockIdx.y;
  const int b = bg / Hkv, gk = bg % Hkv;
  const int G = Hq / Hkv;  // query heads per kv head (<= 16)
  const int64_t L = kv_len[b];
  const float scale2 = sm_scale * kLog2e;
  uint8_t* sq = dsm;                                         // [16][128 B]
  uint8_t* wbuf = dsm + 16 * 128 + warp * (2 * 2 * kAttBK * 128);  // per warp: [2 bufs][K,V][64 rows][128 B]
  float* red = (float*)(dsm + 16 * 128 + kDecWarps * 2 * 2 * kAttBK * 128);  // merge area

  int64_t k_lo = 0;
  if (window > 0) k_lo = max64(0, L - window);
  const int64_t span = L - k_lo;
  const int64_t per = (span + splits - 1) / splits;
  const int64_t s_lo = k_lo + (int64_t)split * per;
  const int64_t s_hi = min64(L, s_lo + per);

  // query rows (zero beyond G)
  for (int c = threadIdx.x; c < 16 * 8; c += 128) {
    const int r = c >> 3, ch = c & 7;
    const bool ok = r < G;
    cp_async16(smem_u32(sq) + swz(r, ch), q + ((int64_t)b * Hq + gk * G + (ok ? r : 0)) * kAttD + ch * 8, ok);
  }
  cp_async_commit();
  const int64_t ntile_all = s_hi > s_lo ? (s_hi - s_lo + kAttBK - 1) / kAttBK : 0;
  // a lane copies one 16-byte piece (ch) of rows lane / 8 + 4 i; the page of a
  // row is found from the tile's first page (one modulo per tile) plus its
  // page offset within the tile (at most 4)
  const int* trow_tab = table ? table + (int64_t)b * tstride : nullptr;
  auto load = [&](int buf, int64_t j0) {
    uint8_t* kb = wbuf + buf * (2 * kAttBK * 128);
    uint8_t* vb = kb + kAttBK * 128;
    const int ch = lane & 7;
    const int64_t p0 = j0 >> 4;
    const int32_t lp0 = trow_tab ? (int32_t)(p0 % tstride) : 0;
#pragma unroll 4
    for (int i = 0; i < kAttBK / 4; ++i) {
      const int r = (lane >> 3) + 4 * i;
      const int64_t kj = j0 + r;
      const bool ok = kj < s_hi;
      const int64_t jj = ok ? kj : j0;  // j0 < s_hi: a valid row to point the skipped copy at
      int64_t row;
      if (trow_tab) {
        int32_t lp = lp0 + (int32_t)((jj >> 4) - p0);
        if (lp >= tstride) lp -= tstride;
        row = (int64_t)__ldg(trow_tab + lp) * 16 + (jj & 15);
      } else {
        row = (int64_t)b * max_len + jj;
      }
      const int64_t src = (row * Hkv + gk) * kAttD + ch * 8;
      cp_async16(smem_u32(kb) + swz(r, ch), kc + src, ok);
      cp_async16(smem_u32(vb) + swz(r, ch), vc + src, ok);
    }
  };
  // tiles of this warp: warp, warp + 4, ...
  int64_t my = warp;
  if (my < ntile_all) load(0, s_lo + my * kAttBK);
  cp_async_commit();
  cp_async_wait<0>();
  __syncthreads();
  uint32_t qf[4][4];
#pragma unroll
  for (int kk = 0; kk < 4; ++kk) {
    const int r = lane & 15, ch = 2 * kk + (lane >> 4);
    ldsm_x4(qf[kk], smem_u32(sq) + swz(r, ch));
  }
  const int g = lane >> 2, t4 = lane & 3;
  float m_r = -1e30f, l_r = 0.f;  // row g (rows g+8 are padding)
  float acc[8][2];
#pragma unroll
  for (int i = 0; i < 8; ++i) acc[i][0] = acc[i][1] = 0.f;
  int buf = 0;
  for (; my < ntile_all; my += kDecWarps) {
    const int64_t j0 = s_lo + my * kAttBK;
    if (my + kDecWarps < ntile_all) load(buf ^ 1, j0 + kDecWarps * kAttBK);
    cp_async_commit();
    cp_async_wait<1>();
    __syncwarp();
    const uint8_t* kb = wbuf + buf * (2 * kAttBK * 128);
    const uint8_t* vb = kb + kAttBK * 128;
    float sc[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i) sc[i][0] = sc[i][1] = sc[i][2] = sc[i][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
      for (int kg = 0; kg < 4; ++kg) {
        uint32_t bb[4];
        const int r = kg * 16 + (lane & 7) + ((lane >> 4) << 3), ch = 2 * kk + ((lane >> 3) & 1);
        ldsm_x4(bb, smem_u32(kb) + swz(r, ch));
        mma_16816(sc[2 * kg], qf[kk], bb[0], bb[1]);
        mma_16816(sc[2 * kg + 1], qf[kk], bb[2], bb[3]);
      }
    }
    float mx = -1e30f;
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int64_t kj = j0 + nt * 8 + 2 * t4 + e;
        float s_ = sc[nt][e] * scale2;
        if (kj >= s_hi) s_ = -1e30f;
        sc[nt][e] = s_;
        mx = fmaxf(mx, s_);
      }
    }
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    const float mn = fmaxf(m_r, mx);
    const float corr = exp2f(m_r - mn);
    m_r = mn;
    float rs = 0.f;
    uint32_t pf[4][4];
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      const float p0 = sc[nt][0] <= -1e29f ? 0.f : exp2f(sc[nt][0] - mn);
      const float p1 = sc[nt][1] <= -1e29f ? 0.f : exp2f(sc[nt][1] - mn);
      rs += p0 + p1;
      pf[nt >> 1][(nt & 1) * 2 + 0] = pack_bf16x2(p0, p1);
      pf[nt >> 1][(nt & 1) * 2 + 1] = 0u;  // padding rows
    }
    rs += __shfl_xor_sync(0xffffffffu, rs, 1);
    rs += __shfl_xor_sync(0xffffffffu, rs, 2);
    l_r = l_r * corr + rs;
#pragma unroll
    for (int dt = 0; dt < 8; ++dt) {
      acc[dt][0] *= corr;
      acc[dt][1] *= corr;
    }
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      const uint32_t a[4] = {pf[kk][0], pf[kk][1], pf[kk][2], pf[kk][3]};
#pragma unroll
      for (int dg = 0; dg < 4; ++dg) {
        uint32_t bb[4];
        const int r = kk * 16 + (lane & 7) + (((lane >> 3) & 1) << 3), ch = 2 * dg + (lane >> 4);
        ldsm_x4_t(bb, smem_u32(vb) + swz(r, ch));
        float c0[4] = {acc[2 * dg][0], acc[2 * dg][1], 0.f, 0.f};
        float c1[4] = {acc[2 * dg + 1][0], acc[2 * dg + 1][1], 0.f, 0.f};
        mma_16816(c0, a, bb[0], bb[1]);
        mma_16816(c1, a, bb[2], bb[3]);
        acc[2 * dg][0] = c0[0];
        acc[2 * dg][1] = c0[1];
        acc[2 * dg + 1][0] = c1[0];
        acc[2 * dg + 1][1] = c1[1];
      }
    }
    __syncwarp();
    buf ^= 1;
  }
  cp_async_wait<0>();
  // merge the 4 warps: red layout per warp: m[16], l[16], o[16][64]
  float* rw = red + warp * (16 + 16 + 16 * 64);
  if (t4 == 0) {
    rw[g] = m_r;
    rw[16 + g] = l_r;
  }
#pragma unroll
  for (int dt = 0; dt < 8; ++dt) {
    rw[32 + g * 64 + dt * 8 + 2 * t4] = acc[dt][0];
    rw[32 + g * 64 + dt * 8 + 2 * t4 + 1] = acc[dt][1];
  }
  __syncthreads();
  // thread -> (row, 8 dims): 8 rows x 64 dims = 512 values, 4 per thread
  for (int idx = threadIdx.x; idx < G * kAttD; idx += 128) {
    const int r = idx / kAttD, d = idx % kAttD;
    float m = -1e30f;
    for (int w = 0; w < kDecWarps; ++w) m = fmaxf(m, red[w * (16 + 16 + 16 * 64) + r]);
    float lsum = 0.f, osum = 0.f;
    for (int w = 0; w < kDecWarps; ++w) {
      const float* rw2 = red + w * (16 + 16 + 16 * 64);
      const float f = rw2[r] <= -1e29f ? 0.f : exp2f(rw2[r] - m);
      lsum += rw2[16 + r] * f;
      osum += rw2[32 + r * 64 + d] * f;
    }
    const int h = gk * G + r;
    const int64_t pidx = ((int64_t)b * Hq + h) * splits + split;
    part_o[pidx * kAttD + d] = osum;
    if (d == 0) {
      part_ml[pidx * 2] = m;
      part_ml[pidx * 2 + 1] = lsum;
    }
  }
}

// Merge of the key splits + sink: one warp per (b, h), lanes over dims.
__global__ void attn_decode_merge_kernel(const float* __restrict__ part_o, const float* __restrict__ part_ml,
                                         int64_t BH, int32_t Hq, int32_t splits, const uint16_t* __restrict__ sinks,
                                         uint16_t* __restrict__ o, float* __restrict__ lse) {
  const int64_t bh = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (bh >= BH) return;
  const int h = (int)(bh % Hq);
  float m = -1e30f;
  for (int s = 0; s < splits; ++s) m = fmaxf(m, part_ml[(bh * splits + s) * 2]);
  float lsum = 0.f, o0 = 0.f, o1 = 0.f;
  for (int s = 0; s < splits; ++s) {
    const float ms = part_ml[(bh * splits + s) * 2];
    const float f = ms <= -1e29f ? 0.f : exp2f(ms - m);
    lsum += part_ml[(bh * splits + s) * 2 + 1] * f;
    o0 += part_o[(bh * splits + s) * kAttD + 2 * lane] * f;
    o1 += part_o[(bh * splits + s) * kAttD + 2 * lane + 1] * f;
  }
  const float inv = lsum > 0.f ? 1.0f / lsum : 0.f;
  const float lse2 = m + log2f(lsum);
  if (lse && lane == 0) lse[bh] = lse2;
  float v0 = round_bf16(o0 * inv), v1 = round_bf16(o1 * inv);
  if (sinks) {
    const float ss = sink_scale(lse2, bf16_bits_to_f32(sinks[h]));
    v0 = __fmul_rn(v0, ss);
    v1 = __fmul_rn(v1, ss);
  }
  ((uint32_t*)(o + bh * kAttD))[lane] = (uint32_t)f32_to_bf16_bits(v0) | ((uint32_t)f32_to_bf16_bits(v1) << 16);
}

// ------------------------------------------------------ merge and sink --
// (o1, l1) and (o2, l2) -> (o, l): m = max; w_i = exp2(l_i - m);
// o = (o1 w1 + o2 w2) / (w1 + w2); lse = m + log2(w1 + w2).
__global__ void attn_merge_kernel(const uint16_t* __restrict__ o1, const float* __restrict__ l1,
                                  const uint16_t* __restrict__ o2, const float* __restrict__ l2, int64_t TH, int32_t D,
                                  uint16_t* __restrict__ o, float* __restrict__ lse) {
  const int64_t th = blockIdx.x;
  if (th >= TH) return;
  const float a = l1[th], b = l2[th];
  const float m = fmaxf(a, b);
  const float wa = exp2f(a - m), wb = exp2f(b - m);
  const float den = wa + wb;
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    const int64_t ix = th * D + d;
    o[ix] = f32_to_bf16_bits((bf16_bits_to_f32(o1[ix]) * wa + bf16_bits_to_f32(o2[ix]) * wb) / den);
  }
  if (threadIdx.x == 0 && lse) lse[th] = m + log2f(den);
}

__global__ void sink_rescale_kernel(uint16_t* __restrict__ o, const float* __restrict__ lse,
                                    const uint16_t* __restrict__ sinks, int64_t TH, int32_t Hq, int32_t D) {
  const int64_t th = blockIdx.x;
  if (th >= TH) return;
  const float ss = sink_scale(lse[th], bf16_bits_to_f32(sinks[th % Hq]));
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    const int64_t ix = th * D + d;
    o[ix] = f32_to_bf16_bits(__fmul_rn(bf16_bits_to_f32(o[ix]), ss));
  }
}

// --------------------------------------------------------------- launch --
int launch_qkv_rope(const uint16_t* qkv, const int32_t* pos, const int32_t* slot, int64_t S, int32_t Hq, int32_t Hkv,
                    int32_t D, const float* inv_freq, float conc, uint16_t* q_out, uint16_t* k_cache,
                    uint16_t* v_cache, cudaStream_t s) {
  if (S <= 0) return 0;
  if (D > 256 || D % 2) return -12;
  RopeTable tab;
  for (int i = 0; i < D / 2; ++i) tab.inv_freq[i] = inv_freq[i];
  const dim3 grid((unsigned)S, (unsigned)((Hq + 2 * Hkv + kRopeHeads - 1) / kRopeHeads));
  qkv_rope_kernel<<<grid, 256, 0, s>>>(qkv, pos, slot, S, Hq, Hkv, D, tab, conc, q_out, k_cache, v_cache);
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

int launch_rope(const uint16_t* x, const int32_t* pos, int64_t S, int32_t Hh, int32_t D, const float* inv_freq,
                float conc, uint16_t* out, cudaStream_t s) {
  if (S <= 0) return 0;
  if (D > 256 || D % 2) return -12;
  RopeTable tab;
  for (int i = 0; i < D / 2; ++i) tab.inv_freq[i] = inv_freq[i];
  rope_kernel<<<(unsigned)S, 256, 0, s>>>(x, pos, S, Hh, D, tab, conc, out);
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

int launch_attn_prefill(const uint16_t* q, const uint16_t* k, const uint16_t* v, const uint16_t* sinks, int64_t Sq,
                        int64_t Skv, int32_t Hq, int32_t Hkv, int32_t D, int32_t window, float sm_scale, uint16_t* o,
                        float* lse, cudaStream_t s) {
  if (Sq <= 0) return 0;
  if (D != kAttD || Hq % Hkv || Skv < Sq) return -12;
  if (window > 0 && window <= kAttShortWindow) {
    // a few key blocks per query tile: the 64-query mma.sync kernel's lower
    // fixed cost per CTA wins over the tcgen05 kernel's pipeline fill
    dim3 grid((unsigned)((Sq + kAttBQ - 1) / kAttBQ), (unsigned)Hq);
    attn_prefill_kernel<<<grid, 128, 0, s>>>(q, k, v, sinks, Sq, Skv, Hq, Hkv, window, sm_scale, o, lse);
    return cudaGetLastError() == cudaSuccess ? 0 : -3;
  }
  if (((uintptr_t)q & 15) || ((uintptr_t)k & 15) || ((uintptr_t)v & 15) || ((uintptr_t)o & 15)) return -12;
  // q [Sq, Hq, 64], k / v [Skv, Hkv, 64] bf16: boxes of 64 dims x 1 head x 128 tokens
  CUtensorMap tq, tk, tv;
  const uint32_t box[3] = {64, 1, 128};
  const uint64_t dq[3] = {64, (uint64_t)Hq, (uint64_t)Sq}, sq_[2] = {128, (uint64_t)Hq * 128};
  const uint64_t dk[3] = {64, (uint64_t)Hkv, (uint64_t)Skv}, sk_[2] = {128, (uint64_t)Hkv * 128};
  if (make_tmap_3d(&tq, q, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, dq, sq_, box, CU_TENSOR_MAP_SWIZZLE_128B) ||
      make_tmap_3d(&tk, k, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, dk, sk_, box, CU_TENSOR_MAP_SWIZZLE_128B) ||
      make_tmap_3d(&tv, v, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, dk, sk_, box, CU_TENSOR_MAP_SWIZZLE_128B))
    return -2;
  static FuncSmemAttr attr;
  ensure_dyn_smem(attr, (const void*)attn_prefill_tc_kernel, kTcSmemAlloc);
  dim3 grid((unsigned)((Sq + 2 * kTcBQ - 1) / (2 * kTcBQ)), (unsigned)Hq);
  attn_prefill_tc_kernel<<<grid, kTcThreads, kTcSmemAlloc, s>>>(tq, tk, tv, sinks, Sq, Skv, Hq, Hkv, window,
                                                                sm_scale, o, lse);
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

size_t attn_decode_scratch_bytes(int64_t B, int32_t Hq, int64_t max_len, int32_t splits) {
  (void)max_len;
  return (size_t)B * Hq * splits * (kAttD + 2) * sizeof(float);
}

// Key splits per (sequence, kv head): one per kDecSplitKeys keys of the
// longest span; with few sequences the splits are halved (down to
// kDecMinSplitKeys keys) until about two CTAs per SM are busy, since a
// single-token decode is otherwise latency-bound on a few SMs.
constexpr int64_t kDecTargetCtas = 2 * 148;
constexpr int64_t kDecMinSplitKeys = 128;
int attn_decode_splits(int64_t B, int32_t Hq, int64_t max_len, int32_t window) {
  const int64_t span = window > 0 ? min64(max_len, window) : max_len;
  int64_t splits = max64(1, (span + kDecSplitKeys - 1) / kDecSplitKeys);
  const int64_t units = max64(1, B) * max64(1, Hq / 8);
  while (units * splits < kDecTargetCtas && (span + 2 * splits - 1) / (2 * splits) >= kDecMinSplitKeys) splits *= 2;
  return (int)splits;
}

int launch_attn_decode(const uint16_t* q, const uint16_t* kc, const uint16_t* vc, const int32_t* kv_len, int64_t B,
                       int64_t max_len, int32_t Hq, int32_t Hkv, int32_t D, int32_t window, float sm_scale,
                       const uint16_t* sinks, float* scratch, uint16_t* o, float* lse, cudaStream_t s,
                       const int32_t* table, int32_t tstride) {
  if (B <= 0) return 0;
  if (D != kAttD || Hq % Hkv || Hq / Hkv > 8) return -12;
  const int splits = attn_decode_splits(B, Hq, max_len, window);
  float* part_o = scratch;
  float* part_ml = scratch + (size_t)B * Hq * splits * kAttD;
  const size_t smem = 16 * 128 + kDecWarps * 2 * 2 * kAttBK * 128 + kDecWarps * (16 + 16 + 16 * 64) * 4;
  static FuncSmemAttr attr;
  ensure_dyn_smem(attr, (const void*)attn_decode_kernel, (int)smem);
  dim3 grid((unsigned)(B * Hkv), (unsigned)splits);
  attn_decode_kernel<<<grid, 128, smem, s>>>(q, kc, vc, kv_len, max_len, Hq, Hkv, window, sm_scale, splits, part_o,
                                             part_ml, table, tstride);
  const int64_t BH = B * Hq;
  attn_decode_merge_kernel<<<(unsigned)((BH * 32 + 255) / 256), 256, 0, s>>>(part_o, part_ml, BH, Hq, splits, sinks,
                                                                               o, lse);
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

// Rows of a paged K/V cache <-> contiguous rows: row i of buf_k / buf_v
// ([n, row_elems] bf16) is key position pos0 + i of sequence `seq`, at pool
// row table[seq * tstride + (p / 16) % tstride] * 16 + p % 16.  to_pages: buf
// -> pool, else pool -> buf.  One warp per row, 16-byte pieces.
__global__ void kv_rows_copy_kernel(uint16_t* __restrict__ pool_k, uint16_t* __restrict__ pool_v,
                                    const int32_t* __restrict__ table, int32_t tstride, int32_t seq, int64_t pos0,
                                    int64_t n, int32_t row_elems, uint16_t* __restrict__ buf_k,
                                    uint16_t* __restrict__ buf_v, int32_t to_pages) {
  const int64_t i = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (i >= n) return;
  const int lane = threadIdx.x & 31;
  const int64_t row = kv_row(table, tstride, 0, seq, pos0 + i);
  uint4* pk = (uint4*)(pool_k + row * row_elems);
  uint4* pv = (uint4*)(pool_v + row * row_elems);
  uint4* bk = (uint4*)(buf_k + i * row_elems);
  uint4* bv = (uint4*)(buf_v + i * row_elems);
  for (int c = lane; c < row_elems / 8; c += 32) {
    if (to_pages) {
      pk[c] = bk[c];
      pv[c] = bv[c];
    } else {
      bk[c] = pk[c];
      bv[c] = pv[c];
    }
  }
}

int launch_kv_rows_copy(uint16_t* pool_k, uint16_t* pool_v, const int32_t* table, int32_t tstride, int32_t seq,
                        int64_t pos0, int64_t n, int32_t row_elems, uint16_t* buf_k, uint16_t* buf_v, int32_t to_pages,
                        cudaStream_t s) {
  if (n <= 0) return 0;
  if (row_elems % 8 || !table || tstride <= 0) return -12;
  kv_rows_copy_kernel<<<(unsigned)((n + 7) / 8), 256, 0, s>>>(pool_k, pool_v, table, tstride, seq, pos0, n, row_elems,
                                                              buf_k, buf_v, to_pages);
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

int launch_attn_merge(const uint16_t* o1, const float* l1, const uint16_t* o2, const float* l2, int64_t T, int32_t Hq,
                      int32_t D, uint16_t* o, float* lse, cudaStream_t s) {
  if (T <= 0) return 0;
  attn_merge_kernel<<<(unsigned)(T * Hq), 64, 0, s>>>(o1, l1, o2, l2, T * Hq, D, o, lse);
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

int launch_sink_rescale(uint16_t* o, const float* lse, const uint16_t* sinks, int64_t T, int32_t Hq, int32_t D,
                        cudaStream_t s) {
  if (T <= 0) return 0;
  sink_rescale_kernel<<<(unsigned)(T * Hq), 64, 0, s>>>(o, lse, sinks, T * Hq, Hq, D);
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

}  // namespace gptoss
