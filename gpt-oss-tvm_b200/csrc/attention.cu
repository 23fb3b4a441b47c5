// attention.cu -- gpt-oss attention with learned sinks, sliding-window / full
// causal masks, GQA and YaRN RoPE (model/attention.py:15-256).
//
//   qkv_rope_kernel      split of the fused QKV projection, YaRN RoPE on q and
//                        k (attention.py:96-180), k/v written to cache slots
//                        (the append_mha_kv step, attention.py:214)
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

__global__ void qkv_rope_kernel(const uint16_t* __restrict__ qkv, const int32_t* __restrict__ pos,
                                const int32_t* __restrict__ slot, int64_t S, int32_t Hq, int32_t Hkv, int32_t D,
                                const RopeTable tab, float conc, uint16_t* __restrict__ q_out,
                                uint16_t* __restrict__ k_cache, uint16_t* __restrict__ v_cache) {
  // one block per token; threads over (head, dim) of q, k and v
  const int64_t s = blockIdx.x;
  if (s >= S) return;
  const int32_t Ht = Hq + 2 * Hkv;
  const uint16_t* row = qkv + s * (int64_t)Ht * D;
  const int32_t half = D / 2;
  const float p = (float)pos[s];
  const int64_t dst_slot = slot ? slot[s] : s;
  for (int32_t i = threadIdx.x; i < Ht * D; i += blockDim.x) {
    const int32_t h = i / D, d = i % D;
    const uint16_t* xr = row + (int64_t)h * D;
    if (h >= Hq + Hkv) {  // v: copy
      v_cache[(dst_slot * Hkv + (h - Hq - Hkv)) * D + d] = xr[d];
      continue;
    }
    const int32_t f = d & (half - 1);
    const float ang = __fmul_rn(p, tab.inv_freq[f]);
    float sn, cs;
    sincosf(ang, &sn, &cs);
    const float c = __fmul_rn(cs, conc), sv = __fmul_rn(sn, conc);
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

// --------------------------------------------------------------- decode --
// One CTA = (sequence b, kv head g, key split).  The 8 query heads of the
// group (GQA) are rows 0..7 of a 16-row MMA tile (rows 8..15 are zero).
// Each of the 4 warps walks 64-key tiles of the split with its own
// double-buffered shared-memory tiles and softmax state; the warps merge at
// the end and the CTA writes an unnormalised partial (o, m, l) per head.
// q [B, Hq, 64]; caches [B, max_len, Hkv, 64]; kv_len [B].
constexpr int kDecWarps = 4;
constexpr int kDecSplitKeys = 1024;

__global__ void __launch_bounds__(128) attn_decode_kernel(const uint16_t* __restrict__ q,
                                                           const uint16_t* __restrict__ kc,
                                                           const uint16_t* __restrict__ vc,
                                                           const int32_t* __restrict__ kv_len, int64_t max_len,
                                                           int32_t Hq, int32_t Hkv, int32_t window, float sm_scale,
                                                           int32_t splits, float* __restrict__ part_o,
                                                           float* __restrict__ part_ml) {
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
  auto load = [&](int buf, int64_t j0) {
    uint8_t* kb = wbuf + buf * (2 * kAttBK * 128);
    uint8_t* vb = kb + kAttBK * 128;
    for (int c = lane; c < kAttBK * 8; c += 32) {
      const int r = c >> 3, ch = c & 7;
      const int64_t kj = j0 + r;
      const bool ok = kj < s_hi;
      const int64_t src = (((int64_t)b * max_len + (ok ? kj : 0)) * Hkv + gk) * kAttD + ch * 8;
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
  qkv_rope_kernel<<<(unsigned)S, 256, 0, s>>>(qkv, pos, slot, S, Hq, Hkv, D, tab, conc, q_out, k_cache, v_cache);
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
  dim3 grid((unsigned)((Sq + kAttBQ - 1) / kAttBQ), (unsigned)Hq);
  attn_prefill_kernel<<<grid, 128, 0, s>>>(q, k, v, sinks, Sq, Skv, Hq, Hkv, window, sm_scale, o, lse);
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

size_t attn_decode_scratch_bytes(int64_t B, int32_t Hq, int64_t max_len, int32_t splits) {
  (void)max_len;
  return (size_t)B * Hq * splits * (kAttD + 2) * sizeof(float);
}

int attn_decode_splits(int64_t max_len, int32_t window) {
  const int64_t span = window > 0 ? min64(max_len, window) : max_len;
  return (int)max64(1, (span + kDecSplitKeys - 1) / kDecSplitKeys);
}

int launch_attn_decode(const uint16_t* q, const uint16_t* kc, const uint16_t* vc, const int32_t* kv_len, int64_t B,
                       int64_t max_len, int32_t Hq, int32_t Hkv, int32_t D, int32_t window, float sm_scale,
                       const uint16_t* sinks, float* scratch, uint16_t* o, float* lse, cudaStream_t s) {
  if (B <= 0) return 0;
  if (D != kAttD || Hq % Hkv || Hq / Hkv > 8) return -12;
  const int splits = attn_decode_splits(max_len, window);
  float* part_o = scratch;
  float* part_ml = scratch + (size_t)B * Hq * splits * kAttD;
  const size_t smem = 16 * 128 + kDecWarps * 2 * 2 * kAttBK * 128 + kDecWarps * (16 + 16 + 16 * 64) * 4;
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(attn_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    attr = true;
  }
  dim3 grid((unsigned)(B * Hkv), (unsigned)splits);
  attn_decode_kernel<<<grid, 128, smem, s>>>(q, kc, vc, kv_len, max_len, Hq, Hkv, window, sm_scale, splits, part_o,
                                             part_ml);
  const int64_t BH = B * Hq;
  attn_decode_merge_kernel<<<(unsigned)((BH * 32 + 255) / 256), 256, 0, s>>>(part_o, part_ml, BH, Hq, splits, sinks,
                                                                               o, lse);
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
