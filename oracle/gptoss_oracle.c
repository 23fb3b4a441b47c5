/*
 * gptoss_oracle.c -- CPU restatement of the gpt-oss MoE block and sink/YaRN
 * attention arithmetic, used ONLY as a test checker.
 *
 * TEST INFRASTRUCTURE.  Only tests/, __graft_entry__.smoke() and the
 * cpu_baseline / --impl reference legs of bench.py may load this library.
 * The product path (libgptoss_b200.so) never calls it.
 *
 * Every routine restates, step by step, the arithmetic that the reference's
 * TIR lowers to when compiled by TVM for a CPU target (fp32 temporaries,
 * bf16 storage rounded with round-to-nearest-even, serial loops in the
 * reference's loop order, no fused multiply-add).  Build with
 * -ffp-contract=off so that gcc does not contract a*b+c into an FMA.
 *
 * Parity pin: tests/golden/*.npz hold outputs of the reference itself
 * (model/mlp.py and model/attention.py compiled by TVM's C target), and
 * tests/test_oracle_golden.py checks this file against them bit for bit.
 *
 * Reference files are cited by path inside the brekkylab/gpt-oss-tvm tree.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

/* ---------------------------------------------------------------- bf16 -- */

static inline float bf16_to_f32(uint16_t h) {
  uint32_t u = ((uint32_t)h) << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

/* Round-to-nearest-even fp32 -> bf16 by the bias-add rule that TVM's bf16
 * legalisation emits (finite inputs; NaN payloads are not special-cased,
 * exactly like the generated code). */
static inline uint16_t f32_to_bf16(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  u = u + (((u >> 16) & 1u) + 0x7FFFu);
  return (uint16_t)(u >> 16);
}

static inline float round_bf16(float f) { return bf16_to_f32(f32_to_bf16(f)); }

/* E2M1 code table of model/mlp.py:9-26 (FP4_VALUES); low nibble is the
 * even element (model/mlp.py:300-303). */
static const float kFp4Values[16] = {+0.0f, +0.5f, +1.0f, +1.5f, +2.0f, +3.0f, +4.0f, +6.0f,
                                     -0.0f, -0.5f, -1.0f, -1.5f, -2.0f, -3.0f, -4.0f, -6.0f};

int orc_version(void) { return 1; }

/* ------------------------------------------------------------- RMSNorm -- */
/* nn.RMSNorm(eps) as lowered for model/mlp.py:81-87,375 and
 * model/attention.py:84,193: fp32 upcast, serial fp32 sum of squares in
 * column order, r = 1/sqrtf(sum/H + eps), out = bf16((r*x)*w). */
void orc_rms_norm(const uint16_t* x, const uint16_t* w, int64_t M, int64_t H, float eps,
                  uint16_t* out) {
#pragma omp parallel for schedule(static)
  for (int64_t m = 0; m < M; ++m) {
    const uint16_t* xr = x + m * H;
    float ss = 0.0f;
    for (int64_t k = 0; k < H; ++k) {
      float v = bf16_to_f32(xr[k]);
      float sq = v * v;
      ss = ss + sq;
    }
    float r = 1.0f / sqrtf((ss / (float)H) + eps);
    for (int64_t k = 0; k < H; ++k) {
      float v = (r * bf16_to_f32(xr[k])) * bf16_to_f32(w[k]);
      out[m * H + k] = f32_to_bf16(v);
    }
  }
}

/* -------------------------------------------------------------- router -- */
/* nn.Linear(H, E) with bias, bf16 output (model/mlp.py:88-92,376).  The
 * matmul accumulator is a bf16 buffer: acc = bf16(float(acc) + t*w) for
 * k = 0..H-1 in order; then logits = bf16(float(acc) + float(bias)). */
void orc_router(const uint16_t* t, const uint16_t* W, const uint16_t* b, int64_t M, int64_t E,
                int64_t H, uint16_t* logits) {
#pragma omp parallel for schedule(static)
  for (int64_t m = 0; m < M; ++m) {
    for (int64_t e = 0; e < E; ++e) {
      uint16_t acc = f32_to_bf16(0.0f);
      const uint16_t* tr = t + m * H;
      const uint16_t* wr = W + e * H;
      for (int64_t k = 0; k < H; ++k) {
        float prod = bf16_to_f32(tr[k]) * bf16_to_f32(wr[k]);
        float s = bf16_to_f32(acc) + prod;
        acc = f32_to_bf16(s);
      }
      float lg = bf16_to_f32(acc) + bf16_to_f32(b[e]);
      logits[m * E + e] = f32_to_bf16(lg);
    }
  }
}

/* ------------------------------------------------------- top-k softmax -- */
/* nn.op.topk(g, k, largest=True) (model/mlp.py:381): the k largest logits,
 * ordered by value descending, ties broken toward the lower expert index
 * (+0 and -0 compare equal).  Then nn.op.softmax over the k bf16 values
 * (model/mlp.py:382): max in bf16; e_i = bf16(expf(v_i - max));
 * sum = bf16(sum + e_i) serially; w_i = bf16(e_i / sum). */
void orc_topk_softmax(const uint16_t* logits, int64_t M, int64_t E, int64_t K,
                      uint16_t* weights, int32_t* indices, uint16_t* topk_values) {
#pragma omp parallel for schedule(static)
  for (int64_t m = 0; m < M; ++m) {
    const uint16_t* lr = logits + m * E;
    int32_t sel[64];
    float val[64];
    for (int64_t j = 0; j < K; ++j) {
      int32_t best = -1;
      float bv = 0.0f;
      for (int64_t e = 0; e < E; ++e) {
        int taken = 0;
        for (int64_t q = 0; q < j; ++q) taken |= (sel[q] == (int32_t)e);
        if (taken) continue;
        float v = bf16_to_f32(lr[e]);
        if (best < 0 || v > bv) {
          best = (int32_t)e;
          bv = v;
        }
      }
      sel[j] = best;
      val[j] = bv;
    }
    float mx = bf16_to_f32(f32_to_bf16(-3.402823e+38f));
    for (int64_t j = 0; j < K; ++j) {
      float v = round_bf16(val[j]);
      mx = round_bf16(mx > v ? mx : v);
    }
    float ex[64];
    for (int64_t j = 0; j < K; ++j) ex[j] = round_bf16(expf(round_bf16(val[j]) - mx));
    float sum = round_bf16(0.0f);
    for (int64_t j = 0; j < K; ++j) sum = round_bf16(sum + ex[j]);
    for (int64_t j = 0; j < K; ++j) {
      weights[m * K + j] = f32_to_bf16(ex[j] / sum);
      indices[m * K + j] = sel[j];
      if (topk_values) topk_values[m * K + j] = f32_to_bf16(val[j]);
    }
  }
}

/* --------------------------------------------------------- MXFP4 decode -- */
/* value = FP4_VALUES[nibble] * 2^(scale - 127) (model/mlp.py:146-236,
 * :291-303): low nibble = element 2j, high nibble = element 2j+1, one scale
 * per 32 elements.  blocks [rows, G, 16], scales [rows, G]; out
 * [rows, G*32] bf16 (the dequant kernel's out_dtype). */
void orc_mxfp4_dequant(const uint8_t* blocks, const uint8_t* scales, int64_t rows, int64_t G,
                       uint16_t* out) {
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < rows; ++r) {
    for (int64_t g = 0; g < G; ++g) {
      float sc = exp2f((float)((int32_t)scales[r * G + g] - 127));
      for (int64_t j = 0; j < 16; ++j) {
        uint8_t byte = blocks[(r * G + g) * 16 + j];
        float lo = kFp4Values[byte & 15] * sc;
        float hi = kFp4Values[byte >> 4] * sc;
        out[r * G * 32 + g * 32 + 2 * j] = f32_to_bf16(lo);
        out[r * G * 32 + g * 32 + 2 * j + 1] = f32_to_bf16(hi);
      }
    }
  }
}

/* ------------------------------------------------------- fused einsum -- */
/* run_einsum (model/mlp.py:238-326):
 *   out[s,r,c] = bias[e,c] + sum_{k in order} (x * lut[nib]) * 2^(scale-127)
 * accumulated serially in fp32, e = idx[s,r].  x is either bf16 [S, K]
 * (x_is_f32 = 0, mlp1) or fp32 [S, R, K] (x_is_f32 = 1, mlp2; the 3-D
 * branch at model/mlp.py:306-311).  out is fp32 [S, R, N].  rows_mask, if
 * non-NULL, restricts work to tokens s with rows_mask[s] != 0. */
void orc_moe_einsum(const void* x, int x_is_f32, const int32_t* idx, const uint8_t* blocks,
                    const uint8_t* scales, const uint16_t* bias, int64_t S, int64_t R, int64_t N,
                    int64_t K, const uint8_t* rows_mask, float* out) {
  const int64_t G = K / 32;
#pragma omp parallel for collapse(2) schedule(dynamic, 16)
  for (int64_t s = 0; s < S; ++s) {
    for (int64_t r = 0; r < R; ++r) {
      if (rows_mask && !rows_mask[s]) continue;
      int64_t e = idx[s * R + r];
      for (int64_t c = 0; c < N; ++c) {
        float sum = bf16_to_f32(bias[e * N + c]);
        const uint8_t* brow = blocks + (e * N + c) * G * 16;
        const uint8_t* srow = scales + (e * N + c) * G;
        for (int64_t k = 0; k < K; ++k) {
          float sc = exp2f((float)((int32_t)srow[k >> 5] - 127));
          uint8_t byte = brow[k >> 1];
          float w = kFp4Values[(byte >> ((k & 1) * 4)) & 15];
          float xv = x_is_f32 ? ((const float*)x)[(s * R + r) * K + k]
                              : bf16_to_f32(((const uint16_t*)x)[s * K + k]);
          float p = (xv * w) * sc;
          sum = sum + p;
        }
        out[(s * R + r) * N + c] = sum;
      }
    }
  }
}

/* --------------------------------------------------------------- SwiGLU -- */
/* swiglu(x, alpha, limit, out_dtype="float32") (model/mlp.py:29-60,390):
 * glu = even columns, linear = odd columns; g = min(glu, limit);
 * l = clip(linear, -limit, limit); y = (g * sigmoid(alpha*g)) * (l + 1),
 * sigmoid(v) = 1/(1 + expf(0 - v)), all fp32. in [T, 2D] -> out [T, D]. */
void orc_swiglu(const float* in, int64_t T, int64_t D, float alpha, float limit, float* out) {
#pragma omp parallel for schedule(static)
  for (int64_t t = 0; t < T; ++t) {
    for (int64_t d = 0; d < D; ++d) {
      float glu = in[t * 2 * D + 2 * d];
      float lin = in[t * 2 * D + 2 * d + 1];
      float g = glu < limit ? glu : limit;
      float l0 = lin < limit ? lin : limit;
      float l = l0 > -limit ? l0 : -limit;
      float ag = alpha * g;
      float sg = 1.0f / (1.0f + expf(0.0f - ag));
      float gate = g * sg;
      float lp = l + 1.0f;
      out[t * D + d] = gate * lp;
    }
  }
}

/* ------------------------------------------------- gating + residual -- */
/* run_gating (model/mlp.py:328-369): o[s,c] = bf16(sum_r y[s,r,c]*w[s,r])
 * accumulated serially over r in fp32; then the residual
 * out = bf16(float(x) + float(o)) (model/mlp.py:399-402). */
void orc_gating_residual(const float* y, const uint16_t* w, const uint16_t* x, int64_t S,
                         int64_t R, int64_t H, uint16_t* out_gated, uint16_t* out) {
#pragma omp parallel for schedule(static)
  for (int64_t s = 0; s < S; ++s) {
    for (int64_t c = 0; c < H; ++c) {
      float acc = 0.0f;
      for (int64_t r = 0; r < R; ++r) {
        float p = y[(s * R + r) * H + c] * bf16_to_f32(w[s * R + r]);
        acc = acc + p;
      }
      uint16_t o = f32_to_bf16(acc);
      if (out_gated) out_gated[s * H + c] = o;
      if (out) out[s * H + c] = f32_to_bf16(bf16_to_f32(x[s * H + c]) + bf16_to_f32(o));
    }
  }
}

/* ------------------------------------------------------ MoE permutation -- */
/* Expert-major ordering of the (token, rank) pairs, the layout consumed by
 * the grouped expert kernels of model/mlp_optimized.py:118-170
 * (moe_cumsum / get_indices / get_indptr / moe_expand_indptr, the last at
 * model/mlp_optimized.py:126-148).  Row order within an expert is token
 * ascending (a token selects an expert at most once).
 *   indptr[E+1]           exclusive prefix sum of per-expert counts
 *   token_of_row[S*R]     source token of each permuted row
 *   row_of_pair[S*R]      permuted row of pair (s, r)  (scatter-back index)
 *   expert_of_row[S*R]    expert of each permuted row */
void orc_moe_permute(const int32_t* idx, int64_t S, int64_t R, int64_t E, int32_t* indptr,
                     int32_t* token_of_row, int32_t* row_of_pair, int32_t* expert_of_row) {
  int64_t* count = (int64_t*)calloc((size_t)E + 1, sizeof(int64_t));
  for (int64_t i = 0; i < S * R; ++i) count[idx[i]]++;
  indptr[0] = 0;
  for (int64_t e = 0; e < E; ++e) indptr[e + 1] = indptr[e] + (int32_t)count[e];
  int64_t* fill = (int64_t*)calloc((size_t)E, sizeof(int64_t));
  for (int64_t s = 0; s < S; ++s) {
    for (int64_t r = 0; r < R; ++r) {
      int32_t e = idx[s * R + r];
      int64_t row = indptr[e] + fill[e]++;
      token_of_row[row] = (int32_t)s;
      row_of_pair[s * R + r] = (int32_t)row;
      expert_of_row[row] = e;
    }
  }
  free(count);
  free(fill);
}

/* ---------------------------------------------------------- YaRN RoPE -- */
/* AttentionBlock._rope (model/attention.py:15-67, :96-169) as lowered by
 * TVM for a CPU target: per dim d, f = d % (D/2),
 *   e    = float(2f) / D
 *   ramp = 1 - max(min((f - low) / (high - low), 1), 0)
 *   inv  = (1/(factor*powf(theta,e)))*(1-ramp) + (1/powf(theta,e))*ramp
 *   ang  = float(pos) * inv
 *   out  = d <  D/2 : x[d]*(cos*conc) - x[d+D/2]*(sin*conc)
 *          d >= D/2 : x[d-D/2]*(sin*conc) + x[d]*(cos*conc)
 * rounded once to bf16.  low, high_minus_low and conc are the fp32
 * literals the reference's Python constants become (attention.py:15-36,
 * :148-153).  x [S, Hh, D] bf16, pos [S] int32. */
void orc_rope_yarn(const uint16_t* x, const int32_t* pos, int64_t S, int64_t Hh, int64_t D,
                   float theta, float factor, float low, float high_minus_low, float conc,
                   uint16_t* out) {
  const int64_t half = D / 2;
#pragma omp parallel for schedule(static)
  for (int64_t s = 0; s < S; ++s) {
    for (int64_t h = 0; h < Hh; ++h) {
      const uint16_t* xr = x + (s * Hh + h) * D;
      for (int64_t d = 0; d < D; ++d) {
        int64_t f = d & (half - 1);
        float e = ((float)(f * 2)) / (float)D;
        float v = (((float)f) - low) / high_minus_low;
        float v1 = v < 1.0f ? v : 1.0f;
        float ramp = 1.0f - (v1 > 0.0f ? v1 : 0.0f);
        float inter = 1.0f - ramp;
        float inv = ((1.0f / (factor * powf(theta, e))) * inter) + ((1.0f / powf(theta, e)) * ramp);
        float ang = ((float)pos[s]) * inv;
        float o;
        if (d >= half) {
          o = (bf16_to_f32(xr[d - half]) * (sinf(ang) * conc)) + (bf16_to_f32(xr[d]) * (cosf(ang) * conc));
        } else {
          o = (bf16_to_f32(xr[d]) * (cosf(ang) * conc)) - (bf16_to_f32(xr[d + half]) * (sinf(ang) * conc));
        }
        out[(s * Hh + h) * D + d] = f32_to_bf16(o);
      }
    }
  }
}

/* ------------------------------------------------------ attention core -- */
/* Masked softmax(q k^T) v with base-2 log-sum-exp, restating TVM's CPU
 * attention kernels (_attention_prefill_ragged_cpu / _attention_decode_cpu
 * in tvm/relax/frontend/nn/llm/kv_cache.py, third-party, not in the
 * reference tree) with the sliding-window predicate of
 * tvm_fix.patch:35-47:  query row i of a qo_len chunk whose keys are the
 * last qo_len of kv_len sees key j iff  j < kv_len - qo_len + i + 1  and,
 * for window W > 0,  j >= kv_len - qo_len + i - W + 1.
 * Scores s = (q.k) * log2(e) * sm_scale; m starts at -5e4 and d at 1.0;
 * d = d*exp2(m_old - m) + sum exp2(s - m); o = sum v * exp2(s-m)/d;
 * lse = m + log2(d).  q [qo_len, Hq, D], k/v [kv_len, Hkv, D] bf16;
 * o [qo_len, Hq, D] bf16 (the kernel's dtype); lse [qo_len, Hq] fp32. */
void orc_attention(const uint16_t* q, const uint16_t* k, const uint16_t* v, int64_t qo_len,
                   int64_t kv_len, int64_t Hq, int64_t Hkv, int64_t D, int32_t causal,
                   int32_t window, float sm_scale, uint16_t* o, float* lse) {
  const int64_t group = Hq / Hkv;
  const float log2e = 1.4426950408889634f;
#pragma omp parallel for collapse(2) schedule(dynamic, 4)
  for (int64_t i = 0; i < qo_len; ++i) {
    for (int64_t h = 0; h < Hq; ++h) {
      int64_t hk = h / group;
      float* sc = (float*)malloc(sizeof(float) * (size_t)kv_len);
      float m = -5e4f;
      for (int64_t j = 0; j < kv_len; ++j) {
        int vis = causal ? (j < kv_len - qo_len + i + 1) : (j < kv_len);
        if (causal && window > 0) vis = vis && (j >= kv_len - qo_len + i - window + 1);
        float s;
        if (vis) {
          float acc = 0.0f;
          for (int64_t d = 0; d < D; ++d)
            acc = acc + bf16_to_f32(q[(i * Hq + h) * D + d]) * bf16_to_f32(k[(j * Hkv + hk) * D + d]);
          s = acc * log2e * sm_scale;
        } else {
          s = -5e4f * log2e * sm_scale;
        }
        sc[j] = s;
        m = s > m ? s : m;
      }
      float dsum = 1.0f * exp2f(-5e4f - m);
      float tot = 0.0f;
      for (int64_t j = 0; j < kv_len; ++j) {
        sc[j] = exp2f(sc[j] - m);
        tot = tot + sc[j];
      }
      dsum = dsum + tot;
      for (int64_t d = 0; d < D; ++d) {
        float acc = 0.0f;
        for (int64_t j = 0; j < kv_len; ++j)
          acc = acc + bf16_to_f32(v[(j * Hkv + hk) * D + d]) * (sc[j] / dsum);
        o[(i * Hq + h) * D + d] = f32_to_bf16(acc);
      }
      lse[i * Hq + h] = m + log2f(dsum);
      free(sc);
    }
  }
}

/* Sink rescale (model/attention.py:240-247):
 *   scale = bf16(sigmoid(ln2 * lse - float(sink_h)));  o = bf16(o * scale)
 * sigmoid(v) = 1/(1 + expf(0 - v)). o [T, Hq, D] bf16 in place. */
void orc_sink_rescale(uint16_t* o, const float* lse, const uint16_t* sinks, int64_t T, int64_t Hq,
                      int64_t D) {
  const float ln2 = 0.6931471805599453f;
#pragma omp parallel for schedule(static)
  for (int64_t t = 0; t < T; ++t) {
    for (int64_t h = 0; h < Hq; ++h) {
      float a = ln2 * lse[t * Hq + h];
      float z = a - bf16_to_f32(sinks[h]);
      float sg = 1.0f / (1.0f + expf(0.0f - z));
      float s = round_bf16(sg);
      for (int64_t d = 0; d < D; ++d) {
        float v = bf16_to_f32(o[(t * Hq + h) * D + d]) * s;
        o[(t * Hq + h) * D + d] = f32_to_bf16(v);
      }
    }
  }
}

/* Merge of two partial attention states (o, lse in base 2), the
 * merge_attn_output_inplace step of model/attention.py:225-233, in the
 * arithmetic of TVM's CPU merge kernel (_merge_state_inplace_cpu in
 * tvm/relax/frontend/nn/llm/kv_cache.py, third-party):
 *   m = max(l1, l2); w1 = exp2(l1 - m); w2 = exp2(l2 - m);
 *   o = o1 * (w1/(w1 + w2)) + o2 * (w2/(w1 + w2)); lse = log2(w1 + w2) + m. */
void orc_merge_states(const uint16_t* o1, const float* l1, const uint16_t* o2, const float* l2,
                      int64_t T, int64_t Hq, int64_t D, uint16_t* o, float* lse) {
#pragma omp parallel for schedule(static)
  for (int64_t t = 0; t < T; ++t) {
    for (int64_t h = 0; h < Hq; ++h) {
      float a = l1[t * Hq + h], b = l2[t * Hq + h];
      float m = a > b ? a : b;
      float wa = exp2f(a - m), wb = exp2f(b - m);
      float sa = wa / (wa + wb), sb = wb / (wa + wb);
      for (int64_t d = 0; d < D; ++d) {
        int64_t ix = (t * Hq + h) * D + d;
        float v = (bf16_to_f32(o1[ix]) * sa) + (bf16_to_f32(o2[ix]) * sb);
        o[ix] = f32_to_bf16(v);
      }
      lse[t * Hq + h] = log2f(wa + wb) + m;
    }
  }
}

/* One decode query per sequence over its cached keys, in the arithmetic of
 * TVM's CPU decode kernel (_attention_decode_cpu in kv_cache.py, the
 * cross_attention of model/attention.py:221-224): an online softmax over
 * the keys in order,
 *   s = (q.k) * (sm_scale * log2 e);  m' = max(m, s);
 *   d = d * exp2(m - m') + exp2(s - m');  o = o * exp2(m - m') + v * exp2(s - m');
 * from m = -5e4, d = 1, o = 0; output bf16(o / d), lse = m + log2(d).
 * Sequence b has kv_len[b] keys; a window W > 0 reads only the last W of
 * them (the sliding-window variant, whose chunk starts at the window
 * offset).  q [B, Hq, D]; caches [B, max_len, Hkv, D] bf16; o [B, Hq, D]. */
void orc_attention_decode(const uint16_t* q, const uint16_t* kc, const uint16_t* vc, const int32_t* kv_len,
                          int64_t B, int64_t max_len, int64_t Hq, int64_t Hkv, int64_t D, int32_t window,
                          float sm_scale, uint16_t* o, float* lse) {
  const int64_t group = Hq / Hkv;
  const float scale = sm_scale * 1.4426950408889634f;
#pragma omp parallel for collapse(2) schedule(dynamic, 1)
  for (int64_t b = 0; b < B; ++b) {
    for (int64_t h = 0; h < Hq; ++h) {
      const int64_t hk = h / group, L = kv_len[b];
      const int64_t j0 = (window > 0 && L > window) ? L - window : 0;
      float* acc = (float*)calloc((size_t)D, sizeof(float));
      float m = -5e4f, den = 1.0f;
      for (int64_t j = j0; j < L; ++j) {
        const uint16_t* kr = kc + ((b * max_len + j) * Hkv + hk) * D;
        const uint16_t* vr = vc + ((b * max_len + j) * Hkv + hk) * D;
        float sc = 0.0f;
        for (int64_t d = 0; d < D; ++d) sc = sc + bf16_to_f32(q[(b * Hq + h) * D + d]) * bf16_to_f32(kr[d]);
        sc = sc * scale;
        const float mn = m > sc ? m : sc;
        den = (den * exp2f(m - mn)) + exp2f(sc - mn);
        const float so = exp2f(m - mn);
        for (int64_t d = 0; d < D; ++d) acc[d] = acc[d] * so;
        m = mn;
        const float f = exp2f(sc - m);
        for (int64_t d = 0; d < D; ++d) acc[d] = acc[d] + bf16_to_f32(vr[d]) * f;
      }
      for (int64_t d = 0; d < D; ++d) o[(b * Hq + h) * D + d] = f32_to_bf16(acc[d] / den);
      lse[b * Hq + h] = m + log2f(den);
      free(acc);
    }
  }
}
