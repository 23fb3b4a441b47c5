/*
 * gptoss_b200.h -- C ABI of libgptoss_b200.so, the B200 (sm_100a) kernels for
 * the gpt-oss MXFP4 mixture-of-experts block and sink/YaRN attention.
 *
 * Conventions
 *   - Destination-passing style: the caller owns every input and output
 *     buffer (device memory) and passes plain pointers and sizes.  bf16 data
 *     is passed as uint16_t bit patterns.
 *   - Every call is asynchronous on the given CUDA stream (`stream` is a
 *     cudaStream_t; NULL = legacy default stream) and returns 0 on success
 *     or a negative code; gptoss_last_error() describes the last failure of
 *     the calling host thread.  Calls on one workspace are not re-entrant.
 *   - Device-side failures (a bounded wait that ran out, an expert index out
 *     of range) set bits in the workspace's device error word, read with
 *     gptoss_moe_workspace_error().
 *
 * Each entry point names the reference (brekkylab/gpt-oss-tvm) interface it
 * replaces.  In the reference these are TIR kernels registered with
 * nn.tensor_ir_op (DPS, single stream) and Relax ops inside MLPBlock.forward
 * (model/mlp.py:371-402) and AttentionBlock.forward (model/attention.py:182-256).
 */
#ifndef GPTOSS_B200_H_
#define GPTOSS_B200_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---------------------------------------------------------------- status */
int gptoss_version(void);
const char* gptoss_last_error(void);

/* ------------------------------------------------------------ MoE weights
 * The reference MLPBlock parameters, unchanged (model/mlp.py:81-143):
 *   norm_weight [H], gate_weight [E, H], gate_bias [E] (bf16);
 *   mlp1_blocks [E, 2I, K/32, 16] u8, mlp1_scales [E, 2I, K/32] u8,
 *   mlp1_bias [E, 2I] bf16; mlp2_blocks [E, H, I/32, 16] u8,
 *   mlp2_scales [E, H, I/32] u8, mlp2_bias [E, H] bf16.
 * With expert parallelism the mlp* pointers cover the `num_local_experts`
 * experts [expert_offset, expert_offset + num_local_experts); the router
 * (gate_*) always covers all `num_experts`. */
typedef struct gptoss_moe_weights {
  int32_t num_experts;
  int32_t num_local_experts;
  int32_t expert_offset;
  int32_t hidden;        /* H = 2880 */
  int32_t intermediate;  /* I = 2880 */
  int32_t top_k;         /* 4 */
  float swiglu_alpha;    /* 1.702 */
  float swiglu_limit;    /* 7.0 */
  float rms_eps;         /* 1e-5 */
  const uint16_t* norm_weight;
  const uint16_t* gate_weight;
  const uint16_t* gate_bias;
  const uint8_t* mlp1_blocks;
  const uint8_t* mlp1_scales;
  const uint16_t* mlp1_bias;
  const uint8_t* mlp2_blocks;
  const uint8_t* mlp2_scales;
  const uint16_t* mlp2_bias;
  uint32_t flags;        /* GPTOSS_MOE_* bits, set by gptoss_moe_weights_prepare */
} gptoss_moe_weights;

/* flags bit: every E8M0 scale code is in 104..140 and RMSNorm outputs stay in
 * the f16 range, so the grouped GEMMs may decode the e2m1 weights to f16 with
 * the hardware converter and run on f16 activations (exact weights either way). */
#define GPTOSS_MOE_F16 1u

/* One-time weight check (synchronises `stream`): sets or clears GPTOSS_MOE_F16
 * in w->flags from the scale codes and the norm weight.  Call after loading
 * weights (the reference loads them once, weights.py:102-122). */
int gptoss_moe_weights_prepare(gptoss_moe_weights* w, void* stream);

/* Scratch for gptoss_moe_forward (device memory owned by the library). */
typedef struct gptoss_moe_workspace gptoss_moe_workspace;

gptoss_moe_workspace* gptoss_moe_workspace_create(int64_t max_tokens, int32_t num_experts, int32_t top_k,
                                                  int32_t hidden, int32_t intermediate);
void gptoss_moe_workspace_destroy(gptoss_moe_workspace* ws);
/* Device error word of the workspace (synchronises the device); clears it. */
uint32_t gptoss_moe_workspace_error(gptoss_moe_workspace* ws);

/* MLPBlock.forward (model/mlp.py:371-402): out = x + MoE(RMSNorm(x)).
 * x, out: [M, H] bf16 (may alias).  M <= max_tokens of the workspace. */
int gptoss_moe_forward(const uint16_t* x, int64_t M, const gptoss_moe_weights* w, gptoss_moe_workspace* ws,
                       uint16_t* out, void* stream);

/* ------------------------------------------------------ MoE building blocks */
/* nn.RMSNorm (model/mlp.py:81-87, :375; model/attention.py:84, :193).
 * Bit-exact to the reference's CPU lowering. */
int gptoss_rms_norm(const uint16_t* x, const uint16_t* weight, int64_t M, int32_t H, float eps, uint16_t* out,
                    void* stream);

/* self.gate + nn.op.topk + nn.op.softmax (model/mlp.py:376, :381-382).
 * t [M, H] bf16 (normed), gate_weight [E, H], gate_bias [E] -> logits [M, E]
 * bf16, topk_weights [M, K] bf16, topk_indices [M, K] int32.  Bit-exact.
 * err: optional device word for out-of-range detection (may be NULL). */
int gptoss_moe_router(const uint16_t* t, const uint16_t* gate_weight, const uint16_t* gate_bias, int64_t M,
                      int32_t E, int32_t H, int32_t K, uint16_t* logits, uint16_t* topk_weights,
                      int32_t* topk_indices, uint32_t* err, void* stream);

/* nn.op.topk(largest=True) + nn.op.softmax (model/mlp.py:381-382) on given
 * bf16 logits [M, E] (E <= 256, K <= 8).  Bit-exact. */
int gptoss_moe_topk_softmax(const uint16_t* logits, int64_t M, int32_t E, int32_t K, uint16_t* topk_weights,
                            int32_t* topk_indices, uint32_t* err, void* stream);

/* moe_cumsum / get_indices / get_indptr / moe_expand_indptr
 * (model/mlp_optimized.py:118-148): expert-major order of the M*K
 * (token, rank) pairs, token-ascending within an expert.  Bit-exact.
 *   indptr [E+1], token_of_row [M*K], row_of_pair [M*K], expert_of_row [M*K],
 *   tile_ptr [E+1], tile_rows [E] (token tiles of the grouped GEMMs). */
int gptoss_moe_permute(const int32_t* topk_indices, int64_t M, int32_t K, int32_t E, int32_t* indptr,
                       int32_t* token_of_row, int32_t* row_of_pair, int32_t* expert_of_row, int32_t* tile_ptr,
                       int32_t* tile_rows, uint32_t* err, void* stream);

/* nn.op.take(t, token_indices) (model/mlp_optimized.py:150): act[r] = t[token_of_row[r]],
 * converted to f16 when act_f16 (the f16 GEMM path). */
int gptoss_moe_gather(const uint16_t* t, const int32_t* token_of_row, int64_t rows, int32_t H, int32_t act_f16,
                      uint16_t* act, void* stream);

/* run_einsum(mlp1) + swiglu (model/mlp.py:238-326, :29-60, :387-390;
 * grouped form mxfp4_moe_mlp1_prefill, model/mlp_optimized.py:214-351).
 * act [act_rows, H] expert-major (bf16, or f16 when act_f16); weights of E experts;
 * y [act_rows, I] (same type as act).  Tolerance (bf16) vs. the reference. */
int gptoss_moe_mlp1(const uint16_t* act, int64_t act_rows, const int32_t* indptr, const int32_t* tile_ptr,
                    const int32_t* tile_rows, int32_t E, int32_t H, int32_t I, const uint8_t* blocks,
                    const uint8_t* scales, const uint16_t* bias, float alpha, float limit, int32_t act_f16,
                    uint16_t* y, uint32_t* err, void* stream);

/* run_einsum(mlp2) (model/mlp.py:395; grouped form mxfp4_moe_mlp2_prefill,
 * model/mlp_optimized.py:353-460).  y [rows, I] (bf16, or f16 when act_f16) -> h2 [rows, H] fp32. */
int gptoss_moe_mlp2(const uint16_t* y, int64_t act_rows, const int32_t* indptr, const int32_t* tile_ptr,
                    const int32_t* tile_rows, int32_t E, int32_t H, int32_t I, const uint8_t* blocks,
                    const uint8_t* scales, const uint16_t* bias, int32_t act_f16, float* h2, uint32_t* err,
                    void* stream);

/* The same two grouped GEMMs for decode-size token tiles (rows <= 8 x E) on
 * the block-scaled tensor cores (tcgen05.mma kind::mxf8f6f4): the MXFP4
 * weights and their E8M0 scales feed the MMA as stored; the activations are
 * carried as two e4m3 terms per value with E8M0 exponents per 32 values
 * (the sum is within 2^-8 relative of the bf16/f16 value).  Same semantics
 * as run_einsum / swiglu (model/mlp.py:238-326, :29-60, :395).
 * gptoss_moe_quantize_mx: row r of q [rows, 2K] (K hi codes, then K lo codes)
 * and scales [rows, 192] (hi exponents, then at byte 96 lo exponents; K/32 <= 96)
 * from source row row_index[r] (or r) of src [*, K] (f16 if src_f16, else bf16).
 * gptoss_moe_mlp1_mx -> y [rows, I] f16; gptoss_moe_mlp2_mx -> h2 [rows, H] fp32.
 * blocks must be 32-byte aligned, K a multiple of 64 in 256..3072. */
int gptoss_moe_quantize_mx(const uint16_t* src, int32_t src_f16, const int32_t* row_index, int64_t rows, int32_t K,
                           uint8_t* q, uint8_t* scales, void* stream);
int gptoss_moe_mlp1_mx(const uint8_t* q, const uint8_t* act_scales, int64_t act_rows, const int32_t* indptr,
                       const int32_t* tile_ptr, const int32_t* tile_rows, int32_t E, int32_t H, int32_t I,
                       const uint8_t* blocks, const uint8_t* scales, const uint16_t* bias, float alpha, float limit,
                       uint16_t* y, uint32_t* err, void* stream);
int gptoss_moe_mlp2_mx(const uint8_t* q, const uint8_t* act_scales, int64_t act_rows, const int32_t* indptr,
                       const int32_t* tile_ptr, const int32_t* tile_rows, int32_t E, int32_t H, int32_t I,
                       const uint8_t* blocks, const uint8_t* scales, const uint16_t* bias, float* h2, uint32_t* err,
                       void* stream);

/* 1 when gptoss_moe_forward of M tokens with these weights runs the experts
 * on the block-scaled path above (decode-size tiles, GPTOSS_MOE_MX not 0),
 * 0 when it runs the decode GEMV or the kind::f16 kernels. */
int gptoss_moe_uses_block_scaled(int64_t M, const gptoss_moe_weights* w);

/* run_gating + residual (model/mlp.py:328-369, :398-402):
 * out[m] = bf16(x[m] + bf16(sum_r h2[row_of_pair[m,r]] * w[m,r])). */
int gptoss_moe_combine(const float* h2, const int32_t* row_of_pair, const uint16_t* topk_weights,
                       const uint16_t* x, int64_t M, int32_t K, int32_t H, uint16_t* out, void* stream);

/* MLPBlock.__dequantize_mxfp4_weight (model/mlp.py:146-236): exact decode of
 * MXFP4 blocks [rows, G, 16] + scales [rows, G] to bf16 [rows, G*32]. */
int gptoss_mxfp4_dequant(const uint8_t* blocks, const uint8_t* scales, int64_t rows, int32_t groups,
                         uint16_t* out, void* stream);

/* -------------------------------------------------------------- attention
 * AttentionBlock (model/attention.py:70-256): head_dim 64, GQA (Hq a multiple
 * of Hkv), learned per-head sinks, alternating sliding-window / full causal
 * masks, YaRN RoPE.  Layouts: q [T, Hq, D], k / v [T, Hkv, D] bf16; lse
 * [T, Hq] fp32 in base 2 of the scaled scores (q.k * sm_scale * log2 e),
 * the convention of the reference's TVM kernels (attention.py:237-240). */

/* YaRN inverse frequencies inv_freq [D/2] and the attention concentration
 * (rope_freq_yarn, model/attention.py:15-67, :148-153), computed on the host
 * in fp32 like the reference.  Host memory in and out. */
int gptoss_yarn_inv_freq(int32_t D, float theta, float factor, float beta_fast, float beta_slow,
                         int32_t original_max_position, float* inv_freq, float* concentration);

/* AttentionBlock._rope (model/attention.py:96-169): x [S, heads, D] -> out,
 * rotate-half pairs (d, d + D/2), positions [S] int32 (device), inv_freq host. */
int gptoss_rope_yarn(const uint16_t* x, const int32_t* positions, int64_t S, int32_t heads, int32_t D,
                     const float* inv_freq, float concentration, uint16_t* out, void* stream);

/* qkv split + RoPE on q and k + append_mha_kv (model/attention.py:206-214):
 * qkv [S, (Hq + 2 Hkv) D] -> q_out [S, Hq, D]; k (rotated) and v written to
 * row slots[s] of k_cache / v_cache [num_slots, Hkv, D] (slots NULL: row s). */
int gptoss_qkv_rope_append(const uint16_t* qkv, const int32_t* positions, const int32_t* slots, int64_t S,
                           int32_t Hq, int32_t Hkv, int32_t D, const float* inv_freq, float concentration,
                           uint16_t* q_out, uint16_t* k_cache, uint16_t* v_cache, void* stream);

/* paged_kv_cache.self_attention + the sink rescale (model/attention.py:218-247):
 * Sq queries that are the last Sq of Skv keys, causal, window W > 0 keeps
 * keys >= pos - W + 1 (tvm_fix.patch:35-47), W <= 0 = full.  sinks [Hq]
 * bf16 or NULL (NULL: no rescale, o is the plain attention output).
 * o [Sq, Hq, D] bf16; lse [Sq, Hq] fp32 or NULL. */
int gptoss_attn_prefill(const uint16_t* q, const uint16_t* k, const uint16_t* v, const uint16_t* sinks, int64_t Sq,
                        int64_t Skv, int32_t Hq, int32_t Hkv, int32_t D, int32_t window, float sm_scale, uint16_t* o,
                        float* lse, void* stream);

/* paged_kv_cache.cross_attention for one new token per sequence
 * (model/attention.py:221-224) + sink rescale: q [B, Hq, D]; caches
 * [B, max_len, Hkv, D] with kv_len[b] valid rows (device), the query being
 * the token at kv_len[b] - 1; window as above (decode on windowed layers
 * reads the last W keys, tvm_fix.patch:194-281).  scratch: device memory of
 * gptoss_attn_decode_scratch_bytes() bytes.  o [B, Hq, D]; lse [B, Hq]. */
int64_t gptoss_attn_decode_scratch_bytes(int64_t B, int32_t Hq, int64_t max_len, int32_t window);
int gptoss_attn_decode(const uint16_t* q, const uint16_t* k_cache, const uint16_t* v_cache, const int32_t* kv_len,
                       int64_t B, int64_t max_len, int32_t Hq, int32_t Hkv, int32_t D, int32_t window,
                       float sm_scale, const uint16_t* sinks, float* scratch, int64_t scratch_bytes, uint16_t* o,
                       float* lse, void* stream);

/* The paged KV cache (the reference's PagedKVCache with page size 16,
 * engine.py:93-104; page windowing tvm_fix.patch:194-281).  A layer's keys
 * and values live in page pools k_pages / v_pages [num_pages * 16, Hkv, D]
 * bf16; key position j of sequence b is row
 *   page_table[b * table_stride + (j / 16) % table_stride] * 16 + j % 16.
 * Full-attention layers give each sequence table_stride >= ceil(len / 16)
 * pages; sliding-window layers may give it a ring of table_stride pages
 * (>= ceil(window / 16) + 1) that holds the last keys only.
 * gptoss_attn_decode_paged: gptoss_attn_decode over such a cache (kv_len[b]
 * keys, window as there); scratch as gptoss_attn_decode_scratch_bytes(B, Hq,
 * 16 * table_stride, window). */
int gptoss_attn_decode_paged(const uint16_t* q, const uint16_t* k_pages, const uint16_t* v_pages,
                             const int32_t* page_table, int32_t table_stride, const int32_t* kv_len, int64_t B,
                             int32_t Hq, int32_t Hkv, int32_t D, int32_t window, float sm_scale, const uint16_t* sinks,
                             float* scratch, int64_t scratch_bytes, uint16_t* o, float* lse, void* stream);
/* Rows of positions pos0 .. pos0 + n - 1 of sequence `seq` between the page
 * pools and contiguous rows k_rows / v_rows [n, Hkv, D]: to_pages != 0 writes
 * the pages (append_mha_kv of a prefill chunk), else reads them (the cached
 * keys an extend attends to). */
int gptoss_kv_pages_copy(uint16_t* k_pages, uint16_t* v_pages, int32_t Hkv, int32_t D, const int32_t* page_table,
                         int32_t table_stride, int32_t seq, int64_t pos0, int64_t n, uint16_t* k_rows,
                         uint16_t* v_rows, int32_t to_pages, void* stream);

/* merge_attn_output_inplace (model/attention.py:231-233): two partial
 * attention states over disjoint keys -> one (o bf16 [T, Hq, D], lse). */
int gptoss_attn_merge(const uint16_t* o1, const float* lse1, const uint16_t* o2, const float* lse2, int64_t T,
                      int32_t Hq, int32_t D, uint16_t* o, float* lse, void* stream);

/* Sink rescale alone (model/attention.py:240-247), in place:
 * o *= bf16(sigmoid(ln2 * lse - sink[h])). */
int gptoss_attn_sink_rescale(uint16_t* o, const float* lse, const uint16_t* sinks, int64_t T, int32_t Hq, int32_t D,
                             void* stream);

/* The attention block's dense projections, nn.Linear with bias
 * (model/attention.py:85-92, :206-211, :254), for decode sizes: out [T, N] =
 * bf16(x [T, K] . weight [N, K]^T + bias [N]), fp32 accumulation, one rounding.
 * T up to gptoss_dense_gemv_max_tokens(); bias may be NULL; weight 16-byte
 * aligned, K a multiple of 8 (<= 8192).  Larger T: a library GEMM. */
int gptoss_dense_gemv_max_tokens(void);
int gptoss_dense_gemv(const uint16_t* x, int64_t T, const uint16_t* weight, const uint16_t* bias, int32_t N,
                      int32_t K, uint16_t* out, void* stream);

/* The same projections at every size on the tensor cores (tcgen05.mma
 * kind::f16, TMA-fed, fp32 in TMEM), and the unembedding without bias
 * (model/transformer.py:99-104): out [T, N] = bf16(x [T, K] . weight [N, K]^T
 * (+ bias [N])), one rounding.  T <= 256 streams the weight rows as the MMA's
 * M side (clusters of CTAs split K when the weight tiles are few; the split
 * partials are added in a fixed order, so results are deterministic); larger
 * T runs persistent 128 x 256 tiles.  x, weight and out 16-byte aligned, K a
 * multiple of 8; bias may be NULL; err: optional device word that records a
 * pipeline wait that ran out (the call then leaves out incomplete). */
int gptoss_dense_gemm(const uint16_t* x, int64_t T, const uint16_t* weight, const uint16_t* bias, int32_t N,
                      int32_t K, uint16_t* out, uint32_t* err, void* stream);

/* Engine.sample (engine.py:38-39, :172-174), i.e. TVM's
 * vm.builtin.sample_top_p_from_logits(logits, temperature, top_p,
 * uniform_sample) (src/runtime/vm/lm_support.cc), on the device and batched:
 * row b of logits [B, V] (fp32, device) gives tokens[b] (int32, device): the
 * argmax when temperature < 1e-6, otherwise the top-p draw with
 * uniform[b] (device, B doubles) or, when uniform is NULL, uniform0 for every
 * row -- the reference's float running sums in its order, so the same token.
 * Ties among logits go to the lower index.  scratch: device memory for the
 * rows whose large elements do not fit on chip; gptoss_sample_top_p_scratch_bytes
 * (B, V) bytes run all rows at once, less runs them in groups (at least one
 * row's worth is required unless temperature < 1e-6). */
int64_t gptoss_sample_top_p_scratch_bytes(int64_t B, int64_t V);
int gptoss_sample_top_p_from_logits(const float* logits, int64_t B, int64_t V, double temperature, double top_p,
                                    const double* uniform, double uniform0, void* scratch, int64_t scratch_bytes,
                                    int32_t* tokens, void* stream);

/* The routing half of gptoss_moe_forward for M normalised tokens t (the
 * output of gptoss_rms_norm): router logits, top-k + softmax and the
 * expert-major permutation with its token-tile plan -- the outputs of
 * gptoss_moe_router followed by gptoss_moe_permute, bit for bit.  At decode
 * sizes (M * top_k <= 256, E <= 256) the part after the logits is one
 * launch. */
int gptoss_moe_route(const uint16_t* t, int64_t M, const gptoss_moe_weights* w, uint16_t* logits,
                     uint16_t* topk_weights, int32_t* topk_indices, int32_t* indptr, int32_t* token_of_row,
                     int32_t* row_of_pair, int32_t* expert_of_row, int32_t* tile_ptr, int32_t* tile_rows,
                     uint32_t* err, void* stream);

/* MLPBlock.forward like gptoss_moe_forward, but allocating nothing: no
 * cudaMalloc, no cudaFree, no workspace.  It has no counterpart in the
 * reference.  It is for callers that cannot allocate device memory when the
 * block runs -- a serving loop whose device memory is planned before the
 * first request, code that must not call cudaMalloc because it synchronises
 * the device, or a host without a CUDA allocator of its own.
 * Its scratch is one fixed device array inside this library (about 6.3 MB,
 * held on every GPU that loads the library until the process exits), sized
 * for M <= 64 tokens, <= 128 experts, top_k <= 4 and hidden, intermediate
 * <= 2880; larger sizes are rejected with an error.  All experts must be on
 * this device.  The first call on each device looks up the array's device
 * address (with that device current) and caches it for the process; make
 * that first call before any stream capture, and do not reset the device
 * between calls.  Every call shares the array: calls that overlap on the
 * GPU (two streams, or two host threads) race on it, and the array keeps
 * the last call's contents.  Device-side failures (a bounded wait that ran
 * out, an expert index out of range) set bits in an error word at the end of
 * the array, read with gptoss_moe_noalloc_error().  x, out: [M, H] bf16
 * device memory. */
int gptoss_moe_forward_noalloc(const uint16_t* x, int64_t M, const gptoss_moe_weights* w, uint16_t* out,
                               void* stream);
/* The device error word of gptoss_moe_forward_noalloc on the current device
 * (the DeviceError bits of gptoss_moe_workspace_error); synchronises the
 * device, reads the word and clears it, allocating nothing.  No counterpart
 * in the reference.  Returns 0xFFFFFFFF when the word cannot be read. */
uint32_t gptoss_moe_noalloc_error(void);

/* --------------------------------------------- expert-parallel helpers
 * The reference runs the MoE block on one device (world_size = 1,
 * model/mlp.py:79); expert parallelism is new here.  Each rank owns
 * num_experts / num_ranks experts; token rows travel between ranks with one
 * NCCL all-to-all each way (host code).  These two calls prepare the rows
 * that arrive for the grouped GEMMs and send the results back. */

/* Token tiles of gptoss_moe_mlp1/mlp2 for rows already grouped by expert
 * (indptr [E+1], device): tile_ptr [E+1], tile_rows [E]. */
int gptoss_moe_plan_tiles(const int32_t* indptr, int32_t E, int32_t* tile_ptr, int32_t* tile_rows, void* stream);

/* Reorders rows between source-major order (for each source rank s, the rows
 * of local experts 0..El-1, counts[s*El + e] rows each) and expert-major order
 * (for each expert, the rows of sources 0..P-1).  direction 0: src -> expert
 * major (also writes indptr_local [El+1] when non-NULL); 1: the reverse;
 * 2: the reverse with fp32 source rows of row_bytes rounded to bf16 rows of
 * row_bytes / 2 (the expert outputs travel back in bf16).
 * row_bytes must be a multiple of 16.  counts is device memory. */
int gptoss_moe_segment_copy(const void* src, void* dst, const int32_t* counts, int32_t num_ranks,
                            int32_t local_experts, int64_t row_bytes, int32_t direction, int32_t* indptr_local,
                            void* stream);

/* gptoss_moe_combine with the expert outputs already rounded to bf16 (the
 * expert-parallel return path): out[m] = bf16(x[m] + bf16(sum_r float(h2[..]) * w[m,r])).
 * No counterpart in the reference (it has no expert parallelism). */
int gptoss_moe_combine_bf16(const uint16_t* h2, const int32_t* row_of_pair, const uint16_t* topk_weights,
                            const uint16_t* x, int64_t M, int32_t K, int32_t H, uint16_t* out, void* stream);

/* ----------------------------------------- expert parallelism over peer memory
 * No counterpart in the reference (it runs the block on one device).  The
 * ranks of one node share buffers through CUDA IPC and write each other's
 * rows directly (plain stores over NVLink; no multicast, no device-side
 * waits on other GPUs).  The caller orders the ranks: every writing call
 * ends with a system-scope fence, and the ranks meet at a collective before
 * the written rows are read or written again. */

/* Stream-ordered flags between ranks (no counterpart in the reference).
 * gptoss_stream_set_flag: once the stream's earlier work is done, a system-
 * scope fence and a release store of `value` into the device word `flag`
 * (this GPU's memory, or a peer's through gptoss_ipc_open).
 * gptoss_stream_wait_flag: the stream waits on the device until the word
 * reaches `value` (wrap-safe: (int32_t)(word - value) >= 0), polling at most
 * max_polls times (1..2^26, about 0.1-0.2 us per poll); when the limit runs
 * out it sets bit 1 << 5 (timeout of a flag wait) in the device word `err`
 * (may be NULL) and returns, so later work on the stream still runs.  The
 * waiting and the setting kernel must run on different GPUs (or the flag be
 * set before the wait is launched): two launches that wait on one another
 * are never guaranteed to run at the same time on one GPU. */
int gptoss_stream_set_flag(uint32_t* flag, uint32_t value, void* stream);
int gptoss_stream_wait_flag(const uint32_t* flag, uint32_t value, uint32_t max_polls, uint32_t* err, void* stream);

/* cudaMalloc of `bytes` on the current device, zero-filled; its IPC handle
 * (64 bytes) in `handle`.  Free with gptoss_ipc_free. */
int gptoss_ipc_alloc(uint64_t bytes, void** ptr, void* handle);
/* Map another process's allocation from its 64-byte handle (peer access
 * enabled); unmap with gptoss_ipc_close. */
int gptoss_ipc_open(const void* handle, void** ptr);
int gptoss_ipc_close(void* ptr);
int gptoss_ipc_free(void* ptr);

/* Row addressing of the expert-parallel dispatch, on the device (no host
 * round trip): counts_all [num_ranks, num_ranks * local_experts] int32 holds
 * every rank's rows per global expert (an all-gather of the per-expert counts).
 * Rank d's activation matrix is expert-major over its local experts and
 * source-rank-major inside an expert.  Writes dst_base [num_ranks *
 * local_experts] (first row on rank d of this rank's rows of d's expert e) and
 * indptr_local [local_experts + 1] (this rank's own expert offsets). */
int gptoss_moe_peer_layout(const int32_t* counts_all, int32_t num_ranks, int32_t local_experts, int32_t rank,
                           int32_t* dst_base, int32_t* indptr_local, void* stream);

/* Expert-parallel dispatch: for every send row r of this rank (the
 * expert-major order of gptoss_moe_permute over the global experts), with
 * eg = expert_of_row[r], d = eg / local_experts, e = eg % local_experts:
 *   rank d's rows[dst] = t[token_of_row[r]] (f16 when to_f16), and
 *   rank d's origin[dst] = (rank << 24) | r,
 * dst = dst_base[d * local_experts + e] + r - indptr[eg] (device int32
 * [num_ranks * local_experts]).  peer_rows / peer_origin: host arrays of
 * num_ranks device pointers (this rank's own buffers at index `rank`), each
 * buffer holding cap_rows rows of H elements / cap_rows int32.  num_ranks <= 8,
 * rows < 2^24. */
int gptoss_moe_dispatch_peer(const uint16_t* t, const int32_t* token_of_row, const int32_t* expert_of_row,
                             const int32_t* indptr, int64_t rows, int32_t H, int32_t num_experts,
                             int32_t local_experts, int32_t rank, const int32_t* dst_base, void* const* peer_rows,
                             int32_t* const* peer_origin, int32_t num_ranks, int64_t cap_rows, int32_t to_f16,
                             void* stream);

/* gptoss_moe_mlp2 whose output row r goes to row (origin[r] & 0xFFFFFF) of
 * peer_back[origin[r] >> 24] (row stride H): fp32, or bf16 (rounded to
 * nearest even) when back_bf16.  peer_back: host array of num_ranks device
 * pointers (<= 8), each holding back_rows rows (a row index beyond it, or a
 * rank beyond num_ranks, is dropped). */
int gptoss_moe_mlp2_peer(const uint16_t* y, int64_t act_rows, const int32_t* indptr, const int32_t* tile_ptr,
                         const int32_t* tile_rows, int32_t E, int32_t H, int32_t I, const uint8_t* blocks,
                         const uint8_t* scales, const uint16_t* bias, int32_t act_f16, const int32_t* origin,
                         void* const* peer_back, int32_t num_ranks, int64_t back_rows, int32_t back_bf16,
                         uint32_t* err, void* stream);

/* ------------------------------- expert parallelism at the C boundary
 * No counterpart in the reference (it runs the block on one device).  The
 * experts of an MLPBlock are sharded over `world` ranks of one node, one
 * process per GPU: rank r owns experts [r E / world, (r + 1) E / world) and
 * routes its own tokens.  NCCL (libnccl.so.2, loaded at run time) carries the
 * per-expert row counts and two one-word orderings per step; the token rows
 * and expert outputs move by plain stores into the other ranks' CUDA IPC
 * buffers (NVLink; no multicast, no device-side waits on other GPUs).  Every
 * rank makes the same calls in the same order on its stream. */
typedef struct gptoss_ep gptoss_ep;
/* A new group's NCCL unique id (128 bytes); rank 0 creates it and sends it to
 * the other ranks over any host channel. */
int gptoss_ep_unique_id(void* id);
/* Joins the group (collective): NCCL communicator, this rank's scratch and
 * IPC buffers for max_tokens tokens per rank, the other ranks' buffers
 * mapped.  exact_return: expert outputs travel back in fp32 (the block is
 * then bit-equal to one GPU's) instead of bf16 (half the bytes).  NULL on
 * failure (gptoss_last_error()). */
gptoss_ep* gptoss_ep_init(const void* id, int32_t rank, int32_t world, int64_t max_tokens, int32_t num_experts,
                          int32_t top_k, int32_t hidden, int32_t intermediate, int32_t exact_return, void* stream);
/* Dispatch: RMSNorm, router, top-k and permutation of this rank's tokens x
 * [M, H]; rows stored into the owners' activation matrices.  w: this rank's
 * shard (num_local_experts = E / world, expert_offset = rank E / world). */
int gptoss_ep_dispatch(gptoss_ep* ep, const uint16_t* x, int64_t M, const gptoss_moe_weights* w, void* stream);
/* Combine: the grouped GEMMs on this rank's experts, outputs returned to the
 * tokens' ranks, out [M, H] = x + weighted sum of each token's experts. */
int gptoss_ep_combine(gptoss_ep* ep, const uint16_t* x, int64_t M, const gptoss_moe_weights* w, uint16_t* out,
                      void* stream);
/* gptoss_ep_dispatch then gptoss_ep_combine: MLPBlock.forward (model/mlp.py:371-402). */
int gptoss_ep_forward(gptoss_ep* ep, const uint16_t* x, int64_t M, const gptoss_moe_weights* w, uint16_t* out,
                      void* stream);
/* The group's device error word (bounded-wait expiry, bad routing); synchronises and clears it. */
uint32_t gptoss_ep_error(gptoss_ep* ep);
/* Leaves the group (after every rank's last step has completed). */
void gptoss_ep_destroy(gptoss_ep* ep);

#ifdef __cplusplus
}
#endif

#endif /* GPTOSS_B200_H_ */
