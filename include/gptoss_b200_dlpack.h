/*
 * gptoss_b200_dlpack.h -- DLTensor entry points of libgptoss_b200.so.
 *
 * The reference runs its kernels through TVM's destination-passing calling
 * convention: nn.tensor_ir_op(prim_func, args=[...], out=placeholder) with
 * the arguments as DLTensors (model/mlp.py:321-326, model/attention.py:218-233).
 * These entry points take the same kind of arguments -- any producer of
 * DLPack tensors (a TVM runtime Tensor, torch, cupy) can call them directly --
 * and check what the plain-pointer entry points of gptoss_b200.h cannot:
 * element type, shape (and agreement between tensors), device (CUDA, the
 * current device) and a dense row-major layout (strides NULL or compact).
 * A mismatch returns -1 with a message in gptoss_last_error(); nothing is
 * launched.  Device pointers are data + byte_offset.
 */
#ifndef GPTOSS_B200_DLPACK_H_
#define GPTOSS_B200_DLPACK_H_

#include <dlpack/dlpack.h>

#include "gptoss_b200.h"

#ifdef __cplusplus
extern "C" {
#endif

/* MLPBlock parameters (model/mlp.py:81-143) from DLTensors into `w`, checked:
 * norm_weight [H], gate_weight [E, H], gate_bias [E] bf16; mlp1_blocks
 * [El, 2I, H/32, 16] u8, mlp1_scales [El, 2I, H/32] u8, mlp1_bias [El, 2I]
 * bf16; mlp2_blocks [El, H, I/32, 16] u8, mlp2_scales [El, H, I/32] u8,
 * mlp2_bias [El, H] bf16 (El = E unless expert_offset / a shard is given:
 * experts [expert_offset, expert_offset + El)).  Runs
 * gptoss_moe_weights_prepare (synchronises `stream`).  SwiGLU alpha 1.702. */
int gptoss_moe_weights_init_dl(gptoss_moe_weights* w, const DLTensor* norm_weight, const DLTensor* gate_weight,
                               const DLTensor* gate_bias, const DLTensor* mlp1_blocks, const DLTensor* mlp1_scales,
                               const DLTensor* mlp1_bias, const DLTensor* mlp2_blocks, const DLTensor* mlp2_scales,
                               const DLTensor* mlp2_bias, int32_t top_k, float swiglu_limit, float rms_eps,
                               int32_t expert_offset, void* stream);

/* MLPBlock.forward (model/mlp.py:371-402): x [..., H] bf16 (any leading
 * shape, e.g. [b, s, H]) -> out of the same shape, x + MoE(RMSNorm(x)). */
int gptoss_moe_forward_dl(const DLTensor* x, const gptoss_moe_weights* w, gptoss_moe_workspace* ws, DLTensor* out,
                          void* stream);

/* paged_kv_cache.self_attention + sink rescale (model/attention.py:218-247):
 * q [Sq, Hq, 64], k / v [Skv, Hkv, 64] bf16 (a leading batch dimension of 1 is
 * accepted), sinks [Hq] bf16 or NULL, o like q, lse [Sq, Hq] fp32 or NULL. */
int gptoss_attn_prefill_dl(const DLTensor* q, const DLTensor* k, const DLTensor* v, const DLTensor* sinks,
                           int32_t window, float sm_scale, DLTensor* o, DLTensor* lse, void* stream);

/* paged_kv_cache.cross_attention for one new token per sequence + sink
 * rescale (model/attention.py:221-224): q [B, Hq, 64], caches [B, max_len,
 * Hkv, 64] bf16, kv_len [B] int32, scratch float32 of at least
 * gptoss_attn_decode_scratch_bytes() bytes, o like q, lse [B, Hq] fp32 or NULL. */
int gptoss_attn_decode_dl(const DLTensor* q, const DLTensor* k_cache, const DLTensor* v_cache, const DLTensor* kv_len,
                          int32_t window, float sm_scale, const DLTensor* sinks, DLTensor* scratch, DLTensor* o,
                          DLTensor* lse, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* GPTOSS_B200_DLPACK_H_ */
