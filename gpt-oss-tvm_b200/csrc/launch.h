// launch.h -- host-side launch helpers shared between the kernel files and the C ABI.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <mutex>

#include "../../include/gptoss_b200.h"

namespace gptoss {

// Ranks of one expert-parallel group whose memory the peer kernels address.
constexpr int kMaxPeerRanks = 8;

// Arguments of one grouped expert GEMM (moe_gemm.cu).
struct GemmLaunch {
  const uint16_t* act;   // [act_rows, K] bf16 or f16, expert-major rows
  int64_t act_rows;
  const uint8_t* blocks;  // [E, N, K/32, 16]
  const uint8_t* scales;  // [E, N, K/32]
  const uint16_t* bias;   // [E, N] bf16
  const int32_t* indptr;
  const int32_t* tile_ptr;
  const int32_t* tile_rows;
  void* out;  // mode 0: [act_rows, N/2] (bf16, or f16 when f16); mode 1: [act_rows, N] f32
  int32_t E, N, K, ldo;
  float alpha, limit;
  uint32_t* err;
  int grid;
  int f16;  // 1: f16 activations and hardware e2m1 -> f16 weight decode
  // mode 1 only, optional: output row r goes to row (row_dst[r] & 0xFFFFFF) of
  // peer_out[row_dst[r] >> 24] (row stride ldo), as bf16 when out_bf16
  const int32_t* row_dst = nullptr;
  void* peer_out[kMaxPeerRanks] = {};
  int64_t peer_out_rows = 0;  // rows of each peer_out buffer; stores beyond it are dropped
  int out_bf16 = 0;
  // optional, decode GEMV only (moe_gemm_gathers): act holds bf16 token rows
  // and activation row r is f16(act[act_gather[r]]) -- the gather into the
  // expert-major rows happens while the GEMV stages its token rows
  const int32_t* act_gather = nullptr;
};
int launch_moe_gemm(int mode, const GemmLaunch& L, cudaStream_t stream);
// Whether launch_moe_gemm takes L to the decode GEMV, the one form that can
// gather its activation rows itself (act_gather).
bool moe_gemm_gathers(const GemmLaunch& L);
// dense.cu: y = x W^T + b for at most dense_gemv_max_tokens() token rows
int dense_gemv_max_tokens();
int launch_dense_gemv(const uint16_t* x, int64_t T, const uint16_t* W, const uint16_t* bias, int32_t N, int32_t K,
                      uint16_t* out, cudaStream_t s);
// router_bf16.cu: router logits on the bf16 FMA pipe, stage-checked against
// the double-rounding case (bit-exact to launch_router's serial fp32 chains)
int launch_router_bf16(const uint16_t* t, const uint16_t* W, const uint16_t* b, int64_t M, int32_t E, int32_t H,
                       uint16_t* logits, uint32_t* err, cudaStream_t s);
// sample.cu: top-p sampling from fp32 logits, one CTA per row
int64_t sample_top_p_scratch_bytes_per_row(int64_t V);
int launch_sample_top_p(const float* logits, int64_t B, int64_t V, double temperature, double top_p,
                        const double* uniform, double uniform0, void* scratch, int64_t scratch_bytes, int32_t* out,
                        cudaStream_t s);
// SM count of the current device (cached per device)
int device_sm_count();

// A kernel's dynamic shared-memory limit, raised on the current device the
// first time a launch needs more than what was set there (function
// attributes are per device; thread-safe; never lowered).
constexpr int kMaxAttrDevices = 64;
struct FuncSmemAttr {
  std::atomic<int> bytes[kMaxAttrDevices] = {};
  std::mutex mu;
};
inline void ensure_dyn_smem(FuncSmemAttr& a, const void* func, int bytes, int carveout = -1) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxAttrDevices) {
    (void)cudaGetLastError();
    dev = 0;
  }
  if (a.bytes[dev].load(std::memory_order_acquire) >= bytes) return;
  std::lock_guard<std::mutex> g(a.mu);
  if (a.bytes[dev].load(std::memory_order_relaxed) >= bytes) return;
  cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (carveout >= 0) cudaFuncSetAttribute(func, cudaFuncAttributePreferredSharedMemoryCarveout, carveout);
  a.bytes[dev].store(bytes, std::memory_order_release);
}
// dense_tc.cu: the same product at any T on the tensor cores
int launch_dense_gemm(const uint16_t* x, int64_t T, const uint16_t* W, const uint16_t* bias, int32_t N, int32_t K,
                      uint16_t* out, uint32_t* err, cudaStream_t s);
// moe_gemv.cu: the decode-size form of the same GEMMs (f16 path, local outputs)
bool moe_gemv_supported(const GemmLaunch& L);
int launch_moe_gemv(int mode, const GemmLaunch& L, cudaStream_t stream);

// Default of the block-scaled decode GEMMs (environment GPTOSS_MOE_MX overrides).
constexpr bool kMoeMxDefault = true;
bool moe_mx_enabled();

// moe_mx.cu: decode-size GEMMs on the block-scaled tensor cores (quantized activations)
bool moe_mx_supported(int64_t act_rows, int32_t E, int32_t N, int32_t K, const void* blocks);
int launch_quantize_mx(const uint16_t* src, int src_f16, const int32_t* idx, int64_t rows, int32_t K, uint8_t* q,
                       uint8_t* sc, cudaStream_t stream);
int launch_moe_gemm_mx(int mode, const GemmLaunch& L, const uint8_t* q, const uint8_t* act_sc, cudaStream_t stream);

// moe_route.cu
int launch_rmsnorm(const uint16_t*, const uint16_t*, int64_t, int32_t, float, uint16_t*, uint32_t*, cudaStream_t);
int launch_router(const uint16_t*, const uint16_t*, const uint16_t*, int64_t, int32_t, int32_t, uint16_t*,
                  uint32_t* err, cudaStream_t);
int launch_topk_softmax(const uint16_t*, int64_t, int32_t, int32_t, uint16_t*, int32_t*, uint32_t*, cudaStream_t);
// top-k + softmax + the permutation in one launch for M * K <= route_small_max_pairs()
int route_small_max_pairs();
int launch_route_small(const uint16_t* logits, int64_t M, int32_t E, int32_t K, uint16_t* weights,
                       int32_t* indices, int32_t* indptr, int32_t* tile_ptr, int32_t* tile_rows,
                       int32_t* token_of_row, int32_t* row_of_pair, int32_t* expert_of_row, uint32_t* err,
                       cudaStream_t s);
int launch_permute(const int32_t*, int64_t, int32_t, int32_t, int32_t*, int32_t*, int32_t*, int32_t*, int32_t*,
                   int32_t*, uint32_t*, cudaStream_t);
int launch_gather(const uint16_t*, const int32_t*, int64_t, int32_t, uint16_t*, int32_t to_f16, cudaStream_t);
int launch_combine(const float*, const int32_t*, const uint16_t*, const uint16_t*, int64_t, int32_t, int32_t,
                   uint16_t*, cudaStream_t);
int launch_mxfp4_dequant(const uint8_t*, const uint8_t*, int64_t, uint16_t*, cudaStream_t);
int launch_plan_tiles(const int32_t*, int32_t, int32_t*, int32_t*, cudaStream_t);
int launch_combine_bf16(const uint16_t* h2, const int32_t* row_of_pair, const uint16_t* w, const uint16_t* x,
                        int64_t M, int32_t K, int32_t H, uint16_t* out, cudaStream_t s);
int launch_segment_copy(const void*, void*, const int32_t*, int32_t, int32_t, int64_t, int32_t, int32_t*,
                        cudaStream_t);
int launch_weight_ranges(const uint8_t* s1, int64_t n1, const uint8_t* s2, int64_t n2, const uint16_t* norm_w,
                         int32_t H, uint32_t* out4, cudaStream_t);

// moe_peer.cu
int launch_peer_layout(const int32_t* counts, int32_t P, int32_t El, int32_t rank, int32_t* dst_base,
                       int32_t* indptr_local, cudaStream_t s);
int launch_dispatch_peer(const uint16_t* t, const int32_t* token_of_row, const int32_t* expert_of_row,
                         const int32_t* indptr, int64_t rows, int32_t H, int32_t E, int32_t El, int32_t rank,
                         const int32_t* dst_base, void* const* peer_rows, int32_t* const* peer_origin,
                         int32_t num_ranks, int64_t cap_rows, int32_t to_f16, cudaStream_t s);
int launch_set_flag(uint32_t* flag, uint32_t value, cudaStream_t s);
int launch_wait_flag(const uint32_t* flag, uint32_t value, uint32_t max_polls, uint32_t* err, cudaStream_t s);

// attention.cu
int launch_qkv_rope(const uint16_t* qkv, const int32_t* pos, const int32_t* slot, int64_t S, int32_t Hq, int32_t Hkv,
                    int32_t D, const float* inv_freq, float conc, uint16_t* q_out, uint16_t* k_cache,
                    uint16_t* v_cache, cudaStream_t s);
int launch_rope(const uint16_t* x, const int32_t* pos, int64_t S, int32_t Hh, int32_t D, const float* inv_freq,
                float conc, uint16_t* out, cudaStream_t s);
int make_tmap_3d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype, const uint64_t dims[3],
                 const uint64_t strides[2], const uint32_t box[3], CUtensorMapSwizzle swz);
int launch_attn_prefill(const uint16_t* q, const uint16_t* k, const uint16_t* v, const uint16_t* sinks, int64_t Sq,
                        int64_t Skv, int32_t Hq, int32_t Hkv, int32_t D, int32_t window, float sm_scale, uint16_t* o,
                        float* lse, cudaStream_t s);
size_t attn_decode_scratch_bytes(int64_t B, int32_t Hq, int64_t max_len, int32_t splits);
int attn_decode_splits(int64_t B, int32_t Hq, int64_t max_len, int32_t window);
int launch_attn_decode(const uint16_t* q, const uint16_t* kc, const uint16_t* vc, const int32_t* kv_len, int64_t B,
                       int64_t max_len, int32_t Hq, int32_t Hkv, int32_t D, int32_t window, float sm_scale,
                       const uint16_t* sinks, float* scratch, uint16_t* o, float* lse, cudaStream_t s,
                       const int32_t* table = nullptr, int32_t tstride = 0);
int launch_kv_rows_copy(uint16_t* pool_k, uint16_t* pool_v, const int32_t* table, int32_t tstride, int32_t seq,
                        int64_t pos0, int64_t n, int32_t row_elems, uint16_t* buf_k, uint16_t* buf_v, int32_t to_pages,
                        cudaStream_t s);
int launch_attn_merge(const uint16_t* o1, const float* l1, const uint16_t* o2, const float* l2, int64_t T, int32_t Hq,
                      int32_t D, uint16_t* o, float* lse, cudaStream_t s);
int launch_sink_rescale(uint16_t* o, const float* lse, const uint16_t* sinks, int64_t T, int32_t Hq, int32_t D,
                        cudaStream_t s);

// capi.cu: the expert part of the MoE block (gather or quantize, both grouped
// GEMMs) on the path the sizes and GPTOSS_MOE_MX select; shared by the
// workspace and the no-allocation forwards
int moe_route(const uint16_t* t, int64_t M, const gptoss_moe_weights* w, uint16_t* logits, uint16_t* topk_w,
              int32_t* topk_idx, int32_t* indptr, int32_t* token_of_row, int32_t* row_of_pair,
              int32_t* expert_of_row, int32_t* tile_ptr, int32_t* tile_rows, uint32_t* err, void* stream);
int moe_experts_forward(const uint16_t* t, int64_t M, const gptoss_moe_weights* w, const int32_t* indptr,
                        const int32_t* tile_ptr, const int32_t* tile_rows, const int32_t* token_of_row, uint16_t* act,
                        uint16_t* y, float* h2, uint8_t* qs, uint32_t* err, void* stream);

// capi.cu: records a message for gptoss_last_error()
int set_last_error(int code, const char* msg);

}  // namespace gptoss
