// capi.cu -- the extern "C" boundary of libgptoss_b200.so (see include/gptoss_b200.h).
#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <string>

#include "../../include/gptoss_b200.h"
#include "common.cuh"

#include "launch.h"

using namespace gptoss;

static thread_local std::string g_last_error;

static int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

namespace gptoss {
// Records a message for gptoss_last_error() (used by entry points defined in other files).
int set_last_error(int code, const char* msg) { return fail(code, "%s", msg); }
}  // namespace gptoss

static int check_launch(int rc, const char* what) {
  if (rc == 0) return 0;
  cudaError_t e = cudaGetLastError();
  return fail(rc < 0 ? rc : -3, "%s failed (code %d, cuda: %s)", what, rc, cudaGetErrorString(e));
}

// SM count of the current device, cached per device (atomics: host threads
// may make their first calls at the same time; they store the same value).
static int num_sms() {
  constexpr int kMaxDev = 64;
  static std::atomic<int> cached[kMaxDev];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDev) {
    (void)cudaGetLastError();
    return 148;
  }
  int n = cached[dev].load(std::memory_order_relaxed);
  if (n <= 0) {
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) {
      (void)cudaGetLastError();
      n = 148;
    }
    cached[dev].store(n, std::memory_order_relaxed);
  }
  return n;
}

namespace gptoss {
int device_sm_count() { return num_sms(); }
}  // namespace gptoss

#define GPTOSS_STREAM(s) ((cudaStream_t)(s))

extern "C" {

int gptoss_version(void) { return 1; }
const char* gptoss_last_error(void) { return g_last_error.c_str(); }

// ---------------------------------------------------------------- pieces --
int gptoss_rms_norm(const uint16_t* x, const uint16_t* weight, int64_t M, int32_t H, float eps, uint16_t* out,
                    void* stream) {
  if (M < 0 || H <= 0 || (H & 1)) return fail(-1, "gptoss_rms_norm: bad shape M=%lld H=%d", (long long)M, H);
  if (M && (!x || !weight || !out)) return fail(-1, "gptoss_rms_norm: null pointer");
  return check_launch(launch_rmsnorm(x, weight, M, H, eps, out, nullptr, GPTOSS_STREAM(stream)), "rms_norm");
}

int gptoss_moe_router(const uint16_t* t, const uint16_t* gate_weight, const uint16_t* gate_bias, int64_t M,
                      int32_t E, int32_t H, int32_t K, uint16_t* logits, uint16_t* topk_weights,
                      int32_t* topk_indices, uint32_t* err, void* stream) {
  if (M < 0 || E <= 0 || E > 256 || E % 8 || K < 1 || K > 8 || K > E || H <= 0)
    return fail(-1, "gptoss_moe_router: unsupported shape M=%lld E=%d H=%d K=%d (E must be a multiple of 8, <= 256)",
                (long long)M, E, H, K);
  int rc = launch_router(t, gate_weight, gate_bias, M, E, H, logits, err, GPTOSS_STREAM(stream));
  if (rc) return check_launch(rc, "router");
  return check_launch(launch_topk_softmax(logits, M, E, K, topk_weights, topk_indices, err, GPTOSS_STREAM(stream)),
                      "topk_softmax");
}

int gptoss_moe_topk_softmax(const uint16_t* logits, int64_t M, int32_t E, int32_t K, uint16_t* topk_weights,
                            int32_t* topk_indices, uint32_t* err, void* stream) {
  if (M < 0 || E <= 0 || E > 256 || K < 1 || K > 8 || K > E)
    return fail(-1, "gptoss_moe_topk_softmax: unsupported shape M=%lld E=%d K=%d", (long long)M, E, K);
  return check_launch(launch_topk_softmax(logits, M, E, K, topk_weights, topk_indices, err, GPTOSS_STREAM(stream)),
                      "topk_softmax");
}

int gptoss_moe_permute(const int32_t* topk_indices, int64_t M, int32_t K, int32_t E, int32_t* indptr,
                       int32_t* token_of_row, int32_t* row_of_pair, int32_t* expert_of_row, int32_t* tile_ptr,
                       int32_t* tile_rows, uint32_t* err, void* stream) {
  if (M < 0 || K < 1 || E < 1 || E > 4096) return fail(-1, "gptoss_moe_permute: bad shape");
  return check_launch(launch_permute(topk_indices, M, K, E, indptr, tile_ptr, tile_rows, token_of_row, row_of_pair,
                                     expert_of_row, err, GPTOSS_STREAM(stream)),
                      "permute");
}

int gptoss_moe_gather(const uint16_t* t, const int32_t* token_of_row, int64_t rows, int32_t H, int32_t act_f16,
                      uint16_t* act, void* stream) {
  if (rows < 0 || H <= 0 || H % 8) return fail(-1, "gptoss_moe_gather: H must be a multiple of 8");
  return check_launch(launch_gather(t, token_of_row, rows, H, act, act_f16, GPTOSS_STREAM(stream)), "gather");
}

static int gemm_common(int mode, const uint16_t* act, int64_t act_rows, const int32_t* indptr,
                       const int32_t* tile_ptr, const int32_t* tile_rows, int32_t E, int32_t N, int32_t K,
                       const uint8_t* blocks, const uint8_t* scales, const uint16_t* bias, float alpha, float limit,
                       void* out, int32_t ldo, int32_t act_f16, uint32_t* err, void* stream) {
  if (act_rows <= 0) return 0;
  if (E <= 0 || N <= 0 || K <= 0 || K % 64)
    return fail(-1, "moe gemm: K must be a positive multiple of 64 (got %d)", K);
  if (((uintptr_t)act & 15) || ((uintptr_t)blocks & 15) || ((uintptr_t)scales & 15))
    return fail(-1, "moe gemm: act, blocks and scales must be 16-byte aligned");
  GemmLaunch L;
  L.act = act;
  L.act_rows = act_rows;
  L.blocks = blocks;
  L.scales = scales;
  L.bias = bias;
  L.indptr = indptr;
  L.tile_ptr = tile_ptr;
  L.tile_rows = tile_rows;
  L.out = out;
  L.E = E;
  L.N = N;
  L.K = K;
  L.ldo = ldo;
  L.alpha = alpha;
  L.limit = limit;
  L.err = err;
  L.grid = num_sms();
  L.f16 = act_f16 ? 1 : 0;
  return check_launch(launch_moe_gemm(mode, L, GPTOSS_STREAM(stream)), mode == 0 ? "moe_mlp1" : "moe_mlp2");
}

int gptoss_moe_mlp1(const uint16_t* act, int64_t act_rows, const int32_t* indptr, const int32_t* tile_ptr,
                    const int32_t* tile_rows, int32_t E, int32_t H, int32_t I, const uint8_t* blocks,
                    const uint8_t* scales, const uint16_t* bias, float alpha, float limit, int32_t act_f16,
                    uint16_t* y, uint32_t* err, void* stream) {
  return gemm_common(0, act, act_rows, indptr, tile_ptr, tile_rows, E, 2 * I, H, blocks, scales, bias, alpha, limit,
                     y, I, act_f16, err, stream);
}

int gptoss_moe_mlp2(const uint16_t* y, int64_t act_rows, const int32_t* indptr, const int32_t* tile_ptr,
                    const int32_t* tile_rows, int32_t E, int32_t H, int32_t I, const uint8_t* blocks,
                    const uint8_t* scales, const uint16_t* bias, int32_t act_f16, float* h2, uint32_t* err,
                    void* stream) {
  return gemm_common(1, y, act_rows, indptr, tile_ptr, tile_rows, E, H, I, blocks, scales, bias, 0.f, 0.f, h2, H,
                     act_f16, err, stream);
}

int gptoss_moe_quantize_mx(const uint16_t* src, int32_t src_f16, const int32_t* row_index, int64_t rows,
                           int32_t K, uint8_t* q, uint8_t* scales, void* stream) {
  if (rows < 0 || K <= 0 || K % 32 || K > 3072)
    return fail(-1, "gptoss_moe_quantize_mx: K must be a positive multiple of 32 up to 3072 (got %d)", K);
  if (rows && (!src || !q || !scales)) return fail(-1, "gptoss_moe_quantize_mx: null pointer");
  if (((uintptr_t)src & 15) || ((uintptr_t)q & 15))
    return fail(-1, "gptoss_moe_quantize_mx: src and q must be 16-byte aligned");
  return check_launch(launch_quantize_mx(src, src_f16, row_index, rows, K, q, scales, GPTOSS_STREAM(stream)),
                      "moe_quantize_mx");
}

static int gemm_mx_common(int mode, const uint8_t* q, const uint8_t* act_scales, int64_t act_rows,
                          const int32_t* indptr, const int32_t* tile_ptr, const int32_t* tile_rows, int32_t E,
                          int32_t N, int32_t K, const uint8_t* blocks, const uint8_t* scales, const uint16_t* bias,
                          float alpha, float limit, void* out, int32_t ldo, uint32_t* err, void* stream) {
  if (act_rows <= 0) return 0;
  if (!moe_mx_supported(act_rows, E, N, K, blocks))
    return fail(-1,
                "moe gemm (block-scaled): needs decode-size tiles (rows <= 8 x experts), K a multiple of 64 in "
                "256..3072, 32-byte aligned blocks (rows=%lld E=%d N=%d K=%d)",
                (long long)act_rows, E, N, K);
  if (((uintptr_t)q & 15) || ((uintptr_t)act_scales & 15) || ((uintptr_t)scales & 15))
    return fail(-1, "moe gemm (block-scaled): q, act_scales and scales must be 16-byte aligned");
  GemmLaunch L;
  L.act = nullptr;
  L.act_rows = act_rows;
  L.blocks = blocks;
  L.scales = scales;
  L.bias = bias;
  L.indptr = indptr;
  L.tile_ptr = tile_ptr;
  L.tile_rows = tile_rows;
  L.out = out;
  L.E = E;
  L.N = N;
  L.K = K;
  L.ldo = ldo;
  L.alpha = alpha;
  L.limit = limit;
  L.err = err;
  L.grid = num_sms();
  L.f16 = 1;
  return check_launch(launch_moe_gemm_mx(mode, L, q, act_scales, GPTOSS_STREAM(stream)),
                      mode == 0 ? "moe_mlp1_mx" : "moe_mlp2_mx");
}

int gptoss_moe_mlp1_mx(const uint8_t* q, const uint8_t* act_scales, int64_t act_rows, const int32_t* indptr,
                       const int32_t* tile_ptr, const int32_t* tile_rows, int32_t E, int32_t H, int32_t I,
                       const uint8_t* blocks, const uint8_t* scales, const uint16_t* bias, float alpha, float limit,
                       uint16_t* y, uint32_t* err, void* stream) {
  return gemm_mx_common(0, q, act_scales, act_rows, indptr, tile_ptr, tile_rows, E, 2 * I, H, blocks, scales, bias,
                        alpha, limit, y, I, err, stream);
}

int gptoss_moe_mlp2_mx(const uint8_t* q, const uint8_t* act_scales, int64_t act_rows, const int32_t* indptr,
                       const int32_t* tile_ptr, const int32_t* tile_rows, int32_t E, int32_t H, int32_t I,
                       const uint8_t* blocks, const uint8_t* scales, const uint16_t* bias, float* h2, uint32_t* err,
                       void* stream) {
  return gemm_mx_common(1, q, act_scales, act_rows, indptr, tile_ptr, tile_rows, E, H, I, blocks, scales, bias, 0.f,
                        0.f, h2, H, err, stream);
}

int gptoss_moe_mlp2_peer(const uint16_t* y, int64_t act_rows, const int32_t* indptr, const int32_t* tile_ptr,
                         const int32_t* tile_rows, int32_t E, int32_t H, int32_t I, const uint8_t* blocks,
                         const uint8_t* scales, const uint16_t* bias, int32_t act_f16, const int32_t* origin,
                         void* const* peer_back, int32_t num_ranks, int64_t back_rows, int32_t back_bf16,
                         uint32_t* err, void* stream) {
  if (act_rows <= 0) return 0;
  if (!origin || !peer_back || num_ranks < 1 || num_ranks > kMaxPeerRanks)
    return fail(-1, "moe_mlp2_peer: origin, peer_back and 1 <= num_ranks <= %d required", kMaxPeerRanks);
  if (E <= 0 || H <= 0 || I <= 0 || I % 64)
    return fail(-1, "moe_mlp2_peer: I must be a positive multiple of 64 (got %d)", I);
  if (((uintptr_t)y & 15) || ((uintptr_t)blocks & 15) || ((uintptr_t)scales & 15))
    return fail(-1, "moe_mlp2_peer: y, blocks and scales must be 16-byte aligned");
  GemmLaunch L;
  L.act = y;
  L.act_rows = act_rows;
  L.blocks = blocks;
  L.scales = scales;
  L.bias = bias;
  L.indptr = indptr;
  L.tile_ptr = tile_ptr;
  L.tile_rows = tile_rows;
  L.out = nullptr;
  L.E = E;
  L.N = H;
  L.K = I;
  L.ldo = H;
  L.alpha = 0.f;
  L.limit = 0.f;
  L.err = err;
  L.grid = num_sms();
  L.f16 = act_f16 ? 1 : 0;
  L.row_dst = origin;
  for (int i = 0; i < num_ranks; ++i) L.peer_out[i] = peer_back[i];
  L.peer_out_rows = back_rows;
  L.out_bf16 = back_bf16 ? 1 : 0;
  return check_launch(launch_moe_gemm(1, L, GPTOSS_STREAM(stream)), "moe_mlp2_peer");
}

int gptoss_moe_peer_layout(const int32_t* counts_all, int32_t num_ranks, int32_t local_experts, int32_t rank,
                           int32_t* dst_base, int32_t* indptr_local, void* stream) {
  return check_launch(launch_peer_layout(counts_all, num_ranks, local_experts, rank, dst_base, indptr_local,
                                         GPTOSS_STREAM(stream)),
                      "moe_peer_layout");
}

int gptoss_moe_dispatch_peer(const uint16_t* t, const int32_t* token_of_row, const int32_t* expert_of_row,
                             const int32_t* indptr, int64_t rows, int32_t H, int32_t num_experts,
                             int32_t local_experts, int32_t rank, const int32_t* dst_base, void* const* peer_rows,
                             int32_t* const* peer_origin, int32_t num_ranks, int64_t cap_rows, int32_t to_f16,
                             void* stream) {
  if (rows > 0 && (!peer_rows || !peer_origin || !dst_base))
    return fail(-1, "moe_dispatch_peer: peer_rows, peer_origin and dst_base required");
  return check_launch(launch_dispatch_peer(t, token_of_row, expert_of_row, indptr, rows, H, num_experts,
                                           local_experts, rank, dst_base, peer_rows, peer_origin, num_ranks,
                                           cap_rows, to_f16, GPTOSS_STREAM(stream)),
                      "moe_dispatch_peer");
}

int gptoss_stream_set_flag(uint32_t* flag, uint32_t value, void* stream) {
  if (!flag || ((uintptr_t)flag & 3)) return fail(-1, "gptoss_stream_set_flag: flag must be a 4-byte aligned device word");
  return check_launch(launch_set_flag(flag, value, GPTOSS_STREAM(stream)), "stream_set_flag");
}

int gptoss_stream_wait_flag(const uint32_t* flag, uint32_t value, uint32_t max_polls, uint32_t* err, void* stream) {
  if (!flag || ((uintptr_t)flag & 3)) return fail(-1, "gptoss_stream_wait_flag: flag must be a 4-byte aligned device word");
  if (max_polls == 0 || max_polls > (1u << 26))
    return fail(-1, "gptoss_stream_wait_flag: max_polls must be 1..2^26 (got %u)", max_polls);
  return check_launch(launch_wait_flag(flag, value, max_polls, err, GPTOSS_STREAM(stream)), "stream_wait_flag");
}

int gptoss_ipc_alloc(uint64_t bytes, void** ptr, void* handle) {
  if (!ptr || !handle || bytes == 0) return fail(-1, "ipc_alloc: null output or zero size");
  *ptr = nullptr;
  if (cudaMalloc(ptr, bytes) != cudaSuccess) {
    cudaGetLastError();
    return fail(-4, "ipc_alloc: cudaMalloc(%llu) failed", (unsigned long long)bytes);
  }
  // zero-filled: an origin word never written decodes to a valid (rank 0, row 0)
  if (cudaMemset(*ptr, 0, bytes) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess) {
    cudaGetLastError();
    cudaFree(*ptr);
    *ptr = nullptr;
    return fail(-4, "ipc_alloc: cudaMemset failed");
  }
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, *ptr) != cudaSuccess) {
    cudaGetLastError();
    cudaFree(*ptr);
    *ptr = nullptr;
    return fail(-4, "ipc_alloc: cudaIpcGetMemHandle failed");
  }
  static_assert(sizeof(h) == 64, "IPC handle size");
  memcpy(handle, &h, sizeof(h));
  return 0;
}

int gptoss_ipc_open(const void* handle, void** ptr) {
  if (!ptr || !handle) return fail(-1, "ipc_open: null handle or output");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  *ptr = nullptr;
  if (cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
    const cudaError_t e = cudaGetLastError();
    return fail(-4, "ipc_open: cudaIpcOpenMemHandle failed (%s)", cudaGetErrorString(e));
  }
  return 0;
}

int gptoss_ipc_close(void* ptr) {
  if (ptr && cudaIpcCloseMemHandle(ptr) != cudaSuccess) {
    cudaGetLastError();
    return fail(-4, "ipc_close: cudaIpcCloseMemHandle failed");
  }
  return 0;
}

int gptoss_ipc_free(void* ptr) {
  if (ptr && cudaFree(ptr) != cudaSuccess) {
    cudaGetLastError();
    return fail(-4, "ipc_free: cudaFree failed");
  }
  return 0;
}

int gptoss_moe_weights_prepare(gptoss_moe_weights* w, void* stream) {
  if (!w) return fail(-1, "gptoss_moe_weights_prepare: null weights");
  const int64_t El = w->num_local_experts;
  const int64_t n1 = El * 2 * w->intermediate * (w->hidden / 32);
  const int64_t n2 = El * w->hidden * (w->intermediate / 32);
  uint32_t* d = nullptr;
  if (cudaMalloc(&d, 16) != cudaSuccess) {
    cudaGetLastError();
    return fail(-4, "gptoss_moe_weights_prepare: cudaMalloc failed");
  }
  const uint32_t init[4] = {255u, 0u, 0u, 0u};
  cudaStream_t s = GPTOSS_STREAM(stream);
  cudaMemcpyAsync(d, init, 16, cudaMemcpyHostToDevice, s);
  int rc = launch_weight_ranges(w->mlp1_scales, n1, w->mlp2_scales, n2, w->norm_weight, w->hidden, d, s);
  uint32_t h[4] = {0, 0, 0, 0};
  if (rc == 0) cudaMemcpyAsync(h, d, 16, cudaMemcpyDeviceToHost, s);
  cudaStreamSynchronize(s);
  cudaFree(d);
  if (rc) return check_launch(rc, "weights_prepare");
  float max_norm;
  memcpy(&max_norm, &h[2], 4);
  // f16 path: every e2m1 x 2^(s-127) is an exact f16 for s in 104..140, and the
  // RMSNorm output stays below sqrt(H) * max|norm weight| < 32768
  const bool f16_ok = h[0] >= 104u && h[1] <= 140u && max_norm * sqrtf((float)w->hidden) < 32768.0f;
  w->flags = (w->flags & ~(uint32_t)GPTOSS_MOE_F16) | (f16_ok ? (uint32_t)GPTOSS_MOE_F16 : 0u);
  return 0;
}

int gptoss_moe_combine(const float* h2, const int32_t* row_of_pair, const uint16_t* topk_weights,
                       const uint16_t* x, int64_t M, int32_t K, int32_t H, uint16_t* out, void* stream) {
  if (M < 0 || K < 1 || K > 8 || H <= 0 || H % 4) return fail(-1, "gptoss_moe_combine: bad shape");
  return check_launch(launch_combine(h2, row_of_pair, topk_weights, x, M, K, H, out, GPTOSS_STREAM(stream)),
                      "combine");
}

int gptoss_moe_combine_bf16(const uint16_t* h2, const int32_t* row_of_pair, const uint16_t* topk_weights,
                            const uint16_t* x, int64_t M, int32_t K, int32_t H, uint16_t* out, void* stream) {
  if (M < 0 || K < 1 || K > 8 || H <= 0 || H % 4) return fail(-1, "gptoss_moe_combine_bf16: bad shape");
  return check_launch(launch_combine_bf16(h2, row_of_pair, topk_weights, x, M, K, H, out, GPTOSS_STREAM(stream)),
                      "combine_bf16");
}

int gptoss_mxfp4_dequant(const uint8_t* blocks, const uint8_t* scales, int64_t rows, int32_t groups,
                         uint16_t* out, void* stream) {
  if (rows < 0 || groups <= 0) return fail(-1, "gptoss_mxfp4_dequant: bad shape");
  if (((uintptr_t)blocks & 15) || ((uintptr_t)out & 15)) return fail(-1, "gptoss_mxfp4_dequant: 16-byte alignment");
  return check_launch(launch_mxfp4_dequant(blocks, scales, rows * (int64_t)groups, out, GPTOSS_STREAM(stream)),
                      "mxfp4_dequant");
}

int gptoss_moe_plan_tiles(const int32_t* indptr, int32_t E, int32_t* tile_ptr, int32_t* tile_rows, void* stream) {
  if (E <= 0) return fail(-1, "gptoss_moe_plan_tiles: bad E");
  return check_launch(launch_plan_tiles(indptr, E, tile_ptr, tile_rows, GPTOSS_STREAM(stream)), "plan_tiles");
}

int gptoss_moe_segment_copy(const void* src, void* dst, const int32_t* counts, int32_t num_ranks,
                            int32_t local_experts, int64_t row_bytes, int32_t direction, int32_t* indptr_local,
                            void* stream) {
  if (num_ranks <= 0 || local_experts <= 0 || row_bytes <= 0 || row_bytes % 16 || direction < 0 || direction > 2)
    return fail(-1, "gptoss_moe_segment_copy: bad arguments");
  if (local_experts + 1 > 256 && indptr_local) return fail(-1, "gptoss_moe_segment_copy: at most 255 local experts");
  return check_launch(launch_segment_copy(src, dst, counts, num_ranks, local_experts, row_bytes, direction,
                                          indptr_local, GPTOSS_STREAM(stream)),
                      "segment_copy");
}

// -------------------------------------------------------------- attention --
int gptoss_yarn_inv_freq(int32_t D, float theta, float factor, float beta_fast, float beta_slow,
                         int32_t original_max_position, float* inv_freq, float* concentration) {
  if (D <= 0 || D % 2 || D > 256 || !inv_freq) return fail(-1, "gptoss_yarn_inv_freq: bad arguments");
  // correction range in double precision (model/attention.py:15-36), then the
  // per-dimension blend in fp32 (attention.py:39-61)
  const double pi = 3.14159265358979323846;
  auto corr_dim = [&](double rot) {
    return (D * std::log((double)original_max_position / (rot * 2 * pi))) / (2 * std::log((double)theta));
  };
  double low = std::max(corr_dim(beta_fast), 0.0);
  double high = std::min(corr_dim(beta_slow), (double)(D - 1));
  if (low == high) high += 0.001;
  const float lo_f = (float)low, hmlo_f = (float)(high - low);
  for (int32_t f = 0; f < D / 2; ++f) {
    const float e = (float)(f * 2 % D) / (float)D;
    const float fp = powf(theta, e);
    const float extra = 1.0f / fp;
    const float inter = 1.0f / (factor * fp);
    float v = ((float)f - lo_f) / hmlo_f;
    v = v < 1.0f ? v : 1.0f;
    const float ramp = 1.0f - (v > 0.0f ? v : 0.0f);
    inv_freq[f] = inter * (1.0f - ramp) + extra * ramp;
  }
  if (concentration) concentration[0] = factor > 1.0f ? (float)(0.1 * std::log((double)factor) + 1.0) : 1.0f;
  return 0;
}

int gptoss_rope_yarn(const uint16_t* x, const int32_t* positions, int64_t S, int32_t heads, int32_t D,
                     const float* inv_freq, float concentration, uint16_t* out, void* stream) {
  if (S < 0 || heads <= 0 || D <= 0 || D % 2 || D > 256 || !inv_freq) return fail(-1, "gptoss_rope_yarn: bad shape");
  return check_launch(launch_rope(x, positions, S, heads, D, inv_freq, concentration, out, GPTOSS_STREAM(stream)),
                      "rope_yarn");
}

int gptoss_qkv_rope_append(const uint16_t* qkv, const int32_t* positions, const int32_t* slots, int64_t S,
                           int32_t Hq, int32_t Hkv, int32_t D, const float* inv_freq, float concentration,
                           uint16_t* q_out, uint16_t* k_cache, uint16_t* v_cache, void* stream) {
  if (S < 0 || Hq <= 0 || Hkv <= 0 || D <= 0 || D % 2 || D > 256 || !inv_freq)
    return fail(-1, "gptoss_qkv_rope_append: bad shape");
  return check_launch(launch_qkv_rope(qkv, positions, slots, S, Hq, Hkv, D, inv_freq, concentration, q_out, k_cache,
                                      v_cache, GPTOSS_STREAM(stream)),
                      "qkv_rope_append");
}

int gptoss_attn_prefill(const uint16_t* q, const uint16_t* k, const uint16_t* v, const uint16_t* sinks, int64_t Sq,
                        int64_t Skv, int32_t Hq, int32_t Hkv, int32_t D, int32_t window, float sm_scale, uint16_t* o,
                        float* lse, void* stream) {
  if (D != 64) return fail(-1, "gptoss_attn_prefill: head_dim must be 64");
  if (Sq < 0 || Skv < Sq || Hq <= 0 || Hkv <= 0 || Hq % Hkv)
    return fail(-1, "gptoss_attn_prefill: need 0 <= Sq <= Skv and Hq a multiple of Hkv");
  return check_launch(launch_attn_prefill(q, k, v, sinks, Sq, Skv, Hq, Hkv, D, window, sm_scale, o, lse,
                                          GPTOSS_STREAM(stream)),
                      "attn_prefill");
}

int64_t gptoss_attn_decode_scratch_bytes(int64_t B, int32_t Hq, int64_t max_len, int32_t window) {
  return (int64_t)attn_decode_scratch_bytes(B, Hq, max_len, attn_decode_splits(B, Hq, max_len, window));
}

int gptoss_attn_decode(const uint16_t* q, const uint16_t* k_cache, const uint16_t* v_cache, const int32_t* kv_len,
                       int64_t B, int64_t max_len, int32_t Hq, int32_t Hkv, int32_t D, int32_t window,
                       float sm_scale, const uint16_t* sinks, float* scratch, int64_t scratch_bytes, uint16_t* o,
                       float* lse, void* stream) {
  if (D != 64) return fail(-1, "gptoss_attn_decode: head_dim must be 64");
  if (B < 0 || max_len <= 0 || Hq <= 0 || Hkv <= 0 || Hq % Hkv || Hq / Hkv > 8)
    return fail(-1, "gptoss_attn_decode: bad shape (Hq/Hkv must be <= 8)");
  if (scratch_bytes < gptoss_attn_decode_scratch_bytes(B, Hq, max_len, window))
    return fail(-1, "gptoss_attn_decode: scratch smaller than gptoss_attn_decode_scratch_bytes()");
  return check_launch(launch_attn_decode(q, k_cache, v_cache, kv_len, B, max_len, Hq, Hkv, D, window, sm_scale, sinks,
                                         scratch, o, lse, GPTOSS_STREAM(stream)),
                      "attn_decode");
}

int gptoss_attn_decode_paged(const uint16_t* q, const uint16_t* k_pages, const uint16_t* v_pages,
                             const int32_t* page_table, int32_t table_stride, const int32_t* kv_len, int64_t B,
                             int32_t Hq, int32_t Hkv, int32_t D, int32_t window, float sm_scale, const uint16_t* sinks,
                             float* scratch, int64_t scratch_bytes, uint16_t* o, float* lse, void* stream) {
  if (D != 64) return fail(-1, "gptoss_attn_decode_paged: head_dim must be 64");
  if (B < 0 || Hq <= 0 || Hkv <= 0 || Hq % Hkv || Hq / Hkv > 8 || table_stride <= 0)
    return fail(-1, "gptoss_attn_decode_paged: bad shape (Hq/Hkv must be <= 8, table_stride > 0)");
  if (B > 0 && !page_table) return fail(-1, "gptoss_attn_decode_paged: page_table is required");
  const int64_t max_len = (int64_t)table_stride * 16;
  if (scratch_bytes < gptoss_attn_decode_scratch_bytes(B, Hq, max_len, window))
    return fail(-1, "gptoss_attn_decode_paged: scratch smaller than gptoss_attn_decode_scratch_bytes(B, Hq, "
                    "16 * table_stride, window)");
  return check_launch(launch_attn_decode(q, k_pages, v_pages, kv_len, B, max_len, Hq, Hkv, D, window, sm_scale, sinks,
                                         scratch, o, lse, GPTOSS_STREAM(stream), page_table, table_stride),
                      "attn_decode_paged");
}

int gptoss_kv_pages_copy(uint16_t* k_pages, uint16_t* v_pages, int32_t Hkv, int32_t D, const int32_t* page_table,
                         int32_t table_stride, int32_t seq, int64_t pos0, int64_t n, uint16_t* k_rows,
                         uint16_t* v_rows, int32_t to_pages, void* stream) {
  if (n < 0 || pos0 < 0 || seq < 0 || Hkv <= 0 || D <= 0 || (Hkv * D) % 8 || table_stride <= 0)
    return fail(-1, "gptoss_kv_pages_copy: bad arguments");
  if (n > 0 && (!page_table || !k_pages || !v_pages || !k_rows || !v_rows))
    return fail(-1, "gptoss_kv_pages_copy: null pointer");
  return check_launch(launch_kv_rows_copy(k_pages, v_pages, page_table, table_stride, seq, pos0, n, Hkv * D, k_rows,
                                          v_rows, to_pages, GPTOSS_STREAM(stream)),
                      "kv_pages_copy");
}

int gptoss_attn_merge(const uint16_t* o1, const float* lse1, const uint16_t* o2, const float* lse2, int64_t T,
                      int32_t Hq, int32_t D, uint16_t* o, float* lse, void* stream) {
  if (T < 0 || Hq <= 0 || D <= 0) return fail(-1, "gptoss_attn_merge: bad shape");
  return check_launch(launch_attn_merge(o1, lse1, o2, lse2, T, Hq, D, o, lse, GPTOSS_STREAM(stream)), "attn_merge");
}

int gptoss_attn_sink_rescale(uint16_t* o, const float* lse, const uint16_t* sinks, int64_t T, int32_t Hq, int32_t D,
                             void* stream) {
  if (T < 0 || Hq <= 0 || D <= 0) return fail(-1, "gptoss_attn_sink_rescale: bad shape");
  return check_launch(launch_sink_rescale(o, lse, sinks, T, Hq, D, GPTOSS_STREAM(stream)), "sink_rescale");
}

int gptoss_dense_gemv_max_tokens(void) { return dense_gemv_max_tokens(); }

int gptoss_dense_gemv(const uint16_t* x, int64_t T, const uint16_t* weight, const uint16_t* bias, int32_t N,
                      int32_t K, uint16_t* out, void* stream) {
  if (T < 0 || T > dense_gemv_max_tokens() || N <= 0 || K <= 0 || K % 8 || K > 8192)
    return fail(-1, "gptoss_dense_gemv: T must be 0..%d, K a multiple of 8 up to 8192 (T=%lld N=%d K=%d)",
                dense_gemv_max_tokens(), (long long)T, N, K);
  if (((uintptr_t)weight & 15)) return fail(-1, "gptoss_dense_gemv: weight must be 16-byte aligned");
  return check_launch(launch_dense_gemv(x, T, weight, bias, N, K, out, GPTOSS_STREAM(stream)), "dense_gemv");
}

int64_t gptoss_sample_top_p_scratch_bytes(int64_t B, int64_t V) {
  return (B > 0 && V > 0) ? B * sample_top_p_scratch_bytes_per_row(V) : 0;
}

int gptoss_sample_top_p_from_logits(const float* logits, int64_t B, int64_t V, double temperature, double top_p,
                                    const double* uniform, double uniform0, void* scratch, int64_t scratch_bytes,
                                    int32_t* tokens, void* stream) {
  if (B < 0 || V <= 0 || V > 0x7FFFFFFF || !(top_p > 0.0) || top_p > 1.0)
    return fail(-1, "gptoss_sample_top_p_from_logits: need B >= 0, 0 < V < 2^31, 0 < top_p <= 1 (B=%lld V=%lld top_p=%g)",
                (long long)B, (long long)V, top_p);
  if (!uniform && !(uniform0 >= 0.0 && uniform0 < 1.0))
    return fail(-1, "gptoss_sample_top_p_from_logits: the uniform draw must be in [0, 1) (got %g)", uniform0);
  if (B && (!logits || !tokens)) return fail(-1, "gptoss_sample_top_p_from_logits: null pointer");
  if (B && temperature >= 1e-6 && (!scratch || scratch_bytes < sample_top_p_scratch_bytes_per_row(V)))
    return fail(-1, "gptoss_sample_top_p_from_logits: scratch of at least %lld bytes (one row) is required",
                (long long)sample_top_p_scratch_bytes_per_row(V));
  return check_launch(launch_sample_top_p(logits, B, V, temperature, top_p, uniform, uniform0, scratch,
                                          scratch_bytes, tokens, GPTOSS_STREAM(stream)),
                      "sample_top_p");
}

int gptoss_dense_gemm(const uint16_t* x, int64_t T, const uint16_t* weight, const uint16_t* bias, int32_t N,
                      int32_t K, uint16_t* out, uint32_t* err, void* stream) {
  if (T < 0 || T > 0x7FFFFFFF || N <= 0 || K <= 0 || K % 8)
    return fail(-1, "gptoss_dense_gemm: T must be >= 0, N > 0, K a positive multiple of 8 (T=%lld N=%d K=%d)",
                (long long)T, N, K);
  if (((uintptr_t)x & 15) || ((uintptr_t)weight & 15) || ((uintptr_t)out & 15))
    return fail(-1, "gptoss_dense_gemm: x, weight and out must be 16-byte aligned");
  return check_launch(launch_dense_gemm(x, T, weight, bias, N, K, out, err, GPTOSS_STREAM(stream)), "dense_gemm");
}

}  // extern "C"

// ------------------------------------------------------------- workspace --
struct gptoss_moe_workspace {
  int64_t max_tokens;
  int32_t E, K, H, I;
  void* base;
  size_t bytes;
  uint16_t* t;
  uint16_t* logits;
  uint16_t* topk_w;
  int32_t* topk_idx;
  int32_t* indptr;
  int32_t* tile_ptr;
  int32_t* tile_rows;
  int32_t* token_of_row;
  int32_t* row_of_pair;
  int32_t* expert_of_row;
  uint16_t* act;
  uint16_t* y;
  float* h2;
  uint8_t* qs;  // [max_tokens * top_k, 192] exponents of the block-scaled GEMMs' activation terms
  uint32_t* err;
};

static size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

namespace gptoss {
// Decode-size expert GEMMs run on the block-scaled tensor cores unless
// GPTOSS_MOE_MX=0 (GPTOSS_MOE_MX=1 forces them wherever they apply).
bool moe_mx_enabled() {
  const char* e = getenv("GPTOSS_MOE_MX");
  if (e && e[0] == '0') return false;
  if (e && e[0] == '1') return true;
  return kMoeMxDefault;
}
}  // namespace gptoss

// The expert part of the block for M routed tokens (t normalised, the
// permutation and token tiles already planned): gather + both grouped GEMMs.
// Decode-size tiles whose GEMMs fit the block-scaled kernel quantize the
// activations into `act` (two e4m3 terms per value, exponents in `qs`) and
// run moe_gemm_mx_kernel; everything else gathers f16 / bf16 rows into `act`
// for the decode GEMV or the kind::f16 kernels.  h2 receives the fp32 expert
// outputs; y is the SwiGLU output (f16 on the f16 and block-scaled paths).
// The decode GEMV keeps the routed rows of a single token (top-k rows): in
// the gpt-oss-20b decode graphs (ms per step, GEMV / block-scaled) batch 1
// 3.18 / 3.37, batch 2 3.77 / 3.75, batch 4 4.58 / 4.23, batch 8 5.70 /
// 4.94, batch 16 7.32 / 5.53.  Without the block-scaled kernels (or weights
// it does not take) the GEMV still serves up to 64 rows.
constexpr int64_t kGemvBeforeMxRows = 4;
static bool experts_block_scaled(int64_t M, const gptoss_moe_weights* w) {
  const int64_t R = M * w->top_k;
  const bool gemv = (w->flags & GPTOSS_MOE_F16) && R <= kGemvBeforeMxRows;
  return !gemv && moe_mx_enabled() && moe_mx_supported(R, w->num_experts, 2 * w->intermediate, w->hidden, w->mlp1_blocks) &&
         moe_mx_supported(R, w->num_experts, w->hidden, w->intermediate, w->mlp2_blocks);
}

extern "C" int gptoss_moe_uses_block_scaled(int64_t M, const gptoss_moe_weights* w) {
  return (w && M > 0 && experts_block_scaled(M, w)) ? 1 : 0;
}

// Router logits, top-k + softmax and the expert-major permutation of M
// normalised tokens t: one fused launch after the logits at decode sizes,
// the separate kernels otherwise (same results either way).
int gptoss::moe_route(const uint16_t* t, int64_t M, const gptoss_moe_weights* w, uint16_t* logits,
                      uint16_t* topk_w, int32_t* topk_idx, int32_t* indptr, int32_t* token_of_row,
                      int32_t* row_of_pair, int32_t* expert_of_row, int32_t* tile_ptr, int32_t* tile_rows,
                      uint32_t* err, void* stream) {
  const int32_t E = w->num_experts, K = w->top_k, H = w->hidden;
  // (one CTA runs every token's top-k: it wins below ~64 tokens, the parallel kernels above)
  if (M * K <= 256 && M * K <= route_small_max_pairs() && E <= 256 && E % 8 == 0 && K <= 8) {
    int rc = launch_router(t, w->gate_weight, w->gate_bias, M, E, H, logits, err, GPTOSS_STREAM(stream));
    if (rc) return check_launch(rc, "router");
    return check_launch(launch_route_small(logits, M, E, K, topk_w, topk_idx, indptr, tile_ptr, tile_rows,
                                           token_of_row, row_of_pair, expert_of_row, err, GPTOSS_STREAM(stream)),
                        "route_small");
  }
  int rc;
  if ((rc = gptoss_moe_router(t, w->gate_weight, w->gate_bias, M, E, H, K, logits, topk_w, topk_idx, err, stream)))
    return rc;
  return gptoss_moe_permute(topk_idx, M, K, E, indptr, token_of_row, row_of_pair, expert_of_row, tile_ptr, tile_rows,
                            err, stream);
}

extern "C" int gptoss_moe_route(const uint16_t* t, int64_t M, const gptoss_moe_weights* w, uint16_t* logits,
                                uint16_t* topk_weights, int32_t* topk_indices, int32_t* indptr, int32_t* token_of_row,
                                int32_t* row_of_pair, int32_t* expert_of_row, int32_t* tile_ptr, int32_t* tile_rows,
                                uint32_t* err, void* stream) {
  if (!w || M < 0) return fail(-1, "gptoss_moe_route: null weights or M < 0");
  if (M == 0) return 0;
  return gptoss::moe_route(t, M, w, logits, topk_weights, topk_indices, indptr, token_of_row, row_of_pair,
                           expert_of_row, tile_ptr, tile_rows, err, stream);
}

int gptoss::moe_experts_forward(const uint16_t* t, int64_t M, const gptoss_moe_weights* w, const int32_t* indptr,
                                const int32_t* tile_ptr, const int32_t* tile_rows, const int32_t* token_of_row,
                                uint16_t* act, uint16_t* y, float* h2, uint8_t* qs, uint32_t* err, void* stream) {
  const int32_t E = w->num_experts, K = w->top_k, H = w->hidden, I = w->intermediate;
  const int32_t f16 = (w->flags & GPTOSS_MOE_F16) ? 1 : 0;
  const int64_t R = M * K;
  int rc;
  if (experts_block_scaled(M, w)) {
    uint8_t* q = (uint8_t*)act;  // R x 2K bytes: the same size as the f16 rows
    if ((rc = gptoss_moe_quantize_mx(t, 0, token_of_row, R, H, q, qs, stream))) return rc;
    if ((rc = gptoss_moe_mlp1_mx(q, qs, R, indptr, tile_ptr, tile_rows, E, H, I, w->mlp1_blocks, w->mlp1_scales,
                                 w->mlp1_bias, w->swiglu_alpha, w->swiglu_limit, y, err, stream)))
      return rc;
    if ((rc = gptoss_moe_quantize_mx(y, 1, nullptr, R, I, q, qs, stream))) return rc;
    return gptoss_moe_mlp2_mx(q, qs, R, indptr, tile_ptr, tile_rows, E, H, I, w->mlp2_blocks, w->mlp2_scales,
                              w->mlp2_bias, h2, err, stream);
  }
  bool gathered = false;
  if (f16 && token_of_row) {
    // the decode GEMV stages its token rows straight from t (no gather launch)
    GemmLaunch L;
    L.act = t;
    L.act_rows = R;
    L.blocks = w->mlp1_blocks;
    L.scales = w->mlp1_scales;
    L.bias = w->mlp1_bias;
    L.indptr = indptr;
    L.tile_ptr = tile_ptr;
    L.tile_rows = tile_rows;
    L.out = y;
    L.E = E;
    L.N = 2 * I;
    L.K = H;
    L.ldo = I;
    L.alpha = w->swiglu_alpha;
    L.limit = w->swiglu_limit;
    L.err = err;
    L.grid = num_sms();
    L.f16 = 1;
    L.act_gather = token_of_row;
    if (moe_gemm_gathers(L)) {
      if ((rc = check_launch(launch_moe_gemm(0, L, GPTOSS_STREAM(stream)), "moe_mlp1"))) return rc;
      gathered = true;
    }
  }
  if (!gathered) {
    if ((rc = gptoss_moe_gather(t, token_of_row, R, H, f16, act, stream))) return rc;
    if ((rc = gptoss_moe_mlp1(act, R, indptr, tile_ptr, tile_rows, E, H, I, w->mlp1_blocks, w->mlp1_scales,
                              w->mlp1_bias, w->swiglu_alpha, w->swiglu_limit, f16, y, err, stream)))
      return rc;
  }
  return gptoss_moe_mlp2(y, R, indptr, tile_ptr, tile_rows, E, H, I, w->mlp2_blocks, w->mlp2_scales, w->mlp2_bias, f16,
                         h2, err, stream);
}

extern "C" {

gptoss_moe_workspace* gptoss_moe_workspace_create(int64_t max_tokens, int32_t num_experts, int32_t top_k,
                                                  int32_t hidden, int32_t intermediate) {
  if (max_tokens <= 0 || num_experts <= 0 || top_k <= 0 || hidden <= 0 || intermediate <= 0) {
    fail(-1, "gptoss_moe_workspace_create: bad sizes");
    return nullptr;
  }
  gptoss_moe_workspace* ws = new gptoss_moe_workspace();
  ws->max_tokens = max_tokens;
  ws->E = num_experts;
  ws->K = top_k;
  ws->H = hidden;
  ws->I = intermediate;
  const int64_t M = max_tokens, R = max_tokens * top_k, E = num_experts;
  size_t off[16], o = 0;
  int i = 0;
  off[i++] = o; o = align256(o + (size_t)M * hidden * 2);        // t
  off[i++] = o; o = align256(o + (size_t)M * E * 2);             // logits
  off[i++] = o; o = align256(o + (size_t)M * top_k * 2);         // topk_w
  off[i++] = o; o = align256(o + (size_t)M * top_k * 4);         // topk_idx
  off[i++] = o; o = align256(o + (size_t)(E + 1) * 4);           // indptr
  off[i++] = o; o = align256(o + (size_t)(E + 1) * 4);           // tile_ptr
  off[i++] = o; o = align256(o + (size_t)E * 4);                 // tile_rows
  off[i++] = o; o = align256(o + (size_t)R * 4);                 // token_of_row
  off[i++] = o; o = align256(o + (size_t)R * 4);                 // row_of_pair
  off[i++] = o; o = align256(o + (size_t)R * 4);                 // expert_of_row
  off[i++] = o; o = align256(o + (size_t)R * hidden * 2);        // act
  off[i++] = o; o = align256(o + (size_t)R * intermediate * 2);  // y
  off[i++] = o; o = align256(o + (size_t)R * hidden * 4);        // h2
  off[i++] = o; o = align256(o + (size_t)R * 192);               // qs
  off[i++] = o; o = align256(o + 256);                           // err
  ws->bytes = o;
  if (cudaMalloc(&ws->base, o) != cudaSuccess) {
    cudaGetLastError();
    fail(-4, "gptoss_moe_workspace_create: cudaMalloc of %zu bytes failed", o);
    delete ws;
    return nullptr;
  }
  char* b = (char*)ws->base;
  i = 0;
  ws->t = (uint16_t*)(b + off[i++]);
  ws->logits = (uint16_t*)(b + off[i++]);
  ws->topk_w = (uint16_t*)(b + off[i++]);
  ws->topk_idx = (int32_t*)(b + off[i++]);
  ws->indptr = (int32_t*)(b + off[i++]);
  ws->tile_ptr = (int32_t*)(b + off[i++]);
  ws->tile_rows = (int32_t*)(b + off[i++]);
  ws->token_of_row = (int32_t*)(b + off[i++]);
  ws->row_of_pair = (int32_t*)(b + off[i++]);
  ws->expert_of_row = (int32_t*)(b + off[i++]);
  ws->act = (uint16_t*)(b + off[i++]);
  ws->y = (uint16_t*)(b + off[i++]);
  ws->h2 = (float*)(b + off[i++]);
  ws->qs = (uint8_t*)(b + off[i++]);
  ws->err = (uint32_t*)(b + off[i++]);
  cudaMemset(ws->err, 0, 256);
  return ws;
}

void gptoss_moe_workspace_destroy(gptoss_moe_workspace* ws) {
  if (!ws) return;
  cudaFree(ws->base);
  delete ws;
}

uint32_t gptoss_moe_workspace_error(gptoss_moe_workspace* ws) {
  if (!ws) return 0;
  uint32_t v = 0;
  cudaDeviceSynchronize();
  cudaMemcpy(&v, ws->err, 4, cudaMemcpyDeviceToHost);
  cudaMemset(ws->err, 0, 4);
  return v;
}

int gptoss_moe_forward(const uint16_t* x, int64_t M, const gptoss_moe_weights* w, gptoss_moe_workspace* ws,
                       uint16_t* out, void* stream) {
  if (!w || !ws) return fail(-1, "gptoss_moe_forward: null weights or workspace");
  if (M < 0 || M > ws->max_tokens)
    return fail(-1, "gptoss_moe_forward: M=%lld exceeds workspace max_tokens=%lld", (long long)M,
                (long long)ws->max_tokens);
  if (w->num_experts != ws->E || w->top_k != ws->K || w->hidden != ws->H || w->intermediate != ws->I)
    return fail(-1, "gptoss_moe_forward: weights and workspace disagree on shapes");
  if (w->num_local_experts != w->num_experts || w->expert_offset != 0)
    return fail(-1, "gptoss_moe_forward: expert-parallel weights need the dispatch/combine path");
  if (M == 0) return 0;
  const int32_t E = w->num_experts, K = w->top_k, H = w->hidden;
  int rc;
  if ((rc = gptoss_rms_norm(x, w->norm_weight, M, H, w->rms_eps, ws->t, stream))) return rc;
  if ((rc = moe_route(ws->t, M, w, ws->logits, ws->topk_w, ws->topk_idx, ws->indptr, ws->token_of_row,
                      ws->row_of_pair, ws->expert_of_row, ws->tile_ptr, ws->tile_rows, ws->err, stream)))
    return rc;
  if ((rc = moe_experts_forward(ws->t, M, w, ws->indptr, ws->tile_ptr, ws->tile_rows, ws->token_of_row, ws->act,
                                 ws->y, ws->h2, ws->qs, ws->err, stream)))
    return rc;
  return gptoss_moe_combine(ws->h2, ws->row_of_pair, ws->topk_w, x, M, K, H, out, stream);
}

}  // extern "C"
