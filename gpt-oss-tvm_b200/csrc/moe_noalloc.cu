// moe_noalloc.cu -- gptoss_moe_forward_noalloc: the MoE block forward without
// any device allocation.
//
// Some callers cannot allocate device memory when they run the block: a
// serving loop whose device memory is fully planned before the first request
// (the way a compiled graph executor plans every buffer up front), code that
// must not call cudaMalloc because it synchronises the device and stalls the
// other streams of the process, or a host that has no CUDA allocator of its
// own.  For them the scratch of the block lives in one fixed array of this
// library, sized for at most kNoAllocMaxTokens tokens.  Every GPU that loads
// the library holds that array (about 6.3 MB) until the process exits.
//
// The array is shared by every call, and keeps what the last call left in it;
// nothing in it has to start at zero, because every stage writes all the
// scratch it later reads.  Calls that overlap on the GPU (two streams, or two
// host threads) race on it.
#include <mutex>

#include "../../include/gptoss_b200.h"
#include "common.cuh"

namespace {

constexpr int64_t kNoAllocMaxTokens = 64;
constexpr int32_t kNoAllocMaxExperts = 128;
constexpr int32_t kNoAllocMaxTopK = 4;
constexpr int32_t kNoAllocMaxHidden = 2880;
constexpr int32_t kNoAllocMaxInter = 2880;
constexpr int64_t kRows = kNoAllocMaxTokens * kNoAllocMaxTopK;

constexpr size_t up256(size_t x) { return (x + 255) & ~(size_t)255; }

// Fixed layout of the scratch array (offsets in bytes).
constexpr size_t kOffT = 0;                                                                   // t [M, H] bf16
constexpr size_t kOffLogits = kOffT + up256((size_t)kNoAllocMaxTokens * kNoAllocMaxHidden * 2);  // [M, E] bf16
constexpr size_t kOffW = kOffLogits + up256((size_t)kNoAllocMaxTokens * kNoAllocMaxExperts * 2);  // [M, K] bf16
constexpr size_t kOffIdx = kOffW + up256((size_t)kRows * 2);                                  // [M, K] int32
constexpr size_t kOffIndptr = kOffIdx + up256((size_t)kRows * 4);                             // [E+1]
constexpr size_t kOffTilePtr = kOffIndptr + up256((size_t)(kNoAllocMaxExperts + 1) * 4);      // [E+1]
constexpr size_t kOffTileRows = kOffTilePtr + up256((size_t)(kNoAllocMaxExperts + 1) * 4);    // [E]
constexpr size_t kOffTok = kOffTileRows + up256((size_t)kNoAllocMaxExperts * 4);              // [M*K]
constexpr size_t kOffRev = kOffTok + up256((size_t)kRows * 4);                                // [M*K]
constexpr size_t kOffExp = kOffRev + up256((size_t)kRows * 4);                                // [M*K]
constexpr size_t kOffAct = kOffExp + up256((size_t)kRows * 4);                                // [M*K, H] bf16
constexpr size_t kOffY = kOffAct + up256((size_t)kRows * kNoAllocMaxHidden * 2);              // [M*K, I] bf16
constexpr size_t kOffH2 = kOffY + up256((size_t)kRows * kNoAllocMaxInter * 2);                // [M*K, H] f32
constexpr size_t kScratchBytes = kOffH2 + up256((size_t)kRows * kNoAllocMaxHidden * 4);

static __device__ __align__(256) uint8_t g_moe_noalloc_scratch[kScratchBytes];

// Device address of the array, per device.  In host code the array's name is
// only a host-side stand-in, so the address is looked up once per device.
constexpr int kMaxDevices = 64;
uint8_t* g_scratch_addr[kMaxDevices] = {nullptr};
std::mutex g_scratch_mu;

}  // namespace

namespace gptoss {
int set_last_error(int code, const char* msg);
}

static int noalloc_fail(int code, const char* msg) { return gptoss::set_last_error(code, msg); }

extern "C" int gptoss_moe_forward_noalloc(const uint16_t* x, int64_t M, const gptoss_moe_weights* w, uint16_t* out,
                                          void* stream) {
  if (!w) return noalloc_fail(-1, "gptoss_moe_forward_noalloc: null weights");
  if (M < 0 || M > kNoAllocMaxTokens)
    return noalloc_fail(-1, "gptoss_moe_forward_noalloc: at most 64 tokens per call (the fixed scratch holds 64)");
  if (w->num_experts <= 0 || w->num_experts > kNoAllocMaxExperts || w->top_k <= 0 || w->top_k > kNoAllocMaxTopK ||
      w->hidden <= 0 || w->hidden > kNoAllocMaxHidden || w->intermediate <= 0 ||
      w->intermediate > kNoAllocMaxInter)
    return noalloc_fail(-1,
                        "gptoss_moe_forward_noalloc: supports at most 128 experts, top-4, hidden and intermediate "
                        "sizes up to 2880");
  if (w->num_local_experts != w->num_experts || w->expert_offset != 0)
    return noalloc_fail(-1, "gptoss_moe_forward_noalloc: needs all experts on this device");
  if (M == 0) return 0;

  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    cudaGetLastError();
    return noalloc_fail(-4, "gptoss_moe_forward_noalloc: no current CUDA device");
  }
  uint8_t* base = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_scratch_mu);
    if (!g_scratch_addr[dev]) {
      // first call on this device (this device is current): resolve the device address
      void* p = nullptr;
      cudaError_t rc = cudaGetSymbolAddress(&p, g_moe_noalloc_scratch);
      if (rc != cudaSuccess || p == nullptr) {
        cudaGetLastError();
        return noalloc_fail(-4, "gptoss_moe_forward_noalloc: cudaGetSymbolAddress of the scratch array failed");
      }
      g_scratch_addr[dev] = (uint8_t*)p;
    }
    base = g_scratch_addr[dev];
  }

  uint16_t* t = (uint16_t*)(base + kOffT);
  uint16_t* logits = (uint16_t*)(base + kOffLogits);
  uint16_t* topk_w = (uint16_t*)(base + kOffW);
  int32_t* topk_idx = (int32_t*)(base + kOffIdx);
  int32_t* indptr = (int32_t*)(base + kOffIndptr);
  int32_t* tile_ptr = (int32_t*)(base + kOffTilePtr);
  int32_t* tile_rows = (int32_t*)(base + kOffTileRows);
  int32_t* tok = (int32_t*)(base + kOffTok);
  int32_t* rev = (int32_t*)(base + kOffRev);
  int32_t* exr = (int32_t*)(base + kOffExp);
  uint16_t* act = (uint16_t*)(base + kOffAct);
  uint16_t* y = (uint16_t*)(base + kOffY);
  float* h2 = (float*)(base + kOffH2);

  const int32_t E = w->num_experts, K = w->top_k, H = w->hidden, I = w->intermediate;
  const int32_t f16 = (w->flags & GPTOSS_MOE_F16) ? 1 : 0;
  const int64_t R = M * K;
  int rc;
  if ((rc = gptoss_rms_norm(x, w->norm_weight, M, H, w->rms_eps, t, stream))) return rc;
  if ((rc = gptoss_moe_router(t, w->gate_weight, w->gate_bias, M, E, H, K, logits, topk_w, topk_idx, nullptr,
                              stream)))
    return rc;
  if ((rc = gptoss_moe_permute(topk_idx, M, K, E, indptr, tok, rev, exr, tile_ptr, tile_rows, nullptr, stream)))
    return rc;
  if ((rc = gptoss_moe_gather(t, tok, R, H, f16, act, stream))) return rc;
  if ((rc = gptoss_moe_mlp1(act, R, indptr, tile_ptr, tile_rows, E, H, I, w->mlp1_blocks, w->mlp1_scales,
                            w->mlp1_bias, w->swiglu_alpha, w->swiglu_limit, f16, y, nullptr, stream)))
    return rc;
  if ((rc = gptoss_moe_mlp2(y, R, indptr, tile_ptr, tile_rows, E, H, I, w->mlp2_blocks, w->mlp2_scales, w->mlp2_bias,
                            f16, h2, nullptr, stream)))
    return rc;
  return gptoss_moe_combine(h2, rev, topk_w, x, M, K, H, out, stream);
}
