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
// The array is shared by every call, and keeps what the last call left in it.
// Only its last 256 bytes must start at zero: the device error word that the
// router, the permutation and both expert GEMMs set when a bounded wait runs
// out or an expert index is out of range (static device memory starts zeroed,
// and gptoss_moe_noalloc_error() clears the word when it reads it).  Every
// other stage writes all the scratch it later reads before reading it.  Calls
// that overlap on the GPU (two streams, or two host threads) race on it.
//
// The device address of the array is looked up once per device and cached for
// the life of the process; it does not survive cudaDeviceReset() (the module
// and its array are reloaded at a new address), so do not reset a device
// between calls.
#include <mutex>
#include <string>

#include "../../include/gptoss_b200.h"
#include "common.cuh"
#include "launch.h"

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
constexpr size_t kOffQs = kOffH2 + up256((size_t)kRows * kNoAllocMaxHidden * 4);   // [M*K, 192] exponents
constexpr size_t kOffErr = kOffQs + up256((size_t)kRows * 192);                      // error word (256 B)
constexpr size_t kScratchBytes = kOffErr + 256;

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

// Device address of the scratch array on the current device; the first call
// on a device (with that device current) looks it up and caches it.
static int scratch_base(const char* who, uint8_t** base) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    cudaGetLastError();
    std::string m = std::string(who) + ": no current CUDA device";
    return noalloc_fail(-4, m.c_str());
  }
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (!g_scratch_addr[dev]) {
    void* p = nullptr;
    const cudaError_t rc = cudaGetSymbolAddress(&p, g_moe_noalloc_scratch);
    if (rc != cudaSuccess || p == nullptr) {
      cudaGetLastError();
      std::string m = std::string(who) + ": cudaGetSymbolAddress of the scratch array failed";
      return noalloc_fail(-4, m.c_str());
    }
    g_scratch_addr[dev] = (uint8_t*)p;
  }
  *base = g_scratch_addr[dev];
  return 0;
}

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

  uint8_t* base = nullptr;
  if (int rc = scratch_base("gptoss_moe_forward_noalloc", &base)) return rc;

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
  uint8_t* qs = base + kOffQs;
  uint32_t* err = (uint32_t*)(base + kOffErr);

  const int32_t E = w->num_experts, K = w->top_k, H = w->hidden;
  int rc;
  if ((rc = gptoss_rms_norm(x, w->norm_weight, M, H, w->rms_eps, t, stream))) return rc;
  if ((rc = gptoss::moe_route(t, M, w, logits, topk_w, topk_idx, indptr, tok, rev, exr, tile_ptr, tile_rows, err,
                              stream)))
    return rc;
  if ((rc = gptoss::moe_experts_forward(t, M, w, indptr, tile_ptr, tile_rows, tok, act, y, h2, qs, err, stream)))
    return rc;
  return gptoss_moe_combine(h2, rev, topk_w, x, M, K, H, out, stream);
}

extern "C" uint32_t gptoss_moe_noalloc_error(void) {
  uint8_t* base = nullptr;
  if (scratch_base("gptoss_moe_noalloc_error", &base)) return 0xFFFFFFFFu;
  // synchronous copies out of and into the array: no allocation, and they wait
  // for the device's work that is still in flight
  uint32_t v = 0;
  if (cudaDeviceSynchronize() != cudaSuccess ||
      cudaMemcpy(&v, base + kOffErr, sizeof(v), cudaMemcpyDeviceToHost) != cudaSuccess ||
      cudaMemset(base + kOffErr, 0, sizeof(v)) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess) {
    cudaGetLastError();
    noalloc_fail(-4, "gptoss_moe_noalloc_error: reading the error word failed");
    return 0xFFFFFFFFu;
  }
  return v;
}
