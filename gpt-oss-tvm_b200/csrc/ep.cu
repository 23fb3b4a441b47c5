// ep.cu -- expert parallelism at the C boundary (gptoss_ep_*): the MoE block
// with its experts sharded over the ranks of one node, one process per GPU.
//
// The same data path as the Python orchestration in ep.py (peer memory):
//   dispatch: RMSNorm, router, top-k and the expert-major permutation over the
//     global experts on this rank's tokens; an NCCL all-gather of the
//     per-expert row counts; the row layout on the device; every token row
//     stored straight into the owning rank's expert-major activation matrix
//     (CUDA IPC buffers, plain NVLink stores); a one-word NCCL all-reduce so
//     that no rank reads rows before every rank's stores are visible.
//   combine: the token-tile plan and both grouped GEMMs on this rank's experts,
//     the down-projection's epilogue storing each output row into the return
//     buffer of the rank that owns the token; a one-word all-reduce; the
//     weighted sum of each token's experts plus the residual.
// NCCL is loaded at run time (dlopen of libnccl.so.2, the library torch and
// the system ship), so the library does not depend on it unless these entry
// points are used.  Every collective of a step is issued in the same order on
// every rank, on the caller's stream.
#include <dlfcn.h>

#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <vector>

#include <nccl.h>

#include "../../include/gptoss_b200.h"
#include "launch.h"

namespace {

struct NcclApi {
  ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
  ncclResult_t (*CommInitRank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
  ncclResult_t (*AllGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*AllReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                            cudaStream_t) = nullptr;
  const char* (*GetErrorString)(ncclResult_t) = nullptr;
  bool ok = false;
};

NcclApi g_nccl;
std::once_flag g_nccl_once;

const NcclApi& nccl() {
  std::call_once(g_nccl_once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) return;
    g_nccl.GetUniqueId = (decltype(g_nccl.GetUniqueId))dlsym(h, "ncclGetUniqueId");
    g_nccl.CommInitRank = (decltype(g_nccl.CommInitRank))dlsym(h, "ncclCommInitRank");
    g_nccl.CommDestroy = (decltype(g_nccl.CommDestroy))dlsym(h, "ncclCommDestroy");
    g_nccl.AllGather = (decltype(g_nccl.AllGather))dlsym(h, "ncclAllGather");
    g_nccl.AllReduce = (decltype(g_nccl.AllReduce))dlsym(h, "ncclAllReduce");
    g_nccl.GetErrorString = (decltype(g_nccl.GetErrorString))dlsym(h, "ncclGetErrorString");
    g_nccl.ok = g_nccl.GetUniqueId && g_nccl.CommInitRank && g_nccl.CommDestroy && g_nccl.AllGather &&
                g_nccl.AllReduce && g_nccl.GetErrorString;
  });
  return g_nccl;
}

int ep_fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  return gptoss::set_last_error(code, buf);
}

size_t up256(size_t x) { return (x + 255) & ~(size_t)255; }

// counts[e] = indptr[e + 1] - indptr[e]: this rank's rows per global expert
__global__ void counts_kernel(const int32_t* __restrict__ indptr, int32_t E, int32_t* __restrict__ counts) {
  for (int32_t e = blockIdx.x * blockDim.x + threadIdx.x; e < E; e += gridDim.x * blockDim.x)
    counts[e] = indptr[e + 1] - indptr[e];
}

}  // namespace

struct gptoss_ep {
  int32_t rank, world;
  int64_t max_tokens;
  int32_t E, El, K, H, I;
  int32_t exact_return;
  ncclComm_t comm = nullptr;
  // this rank's scratch (one cudaMalloc)
  void* base = nullptr;
  uint16_t* t;
  uint16_t* logits;
  uint16_t* topk_w;
  int32_t *topk_idx, *indptr, *tile_ptr_g, *tile_rows_g, *tok, *rev, *exr;
  int32_t *counts_all, *dst_base, *indptr_local, *tile_ptr, *tile_rows, *one;
  uint16_t* y;
  uint32_t* err;
  // IPC buffers: activation rows (f16 / bf16), row origins, return rows
  int64_t cap;  // rows of the activation matrix (every rank's rows)
  void* own[3] = {nullptr, nullptr, nullptr};
  std::vector<void*> opened;
  std::vector<void*> rows, origin, back;  // per rank
  int32_t f16 = -1;  // activation type of the step in flight (rows travel in the GEMM's type)
};

extern "C" int gptoss_ep_unique_id(void* id) {
  const NcclApi& n = nccl();
  if (!n.ok) return ep_fail(-5, "gptoss_ep_unique_id: libnccl.so.2 could not be loaded");
  if (!id) return ep_fail(-1, "gptoss_ep_unique_id: null output");
  ncclUniqueId u;
  const ncclResult_t r = n.GetUniqueId(&u);
  if (r != ncclSuccess) return ep_fail(-5, "ncclGetUniqueId: %s", n.GetErrorString(r));
  static_assert(sizeof(u) == 128, "ncclUniqueId is 128 bytes");
  memcpy(id, &u, sizeof(u));
  return 0;
}

extern "C" void gptoss_ep_destroy(gptoss_ep* ep) {
  if (!ep) return;
  cudaDeviceSynchronize();
  for (void* p : ep->opened) gptoss_ipc_close(p);
  for (void* p : ep->own)
    if (p) gptoss_ipc_free(p);
  if (ep->base) cudaFree(ep->base);
  if (ep->comm) nccl().CommDestroy(ep->comm);
  cudaGetLastError();
  delete ep;
}

extern "C" gptoss_ep* gptoss_ep_init(const void* id, int32_t rank, int32_t world, int64_t max_tokens,
                                     int32_t num_experts, int32_t top_k, int32_t hidden, int32_t intermediate,
                                     int32_t exact_return, void* stream) {
  const NcclApi& n = nccl();
  if (!n.ok) {
    ep_fail(-5, "gptoss_ep_init: libnccl.so.2 could not be loaded");
    return nullptr;
  }
  if (!id || world < 1 || world > gptoss::kMaxPeerRanks || rank < 0 || rank >= world || max_tokens < 1 ||
      num_experts % world || top_k < 1 || top_k > 8 || hidden <= 0 || intermediate <= 0 ||
      (int64_t)world * max_tokens * top_k >= (1 << 24)) {
    ep_fail(-1, "gptoss_ep_init: bad arguments (1 <= world <= %d, experts divisible by world, rows < 2^24)",
            gptoss::kMaxPeerRanks);
    return nullptr;
  }
  gptoss_ep* ep = new gptoss_ep();
  ep->rank = rank;
  ep->world = world;
  ep->max_tokens = max_tokens;
  ep->E = num_experts;
  ep->El = num_experts / world;
  ep->K = top_k;
  ep->H = hidden;
  ep->I = intermediate;
  ep->exact_return = exact_return ? 1 : 0;
  ep->cap = (int64_t)world * max_tokens * top_k;
  cudaStream_t s = (cudaStream_t)stream;
  ncclUniqueId u;
  memcpy(&u, id, sizeof(u));
  ncclResult_t r = n.CommInitRank(&ep->comm, world, u, rank);
  if (r != ncclSuccess) {
    ep->comm = nullptr;
    ep_fail(-5, "ncclCommInitRank: %s", n.GetErrorString(r));
    gptoss_ep_destroy(ep);
    return nullptr;
  }
  // scratch of this rank
  const int64_t M = max_tokens, R = max_tokens * top_k, E = num_experts, El = ep->El;
  size_t off[18], o = 0;
  int i = 0;
  off[i++] = o; o = up256(o + (size_t)M * hidden * 2);            // t
  off[i++] = o; o = up256(o + (size_t)M * E * 2);                 // logits
  off[i++] = o; o = up256(o + (size_t)M * top_k * 2);             // topk_w
  off[i++] = o; o = up256(o + (size_t)M * top_k * 4);             // topk_idx
  off[i++] = o; o = up256(o + (size_t)(E + 1) * 4);               // indptr
  off[i++] = o; o = up256(o + (size_t)(E + 1) * 4);               // tile_ptr_g
  off[i++] = o; o = up256(o + (size_t)E * 4);                     // tile_rows_g
  off[i++] = o; o = up256(o + (size_t)R * 4);                     // tok
  off[i++] = o; o = up256(o + (size_t)R * 4);                     // rev
  off[i++] = o; o = up256(o + (size_t)R * 4);                     // exr
  off[i++] = o; o = up256(o + (size_t)world * E * 4);             // counts_all
  off[i++] = o; o = up256(o + (size_t)world * El * 4);            // dst_base
  off[i++] = o; o = up256(o + (size_t)(El + 1) * 4);              // indptr_local
  off[i++] = o; o = up256(o + (size_t)(El + 1) * 4);              // tile_ptr
  off[i++] = o; o = up256(o + (size_t)El * 4);                    // tile_rows
  off[i++] = o; o = up256(o + 256);                               // one (ordering word) + handles
  off[i++] = o; o = up256(o + (size_t)ep->cap * intermediate * 2);  // y
  off[i++] = o; o = up256(o + 256);                               // err
  if (cudaMalloc(&ep->base, o) != cudaSuccess || cudaMemset(ep->base, 0, o) != cudaSuccess) {
    cudaGetLastError();
    ep->base = nullptr;
    ep_fail(-4, "gptoss_ep_init: cudaMalloc of %zu bytes failed", o);
    gptoss_ep_destroy(ep);
    return nullptr;
  }
  char* b = (char*)ep->base;
  i = 0;
  ep->t = (uint16_t*)(b + off[i++]);
  ep->logits = (uint16_t*)(b + off[i++]);
  ep->topk_w = (uint16_t*)(b + off[i++]);
  ep->topk_idx = (int32_t*)(b + off[i++]);
  ep->indptr = (int32_t*)(b + off[i++]);
  ep->tile_ptr_g = (int32_t*)(b + off[i++]);
  ep->tile_rows_g = (int32_t*)(b + off[i++]);
  ep->tok = (int32_t*)(b + off[i++]);
  ep->rev = (int32_t*)(b + off[i++]);
  ep->exr = (int32_t*)(b + off[i++]);
  ep->counts_all = (int32_t*)(b + off[i++]);
  ep->dst_base = (int32_t*)(b + off[i++]);
  ep->indptr_local = (int32_t*)(b + off[i++]);
  ep->tile_ptr = (int32_t*)(b + off[i++]);
  ep->tile_rows = (int32_t*)(b + off[i++]);
  ep->one = (int32_t*)(b + off[i++]);
  ep->y = (uint16_t*)(b + off[i++]);
  ep->err = (uint32_t*)(b + off[i++]);
  // IPC buffers, their handles exchanged with one all-gather (192 bytes per rank)
  const size_t sizes[3] = {(size_t)ep->cap * hidden * 2, (size_t)ep->cap * 4,
                           (size_t)R * hidden * (ep->exact_return ? 4 : 2)};
  std::vector<uint8_t> mine(3 * 64), all((size_t)world * 3 * 64);
  for (int k = 0; k < 3; ++k) {
    if (gptoss_ipc_alloc(sizes[k], &ep->own[k], mine.data() + 64 * k)) {
      gptoss_ep_destroy(ep);
      return nullptr;
    }
  }
  uint8_t* dh = nullptr;
  if (cudaMalloc(&dh, all.size()) != cudaSuccess) {
    cudaGetLastError();
    ep_fail(-4, "gptoss_ep_init: cudaMalloc for the handle exchange failed");
    gptoss_ep_destroy(ep);
    return nullptr;
  }
  cudaMemcpyAsync(dh + (size_t)rank * 192, mine.data(), 192, cudaMemcpyHostToDevice, s);
  r = n.AllGather(dh + (size_t)rank * 192, dh, 192, ncclUint8, ep->comm, s);
  cudaMemcpyAsync(all.data(), dh, all.size(), cudaMemcpyDeviceToHost, s);
  const cudaError_t ce = cudaStreamSynchronize(s);
  cudaFree(dh);
  if (r != ncclSuccess || ce != cudaSuccess) {
    cudaGetLastError();
    ep_fail(-5, "gptoss_ep_init: handle exchange failed (%s)", r != ncclSuccess ? n.GetErrorString(r) : "cuda");
    gptoss_ep_destroy(ep);
    return nullptr;
  }
  ep->rows.assign(world, nullptr);
  ep->origin.assign(world, nullptr);
  ep->back.assign(world, nullptr);
  std::vector<void*>* dst[3] = {&ep->rows, &ep->origin, &ep->back};
  for (int rr = 0; rr < world; ++rr) {
    for (int k = 0; k < 3; ++k) {
      if (rr == rank) {
        (*dst[k])[rr] = ep->own[k];
        continue;
      }
      void* p = nullptr;
      if (gptoss_ipc_open(all.data() + ((size_t)rr * 3 + k) * 64, &p)) {
        gptoss_ep_destroy(ep);
        return nullptr;
      }
      ep->opened.push_back(p);
      (*dst[k])[rr] = p;
    }
  }
  return ep;
}

namespace {

int ep_check_weights(const gptoss_ep* ep, const gptoss_moe_weights* w, const char* fn) {
  if (!ep || !w) return ep_fail(-1, "%s: null group or weights", fn);
  if (w->num_experts != ep->E || w->num_local_experts != ep->El || w->expert_offset != ep->rank * ep->El ||
      w->top_k != ep->K || w->hidden != ep->H || w->intermediate != ep->I)
    return ep_fail(-1, "%s: the weights must be this rank's shard (experts [%d, %d) of %d, top-%d, %d x %d)", fn,
                   ep->rank * ep->El, (ep->rank + 1) * ep->El, ep->E, ep->K, ep->H, ep->I);
  return 0;
}

// One-word all-reduce: every rank's kernels issued before it on its stream
// have completed, so their peer stores are visible everywhere.
int ep_order(gptoss_ep* ep, cudaStream_t s) {
  const ncclResult_t r = nccl().AllReduce(ep->one, ep->one, 1, ncclInt32, ncclMax, ep->comm, s);
  return r == ncclSuccess ? 0 : ep_fail(-5, "ncclAllReduce: %s", nccl().GetErrorString(r));
}

}  // namespace

extern "C" int gptoss_ep_dispatch(gptoss_ep* ep, const uint16_t* x, int64_t M, const gptoss_moe_weights* w,
                                  void* stream) {
  if (int rc = ep_check_weights(ep, w, "gptoss_ep_dispatch")) return rc;
  if (M < 0 || M > ep->max_tokens)
    return ep_fail(-1, "gptoss_ep_dispatch: %lld tokens exceed max_tokens=%lld", (long long)M,
                   (long long)ep->max_tokens);
  cudaStream_t s = (cudaStream_t)stream;
  const int32_t E = ep->E, K = ep->K, H = ep->H;
  ep->f16 = (w->flags & GPTOSS_MOE_F16) ? 1 : 0;
  int rc;
  if ((rc = gptoss_rms_norm(x, w->norm_weight, M, H, w->rms_eps, ep->t, s))) return rc;
  if ((rc = gptoss_moe_router(ep->t, w->gate_weight, w->gate_bias, M, E, H, K, ep->logits, ep->topk_w, ep->topk_idx,
                              ep->err, s)))
    return rc;
  if ((rc = gptoss_moe_permute(ep->topk_idx, M, K, E, ep->indptr, ep->tok, ep->rev, ep->exr, ep->tile_ptr_g,
                               ep->tile_rows_g, ep->err, s)))
    return rc;
  // this rank's rows per global expert, written into its slot of the
  // all-gathered [world, E] counts (an in-place all-gather)
  int32_t* counts = ep->counts_all + (size_t)ep->rank * E;
  counts_kernel<<<(E + 255) / 256, 256, 0, s>>>(ep->indptr, E, counts);
  if (cudaGetLastError() != cudaSuccess) return ep_fail(-3, "gptoss_ep_dispatch: counts kernel launch failed");
  ncclResult_t r = nccl().AllGather(counts, ep->counts_all, (size_t)E, ncclInt32, ep->comm, s);
  if (r != ncclSuccess) return ep_fail(-5, "ncclAllGather: %s", nccl().GetErrorString(r));
  if ((rc = gptoss_moe_peer_layout(ep->counts_all, ep->world, ep->El, ep->rank, ep->dst_base, ep->indptr_local, s)))
    return rc;
  if ((rc = gptoss_moe_dispatch_peer(ep->t, ep->tok, ep->exr, ep->indptr, M * K, H, E, ep->El, ep->rank,
                                     ep->dst_base, ep->rows.data(), (int32_t* const*)ep->origin.data(), ep->world,
                                     ep->cap, ep->f16, s)))
    return rc;
  return ep_order(ep, s);
}

extern "C" int gptoss_ep_combine(gptoss_ep* ep, const uint16_t* x, int64_t M, const gptoss_moe_weights* w,
                                 uint16_t* out, void* stream) {
  if (int rc = ep_check_weights(ep, w, "gptoss_ep_combine")) return rc;
  if (ep->f16 < 0) return ep_fail(-1, "gptoss_ep_combine: no dispatch before it");
  cudaStream_t s = (cudaStream_t)stream;
  const int32_t H = ep->H, I = ep->I, El = ep->El;
  int rc;
  if ((rc = gptoss_moe_plan_tiles(ep->indptr_local, El, ep->tile_ptr, ep->tile_rows, s))) return rc;
  // launched on the buffer capacity: the tiles come from the device-side plan
  if ((rc = gptoss_moe_mlp1((const uint16_t*)ep->own[0], ep->cap, ep->indptr_local, ep->tile_ptr, ep->tile_rows, El,
                            H, I, w->mlp1_blocks, w->mlp1_scales, w->mlp1_bias, w->swiglu_alpha, w->swiglu_limit,
                            ep->f16, ep->y, ep->err, s)))
    return rc;
  if ((rc = gptoss_moe_mlp2_peer(ep->y, ep->cap, ep->indptr_local, ep->tile_ptr, ep->tile_rows, El, H, I,
                                 w->mlp2_blocks, w->mlp2_scales, w->mlp2_bias, ep->f16, (const int32_t*)ep->own[1],
                                 ep->back.data(), ep->world, ep->max_tokens * ep->K, ep->exact_return ? 0 : 1,
                                 ep->err, s)))
    return rc;
  if ((rc = ep_order(ep, s))) return rc;
  ep->f16 = -1;
  if (M == 0) return 0;
  if (ep->exact_return)
    return gptoss_moe_combine((const float*)ep->own[2], ep->rev, ep->topk_w, x, M, ep->K, H, out, s);
  return gptoss_moe_combine_bf16((const uint16_t*)ep->own[2], ep->rev, ep->topk_w, x, M, ep->K, H, out, s);
}

extern "C" int gptoss_ep_forward(gptoss_ep* ep, const uint16_t* x, int64_t M, const gptoss_moe_weights* w,
                                 uint16_t* out, void* stream) {
  if (int rc = gptoss_ep_dispatch(ep, x, M, w, stream)) return rc;
  return gptoss_ep_combine(ep, x, M, w, out, stream);
}

extern "C" uint32_t gptoss_ep_error(gptoss_ep* ep) {
  if (!ep) return 0;
  uint32_t v = 0;
  cudaDeviceSynchronize();
  cudaMemcpy(&v, ep->err, 4, cudaMemcpyDeviceToHost);
  cudaMemset(ep->err, 0, 4);
  return v;
}
