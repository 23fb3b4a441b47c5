// moe_peer.cu -- expert-parallel data movement over peer memory (NVLink).
//
// The expert-parallel MoE block (gpt-oss-tvm_b200/ep.py) shards the experts of
// the block over the ranks of one node (one process per GPU).  Instead of
// all-to-all exchanges through NCCL plus reorder passes, each rank writes the
// rows straight into the rank that uses them:
//   * dispatch: the token row of every (token, expert) pair is stored into
//     the owning rank's expert-major activation matrix at its final row, in
//     the GEMM's activation type, together with the row's origin;
//   * return: the down-projection GEMM's epilogue stores each output row into
//     the return buffer of the rank that owns the token (moe_gemm.cu).
// Buffers are plain cudaMalloc allocations shared with cudaIpc handles; the
// kernels use ordinary stores to peer addresses (no multicast, no waits on
// other GPUs).  Ordering between ranks is the host's: every writing kernel
// ends with a system-scope fence and the ranks meet at a collective before
// the rows are read.
#include "common.cuh"
#include "launch.h"

namespace gptoss {

struct PeerRows {
  void* rows[kMaxPeerRanks];      // per destination rank: activation matrix [cap_rows, H]
  int32_t* origin[kMaxPeerRanks];  // per destination rank: origin of each row (rank << 24 | send row)
};

// Send row r (this rank's expert-major order over the global experts) of
// expert eg goes to rank d = eg / El, local expert e = eg % El, row
// dst_base[d * El + e] + (r - indptr[eg]): the block of this rank's rows of
// expert e on rank d, in this rank's order.  One warp per row, 16-byte
// pieces, bf16 -> f16 on the way for the f16 GEMM path (as gather_rows_kernel).
template <bool kToF16>
__global__ void dispatch_peer_kernel(const uint16_t* __restrict__ t, const int32_t* __restrict__ token_of_row,
                                     const int32_t* __restrict__ expert_of_row, const int32_t* __restrict__ indptr,
                                     int64_t rows, int32_t H, int32_t E, int32_t El, int32_t rank,
                                     const int32_t* __restrict__ dst_base, int64_t cap_rows, const PeerRows peers) {
  const int64_t r = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (r >= rows) return;
  const int lane = threadIdx.x & 31;
  const int32_t eg = expert_of_row[r];
  if (eg < 0 || eg >= E) return;  // routing errors are reported by the router
  const int32_t d = eg / El, e = eg - d * El;
  const int64_t dst = (int64_t)dst_base[d * El + e] + (r - indptr[eg]);
  if (dst < 0 || dst >= cap_rows) return;  // (capacities hold every rank's rows)
  const uint4* s = (const uint4*)(t + (int64_t)token_of_row[r] * H);
  uint4* o = (uint4*)((uint16_t*)peers.rows[d] + dst * H);
  for (int32_t i = lane; i < H / 8; i += 32) {
    uint4 v = s[i];
    if (kToF16) {
      uint32_t* w = (uint32_t*)&v;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const __half2 h = __floats2half2_rn(__uint_as_float(w[q] << 16), __uint_as_float(w[q] & 0xFFFF0000u));
        w[q] = *(const uint32_t*)&h;
      }
    }
    o[i] = v;
  }
  if (lane == 0) peers.origin[d][dst] = (rank << 24) | (int32_t)r;
  __threadfence_system();
}

// Row addressing of the peer path from the all-gathered counts
// [num_ranks, num_ranks * El] (rows of source rank s for each global expert),
// as peer_layout in ep.py: rank d's matrix is expert-major over its local
// experts and source-major inside an expert.
//   dst_base[d * El + e] = first row on rank d of this rank's rows of e;
//   indptr_local[e] = first row of this rank's own local expert e.
__global__ void peer_layout_kernel(const int32_t* __restrict__ counts, int32_t P, int32_t El, int32_t rank,
                                   int32_t* __restrict__ dst_base, int32_t* __restrict__ indptr_local) {
  const int32_t E = P * El;
  for (int32_t i = threadIdx.x; i < P * El; i += blockDim.x) {
    const int32_t d = i / El, e = i % El;
    int32_t v = 0;
    for (int32_t ep = 0; ep < e; ++ep)
      for (int32_t s = 0; s < P; ++s) v += counts[s * E + d * El + ep];
    for (int32_t s = 0; s < rank; ++s) v += counts[s * E + d * El + e];
    dst_base[i] = v;
  }
  for (int32_t e = threadIdx.x; e <= El; e += blockDim.x) {
    int32_t v = 0;
    for (int32_t ep = 0; ep < e; ++ep)
      for (int32_t s = 0; s < P; ++s) v += counts[s * E + rank * El + ep];
    indptr_local[e] = v;
  }
}

int launch_peer_layout(const int32_t* counts, int32_t P, int32_t El, int32_t rank, int32_t* dst_base,
                       int32_t* indptr_local, cudaStream_t s) {
  if (P < 1 || P > kMaxPeerRanks || El <= 0 || rank < 0 || rank >= P) return -12;
  peer_layout_kernel<<<1, 256, 0, s>>>(counts, P, El, rank, dst_base, indptr_local);
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

int launch_dispatch_peer(const uint16_t* t, const int32_t* token_of_row, const int32_t* expert_of_row,
                         const int32_t* indptr, int64_t rows, int32_t H, int32_t E, int32_t El, int32_t rank,
                         const int32_t* dst_base, void* const* peer_rows, int32_t* const* peer_origin,
                         int32_t num_ranks, int64_t cap_rows, int32_t to_f16, cudaStream_t s) {
  if (rows <= 0) return 0;
  if (H % 8 || num_ranks < 1 || num_ranks > kMaxPeerRanks || El <= 0 || E != El * num_ranks || rank < 0 ||
      rank >= num_ranks || rows >= (1 << 24))
    return -12;
  PeerRows pr;
  for (int i = 0; i < kMaxPeerRanks; ++i) {
    pr.rows[i] = i < num_ranks ? peer_rows[i] : nullptr;
    pr.origin[i] = i < num_ranks ? peer_origin[i] : nullptr;
  }
  const unsigned blocks = (unsigned)((rows + 7) / 8);
  if (to_f16)
    dispatch_peer_kernel<true><<<blocks, 256, 0, s>>>(t, token_of_row, expert_of_row, indptr, rows, H, E, El, rank,
                                                       dst_base, cap_rows, pr);
  else
    dispatch_peer_kernel<false><<<blocks, 256, 0, s>>>(t, token_of_row, expert_of_row, indptr, rows, H, E, El, rank,
                                                        dst_base, cap_rows, pr);
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

// ---------------------------------------------- stream-ordered rank flags --
// One rank publishes a step number in a 32-bit word (its own memory, or a
// peer's through an IPC mapping) once its earlier work on the stream is
// visible system-wide; another rank's stream waits on the device until the
// word reaches that number.  The wait is bounded: after max_polls polls
// (about 0.1-0.2 us each) it sets kErrTimeoutFlag in *err and returns, so a
// rank that never arrives leaves an error bit instead of a stuck stream.
// The comparison is wrap-safe (the word counts steps modulo 2^32).
__global__ void set_flag_kernel(uint32_t* flag, uint32_t value) {
  if (threadIdx.x == 0) {
    __threadfence_system();
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(flag), "r"(value) : "memory");
  }
}

__global__ void wait_flag_kernel(const uint32_t* flag, uint32_t value, uint32_t max_polls, uint32_t* err) {
  if (threadIdx.x != 0) return;
  for (uint32_t i = 0; i < max_polls; ++i) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(flag) : "memory");
    if ((int32_t)(v - value) >= 0) return;
    __nanosleep(128);
  }
  raise_error(err, kErrTimeoutFlag);
}

int launch_set_flag(uint32_t* flag, uint32_t value, cudaStream_t s) {
  set_flag_kernel<<<1, 32, 0, s>>>(flag, value);
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

int launch_wait_flag(const uint32_t* flag, uint32_t value, uint32_t max_polls, uint32_t* err, cudaStream_t s) {
  wait_flag_kernel<<<1, 32, 0, s>>>(flag, value, max_polls, err);
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

}  // namespace gptoss
