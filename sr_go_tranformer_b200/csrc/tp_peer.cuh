// tp_peer.cuh -- the tensor-parallel all-reduce over NVLink peer memory.
//
// The ranks' partial sums of o_proj / down_proj (the row-parallel halves of
// the step, cmd/monolith/monolith.go:6398-6400 and 6415-6417) live in buffers
// that every rank maps through CUDA IPC, so the all-reduce is two plain kernels
// of peer loads and stores instead of a library collective:
//   k_peer_reduce   every rank signals "partials complete" (barrier B0) to all
//                   ranks, waits for all of theirs, then sums its own chunk of
//                   the n x d array over the ranks in rank order (q = 0, 1, ...),
//                   writing the sum in place; the last CTA to finish signals
//                   "chunk reduced" (barrier B1);
//   k_peer_gather   waits for B1 from every rank and copies the other ranks'
//                   reduced chunks into this rank's buffer.
// Each chunk is reduced once, by its owner, in a fixed order, so every rank
// ends with bit-identical sums.  Two buffers alternate between consecutive
// all-reduces: a rank writes buffer k%2 again only for all-reduce k+2, after
// every rank has signalled B0 of all-reduce k+1 and so has finished reading
// buffer k%2.  Barrier slots hold the all-reduce's epoch (monotonic), so they
// never need resetting.  Every wait is bounded (globaltimer); on expiry the
// kernel raises an error flag and returns, and the host reports SR_ETIMEOUT.
// Only plain loads (L2, not L1: __ldcg) and stores reach peer memory (no
// multicast, no TMA).
#pragma once

#include <cuda_runtime.h>

#include "tc_gemm.cuh"

namespace sr {
namespace peer {

constexpr int kMaxRanks = 64;
constexpr int kSlots = 2 * kMaxRanks;  // B0 slots, then B1 slots, one per source rank
constexpr int kThreads = 256;

struct Args {
  float* const* bufs;  // [size] this all-reduce's buffer of every rank (own one included)
  int* const* flags;   // [size] every rank's barrier slots
  int* counter;        // this rank's finished-CTA counter of k_peer_reduce
  int* err;
  int64_t count;       // floats in the n x d array (a multiple of 4)
  int64_t chunk;       // floats per rank (a multiple of 4)
  uint32_t epoch;
  int rank, size;
};

__device__ __forceinline__ void st_release_sys(int* p, int v) {
  asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ int ld_acquire_sys(const int* p) {
  int v;
  asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Thread q < size watches this rank's slot of barrier b for rank q.  Returns
// false for the whole block when a wait expired (or another one already did).
__device__ bool wait_all(const Args& a, int b) {
  __shared__ int failed;
  if (threadIdx.x == 0) failed = 0;
  __syncthreads();
  if (threadIdx.x < a.size) {
    const int* slot = a.flags[a.rank] + b * kMaxRanks + threadIdx.x;
    uint64_t t0 = 0;
    for (uint32_t it = 0;; it++) {
      if ((int)((uint32_t)ld_acquire_sys(slot) - a.epoch) >= 0) break;
      if ((it & 63) == 0) {
        if (*(volatile int*)a.err) {
          failed = 1;
          break;
        }
        const uint64_t now = tc::globaltimer();
        if (t0 == 0) t0 = now;
        else if (now - t0 > tc::kWaitNs) {
          atomicExch(a.err, 1);
          failed = 1;
          break;
        }
      }
    }
  }
  __syncthreads();
  return failed == 0;
}

__global__ void __launch_bounds__(kThreads) k_peer_reduce(Args a) {
  // B0: this rank's partials (written by earlier kernels on this stream) are
  // complete; tell every rank, including this one.
  if (blockIdx.x == 0 && threadIdx.x < a.size) {
    __threadfence_system();
    st_release_sys(a.flags[threadIdx.x] + a.rank, (int)a.epoch);
  }
  if (!wait_all(a, 0)) return;
  const int64_t lo = (int64_t)a.rank * a.chunk;
  const int64_t hi = min(a.count, lo + a.chunk);
  float4* own = (float4*)a.bufs[a.rank];
  for (int64_t i = lo / 4 + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < hi / 4;
       i += (int64_t)gridDim.x * blockDim.x) {
    float4 s = __ldcg((const float4*)a.bufs[0] + i);
    for (int q = 1; q < a.size; q++) {
      const float4 v = __ldcg((const float4*)a.bufs[q] + i);
      s.x += v.x;
      s.y += v.y;
      s.z += v.z;
      s.w += v.w;
    }
    own[i] = s;
  }
  // B1 once every CTA's sums are stored: the last CTA to count itself signals.
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned t = atomicAdd((unsigned*)a.counter, 1u);
    if (t == gridDim.x - 1) {
      atomicExch(a.counter, 0);
      __threadfence_system();
      for (int q = 0; q < a.size; q++) st_release_sys(a.flags[q] + kMaxRanks + a.rank, (int)a.epoch);
    }
  }
}

__global__ void __launch_bounds__(kThreads) k_peer_gather(Args a) {
  if (!wait_all(a, 1)) return;
  const int64_t c4 = a.chunk / 4;
  float4* own = (float4*)a.bufs[a.rank];
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < a.count / 4;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int q = (int)(i / c4);
    if (q != a.rank) own[i] = __ldcg((const float4*)a.bufs[q] + i);
  }
}

}  // namespace peer
}  // namespace sr
