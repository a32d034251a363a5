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

// ------------------------------------------------------------ LL protocol --
// The flags travel with the data: a 16-byte line holds two values, each next
// to the all-reduce's epoch ({v0, e, v1, e}), written by one 16-byte store
// and read by one 16-byte load, so a reader that sees both flags equal to the
// epoch also sees both values (the word-level flag scheme of NCCL's LL
// protocol).  No separate barrier: every consumer waits on the lines it reads.
__device__ __forceinline__ void st_line(uint4* p, uint4 v) {
  asm volatile("st.volatile.global.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}
__device__ __forceinline__ uint4 ld_line(const uint4* p) {
  uint4 v;
  asm volatile("ld.volatile.global.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p)
               : "memory");
  return v;
}
// Bounded wait for a line of epoch e.  After an expiry (here or anywhere:
// *err) the caller's ok turns false and no further line is waited for.
__device__ __forceinline__ uint4 wait_line(const uint4* p, uint32_t e, int* err, bool& ok) {
  uint64_t t0 = 0;
  for (uint32_t it = 0;; it++) {
    const uint4 v = ld_line(p);
    if ((v.y == e && v.w == e) || !ok) return v;
    if ((it & 63) == 0) {
      if (*(volatile int*)err) {
        ok = false;
        return v;
      }
      const uint64_t now = tc::globaltimer();
      if (t0 == 0) t0 = now;
      else if (now - t0 > tc::kWaitNs) {
        atomicExch(err, 1);
        ok = false;
        return v;
      }
    }
  }
}

struct LLArgs {
  const float* part;  // this rank's partial sums, count floats
  uint4* const* rb;   // [size] every rank's reduce buffer: [size source slots][chunk/2 lines]
  uint4* const* gb;   // [size] every rank's gather buffer: [count/2 lines]
  int* err;
  int64_t count, chunk;  // floats; both multiples of 4
  uint32_t epoch;
  int rank, size;
};

// The whole all-reduce in one kernel.  Line L of chunk q of this rank's
// partials goes to rank q's reduce buffer (slot = this rank); then this rank's
// own chunk is summed line by line over the slots in rank order (q = 0, 1, ...,
// the same order as k_peer_reduce) as the lines arrive, and each sum line goes
// to every rank's gather buffer.  A CTA pushes before it waits and every rank
// runs the same grid over the same lines, so no CTA waits on another CTA of its
// own GPU.  grid <= the resident CTAs (256 threads, no shared memory).
__global__ void __launch_bounds__(kThreads) k_peer_ll(LLArgs a) {
  const int64_t cl = a.chunk / 2;
  const int64_t t0 = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int q = 0; q < a.size; q++) {
    const int64_t lo = (int64_t)q * a.chunk;
    const int64_t nl = (min(a.count, lo + a.chunk) - lo) / 2;
    uint4* dst = a.rb[q] + (int64_t)a.rank * cl;
    for (int64_t L = t0; L < nl; L += stride) {
      const float2 v = *(const float2*)(a.part + lo + 2 * L);
      st_line(dst + L, make_uint4(__float_as_uint(v.x), a.epoch, __float_as_uint(v.y), a.epoch));
    }
  }
  const int64_t lo = (int64_t)a.rank * a.chunk;
  const int64_t nl = (min(a.count, lo + a.chunk) - lo) / 2;
  const uint4* src = a.rb[a.rank];
  bool ok = true;
  for (int64_t L = t0; L < nl; L += stride) {
    float s0 = 0.f, s1 = 0.f;
    for (int q = 0; q < a.size; q++) {
      const uint4 w = wait_line(src + (int64_t)q * cl + L, a.epoch, a.err, ok);
      if (q == 0) {
        s0 = __uint_as_float(w.x);
        s1 = __uint_as_float(w.z);
      } else {
        s0 += __uint_as_float(w.x);
        s1 += __uint_as_float(w.z);
      }
    }
    const uint4 line = make_uint4(__float_as_uint(s0), a.epoch, __float_as_uint(s1), a.epoch);
    for (int p = 0; p < a.size; p++) st_line(a.gb[p] + lo / 2 + L, line);
  }
}

// X += the all-reduced sums read from this rank's gather buffer (tp_add for
// the LL protocol: exact mode, and the last layer before the final norm).
__global__ void k_add_ll(float* __restrict__ X, const uint4* __restrict__ G, uint32_t epoch, int* err,
                         int64_t count) {
  bool ok = true;
  for (int64_t L = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; L < count / 2; L += (int64_t)gridDim.x * blockDim.x) {
    const uint4 w = wait_line(G + L, epoch, err, ok);
    X[2 * L] += __uint_as_float(w.x);
    X[2 * L + 1] += __uint_as_float(w.z);
  }
}

}  // namespace peer
}  // namespace sr
