// tc_gemm2.cuh -- the tensor-core projection on pairs of SMs (tcgen05
// cta_group::2), for steps of more than 128 rows with the bf16 code cache.
//
// Same arithmetic, stream-K schedule, epilogue and partial-tile layout as
// k_gemm_q (tc_gemm.cuh); what changes is the MMA shape.  A cluster of two
// CTAs on two SMs owns a 256-feature x 256-row tile:
//   * CTA r (rank in the pair) loads the weight tile's features r*128..+127
//     (16 KiB of the cache's pre-swizzled 32 KiB tile) and the activation rows
//     r*128..+127 of the hi and lo planes (16 KiB each), all by TMA, with
//     completion signalled on the first CTA's ("leader's") stage barrier;
//   * one thread of the leader issues M=256 x N=256 x K=16 MMAs: each SM's
//     tensor core reads its own weight half and both SMs' activation halves,
//     so each SM supplies half of every activation tile from its shared
//     memory instead of all of it (k_gemm_q's 256-feature MMA pair reads each
//     activation slice twice from one SM), which is the shared-memory
//     bandwidth k_gemm_q is bound by;
//   * each CTA's TMEM holds its 128 features x 256 rows (two such buffers);
//     its 8 epilogue warps read them as k_gemm_q's do (lane quarter x row
//     half), apply the per-block scales and store whole tiles or write the
//     1-SM partial slots (row tile 2*j + half) that k_sk_reduce adds.
// The commit that frees a stage or fills an accumulator arrives on both CTAs'
// barriers (multicast commit); the epilogue warps of both CTAs arrive on the
// leader's accumulator-free barrier.  No load is multicast: every CTA loads
// its own halves.  Every wait is bounded (tc_gemm.cuh's mbar_wait).
#pragma once

#include "tc_gemm.cuh"

namespace sr {
namespace tc {

constexpr int kN2 = 256;          // step rows per pair tile (MMA N)
constexpr int kStages2 = 4;
constexpr uint32_t kTileA2 = kM * kKB * 2;   // 16 KiB: this CTA's 128 features of the weight tile
constexpr uint32_t kStageBytes2 = kTileA2 + 2 * kTileB;  // + its 128 rows of the hi and lo planes
constexpr size_t kSmemBytes2 = (size_t)kStages2 * kStageBytes2 + 1024 /*align*/ + 256 /*barriers, slot*/;
static_assert(kAcc * kN2 == 512, "two 256-column accumulators fill TMEM");

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// shared::cluster address of the same shared variable in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t cluster_addr(const void* p, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
  return r;
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// TMA tile load into this CTA's shared memory, completing on a barrier that
// may be the pair's other CTA's (cta_group::2; no multicast).
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* map, uint32_t bar_cluster, int c0,
                                                 int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], "
      "[%2];" ::"r"(smem_u32(dst)),
      "l"(map), "r"(bar_cluster), "r"(c0), "r"(c1)
      : "memory");
}
__device__ __forceinline__ void umma_bf16_pair(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                               uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, {%5, %5, %5, %5, %5, %5, %5, %5}, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(0));
}
// Arrive (once) on the barrier at this shared offset in both CTAs of the pair
// when the MMAs issued so far have completed.
__device__ __forceinline__ void umma_commit_pair(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          smem_u32(bar)),
      "h"((uint16_t)3)
      : "memory");
}
// Arrive on a barrier of either CTA of the pair (default .release.cta
// semantics: the arrival only hands back a TMEM buffer, whose reads the
// caller ordered with tcgen05.fence::before_thread_sync; a cluster-scope
// release would make every epilogue warp wait for its earlier global stores).
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t bar_cluster) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(bar_cluster) : "memory");
}

// grid: ngroups * nt2 clusters of 2 CTAs (cluster dims 2), one CTA per SM.
// a.nt is the number of 128-row tiles (2 per pair tile), as k_sk_reduce reads it.
__global__ void __launch_bounds__(kThreads, 1)
k_gemm_q2(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_xh,
          const __grid_constant__ CUtensorMap tm_xl, GemmArgs a) {
  extern __shared__ __align__(1024) uint8_t gsm2_raw[];
  uint8_t* gsm = (uint8_t*)(((uintptr_t)gsm2_raw + 1023) & ~(uintptr_t)1023);
  uint64_t* full = (uint64_t*)(gsm + kStages2 * kStageBytes2);
  uint64_t* empty = full + kStages2;
  uint64_t* tfull = empty + kStages2;
  uint64_t* tempty = tfull + kAcc;
  uint32_t* tmem_slot = (uint32_t*)(tempty + kAcc);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const int nt2 = a.nt / 2;
  const int pair = blockIdx.x >> 1;
  const int g = pair / nt2, j2 = pair % nt2;  // stream-K group, 256-row tile
  const int K = a.groups;
  const int units = a.mt * K;
  const int ub = sk_begin(g, units, a.ngroups), ue = sk_begin(g + 1, units, a.ngroups);
  const int nu = ue - ub;
  const int m_first = ub / K, kb_first = ub - m_first * K;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages2; s++) {
      mbar_init(&full[s], 1);   // the leader's producer (expect_tx for both CTAs' bytes)
      mbar_init(&empty[s], 1);  // the MMA commit
    }
    for (int b = 0; b < kAcc; b++) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 2 * kEpiWarps);  // the epilogue warps of both CTAs
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {  // the same warp of both CTAs allocates the pair's TMEM
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(kAcc * kN2));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
  }
  tc_fence_before();
  cluster_sync();  // both CTAs' barriers are initialised before either signals the other's
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {  // TMA producer of this CTA's halves
      if (nu > 0) prefetch_tile_scales(a, m_first);
      int m = m_first, kb = kb_first;
      for (int i = 0; i < nu; i++, kb = (kb + 1 == K) ? 0 : kb + 1, m += (kb == 0) ? 1 : 0) {
        if (i == 0 || kb == 0) prefetch_tile_scales(a, m + 1);
        const int s = i % kStages2, use = i / kStages2;
        if (use > 0 && !mbar_wait(&empty[s], (use - 1) & 1, a.err)) break;
        uint8_t* st = gsm + s * kStageBytes2;
        const uint32_t bar = cluster_addr(&full[s], 0);
        if (rank == 0) mbar_expect_tx(&full[s], 2 * kStageBytes2);
        tma_load_2d_pair(st, &tm_w, bar, 0, (m * K + kb) * kMC + (int)rank * kM);
        tma_load_2d_pair(st + kTileA2, &tm_xh, bar, kb * kKB, j2 * kN2 + (int)rank * kN);
        tma_load_2d_pair(st + kTileA2 + kTileB, &tm_xl, bar, kb * kKB, j2 * kN2 + (int)rank * kN);
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && rank == 0) {  // MMA issuer for the pair
      const uint32_t idesc = idesc_bf16(2 * kM, kN2);
      for (int i = 0; i < nu; i++) {
        const int s = i % kStages2, b = i % kAcc;
        if (!mbar_wait(&full[s], (i / kStages2) & 1, a.err)) break;
        if (i >= kAcc && !mbar_wait(&tempty[b], ((i / kAcc) - 1) & 1, a.err)) break;
        tc_fence_after();
        const uint8_t* st = gsm + s * kStageBytes2;
        const uint64_t da = sw128_desc(st), dh = sw128_desc(st + kTileA2), dl = sw128_desc(st + kTileA2 + kTileB);
        const uint32_t td = tmem + b * kN2;
#pragma unroll
        for (int k = 0; k < kKB / 16; k++) umma_bf16_pair(td, da + 2 * k, dh + 2 * k, idesc, k > 0 ? 1u : 0u);
#pragma unroll
        for (int k = 0; k < kKB / 16; k++) umma_bf16_pair(td, da + 2 * k, dl + 2 * k, idesc, 1u);
        umma_commit_pair(&empty[s]);
        umma_commit_pair(&tfull[b]);
      }
    }
  } else {  // epilogue warps 2..9: TMEM lane quarter = warp % 4, row half = (warp - 2) / 4
    const int q = warp & 3, h = (warp - kEpiWarp0) >> 2;
    const int f = (int)rank * kM + q * 32 + lane;  // feature within the 256-feature tile
    const int n0 = j2 * kN2 + h * kN;               // first step row of this warp's accumulator half
    const int jt = 2 * j2 + h;                      // its 128-row tile (partial-slot layout of k_gemm_q)
    const uint32_t tempty_leader[2] = {cluster_addr(&tempty[0], 0), cluster_addr(&tempty[1], 0)};
    bool ok = true;
    float acc[kN];
#pragma unroll
    for (int jj = 0; jj < kN; jj++) acc[jj] = 0.f;
    int kb_s = kb_first;
    int m = m_first, kb = kb_first;
    for (int i = 0; i < nu; i++, kb = (kb + 1 == K) ? 0 : kb + 1, m += (kb == 0) ? 1 : 0) {
      const int b = i & 1;
      const int o = m * kMC + f;
      if (kb == 0) kb_s = 0;
      const float sc = a.scales[(int64_t)min(o, a.out - 1) * K + kb];
      ok = ok && mbar_wait(&tfull[b], (i >> 1) & 1, a.err);
      if (ok) {
        tc_fence_after();
        const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16) + b * kN2 + h * kN;
        uint32_t va[16], vb[16];
        tmem_ld16(taddr, va);
        tmem_wait_ld16(va);
#pragma unroll
        for (int c = 0; c < kN; c += 32) {
          tmem_ld16(taddr + c + 16, vb);
#pragma unroll
          for (int jj = 0; jj < 16; jj++) acc[c + jj] = fmaf(__uint_as_float(va[jj]), sc, acc[c + jj]);
          tmem_wait_ld16(vb);
          if (c + 32 < kN) {
            tmem_ld16(taddr + c + 32, va);
          } else {  // buffer fully read: hand it back (to the leader's barrier) before the last FMAs
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(tempty_leader[b]);
          }
#pragma unroll
          for (int jj = 0; jj < 16; jj++) acc[c + 16 + jj] = fmaf(__uint_as_float(vb[jj]), sc, acc[c + 16 + jj]);
          if (c + 32 < kN) tmem_wait_ld16(va);
        }
      }
      if (kb != K - 1 && i != nu - 1) continue;
      const int kb_e = kb;
      // ---- this group's segment of tile m ends here: as in k_gemm_q.
      const bool whole = (kb_s == 0 && kb_e == K - 1);
      bool direct = false;
      float* dst;
      int ld;
      bool hb = false;
      float bias = 0.f;
      if (whole && o < a.out) {
        const OutCol oc = out_col(a, o);
        direct = !oc.resid && !a.out_map;
        if (direct) {
          dst = oc.y + (int64_t)n0 * oc.ldy;
          ld = oc.ldy;
          hb = oc.has_bias;
          bias = oc.bias;
        }
      }
      if (!direct) {
        dst = a.partial + (((int64_t)g * a.nt + jt) * 2 + ((m == m_first) ? 0 : 1)) * kN * kMC + f;
        ld = kMC;
      }
      const bool write = direct || !whole || o < a.out;
      const int nr = write ? min(kN, a.n - n0) : 0;
      if (hb) {
#pragma unroll
        for (int jj = 0; jj < kN; jj++) acc[jj] += bias;
      }
#pragma unroll
      for (int jj = 0; jj < kN; jj++) {
        if (jj < nr) dst[jj * ld] = acc[jj];
        acc[jj] = 0.f;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // neither CTA leaves while the pair's MMAs or barriers may still touch its shared memory
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kAcc * kN2));
  }
}

}  // namespace tc
}  // namespace sr
