// tc_gemm.cuh -- SR_MODE_FAST projections on the 5th-generation tensor cores.
//
// Y[n, out] = X[n, in] W[out, in]^T for Q8/Q4 weights (linearQ8Into / linearQ4Into,
// cmd/monolith/monolith.go:4074-4511) restated for tcgen05:
//   * W's integer codes are held as bf16 (exact: |q| <= 127) in a shadow copy
//     laid out as contiguous 32 KiB (256-feature, 64-column) tiles that are
//     already in the MMA's 128-byte-swizzled shared-memory order, so each
//     weight tile is one bulk copy (a few DRAM pages, not 256 strided rows);
//     the fp32 activations are split into bf16 hi + lo planes, so each 64-column
//     block's partial sum  sum_j x_j q_j  is formed by two MMA passes with fp32
//     accumulation in TMEM (relative error ~2^-16 per term);
//   * "swap AB": the 128-row MMA M dimension runs over output features, N over
//     step rows, so a thread of the epilogue owns one output feature and its
//     per-block scale (the reference's s += p*scale) is a scalar FMA on
//     registers after each block's accumulator is read from TMEM;
//   * a CTA computes 256 output features (two M=128 MMA halves sharing each
//     activation tile) for one 128-row tile of the step; TMA (SWIZZLE_128B)
//     feeds a 3-stage mbarrier pipeline of 64 KiB stages; one thread issues
//     MMAs; TMEM holds two accumulator buffers so block b+1's MMAs overlap
//     block b's epilogue;
//   * persistent stream-K schedule: the (256-feature tile, 64-column block)
//     units of the matrix are cut into one contiguous range per group of CTAs
//     (a group holds one CTA per 128-row tile, so the CTAs that read the same
//     weight tile run together and share it in L2); the pipeline runs through
//     tile boundaries without refilling.  A tile whose blocks span several
//     groups leaves one partial sum per group, and k_sk_reduce adds them in
//     block order (deterministic) and applies the epilogue.
// Every mbarrier wait is bounded (globaltimer); on expiry the kernel records an
// error flag, stops waiting and finishes, and the host reports SR_ETIMEOUT.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>

#include "common.cuh"

namespace sr {
namespace tc {

constexpr int kM = 128;          // output features per MMA (MMA M)
constexpr int kMH = 2;           // MMA halves per CTA: a CTA owns kMC = 256 output features
constexpr int kMC = kM * kMH;
constexpr int kN = 128;          // step rows per tile (MMA N)
constexpr int kKB = 64;          // K per block (one scale block, one 128-byte bf16 row)
constexpr int kStages = 3;
constexpr int kAcc = 2;          // TMEM accumulator buffers, each kMH*kN columns (512 in all)
static_assert(kAcc == 2, "the epilogue indexes TMEM buffers as i & 1");
constexpr int kThreads = 320;    // warp 0: TMA, warp 1: MMA, warps 2-9: epilogue
constexpr int kEpiWarps = 8;     // lane quarter (warp % 4) x MMA half ((warp - 2) / 4)
constexpr int kEpiWarp0 = 2;
constexpr uint32_t kTileA = kMC * kKB * 2;  // 32 KiB of weight codes
constexpr uint32_t kTileB = kN * kKB * 2;   // 16 KiB per activation plane
constexpr uint32_t kStageBytes = kTileA + 2 * kTileB;
constexpr size_t kSmemBytes = (size_t)kStages * kStageBytes + 1024 /*align*/ + 256 /*barriers, flags*/;
constexpr uint64_t kWaitNs = 2000000000ull;  // 2 s per wait, then abort

struct Segment {
  int32_t rows;        // output features in this segment
  int32_t ldy;
  float* y;
  const float* bias;
  const float* resid;  // may alias y
};

struct GemmArgs {
  const uint8_t* wt;  // tiled weight codes: tile (m, kb) at (m * groups + kb) * kTileA bytes
  int n;             // step rows
  int out;           // total output features (sum of segment rows)
  int in;            // K
  int groups;        // ceil(in/64) scale blocks per output row
  int mt, nt;        // 256-feature tiles, 128-row tiles
  int ngroups;       // stream-K groups (nt CTAs each); grid = ngroups * nt
  const float* scales;   // [out][groups] (concatenated for fused segments)
  float* partial;        // [ngroups*nt][2][kN][kMC] partial tiles (first / last segment of a CTA)
  const int32_t* out_map;  // compacted head rows -> destination row (never combined with a residual)
  Segment seg[3];
  int nseg;
  int* err;
  int fmt;  // kQ8 or kQ4: the code format k_gemm_direct reads (tc_gemm_direct.cuh)
};

// Stream-K range of group g over the mt*groups (tile, block) units.  32-bit
// arithmetic: g, ngroups <= 148 and units < 2^24 (checked on the host).
__host__ __device__ inline int sk_begin(int g, int units, int ngroups) {
  return (int)((unsigned)(g * units) / (unsigned)ngroups);
}
__host__ __device__ inline int sk_group_of(int u, int units, int ngroups) {
  int g = (int)((unsigned)(u * ngroups) / (unsigned)units);
  while (g + 1 < ngroups && sk_begin(g + 1, units, ngroups) <= u) g++;
  while (g > 0 && sk_begin(g, units, ngroups) > u) g--;
  return g;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
// Bounded parity wait.  Returns false (and raises *err) when it expires or
// when another thread already raised the error.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* err) {
  const uint32_t addr = smem_u32(bar);
  uint64_t t0 = 0;
  for (uint32_t it = 0;; it++) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(addr), "r"(parity)
        : "memory");
    if (done) return true;
    if ((it & 63) == 0) {
      if (*(volatile int*)err) return false;
      const uint64_t now = globaltimer();
      if (t0 == 0) t0 = now;
      else if (now - t0 > kWaitNs) {
        atomicExch(err, 1);
        return false;
      }
    }
  }
}
// Contiguous global -> shared bulk copy completing on an mbarrier (16-byte
// aligned addresses, size a multiple of 16).
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          smem_u32(dst)),
      "l"(map), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}
// Bring [p, p + bytes) into L2 (a hint: no shared memory, no barrier).
__device__ __forceinline__ void prefetch_l2(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}
// The per-block scales of 256-feature tile m (contiguous: rows m*256.. of a
// [out][groups] array), so that the epilogue's scale loads hit L2.
__device__ __forceinline__ void prefetch_tile_scales(const GemmArgs& a, int m) {
  if (m >= a.mt) return;
  const int rows = min(kMC, a.out - m * kMC);
  const uint32_t bytes = ((uint32_t)rows * a.groups * 4u) & ~15u;  // bulk sizes are multiples of 16
  if (bytes) prefetch_l2(a.scales + (int64_t)m * kMC * a.groups, bytes);
}
// K-major, SWIZZLE_128B shared-memory matrix descriptor (rows of 128 bytes,
// 8-row groups 1024 bytes apart).
__device__ __forceinline__ uint64_t sw128_desc(const void* tile) {
  const uint64_t addr = smem_u32(tile);
  uint64_t d = (addr >> 4) & 0x3FFFull;
  d |= 1ull << 16;                // leading byte offset (unused for swizzled K-major)
  d |= (uint64_t)(1024 >> 4) << 32;  // stride byte offset
  d |= 1ull << 46;                // descriptor version
  d |= 2ull << 61;                // SWIZZLE_128B
  return d;
}
// kind::f16 instruction descriptor: bf16 x bf16 -> f32, both K-major.
__host__ __device__ constexpr uint32_t idesc_bf16(int m, int n) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}
__device__ __forceinline__ void umma_bf16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(0), "r"(0), "r"(0), "r"(0));
}
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,"
      "%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
        "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]), "=r"(v[16]),
        "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]),
        "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
        "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
      : "r"(taddr));
}
// Wait for this thread's outstanding TMEM loads.  The registers of the load
// being waited for are in/out operands, so no use of them can be scheduled
// before the wait.
__device__ __forceinline__ void tmem_wait_ld16(uint32_t (&v)[16]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(v[0]), "+r"(v[1]), "+r"(v[2]), "+r"(v[3]), "+r"(v[4]), "+r"(v[5]), "+r"(v[6]), "+r"(v[7]),
                 "+r"(v[8]), "+r"(v[9]), "+r"(v[10]), "+r"(v[11]), "+r"(v[12]), "+r"(v[13]), "+r"(v[14]), "+r"(v[15])
               :
               : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Output column of feature o: its segment's destination, stride, bias and
// residual, resolved once per thread.
struct OutCol {
  float* y;
  const float* resid;
  float bias;
  int ldy;
  bool has_bias;
};
__device__ __forceinline__ OutCol out_col(const GemmArgs& a, int o) {
  // constant indices into a.seg (a dynamic index would copy it to local memory)
  const int r0 = a.seg[0].rows, r1 = a.seg[1].rows;
  const int s = (a.nseg > 1 && o >= r0) ? ((a.nseg > 2 && o >= r0 + r1) ? 2 : 1) : 0;
  const Segment& g = s == 0 ? a.seg[0] : (s == 1 ? a.seg[1] : a.seg[2]);
  const int ol = o - (s == 0 ? 0 : (s == 1 ? r0 : r0 + r1));
  OutCol c;
  c.y = g.y + ol;
  c.resid = g.resid ? g.resid + ol : nullptr;
  c.has_bias = g.bias != nullptr;
  c.bias = g.bias ? g.bias[ol] : 0.f;
  c.ldy = g.ldy;
  return c;
}

// grid: ngroups * nt CTAs, one per SM (197 KiB of shared memory each).
__global__ void __launch_bounds__(kThreads, 1)
k_gemm_q(const __grid_constant__ CUtensorMap tm_xh, const __grid_constant__ CUtensorMap tm_xl, GemmArgs a) {
  extern __shared__ __align__(1024) uint8_t gsm_raw[];
  uint8_t* gsm = (uint8_t*)(((uintptr_t)gsm_raw + 1023) & ~(uintptr_t)1023);
  uint64_t* full = (uint64_t*)(gsm + kStages * kStageBytes);
  uint64_t* empty = full + kStages;
  uint64_t* tfull = empty + kStages;
  uint64_t* tempty = tfull + kAcc;
  uint32_t* tmem_slot = (uint32_t*)(tempty + kAcc);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = blockIdx.x / a.nt, j = blockIdx.x % a.nt;  // stream-K group, row tile
  const int K = a.groups;
  const int units = a.mt * K;
  const int ub = sk_begin(g, units, a.ngroups), ue = sk_begin(g + 1, units, a.ngroups);
  const int nu = ue - ub;
  const int m_first = ub / K, kb_first = ub - m_first * K;
  const int n0 = j * kN;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < kAcc; b++) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], kEpiWarps);  // one arrive per epilogue warp
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {  // one warp allocates kAcc*kMH*kN TMEM columns
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(kAcc * kMH * kN));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {  // TMA producer
      // The epilogue reads one scale per unit right before its FMAs: bring
      // each tile's scales (and the next tile's) into L2 when the tile starts.
      if (nu > 0) prefetch_tile_scales(a, m_first);
      int m = m_first, kb = kb_first;
      for (int i = 0; i < nu; i++, kb = (kb + 1 == K) ? 0 : kb + 1, m += (kb == 0) ? 1 : 0) {
        if (i == 0 || kb == 0) prefetch_tile_scales(a, m + 1);
        const int s = i % kStages, use = i / kStages;
        if (use > 0 && !mbar_wait(&empty[s], (use - 1) & 1, a.err)) break;
        uint8_t* st = gsm + s * kStageBytes;
        mbar_expect_tx(&full[s], kStageBytes);
        bulk_load(st, a.wt + ((int64_t)m * K + kb) * kTileA, kTileA, &full[s]);
        tma_load_2d(st + kTileA, &tm_xh, &full[s], kb * kKB, n0);
        tma_load_2d(st + kTileA + kTileB, &tm_xl, &full[s], kb * kKB, n0);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {  // MMA issuer
      const uint32_t idesc = idesc_bf16(kM, kN);
      for (int i = 0; i < nu; i++) {
        const int s = i % kStages, b = i % kAcc;
        if (!mbar_wait(&full[s], (i / kStages) & 1, a.err)) break;
        if (i >= kAcc && !mbar_wait(&tempty[b], ((i / kAcc) - 1) & 1, a.err)) break;
        tc_fence_after();
        const uint8_t* st = gsm + s * kStageBytes;
        const uint64_t dh = sw128_desc(st + kTileA), dl = sw128_desc(st + kTileA + kTileB);
#pragma unroll
        for (int h = 0; h < kMH; h++) {
          const uint64_t da = sw128_desc(st + h * (kTileA / kMH));
          const uint32_t td = tmem + b * (kMH * kN) + h * kN;
#pragma unroll
          for (int k = 0; k < kKB / 16; k++) umma_bf16(td, da + 2 * k, dh + 2 * k, idesc, k > 0 ? 1u : 0u);
#pragma unroll
          for (int k = 0; k < kKB / 16; k++) umma_bf16(td, da + 2 * k, dl + 2 * k, idesc, 1u);
        }
        umma_commit(&empty[s]);
        umma_commit(&tfull[b]);
      }
    }
  } else {  // epilogue warps 2..9: TMEM lane quarter = warp % 4, MMA half = (warp - 2) / 4
    // After an expired wait the warp only skips the TMEM reads.  The loops
    // keep little state besides acc[] so that it stays in registers.
    const int q = warp & 3, h = (warp - kEpiWarp0) >> 2;
    const int f = h * kM + q * 32 + lane;  // feature within the tile
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
        const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16) + b * (kMH * kN) + h * kN;
        // Two 16-column register sets: the load of the next set is in flight
        // while the FMAs consume the current one.
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
          } else {  // buffer fully read: hand it back before the last FMAs
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tempty[b]);
          }
#pragma unroll
          for (int jj = 0; jj < 16; jj++) acc[c + 16 + jj] = fmaf(__uint_as_float(vb[jj]), sc, acc[c + 16 + jj]);
          if (c + 32 < kN) tmem_wait_ld16(va);
        }
      }
      if (kb != K - 1 && i != nu - 1) continue;
      const int kb_e = kb;
      // ---- the group's segment of tile (m, j) ends here.  A whole tile that
      // needs only a bias goes straight to the output; every other segment
      // goes to this CTA's partial slot (first segment: 0, later ones: 1) for
      // k_sk_reduce.  (This store shape keeps acc[] in registers: a per-element
      // select of the bias, or a dynamic row bound inside the loop, did not.)
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
        dst = a.partial + ((int)blockIdx.x * 2 + ((m == m_first) ? 0 : 1)) * kN * kMC + f;
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
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kAcc * kMH * kN));
  }
}

// Tiles a stream-K launch left in partial slots (split tiles, and whole tiles
// that need the residual or the head row map): out[row][o] = the groups'
// partials added in block order, then bias / residual / head row map.
// grid (tiles*nt, kN/kRedBlockRows), block kMC threads (one output feature
// each) over kRedBlockRows rows in chunks of kRedRows.
// by_boundary: blockIdx.x / nt is a group boundary b (1..ngroups-1) and the
// block finishes the tile it cuts (once per tile: at its first inner
// boundary); otherwise blockIdx.x / nt is the tile.  The partials of up to 8
// groups for a chunk are loaded before any add.
constexpr int kRedRows = 8;
constexpr int kRedBlockRows = 32;
__global__ void __launch_bounds__(kMC, 2) k_sk_reduce(GemmArgs a, int by_boundary) {
  const int K = a.groups, units = a.mt * K;
  const int j = blockIdx.x % a.nt;
  int m = blockIdx.x / a.nt;
  if (by_boundary) {
    const int bnd = m + 1, u = sk_begin(bnd, units, a.ngroups);
    m = u / K;
    if (u == m * K) return;                                              // boundary on a tile edge
    if (bnd > 1 && sk_begin(bnd - 1, units, a.ngroups) > m * K) return;  // tile owned by an earlier boundary
  }
  const int gf = sk_group_of(m * K, units, a.ngroups), gl = sk_group_of(m * K + K - 1, units, a.ngroups);
  const int f = threadIdx.x, o = m * kMC + f;
  const int n0 = j * kN;
  if (o >= a.out) return;
  const OutCol oc = out_col(a, o);
  if (gf == gl && !oc.resid && !a.out_map) return;  // the GEMM stored this tile
  const int ns = gl - gf + 1;
  int off[8];  // partial slot of each group (first segment of a group: slot 0)
#pragma unroll
  for (int q = 0; q < 8; q++) {
    const int gs = min(gf + q, gl);
    const int sl = (sk_begin(gs, units, a.ngroups) / K == m) ? 0 : 1;
    off[q] = ((gs * a.nt + j) * 2 + sl) * kN * kMC + f;
  }
  for (int r0 = blockIdx.y * kRedBlockRows; r0 < (int)(blockIdx.y + 1) * kRedBlockRows && n0 + r0 < a.n;
       r0 += kRedRows) {
    float v[kRedRows];
#pragma unroll
    for (int jj = 0; jj < kRedRows; jj++) v[jj] = 0.f;
    if (ns <= 8) {
      float p[8][kRedRows];
#pragma unroll
      for (int q = 0; q < 8; q++)
#pragma unroll
        for (int jj = 0; jj < kRedRows; jj++) p[q][jj] = (q < ns) ? __ldcg(a.partial + off[q] + (r0 + jj) * kMC) : 0.f;
#pragma unroll
      for (int q = 0; q < 8; q++)
#pragma unroll
        for (int jj = 0; jj < kRedRows; jj++)
          if (q < ns) v[jj] += p[q][jj];
    } else {
      for (int gs = gf; gs <= gl; gs++) {
        const int sl = (sk_begin(gs, units, a.ngroups) / K == m) ? 0 : 1;
        const float* P = a.partial + ((gs * a.nt + j) * 2 + sl) * kN * kMC + r0 * kMC + f;
#pragma unroll
        for (int jj = 0; jj < kRedRows; jj++) v[jj] += __ldcg(P + jj * kMC);
      }
    }
    float pre[kRedRows];
#pragma unroll
    for (int jj = 0; jj < kRedRows; jj++) {
      const int row = n0 + r0 + jj;
      pre[jj] = 0.f;
      if (row < a.n) {
        if (a.out_map) pre[jj] = __int_as_float(a.out_map[row]);
        else if (oc.resid) pre[jj] = oc.resid[(int64_t)row * oc.ldy];
      }
    }
#pragma unroll
    for (int jj = 0; jj < kRedRows; jj++) {
      const int row = n0 + r0 + jj;
      if (row < a.n) {
        const int64_t orow = a.out_map ? (int64_t)__float_as_int(pre[jj]) : (int64_t)row;
        float x = v[jj];
        if (oc.has_bias) x += oc.bias;
        if (oc.resid) x = pre[jj] + x;
        oc.y[orow * oc.ldy] = x;
      }
    }
  }
}

// fp32 activations -> bf16 hi/lo planes: x ~= hi + lo, |x - hi - lo| <= 2^-17 |x|.
__global__ void k_split_bf16(const float* __restrict__ X, int n, int in, __nv_bfloat16* __restrict__ H,
                             __nv_bfloat16* __restrict__ Lo) {
  const int64_t total = (int64_t)n * in;
  for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
    const float x = X[t];
    const __nv_bfloat16 h = __float2bfloat16_rn(x);
    H[t] = h;
    Lo[t] = __float2bfloat16_rn(x - __bfloat162float(h));
  }
}

// Integer codes of a Q8/Q4 matrix as bf16 (exact) in the tiled, swizzled
// shadow layout: row r (of a fused matrix, this part starting at row0) and
// 16-byte chunk c (columns 8c..8c+7 of block kb) of tile m = r / 256 go to
// byte ((m * groups + kb) * 256 + r % 256) * 128 + ((c ^ (r % 8)) * 16).
// Columns past cols are written as zero; the caller zeroes rows past the end.
__global__ void k_codes_tiled(const void* __restrict__ values, int fmt, int rows, int cols, int row0, int groups,
                              uint8_t* __restrict__ dst) {
  const int64_t chunks = (int64_t)rows * groups * 8;
  for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < chunks; t += (int64_t)gridDim.x * blockDim.x) {
    const int rl = (int)(t / (groups * 8)), cc = (int)(t % (groups * 8));
    const int kb = cc >> 3, c = cc & 7;
    const int r = row0 + rl, m = r / kMC, rr = r % kMC;
    __align__(16) __nv_bfloat16 v[8];
#pragma unroll
    for (int e = 0; e < 8; e++) {
      const int col = kb * kKB + c * 8 + e;
      float q = 0.f;
      if (col < cols) {
        if (fmt == kQ8) {
          q = (float)((const int8_t*)values)[(int64_t)rl * cols + col];
        } else {
          const uint32_t b = ((const uint8_t*)values)[(int64_t)rl * ((cols + 1) / 2) + col / 2];
          q = (col & 1) ? q4_hi(b) : q4_lo(b);
        }
      }
      v[e] = __float2bfloat16_rn(q);
    }
    const int64_t off = (((int64_t)m * groups + kb) * kMC + rr) * 128 + (int64_t)((c ^ (rr & 7)) * 16);
    *(uint4*)(dst + off) = *(const uint4*)v;
  }
}

}  // namespace tc
}  // namespace sr
