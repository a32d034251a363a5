// tc_gemm_direct.cuh -- the tensor-core projection without the bf16 code
// cache: k_gemm_q (tc_gemm.cuh) with the A operand supplied from the
// reference's own storage (Param, cmd/monolith/monolith.go:3784-3850).
//
//   * the int8 codes [out, in] (or packed nibbles [out, ceil(in/2)]) of one
//     256-feature tile and one 64-column scale block are loaded by 4 TMA boxes
//     of 64 rows from per-parameter tensor maps (so fused Q|K|V and gate|up
//     need only 64-row segment boundaries), kRawSlots tiles in flight, one unit
//     ahead of the activation planes;
//   * two converter warps widen them to bf16 (exact: |q| <= 127; a byte permute
//     places the biased code in a float's mantissa and one subtraction removes
//     the bias) in the MMA's 128-byte swizzled K-major layout, into one of two A
//     tiles;
//   * MMA, epilogue, stream-K schedule and k_sk_reduce are k_gemm_q's.
// It needs no device memory beyond the model's own codes, but moves about 224
// KiB through shared memory per (256-feature, 128-row, 64-column) unit against
// k_gemm_q's 192 KiB (the widening reads 16 and writes 32 KiB), so it runs
// slower; the step uses it when the code cache is off or does not fit.
#pragma once

#include "tc_gemm.cuh"

namespace sr {
namespace tc {

constexpr int kDirRawSlots = 4;   // code tiles in flight
constexpr int kDirBSlots = 3;     // activation tiles in flight
constexpr int kDirASlots = 2;     // widened A tiles
constexpr int kDirConvWarps = 2;  // warps 2-3; epilogue warps 4-11
constexpr int kDirEpiWarp0 = 4;
constexpr int kDirThreads = (kDirEpiWarp0 + kEpiWarps) * 32;
constexpr int kDirSub = 64;  // weight rows per TMA box
constexpr uint32_t kDirRaw = kMC * kKB;  // 16 KiB of int8 codes (Q4: half)
constexpr uint32_t kDirB = 2 * kTileB;   // hi + lo planes of one unit
constexpr size_t kDirSmemBytes = (size_t)kDirBSlots * kDirB + (size_t)kDirASlots * kTileA +
                                 (size_t)kDirRawSlots * kDirRaw + 1024 /*align*/ + 256 /*barriers*/;

// Layout from the 1024-byte aligned base: B slots (1024-aligned, for the
// swizzle), A slots, code slots, then the barriers.
struct DirSmem {
  uint8_t* base;
  __device__ __forceinline__ uint8_t* btile(int s) const { return base + s * kDirB; }
  __device__ __forceinline__ uint8_t* atile(int b) const { return base + kDirBSlots * kDirB + b * kTileA; }
  __device__ __forceinline__ uint8_t* raw(int r) const {
    return base + kDirBSlots * kDirB + kDirASlots * kTileA + r * kDirRaw;
  }
  __device__ __forceinline__ uint64_t* bar(int i) const {
    return (uint64_t*)(base + kDirBSlots * kDirB + kDirASlots * kTileA + kDirRawSlots * kDirRaw) + i;
  }
  __device__ __forceinline__ uint64_t* rfull(int r) const { return bar(r); }
  __device__ __forceinline__ uint64_t* rempty(int r) const { return bar(kDirRawSlots + r); }
  __device__ __forceinline__ uint64_t* bfull(int s) const { return bar(2 * kDirRawSlots + s); }
  __device__ __forceinline__ uint64_t* bempty(int s) const { return bar(2 * kDirRawSlots + kDirBSlots + s); }
  __device__ __forceinline__ uint64_t* afull(int b) const { return bar(2 * kDirRawSlots + 2 * kDirBSlots + b); }
  __device__ __forceinline__ uint64_t* aempty(int b) const {
    return bar(2 * kDirRawSlots + 2 * kDirBSlots + kDirASlots + b);
  }
  __device__ __forceinline__ uint64_t* tfull(int b) const {
    return bar(2 * kDirRawSlots + 2 * kDirBSlots + 2 * kDirASlots + b);
  }
  __device__ __forceinline__ uint64_t* tempty(int b) const {
    return bar(2 * kDirRawSlots + 2 * kDirBSlots + 2 * kDirASlots + kAcc + b);
  }
  __device__ __forceinline__ uint32_t* tmem_slot() const {
    return (uint32_t*)bar(2 * kDirRawSlots + 2 * kDirBSlots + 2 * kDirASlots + 2 * kAcc);
  }
};
__device__ __forceinline__ DirSmem dir_smem() {
  extern __shared__ __align__(1024) uint8_t gsm_raw[];
  return DirSmem{(uint8_t*)(((uintptr_t)gsm_raw + 1023) & ~(uintptr_t)1023)};
}

// Integer codes -> bf16, exactly: the biased code (q + 128 for Q8, q + 8 for
// Q4) goes into the mantissa of 2^23, the bias is subtracted in fp32, and a
// float holding an integer of at most 8 significant bits keeps all of them in
// its top 16 bits (its bf16 value).
__device__ __forceinline__ uint2 i8x4_bf16(uint32_t w) {
  const uint32_t u = w ^ 0x80808080u;
  const float f0 = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7540)) - 8388736.f;
  const float f1 = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7541)) - 8388736.f;
  const float f2 = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7542)) - 8388736.f;
  const float f3 = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7543)) - 8388736.f;
  return make_uint2(__byte_perm(__float_as_uint(f0), __float_as_uint(f1), 0x7632),
                    __byte_perm(__float_as_uint(f2), __float_as_uint(f3), 0x7632));
}
// 8 packed nibbles (q4.put order: column 2b in byte b's low half) -> 4 words of bf16 pairs.
__device__ __forceinline__ uint4 i4x8_bf16(uint32_t w) {
  const uint32_t u = w ^ 0x88888888u;
  const uint32_t lo = u & 0x0f0f0f0fu, hi = (u >> 4) & 0x0f0f0f0fu;
  uint32_t r[4];
#pragma unroll
  for (int b = 0; b < 4; b++) {
    const float fl = __uint_as_float(__byte_perm(lo, 0x4B000000u, 0x7540 + b)) - 8388616.f;
    const float fh = __uint_as_float(__byte_perm(hi, 0x4B000000u, 0x7540 + b)) - 8388616.f;
    r[b] = __byte_perm(__float_as_uint(fl), __float_as_uint(fh), 0x7632);
  }
  return make_uint4(r[0], r[1], r[2], r[3]);
}

// Widen unit u's codes (code slot u % kDirRawSlots) into A tile u & 1, by the
// converter threads ct = 0..63: 16-byte output chunk k = (row r, c) holds
// columns 8c..8c+7 of row r and goes to byte r*128 + ((c ^ (r % 8)) * 16) of
// the tile (the UMMA 128-byte swizzle).  Loads go out in batches of 8 before
// any store (a store could alias a later load, so the compiler keeps them in
// order otherwise).  Returns false if a wait expired.
__device__ __forceinline__ bool dir_convert(const GemmArgs& a, int u, int ct) {
  const DirSmem sm = dir_smem();
  const int r = u % kDirRawSlots, b = u & 1;
  if (!mbar_wait(sm.rfull(r), (u / kDirRawSlots) & 1, a.err)) return false;
  if (u >= kDirASlots && !mbar_wait(sm.aempty(b), ((u >> 1) - 1) & 1, a.err)) return false;
  const uint8_t* raw = sm.raw(r);
  uint8_t* at = sm.atile(b);
  constexpr int kStep = kDirConvWarps * 32, kBatch = 8, kChunks = kMC * 8;
  if (a.fmt == kQ8) {
#pragma unroll 1
    for (int k0 = ct; k0 < kChunks; k0 += kBatch * kStep) {
      uint2 w[kBatch];
#pragma unroll
      for (int e = 0; e < kBatch; e++) {
        const int k = k0 + e * kStep;
        w[e] = *(const uint2*)(raw + (k >> 3) * kKB + (k & 7) * 8);
      }
#pragma unroll
      for (int e = 0; e < kBatch; e++) {
        const int k = k0 + e * kStep, row = k >> 3, c = k & 7;
        const uint2 lo = i8x4_bf16(w[e].x), hi = i8x4_bf16(w[e].y);
        *(uint4*)(at + row * 128 + ((c ^ (row & 7)) << 4)) = make_uint4(lo.x, lo.y, hi.x, hi.y);
      }
    }
  } else {
#pragma unroll 1
    for (int k0 = ct; k0 < kChunks; k0 += kBatch * kStep) {
      uint32_t w[kBatch];
#pragma unroll
      for (int e = 0; e < kBatch; e++) {
        const int k = k0 + e * kStep;
        w[e] = *(const uint32_t*)(raw + (k >> 3) * (kKB / 2) + (k & 7) * 4);
      }
#pragma unroll
      for (int e = 0; e < kBatch; e++) {
        const int k = k0 + e * kStep, row = k >> 3, c = k & 7;
        *(uint4*)(at + row * 128 + ((c ^ (row & 7)) << 4)) = i4x8_bf16(w[e]);
      }
    }
  }
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // the MMA reads the tile through the async proxy
  __syncwarp();
  if ((ct & 31) == 0) {
    mbar_arrive(sm.afull(b));
    mbar_arrive(sm.rempty(r));
  }
  return true;
}

// grid: ngroups * nt CTAs, one per SM.  tm_w*: the segments' code maps
// (uint8, box kDirSub rows x one block's bytes), tm_x*: the activation planes.
// Leaves the same partial slots as k_gemm_q for k_sk_reduce.
__global__ void __launch_bounds__(kDirThreads, 1)
k_gemm_direct(const __grid_constant__ CUtensorMap tm_xh, const __grid_constant__ CUtensorMap tm_xl,
              const __grid_constant__ CUtensorMap tm_w0, const __grid_constant__ CUtensorMap tm_w1,
              const __grid_constant__ CUtensorMap tm_w2, GemmArgs a) {
  const DirSmem sm = dir_smem();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = blockIdx.x / a.nt, j = blockIdx.x % a.nt;  // stream-K group, row tile
  const int K = a.groups;
  const int units = a.mt * K;
  const int ub = sk_begin(g, units, a.ngroups), ue = sk_begin(g + 1, units, a.ngroups);
  const int nu = ue - ub;
  const int m_first = ub / K, kb_first = ub - m_first * K;
  const int n0 = j * kN;
  const uint32_t sub_bytes = (uint32_t)kDirSub * (a.fmt == kQ8 ? kKB : kKB / 2);

  if (threadIdx.x == 0) {
    for (int r = 0; r < kDirRawSlots; r++) {
      mbar_init(sm.rfull(r), 1);
      mbar_init(sm.rempty(r), kDirConvWarps);
    }
    for (int s = 0; s < kDirBSlots; s++) {
      mbar_init(sm.bfull(s), 1);
      mbar_init(sm.bempty(s), 1);
    }
    for (int b = 0; b < kDirASlots; b++) {
      mbar_init(sm.afull(b), kDirConvWarps);
      mbar_init(sm.aempty(b), 1);
    }
    for (int b = 0; b < kAcc; b++) {
      mbar_init(sm.tfull(b), 1);
      mbar_init(sm.tempty(b), kEpiWarps);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(sm.tmem_slot())),
                 "r"(kAcc * kMH * kN));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *sm.tmem_slot();

  if (warp == 0) {
    if (lane == 0) {  // TMA producer: codes of unit u, then the planes of unit u - 1
      if (nu > 0) prefetch_tile_scales(a, m_first);
      const int b1 = a.seg[0].rows, b2 = b1 + a.seg[1].rows;
      int um = m_first, ukb = kb_first, vkb = kb_first;
      for (int u = 0; u <= nu; u++) {
        if (u < nu) {
          const int r = u % kDirRawSlots;
          if (u >= kDirRawSlots && !mbar_wait(sm.rempty(r), ((u / kDirRawSlots) - 1) & 1, a.err)) break;
          if (u == 0 || ukb == 0) prefetch_tile_scales(a, um + 1);
          mbar_expect_tx(sm.rfull(r), 4 * sub_bytes);
          const int xc = ukb * (a.fmt == kQ8 ? kKB : kKB / 2);  // byte column of the block (16-byte multiple)
#pragma unroll
          for (int q = 0; q < kMC / kDirSub; q++) {
            // rows past the last segment read as zeros (TMA out-of-bounds fill)
            const int rg = um * kMC + q * kDirSub;
            const int sg = (a.nseg > 1 && rg >= b1) ? ((a.nseg > 2 && rg >= b2) ? 2 : 1) : 0;
            const CUtensorMap* map = sg == 0 ? &tm_w0 : (sg == 1 ? &tm_w1 : &tm_w2);
            tma_load_2d(sm.raw(r) + q * sub_bytes, map, sm.rfull(r), xc, rg - (sg == 0 ? 0 : (sg == 1 ? b1 : b2)));
          }
          ukb = (ukb + 1 == K) ? 0 : ukb + 1;
          um += (ukb == 0) ? 1 : 0;
        }
        const int v = u - 1;
        if (v >= 0) {
          const int sb = v % kDirBSlots;
          if (v >= kDirBSlots && !mbar_wait(sm.bempty(sb), ((v / kDirBSlots) - 1) & 1, a.err)) break;
          mbar_expect_tx(sm.bfull(sb), kDirB);
          tma_load_2d(sm.btile(sb), &tm_xh, sm.bfull(sb), vkb * kKB, n0);
          tma_load_2d(sm.btile(sb) + kTileB, &tm_xl, sm.bfull(sb), vkb * kKB, n0);
          vkb = (vkb + 1 == K) ? 0 : vkb + 1;
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {  // MMA issuer
      const uint32_t idesc = idesc_bf16(kM, kN);
      for (int i = 0; i < nu; i++) {
        const int sb = i % kDirBSlots, b = i & 1;
        if (!mbar_wait(sm.bfull(sb), (i / kDirBSlots) & 1, a.err)) break;
        if (!mbar_wait(sm.afull(b), (i >> 1) & 1, a.err)) break;
        if (i >= kAcc && !mbar_wait(sm.tempty(b), ((i >> 1) - 1) & 1, a.err)) break;
        tc_fence_after();
        const uint8_t* bt = sm.btile(sb);
        const uint8_t* at = sm.atile(b);
        const uint64_t dh = sw128_desc(bt), dl = sw128_desc(bt + kTileB);
#pragma unroll
        for (int h = 0; h < kMH; h++) {
          const uint64_t da = sw128_desc(at + h * (kTileA / kMH));
          const uint32_t td = tmem + b * (kMH * kN) + h * kN;
#pragma unroll
          for (int k = 0; k < kKB / 16; k++) umma_bf16(td, da + 2 * k, dh + 2 * k, idesc, k > 0 ? 1u : 0u);
#pragma unroll
          for (int k = 0; k < kKB / 16; k++) umma_bf16(td, da + 2 * k, dl + 2 * k, idesc, 1u);
        }
        umma_commit(sm.bempty(sb));
        umma_commit(sm.aempty(b));
        umma_commit(sm.tfull(b));
      }
    }
  } else if (warp < kDirEpiWarp0) {  // converters
    const int ct = threadIdx.x - 2 * 32;
    for (int u = 0; u < nu; u++)
      if (!dir_convert(a, u, ct)) break;
  } else {  // epilogue warps 4..11: TMEM lane quarter = warp % 4, MMA half = (warp - 4) / 4
    // k_gemm_q's epilogue (per-block scale FMAs; whole plain tiles stored,
    // the rest to the CTA's partial slots for k_sk_reduce)
    const int q = warp & 3, h = (warp - kDirEpiWarp0) >> 2;
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
      ok = ok && mbar_wait(sm.tfull(b), (i >> 1) & 1, a.err);
      if (ok) {
        tc_fence_after();
        const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16) + b * (kMH * kN) + h * kN;
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
          } else {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(sm.tempty(b));
          }
#pragma unroll
          for (int jj = 0; jj < 16; jj++) acc[c + 16 + jj] = fmaf(__uint_as_float(vb[jj]), sc, acc[c + 16 + jj]);
          if (c + 32 < kN) tmem_wait_ld16(va);
        }
      }
      if (kb != K - 1 && i != nu - 1) continue;
      const int kb_e = kb;
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

}  // namespace tc
}  // namespace sr
