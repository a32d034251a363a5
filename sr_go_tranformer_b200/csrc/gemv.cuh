// gemv.cuh -- SR_MODE_FAST decode projections for steps of 1 or 2 rows:
// Y[n, out] = X[n, in] W[out, in]^T with
// W in the reference's Q8 / Q4 storage (Param, cmd/monolith/monolith.go:3784-3850),
// read as stored.
//
// linearQ8Into / linearQ4Into (M:4074-4511) restated for a few rows on CUDA
// cores, bound by the weight bytes:
//   * every lane of a warp loads 16 bytes of one weight row per iteration with
//     one 128-bit load (16 Q8 codes or 32 Q4 codes, always inside one
//     64-column scale block), so a warp reads 512 contiguous bytes of each of
//     its kRowsPerWarp rows;
//   * the codes are widened in registers (exact: the byte is placed in the
//     mantissa of 2^23 by a byte permute and the bias subtracted), multiplied
//     with the step rows' activations staged in shared memory, and each lane's
//     partial dot of a block is scaled by the block's scale (s += p * scale,
//     in fp32 FMA);
//   * lanes are summed by warp shuffles at the end (fast mode: reordered sums);
//   * narrow matrices split K over several CTAs; the partial sums go to
//     scratch and the last CTA of each row group to arrive (an atomic counter,
//     no waiting) adds them in split order, so results do not depend on timing.
// The epilogue adds the bias, the residual (y = resid + W x, resid may alias y)
// or scatters rows through the head's row map, like linear_store.
#pragma once

#include "common.cuh"
#include "exact_kernels.cuh"

namespace sr {
namespace gv {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kMaxSeg = 3;
// Rows of the largest instantiation.  With more step rows the FMAs per weight
// byte (one per row) bound the kernel below the tensor cores' time (measured on
// the Mistral-7B step: 1 row 3.8 ms, 2 rows 4.3 ms, 4 rows 7.2 ms against 5.3 ms
// for the tcgen05 path at any row count up to 128).
constexpr int kMaxRows = 2;
// Weight rows per warp (more rows share each staged activation read) and per CTA.
__host__ __device__ constexpr int rows_per_warp(int nr) { return nr <= 2 ? 8 : 4; }
__host__ __device__ constexpr int rows_per_cta(int nr) { return kWarps * rows_per_warp(nr); }
// The most K columns of X one CTA stages (NR x chunk x 4 bytes = 32 KiB, 16 KiB
// at one row); a CTA's K range never exceeds it.
__host__ __device__ constexpr int chunk_for(int nr) { return nr <= 2 ? 4096 : (nr == 4 ? 2048 : 1024); }
// Columns one warp covers per iteration (16 bytes of codes per lane).
__host__ __device__ constexpr int span_for(int fmt) { return fmt == kQ8 ? 512 : 1024; }

struct Seg {
  int32_t rows;   // output features
  int32_t tiles;  // ceil(rows / rows_per_cta(NR))
  const uint8_t* w;     // codes, row stride rb bytes
  const float* scales;  // [rows][groups]
  float* y;
  int32_t ldy;
  const float* bias;
  const float* resid;
};

struct Args {
  const float* x;  // [n][in] fp32
  int n, in, fmt, groups;
  int64_t rb;      // bytes per weight row
  Seg seg[kMaxSeg];
  int nseg;
  const int32_t* out_map;  // compact head rows -> destination rows
  int ksplit, kper;        // K splits; columns per split (a multiple of the span, at most the chunk)
  int total_tiles;
  float* part;             // [ksplit][total_tiles * rows_per_cta][NR] partials (ksplit > 1)
  int* counters;           // [total_tiles], zero between launches
};

// 4 signed bytes -> 4 floats, exactly.
__device__ __forceinline__ void i8x4(uint32_t w, float (&f)[4]) {
  const uint32_t u = w ^ 0x80808080u;  // q + 128 in 0..255
  f[0] = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7540)) - 8388736.f;
  f[1] = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7541)) - 8388736.f;
  f[2] = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7542)) - 8388736.f;
  f[3] = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7543)) - 8388736.f;
}
// 8 signed nibbles (low nibble first: column 2b in byte b's low half) -> 8 floats.
__device__ __forceinline__ void i4x8(uint32_t w, float (&f)[8]) {
  const uint32_t u = w ^ 0x88888888u;  // q + 8 in 0..15
  const uint32_t lo = u & 0x0f0f0f0fu, hi = (u >> 4) & 0x0f0f0f0fu;
  f[0] = __uint_as_float(__byte_perm(lo, 0x4B000000u, 0x7540)) - 8388616.f;
  f[1] = __uint_as_float(__byte_perm(hi, 0x4B000000u, 0x7540)) - 8388616.f;
  f[2] = __uint_as_float(__byte_perm(lo, 0x4B000000u, 0x7541)) - 8388616.f;
  f[3] = __uint_as_float(__byte_perm(hi, 0x4B000000u, 0x7541)) - 8388616.f;
  f[4] = __uint_as_float(__byte_perm(lo, 0x4B000000u, 0x7542)) - 8388616.f;
  f[5] = __uint_as_float(__byte_perm(hi, 0x4B000000u, 0x7542)) - 8388616.f;
  f[6] = __uint_as_float(__byte_perm(lo, 0x4B000000u, 0x7543)) - 8388616.f;
  f[7] = __uint_as_float(__byte_perm(hi, 0x4B000000u, 0x7543)) - 8388616.f;
}

// Segment of global row-group t, and t's first row within it.
__device__ __forceinline__ int seg_of(const Args& a, int t, int rpc, int* row0) {
  int s = 0, base = 0;
  if (a.nseg > 1 && t >= a.seg[0].tiles) {
    s = 1;
    base = a.seg[0].tiles;
    if (a.nseg > 2 && t >= base + a.seg[1].tiles) {
      s = 2;
      base += a.seg[1].tiles;
    }
  }
  *row0 = (t - base) * rpc;
  return s;
}

__device__ __forceinline__ void store_out(const Args& a, const Seg& g, int r, int o, float v) {
  const int64_t orow = a.out_map ? (int64_t)a.out_map[r] : (int64_t)r;
  if (g.bias) v += g.bias[o];
  if (g.resid) v = g.resid[orow * g.ldy + o] + v;
  g.y[orow * g.ldy + o] = v;
}

// grid (total_tiles, ksplit), kThreads threads.  NR: step rows rounded up
// (rows >= n contribute zeros); FMT kQ8 or kQ4.  Each CTA stages its K range
// of X once, then every warp streams its RPW weight rows over it with the next
// iteration's 16-byte loads in flight while the current ones are consumed.
template <int FMT, int NR>
__global__ void __launch_bounds__(kThreads) k_gemv(Args a) {
  constexpr int RPW = rows_per_warp(NR), RPC = rows_per_cta(NR);
  constexpr int kChunk = chunk_for(NR);
  __shared__ __align__(16) float xs[NR][kChunk];
  __shared__ int s_last;
  constexpr int kCols = FMT == kQ8 ? 16 : 32;  // columns per lane per 16-byte load
  constexpr int kSpan = 32 * kCols;             // columns per warp iteration
  constexpr int kW = FMT == kQ8 ? 4 : 8;        // columns per 32-bit word of codes
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int t = blockIdx.x, split = blockIdx.y;
  int row0;
  const int si = seg_of(a, t, RPC, &row0);
  const Seg& g = si == 0 ? a.seg[0] : (si == 1 ? a.seg[1] : a.seg[2]);
  const int c0 = split * a.kper, cn = min(a.in, c0 + a.kper) - c0;  // cn <= kChunk, a multiple of kCols
  const int ob = row0 + warp * RPW;  // this warp's first feature
  const uint8_t* wrow[RPW];
  const float* srow[RPW];
#pragma unroll
  for (int i = 0; i < RPW; i++) {
    const int o = min(ob + i, g.rows - 1);  // rows past the end repeat the last one; never stored
    wrow[i] = g.w + (int64_t)o * a.rb + (FMT == kQ8 ? c0 : c0 / 2);
    srow[i] = g.scales + (int64_t)o * a.groups + c0 / kQBlock;
  }
  // first iteration's codes, in flight while X is staged
  int cc = lane * kCols;
  uint4 wv[RPW];
  float sc[RPW];
#pragma unroll
  for (int i = 0; i < RPW; i++) {
    wv[i] = cc < cn ? __ldg((const uint4*)(wrow[i] + (FMT == kQ8 ? cc : cc / 2))) : make_uint4(0, 0, 0, 0);
    sc[i] = cc < cn ? __ldg(srow[i] + cc / kQBlock) : 0.f;
  }
  for (int idx = tid; idx < NR * (cn / 4); idx += kThreads) {
    const int r = idx / (cn / 4), c = idx - r * (cn / 4);
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (r < a.n) v = *(const float4*)(a.x + (int64_t)r * a.in + c0 + 4 * c);
    *(float4*)&xs[r][4 * c] = v;
  }
  __syncthreads();
  float acc[RPW][NR];
#pragma unroll
  for (int i = 0; i < RPW; i++)
#pragma unroll
    for (int r = 0; r < NR; r++) acc[i][r] = 0.f;
  for (; cc < cn; cc += kSpan) {
    const int nx = cc + kSpan;
    uint4 wn[RPW];
    float sn[RPW];
#pragma unroll
    for (int i = 0; i < RPW; i++) {
      wn[i] = nx < cn ? __ldg((const uint4*)(wrow[i] + (FMT == kQ8 ? nx : nx / 2))) : make_uint4(0, 0, 0, 0);
      sn[i] = nx < cn ? __ldg(srow[i] + nx / kQBlock) : 0.f;
    }
    float p[RPW][NR];
#pragma unroll
    for (int i = 0; i < RPW; i++)
#pragma unroll
      for (int r = 0; r < NR; r++) p[i][r] = 0.f;
#pragma unroll
    for (int q = 0; q < 4; q++) {  // 32-bit word q of every row's 16 bytes
      float f[RPW][kW];
#pragma unroll
      for (int i = 0; i < RPW; i++) {
        const uint32_t word = q == 0 ? wv[i].x : (q == 1 ? wv[i].y : (q == 2 ? wv[i].z : wv[i].w));
        if constexpr (FMT == kQ8) {
          float f4[4];
          i8x4(word, f4);
#pragma unroll
          for (int e = 0; e < 4; e++) f[i][e] = f4[e];
        } else {
          float f8[8];
          i4x8(word, f8);
#pragma unroll
          for (int e = 0; e < 8; e++) f[i][e] = f8[e];
        }
      }
#pragma unroll
      for (int r = 0; r < NR; r++) {
        float xv[kW];
        const float4 v0 = *(const float4*)&xs[r][cc + q * kW];
        xv[0] = v0.x, xv[1] = v0.y, xv[2] = v0.z, xv[3] = v0.w;
        if constexpr (kW == 8) {
          const float4 v1 = *(const float4*)&xs[r][cc + q * kW + 4];
          xv[4] = v1.x, xv[5] = v1.y, xv[6] = v1.z, xv[7] = v1.w;
        }
#pragma unroll
        for (int i = 0; i < RPW; i++)
#pragma unroll
          for (int e = 0; e < kW; e++) p[i][r] = fmaf(f[i][e], xv[e], p[i][r]);
      }
    }
#pragma unroll
    for (int i = 0; i < RPW; i++) {
#pragma unroll
      for (int r = 0; r < NR; r++) acc[i][r] = fmaf(p[i][r], sc[i], acc[i][r]);
      wv[i] = wn[i];
      sc[i] = sn[i];
    }
  }
#pragma unroll
  for (int i = 0; i < RPW; i++)
#pragma unroll
    for (int r = 0; r < NR; r++)
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) acc[i][r] += __shfl_xor_sync(0xffffffffu, acc[i][r], off);
  if (a.ksplit == 1) {
    if (lane == 0)
#pragma unroll
      for (int i = 0; i < RPW; i++)
        if (ob + i < g.rows)
#pragma unroll
          for (int r = 0; r < NR; r++)
            if (r < a.n) store_out(a, g, r, ob + i, acc[i][r]);
    return;
  }
  // split K: publish this split's partials, then the last CTA of the row group
  // adds the splits in order (threadfence reduction; nobody waits)
  const int64_t plane = (int64_t)a.total_tiles * RPC;  // partial slots per split
  const int64_t slot = (int64_t)t * RPC + warp * RPW;
  if (lane == 0)
#pragma unroll
    for (int i = 0; i < RPW; i++)
#pragma unroll
      for (int r = 0; r < NR; r++)
        if (r < a.n) a.part[((int64_t)split * plane + slot + i) * NR + r] = acc[i][r];
  __threadfence();
  __syncthreads();
  if (tid == 0) s_last = atomicAdd(&a.counters[t], 1) == a.ksplit - 1;
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  for (int idx = tid; idx < RPC * a.n; idx += kThreads) {
    const int i = idx / a.n, r = idx - i * a.n;
    const int o = row0 + i;
    if (o >= g.rows) continue;
    float v = 0.f;
    for (int s = 0; s < a.ksplit; s++) v += __ldcg(a.part + ((int64_t)s * plane + (int64_t)t * RPC + i) * NR + r);
    store_out(a, g, r, o, v);
  }
  if (tid == 0) a.counters[t] = 0;  // ready for the next launch on this stream
}

}  // namespace gv
}  // namespace sr
