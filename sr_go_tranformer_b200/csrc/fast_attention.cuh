// fast_attention.cuh -- SR_MODE_FAST paged GQA attention (flash-decoding).
//
// Same mathematics as attend (cmd/monolith/monolith.go:5293-5352), reordered
// for the B200: every (row, KV head) context is cut into splits of kSplit
// positions, one CTA per split.  A CTA stages K/V tiles of kTile positions
// from the page pool into shared memory with cp.async (double-buffered),
// computes the `group` query heads' scores with FFMA, and keeps an online
// softmax (running max, rescaled sum and output).  A combine kernel merges the
// splits with their log-sum-exp weights.  Results match the exact path within
// fp32 rounding (tolerance-checked), not bit for bit.
#pragma once

#include <float.h>
#include "common.cuh"

namespace sr {

constexpr int kFaThreads = 128;
constexpr int kFaTile = 32;    // positions per shared-memory tile
constexpr int kFaSplit = 256;  // positions per CTA

struct FastAttnArgs {
  const float* Q;
  float* A;
  const float* pool;
  StepMeta meta;
  ModelDims dm;
  int layer;
  float scale;
  int max_splits;
  float* part_o;   // [items][group][hd]
  float* part_ml;  // [items][group][2]
};

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  unsigned s = (unsigned)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(s), "l"(gmem));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;\n" ::); }

// Stage K and V rows of positions [t0, t0+tn) (tn <= kFaTile) of one KV head.
template <int HD>
__device__ __forceinline__ void fa_load_tile(const FastAttnArgs& a, float* ks, float* vs, int pbase, int kh, int t0,
                                             int tn) {
  const int pt = a.dm.page_tokens;
  const int64_t lay = (int64_t)a.layer * 2 * pt * a.dm.kvd + (int64_t)kh * HD;
  constexpr int C4 = HD / 4;
  for (int idx = threadIdx.x; idx < tn * C4; idx += kFaThreads) {
    const int s = idx / C4, c = idx % C4, pos = t0 + s;
    const int64_t page = a.meta.page_ids[pbase + pos / pt];
    const float* krow = a.pool + page * a.dm.page_elems + lay + (int64_t)(pos % pt) * a.dm.kvd;
    cp_async16(ks + s * HD + 4 * c, krow + 4 * c);
    cp_async16(vs + s * HD + 4 * c, krow + (int64_t)pt * a.dm.kvd + 4 * c);
  }
}

template <int HD, int G>
__global__ void __launch_bounds__(kFaThreads) k_attn_split(FastAttnArgs a) {
  static_assert(HD == 64 || HD == 128, "head_dim");
  static_assert(G >= 1 && G <= 8, "group");
  constexpr int LPP = HD / 16;        // lanes per position in the score phase
  constexpr int PPW = 32 / LPP;       // positions per warp per pass
  constexpr int PPAR = kFaThreads / HD;  // position-parallel groups in the PV phase
  constexpr int GP = (G + 3) & ~3;    // padded group (float4 p loads)
  extern __shared__ __align__(16) float fsm[];
  float* ks = fsm;                          // [2][kFaTile][HD]
  float* vs = ks + 2 * kFaTile * HD;        // [2][kFaTile][HD]
  float* sc = vs + 2 * kFaTile * HD;        // [G][kFaTile]
  float* ps = sc + G * kFaTile;             // [kFaTile][GP]
  float* alpha_s = ps + kFaTile * GP;       // [GP]
  float* m_s = alpha_s + GP;                // [GP]
  float* l_s = m_s + GP;                    // [GP]
  float* red = l_s + GP;                    // [PPAR][G][HD] partial outputs

  const int split = blockIdx.x, r = blockIdx.y, kh = blockIdx.z;
  const int L = a.meta.row_pos[r] + 1;
  const int s0 = split * kFaSplit;
  if (s0 >= L) return;
  const int s1 = min(L, s0 + kFaSplit);
  const int pbase = a.meta.row_pbase[r];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  // query slices in registers: lane covers dims 4*(lane%LPP) + 4*LPP*i, i < 4
  float4 q[G][4];
  {
    const float* qrow = a.Q + (int64_t)r * a.dm.dim + (int64_t)kh * G * HD;
    const int jl = lane % LPP;
#pragma unroll
    for (int g = 0; g < G; g++)
#pragma unroll
      for (int i = 0; i < 4; i++) {
        float4 v = *(const float4*)(qrow + g * HD + 4 * jl + 4 * LPP * i);
        q[g][i] = make_float4(v.x * a.scale, v.y * a.scale, v.z * a.scale, v.w * a.scale);
      }
  }
  if (tid < GP) {
    m_s[tid] = -INFINITY;
    l_s[tid] = 0.f;
  }
  const int d = tid % HD, par = tid / HD;
  float acc[G];
#pragma unroll
  for (int g = 0; g < G; g++) acc[g] = 0.f;

  const int ntiles = (s1 - s0 + kFaTile - 1) / kFaTile;
  fa_load_tile<HD>(a, ks, vs, pbase, kh, s0, min(kFaTile, s1 - s0));
  cp_async_commit();
  for (int t = 0; t < ntiles; t++) {
    const int t0 = s0 + t * kFaTile, tn = min(kFaTile, s1 - t0);
    float* kt = ks + (t & 1) * kFaTile * HD;
    float* vt = vs + (t & 1) * kFaTile * HD;
    cp_async_wait_all();
    __syncthreads();
    if (t + 1 < ntiles) {
      const int n0 = t0 + kFaTile;
      fa_load_tile<HD>(a, ks + ((t + 1) & 1) * kFaTile * HD, vs + ((t + 1) & 1) * kFaTile * HD, pbase, kh, n0,
                       min(kFaTile, s1 - n0));
    }
    cp_async_commit();
    // scores: warp w handles positions w*PPW*k + lane/LPP
    for (int base = warp * PPW; base < kFaTile; base += 4 * PPW) {
      const int s = base + lane / LPP;
      const int jl = lane % LPP;
      float part[G];
#pragma unroll
      for (int g = 0; g < G; g++) part[g] = 0.f;
      if (s < tn) {
        const float* kr = kt + s * HD + 4 * jl;
#pragma unroll
        for (int i = 0; i < 4; i++) {
          float4 kv = *(const float4*)(kr + 4 * LPP * i);
#pragma unroll
          for (int g = 0; g < G; g++)
            part[g] += q[g][i].x * kv.x + q[g][i].y * kv.y + q[g][i].z * kv.z + q[g][i].w * kv.w;
        }
      }
#pragma unroll
      for (int off = 1; off < LPP; off <<= 1)
#pragma unroll
        for (int g = 0; g < G; g++) part[g] += __shfl_xor_sync(0xffffffffu, part[g], off);
      if (jl == 0 && s < kFaTile)
#pragma unroll
        for (int g = 0; g < G; g++) sc[g * kFaTile + s] = s < tn ? part[g] : -INFINITY;
    }
    __syncthreads();
    // online softmax per head: warp w handles heads w, w+4
    for (int g = warp; g < G; g += 4) {
      const float v = sc[g * kFaTile + lane];
      float mt = v;
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, off));
      const float mo = m_s[g];
      const float mn = fmaxf(mo, mt);
      const float p = (v == -INFINITY) ? 0.f : expf(v - mn);
      float sum = p;
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
      ps[lane * GP + g] = p;
      if (lane == 0) {
        const float al = (mo == -INFINITY) ? 0.f : expf(mo - mn);
        alpha_s[g] = al;
        m_s[g] = mn;
        l_s[g] = l_s[g] * al + sum;
      }
    }
    __syncthreads();
    // PV: thread (d, par) accumulates positions par, par+PPAR, ...
#pragma unroll
    for (int g = 0; g < G; g++) acc[g] *= alpha_s[g];
    for (int s = par; s < tn; s += PPAR) {
      const float v = vt[s * HD + d];
      const float* pp = ps + s * GP;
#pragma unroll
      for (int g = 0; g < G; g++) acc[g] += pp[g] * v;
    }
  }
  // merge position-parallel partials and write this split's (O, m, l)
  __syncthreads();
#pragma unroll
  for (int g = 0; g < G; g++) red[(par * G + g) * HD + d] = acc[g];
  __syncthreads();
  const int64_t item = ((int64_t)r * a.dm.kv_heads + kh) * a.max_splits + split;
  for (int idx = tid; idx < G * HD; idx += kFaThreads) {
    float v = 0.f;
#pragma unroll
    for (int p = 0; p < PPAR; p++) v += red[p * G * HD + idx];
    a.part_o[item * G * HD + idx] = v;
  }
  if (tid < G) {
    a.part_ml[(item * G + tid) * 2] = m_s[tid];
    a.part_ml[(item * G + tid) * 2 + 1] = l_s[tid];
  }
}

// Merge the splits of each (row, query head) and write the attention output.
template <int HD>
__global__ void __launch_bounds__(HD) k_attn_combine(FastAttnArgs a) {
  const int r = blockIdx.x, h = blockIdx.y, d = threadIdx.x;
  const int G = a.dm.group, kh = h / G, g = h % G;
  const int L = a.meta.row_pos[r] + 1;
  const int ns = (L + kFaSplit - 1) / kFaSplit;
  const int64_t base = ((int64_t)r * a.dm.kv_heads + kh) * a.max_splits;
  float M = -INFINITY;
  for (int s = 0; s < ns; s++) M = fmaxf(M, a.part_ml[((base + s) * G + g) * 2]);
  float den = 0.f, num = 0.f;
  for (int s = 0; s < ns; s++) {
    const float w = expf(a.part_ml[((base + s) * G + g) * 2] - M);
    den += w * a.part_ml[((base + s) * G + g) * 2 + 1];
    num += w * a.part_o[((base + s) * G + g) * HD + d];
  }
  a.A[(int64_t)r * a.dm.dim + (int64_t)h * HD + d] = num / den;
}

template <int HD, int G>
inline size_t fa_smem_bytes() {
  constexpr int GP = (G + 3) & ~3;
  constexpr int PPAR = kFaThreads / HD;
  return (size_t)(4 * kFaTile * HD + G * kFaTile + kFaTile * GP + 3 * GP + PPAR * G * HD) * 4;
}

}  // namespace sr
