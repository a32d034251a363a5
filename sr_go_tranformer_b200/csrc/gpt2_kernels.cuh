// gpt2_kernels.cuh -- the GPT-2 profile's own kernels, exact order
// (cmd/monolith/monolith.go, "M:line").  Everything else of the GPT-2 step
// (exact linears with bias and residual, exact attention, embedding gather,
// sampler) is shared with the RMSNorm profiles.
#pragma once

#include "exact_kernels.cuh"

namespace sr {

// Absolute positions (M:6369-6371): X[r] += wpe[pos(r)], float32 adds.
__global__ void k_add_position(float* __restrict__ X, const float* __restrict__ wpe, StepMeta meta, int d) {
  const int r = blockIdx.x;
  const float* p = wpe + (int64_t)meta.row_pos[r] * d;
  float* x = X + (int64_t)r * d;
  for (int j = threadIdx.x; j < d; j += blockDim.x) x[j] = fadd(x[j], p[j]);
}

// layerNormInto (M:5167-5185): fp64 mean, then fp64 sum of squared deviations,
// both in column order (lane 0 adds a warp's staged chunk); then
// y = float32((x - mean) * inv) * w + b in float32.  One warp per row;
// src_map (optional) gathers input rows.
__global__ void __launch_bounds__(kNormWarps * 32)
k_layernorm_exact(const float* __restrict__ X, const int32_t* __restrict__ src_map, const float* __restrict__ w,
                  const float* __restrict__ b, float* __restrict__ Y, int rows, int d, double eps) {
  __shared__ double st[kNormWarps][kNormChunk];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r = blockIdx.x * kNormWarps + warp;
  if (r >= rows) return;
  const int srow = src_map ? src_map[r] : r;
  const float* x = X + (int64_t)srow * d;
  double mean = 0.0;
  for (int c0 = 0; c0 < d; c0 += kNormChunk) {
    const int cn = min(kNormChunk, d - c0);
    for (int j = lane; j < cn; j += 32) st[warp][j] = (double)x[c0 + j];
    __syncwarp();
    if (lane == 0)
      for (int j = 0; j < cn; j++) mean = dadd(mean, st[warp][j]);
    __syncwarp();
  }
  mean = __ddiv_rn(__shfl_sync(0xffffffffu, mean, 0), (double)d);
  double var = 0.0;
  for (int c0 = 0; c0 < d; c0 += kNormChunk) {
    const int cn = min(kNormChunk, d - c0);
    for (int j = lane; j < cn; j += 32) {
      const double z = dsub((double)x[c0 + j], mean);
      st[warp][j] = dmul(z, z);
    }
    __syncwarp();
    if (lane == 0)
      for (int j = 0; j < cn; j++) var = dadd(var, st[warp][j]);
    __syncwarp();
  }
  var = __shfl_sync(0xffffffffu, var, 0);
  const double inv = __ddiv_rn(1.0, __dsqrt_rn(dadd(__ddiv_rn(var, (double)d), eps)));
  float* y = Y + (int64_t)r * d;
  for (int j = lane; j < d; j += 32) y[j] = fadd(fmul((float)dmul(dsub((double)x[j], mean), inv), w[j]), b[j]);
}

// gelu_new as the reference writes it (M:6405-6407), left to right in fp64:
// float32(0.5*x * (1 + tanh(sqrt(2/pi) * (x + 0.044715*x*x*x)))).  The
// constant is the double nearest 2/pi.
__global__ void k_gelu_exact(const float* __restrict__ G, float* __restrict__ H, int64_t count) {
  const double c = __dsqrt_rn(0x1.45f306dc9c883p-1);
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < count; i += (int64_t)gridDim.x * blockDim.x) {
    const double x = (double)G[i];
    const double inner = dmul(c, dadd(x, dmul(dmul(dmul(0.044715, x), x), x)));
    H[i] = (float)dmul(dmul(0.5, x), dadd(1.0, tanh(inner)));
  }
}

// The K/V rows into the row's page without RoPE (KVCache.row M:6038-6043,
// copy M:6393-6395; GPT-2 skips Model.rope, M:6389).
__global__ void k_kv_write_exact(const float* __restrict__ K, const float* __restrict__ V, StepMeta meta,
                                 float* __restrict__ pool, ModelDims dm, int layer) {
  const int r = blockIdx.x;
  const int pos = meta.row_pos[r];
  const int64_t page = meta.page_ids[meta.row_pbase[r] + pos / dm.page_tokens];
  float* kdst = pool + page * dm.page_elems + (int64_t)layer * 2 * dm.page_tokens * dm.kvd +
                (int64_t)(pos % dm.page_tokens) * dm.kvd;
  float* vdst = kdst + (int64_t)dm.page_tokens * dm.kvd;
  for (int j = threadIdx.x; j < dm.kvd; j += blockDim.x) {
    kdst[j] = K[(int64_t)r * dm.kvd + j];
    vdst[j] = V[(int64_t)r * dm.kvd + j];
  }
}

}  // namespace sr
