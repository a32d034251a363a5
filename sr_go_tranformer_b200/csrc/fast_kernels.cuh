// fast_kernels.cuh -- SR_MODE_FAST: fused-multiply-add, split-K and tensor-core
// kernels, checked against the reference within a stated tolerance.  Shapes a
// fast kernel does not cover run on the exact kernels.
#pragma once

#include <algorithm>

#include "common.cuh"
#include "exact_kernels.cuh"
#include "fast_attention.cuh"
#include "gemv.cuh"
#include "srstep_internal.h"
#include "tp_peer.cuh"

namespace sr {

struct FastState {
  float* part_o = nullptr;
  float* part_ml = nullptr;
  size_t items_cap = 0;
  float* gv_part = nullptr;  // decode GEMV split-K partials (grow-only)
  size_t gv_part_floats = 0;
  int* gv_count = nullptr;   // decode GEMV row-group counters (zeroed, reset by the kernel)
  size_t gv_count_cap = 0;
  int* err = nullptr;    // device flag raised by an expired bounded wait
  int* h_err = nullptr;  // pinned host copy
  bool ran = false;      // a kernel that can raise the flag ran since the last check
};

inline FastState* fast_state(sr_model* m) { return (FastState*)m->fast; }

inline int fast_init(sr_model* m) {
  FastState* st = new FastState();
  m->fast = st;
  m->fast_free.push_back([st]() {
    if (st->part_o) cudaFree(st->part_o);
    if (st->part_ml) cudaFree(st->part_ml);
    if (st->gv_part) cudaFree(st->gv_part);
    if (st->gv_count) cudaFree(st->gv_count);
    if (st->err) cudaFree(st->err);
    if (st->h_err) cudaFreeHost(st->h_err);
    delete st;
  });
  if (cudaMalloc((void**)&st->err, 16) != cudaSuccess || cudaMallocHost((void**)&st->h_err, 16) != cudaSuccess ||
      cudaMemset(st->err, 0, 16) != cudaSuccess) {
    cudaGetLastError();
    return sr_fail(SR_ENOMEM, "allocating the attention error flag failed");
  }
  return SR_OK;
}

// After the step's stream synchronize: SR_ETIMEOUT if an attention wait expired.
inline int fast_check(sr_model* m) {
  FastState* st = fast_state(m);
  if (!st || !st->err || !st->ran) return SR_OK;
  st->ran = false;
  if (cudaMemcpy(st->h_err, st->err, 4, cudaMemcpyDeviceToHost) != cudaSuccess) {
    cudaGetLastError();
    return sr_fail(SR_EDEVICE, "reading the attention error flag failed");
  }
  if (*st->h_err) {
    cudaMemset(st->err, 0, 4);
    return sr_fail(SR_ETIMEOUT, "an attention tile wait expired; results of this step are invalid");
  }
  return SR_OK;
}

// ------------------------------------------------------------------ RMSNorm --
// rmsInto (M:6182-6194) with a block-parallel fp64 sum of squares (reordered).
// One 128-thread block per row keeps every SM busy at decode batch sizes.
// With T set (tensor parallel, rows not remapped), the row first takes the
// all-reduced projection: X += T (addInPlace, M:6405/6418), written back.
__global__ void __launch_bounds__(128)
k_rmsnorm_fast(float* __restrict__ X, const int32_t* __restrict__ src_map, const float* __restrict__ w,
               float* __restrict__ Y, int rows, int d, double eps, op16* __restrict__ yh,
               op16* __restrict__ yl, const float* __restrict__ T, const uint4* __restrict__ Tll,
               uint32_t epoch, int* err) {
  __shared__ double red[4];
  const int r = blockIdx.x;
  const int srow = src_map ? src_map[r] : r;
  float* x = X + (int64_t)srow * d;
  const bool vec = (d & 3) == 0;
  if (T) {
    const float* t = T + (int64_t)srow * d;
    for (int j = threadIdx.x; j < d; j += 128) x[j] += t[j];
    __syncthreads();
  } else if (Tll) {  // the LL all-reduce's sums, waited for line by line (peer::k_peer_ll)
    const uint4* t = Tll + (int64_t)srow * d / 2;
    bool ok = true;
    for (int j = threadIdx.x; j < d / 2; j += 128) {
      const uint4 v = peer::wait_line(t + j, epoch, err, ok);
      x[2 * j] += __uint_as_float(v.x);
      x[2 * j + 1] += __uint_as_float(v.z);
    }
    __syncthreads();
  }
  double ss = 0.0;
  if (vec) {
    for (int j = threadIdx.x * 4; j < d; j += 512) {
      const float4 v = *(const float4*)(x + j);
      ss += (double)v.x * v.x + (double)v.y * v.y + (double)v.z * v.z + (double)v.w * v.w;
    }
  } else {
    for (int j = threadIdx.x; j < d; j += 128) ss += (double)x[j] * x[j];
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  ss = red[0] + red[1] + red[2] + red[3];
  const float a = (float)(1.0 / sqrt(ss / (double)d + eps));
  const int64_t o = (int64_t)r * d;
  if (vec) {
    for (int j = threadIdx.x * 4; j < d; j += 512) {
      const float4 v = *(const float4*)(x + j);
      const float4 g = *(const float4*)(w + j);
      const float y0 = v.x * a * g.x, y1 = v.y * a * g.y, y2 = v.z * a * g.z, y3 = v.w * a * g.w;
      if (yh) {
        split_op(y0, yh + o + j, yl + o + j);
        split_op(y1, yh + o + j + 1, yl + o + j + 1);
        split_op(y2, yh + o + j + 2, yl + o + j + 2);
        split_op(y3, yh + o + j + 3, yl + o + j + 3);
      } else {
        *(float4*)(Y + o + j) = make_float4(y0, y1, y2, y3);
      }
    }
  } else {
    for (int j = threadIdx.x; j < d; j += 128) {
      const float y = x[j] * a * w[j];
      if (yh)
        split_op(y, yh + o + j, yl + o + j);
      else
        Y[o + j] = y;
    }
  }
}

inline void fast_rmsnorm(sr_model* m, float* X, const int32_t* src_map, const float* w, float* Y, int rows, int d,
                         double eps, op16* yh = nullptr, op16* yl = nullptr,
                         const float* T = nullptr, const uint4* Tll = nullptr, uint32_t epoch = 0,
                         int* err = nullptr, cudaStream_t stream = nullptr) {
  k_rmsnorm_fast<<<rows, 128, 0, stream ? stream : m->stream>>>(X, src_map, w, Y, rows, d, eps, yh, yl, T, Tll, epoch,
                                                                 err);
}

// SwiGLU h = g/(1+exp(-g)) * u in fp32 (M:6410-6413 reordered), written as the
// down projection's bf16 hi/lo operand planes.
__global__ void k_swiglu_split(const float* __restrict__ G, const float* __restrict__ U,
                               op16* __restrict__ hh, op16* __restrict__ hl, int64_t count) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < count; i += (int64_t)gridDim.x * blockDim.x) {
    const float g = G[i];
    split_op(g / (1.f + __expf(-g)) * U[i], hh + i, hl + i);
  }
}

// ------------------------------------------------------------ GPT-2, fast --
// layerNormInto (M:5167-5185) reordered: one 128-thread block per row, the sum
// and then the sum of squared deviations in fp64 over strided partial sums,
// y = float32((x - mean) * inv) * w + b with an FMA, written as fp32 Y or as the
// next projection's bf16 hi/lo operand planes (yh/yl, row r at r * d).
// src_map (optional) gathers input rows.
__global__ void __launch_bounds__(128)
k_layernorm_fast(const float* __restrict__ X, const int32_t* __restrict__ src_map, const float* __restrict__ w,
                 const float* __restrict__ b, float* __restrict__ Y, int rows, int d, double eps,
                 op16* __restrict__ yh, op16* __restrict__ yl) {
  __shared__ double red[2][4];
  const int r = blockIdx.x;
  const int srow = src_map ? src_map[r] : r;
  const float* x = X + (int64_t)srow * d;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  double s = 0.0;
  for (int j = threadIdx.x; j < d; j += 128) s += (double)x[j];
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
  if (lane == 0) red[0][warp] = s;
  __syncthreads();
  const double mean = (red[0][0] + red[0][1] + red[0][2] + red[0][3]) / (double)d;
  double v = 0.0;
  for (int j = threadIdx.x; j < d; j += 128) {
    const double z = (double)x[j] - mean;
    v += z * z;
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
  if (lane == 0) red[1][warp] = v;
  __syncthreads();
  const double var = red[1][0] + red[1][1] + red[1][2] + red[1][3];
  const double inv = 1.0 / sqrt(var / (double)d + eps);
  const int64_t o = (int64_t)r * d;
  for (int j = threadIdx.x; j < d; j += 128) {
    const float y = fmaf((float)(((double)x[j] - mean) * inv), w[j], b[j]);
    if (yh)
      split_op(y, yh + o + j, yl + o + j);
    else
      Y[o + j] = y;
  }
}

// gelu_new (M:6405-6407) in fp32: 0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3))),
// written as fp32 H or as the c_proj projection's bf16 hi/lo operand planes.
__global__ void k_gelu_fast(const float* __restrict__ G, float* __restrict__ H, op16* __restrict__ hh,
                            op16* __restrict__ hl, int64_t count) {
  const float c = 0.7978845608028654f;  // sqrt(2/pi)
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < count; i += (int64_t)gridDim.x * blockDim.x) {
    const float g = G[i];
    const float y = 0.5f * g * (1.f + tanhf(c * (g + 0.044715f * g * g * g)));
    if (hh)
      split_op(y, hh + i, hl + i);
    else
      H[i] = y;
  }
}

// ---------------------------------------------------------------- attention --
// Work counts of one step's fast attention: all (row, split) items, those of
// rows from 1-token chunks, and the (row group, split) pairs of longer chunks.
struct FaWork {
  int items, single, groups;
};

template <int HD, int G>
inline bool fa_launch(sr_model* m, const FastAttnArgs& a, int n, const FaWork& w, cudaStream_t stream) {
  const size_t smem = fa_smem_bytes<HD, G>();
  if constexpr (HD == 128) {
    if (w.single > 0) {  // decode rows: 4 warps split each row's positions
      cudaFuncSetAttribute(k_attn_warp128<G>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      k_attn_warp128<G><<<dim3(w.single, a.dm.kv_heads), kFaThreads, smem, stream>>>(a);
      sr_count_launch(m);
    }
    if (w.groups > 0) {  // prefill rows
      if constexpr (G == 4) {  // 4 rows x 4 heads: one tensor-core M tile
        cudaFuncSetAttribute(k_attn_mma128, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)MmaSmem::BYTES);
        k_attn_mma128<<<dim3(w.groups, a.dm.kv_heads), kMmWarps * 32, MmaSmem::BYTES, stream>>>(a);
      } else {  // one warp per row, shared K/V tiles
        const size_t rsm = RowsSmem<G>::BYTES;
        cudaFuncSetAttribute(k_attn_rows128<G>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)rsm);
        k_attn_rows128<G><<<dim3(w.groups, a.dm.kv_heads), kFaThreads, rsm, stream>>>(a);
      }
      sr_count_launch(m);
    }
  } else {
    cudaFuncSetAttribute(k_attn_tile<HD, G>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    k_attn_tile<HD, G><<<dim3(w.items, a.dm.kv_heads), kFaThreads, smem, stream>>>(a);
    sr_count_launch(m);
  }
  k_attn_combine<HD><<<dim3(n, a.dm.heads), HD, 0, stream>>>(a);
  sr_count_launch(m);
  return true;
}

template <int HD>
inline bool fa_dispatch_g(sr_model* m, const FastAttnArgs& a, int n, const FaWork& items, cudaStream_t s) {
  switch (a.dm.group) {
    case 1: return fa_launch<HD, 1>(m, a, n, items, s);
    case 2: return fa_launch<HD, 2>(m, a, n, items, s);
    case 3: return fa_launch<HD, 3>(m, a, n, items, s);
    case 4: return fa_launch<HD, 4>(m, a, n, items, s);
    case 5: return fa_launch<HD, 5>(m, a, n, items, s);
    case 6: return fa_launch<HD, 6>(m, a, n, items, s);
    case 7: return fa_launch<HD, 7>(m, a, n, items, s);
    case 8: return fa_launch<HD, 8>(m, a, n, items, s);
    default: return false;
  }
}

// Whether the split-K kernels cover this model shape.
inline bool fast_attention_supported(const ModelDims& dm) {
  return (dm.hd == 64 || dm.hd == 128) && dm.group <= 8;
}
// Scratch floats the split-K attention needs for a step's (row, split) items
// (partial O, then (m, l)); *units_out = items x KV heads.
inline size_t fa_scratch_floats(const ModelDims& dm, int items, size_t* units_out = nullptr) {
  const size_t units = (size_t)items * dm.kv_heads;
  if (units_out) *units_out = units;
  return units * dm.group * (dm.hd + 2);
}

// One half of a split step for the attention: its stream, first row and the
// first entries of its item lists (the halves cut the lists at a session).
struct FaLane {
  cudaStream_t s;
  int row0;
  FaWork base;
};

// Launch split + combine with caller-provided scratch (no allocation).  With
// xh/xl set, the combine writes bf16 hi/lo operand planes instead of fp32 A.
// With a lane, n and items are the half's and xh/xl its planes.
inline bool fast_attention_run(sr_model* m, const float* pool_data, int n, const FaWork& items, int layer, float* part_o,
                               float* part_ml, op16* xh = nullptr, op16* xl = nullptr, const FaLane* lane = nullptr) {
  const ModelDims& dm = m->dm;
  FastAttnArgs a;
  a.Q = m->Q;
  a.A = m->A;
  a.pool = pool_data;
  a.meta = m->meta;
  a.dm = dm;
  a.layer = layer;
  a.scale = (float)(1.0 / std::sqrt((double)dm.hd));
  a.part_o = part_o;
  a.part_ml = part_ml;
  a.xh = xh;
  a.xl = xl;
  a.err = fast_state(m)->err;
  if (lane) {
    a.row0 = lane->row0;
    a.single0 = lane->base.single;
    a.grp0 = lane->base.groups;
    a.item0 = lane->base.items;
  }
  fast_state(m)->ran = true;
  cudaStream_t s = lane ? lane->s : m->stream;
  return dm.hd == 128 ? fa_dispatch_g<128>(m, a, n, items, s) : fa_dispatch_g<64>(m, a, n, items, s);
}

// Grow the split scratch to cover `work_items` (row, split) items; false when
// the shape is unsupported or the scratch would exceed its cap.
inline bool fa_reserve(sr_model* m, int work_items) {
  const ModelDims& dm = m->dm;
  if (!fast_attention_supported(dm)) return false;
  FastState* st = fast_state(m);
  size_t items = 0;
  fa_scratch_floats(dm, work_items, &items);
  const size_t o_bytes = items * dm.group * dm.hd * 4;
  if (o_bytes > ((size_t)1 << 30)) return false;
  if (items > st->items_cap) {
    // Grow by half again (within the 1 GiB cap): the item count creeps up as
    // contexts cross split boundaries, and every reallocation
    // synchronises the device.
    const size_t unit_o = (size_t)dm.group * dm.hd * 4;
    const size_t cap = std::max(items, std::min(st->items_cap + st->items_cap / 2, ((size_t)1 << 30) / unit_o));
    if (st->part_o) cudaFree(st->part_o);
    if (st->part_ml) cudaFree(st->part_ml);
    st->part_o = st->part_ml = nullptr;
    st->items_cap = 0;
    if (cudaMalloc((void**)&st->part_o, cap * unit_o) != cudaSuccess ||
        cudaMalloc((void**)&st->part_ml, cap * dm.group * 2 * 4) != cudaSuccess) {
      cudaGetLastError();
      if (st->part_o) cudaFree(st->part_o);
      st->part_o = nullptr;
      return false;
    }
    st->items_cap = cap;
  }
  return true;
}

// Returns false (exact kernel runs instead) for unsupported shapes or when the
// split scratch would exceed its cap.  The scratch grows on demand (a split
// step reserves it for all its items before its halves start).
inline bool fast_attention_try(sr_model* m, const float* pool_data, int n, const FaWork& work, int layer,
                               op16* xh = nullptr, op16* xl = nullptr, const FaLane* lane = nullptr) {
  const int all_items = lane ? lane->base.items + work.items : work.items;
  if (!fa_reserve(m, all_items)) return false;
  FastState* st = fast_state(m);
  return fast_attention_run(m, pool_data, n, work, layer, st->part_o, st->part_ml, xh, xl, lane);
}

// ------------------------------------------------------------------- linear --
// Returns true when a fast projection kernel handled the call.
bool fast_linear(sr_model* m, const float* X, int n, const Param& W, LinearOut O);

// ------------------------------------------------------------- decode GEMV --
// Whether the decode GEMV covers matrix W for n step rows (1..gv::kMaxRows):
// Q8 rows of a multiple of 16 columns, Q4 of 32 (16-byte aligned rows of codes).
inline bool gemv_covers(const Param& W, int n) {
  if (n < 1 || n > gv::kMaxRows) return false;
  if (W.format == kQ8) return W.cols % 16 == 0;
  if (W.format == kQ4) return W.cols % 32 == 0;
  return false;
}

template <int NR>
inline void gemv_launch(const gv::Args& a, dim3 grid, cudaStream_t s) {
  if (a.fmt == kQ8) gv::k_gemv<kQ8, NR><<<grid, gv::kThreads, 0, s>>>(a);
  else gv::k_gemv<kQ4, NR><<<grid, gv::kThreads, 0, s>>>(a);
}

// Y = X W^T for up to 3 matrices sharing X (same format and width), each with
// its own output.  Returns false when the shapes are not covered or scratch
// cannot be allocated; then nothing was launched and the caller runs the
// tensor-core or exact kernels.
inline bool gemv_run(sr_model* m, const float* X, int n, const Param* const* W, const LinearOut* O, int nseg) {
  if (nseg < 1 || nseg > gv::kMaxSeg) return false;
  for (int i = 0; i < nseg; i++)
    if (!gemv_covers(*W[i], n) || W[i]->format != W[0]->format || W[i]->cols != W[0]->cols ||
        (O[i].out_map != O[0].out_map))
      return false;
  FastState* st = fast_state(m);
  const int nr = n;  // 1 or 2
  gv::Args a;
  a.x = X;
  a.n = n;
  a.in = W[0]->cols;
  a.fmt = W[0]->format;
  a.groups = (a.in + kQBlock - 1) / kQBlock;
  a.rb = a.fmt == kQ8 ? a.in : (a.in + 1) / 2;
  a.nseg = nseg;
  a.out_map = O[0].out_map;
  int tiles = 0;
  const int rpc = gv::rows_per_cta(nr);
  for (int i = 0; i < nseg; i++) {
    gv::Seg& g = a.seg[i];
    g.rows = W[i]->rows;
    g.tiles = (g.rows + rpc - 1) / rpc;
    g.w = (const uint8_t*)W[i]->values;
    g.scales = W[i]->scales;
    g.y = O[i].y;
    g.ldy = O[i].ldy;
    g.bias = O[i].bias;
    g.resid = O[i].resid;
    tiles += g.tiles;
  }
  for (int i = nseg; i < gv::kMaxSeg; i++) a.seg[i] = a.seg[0];
  a.total_tiles = tiles;
  // K splits: at least enough that a CTA's columns fit its staged chunk, more
  // (down to one warp span each) until the launch has about 4 CTAs per SM.
  const int chunk = gv::chunk_for(nr), span = gv::span_for(a.fmt);
  const int min_split = (a.in + chunk - 1) / chunk, max_split = std::max(min_split, (a.in + span - 1) / span);
  const int ksplit = std::max(min_split, std::min(max_split, (148 * 4 + tiles - 1) / tiles));
  a.kper = ((a.in + ksplit - 1) / ksplit + span - 1) / span * span;
  a.ksplit = (a.in + a.kper - 1) / a.kper;
  a.part = nullptr;
  a.counters = nullptr;
  if (a.ksplit > 1) {
    const size_t need = (size_t)a.ksplit * tiles * rpc * nr;
    if (need > st->gv_part_floats) {
      if (st->gv_part) cudaFree(st->gv_part);
      st->gv_part = nullptr;
      st->gv_part_floats = 0;
      const size_t cap = std::max(need, (size_t)1 << 20);
      if (cudaMalloc((void**)&st->gv_part, cap * 4) != cudaSuccess) {
        cudaGetLastError();
        return false;
      }
      st->gv_part_floats = cap;
    }
    if ((size_t)tiles > st->gv_count_cap) {
      if (st->gv_count) cudaFree(st->gv_count);
      st->gv_count = nullptr;
      st->gv_count_cap = 0;
      const size_t cap = std::max((size_t)tiles, (size_t)4096);
      if (cudaMalloc((void**)&st->gv_count, cap * 4) != cudaSuccess ||
          cudaMemsetAsync(st->gv_count, 0, cap * 4, m->stream) != cudaSuccess) {
        cudaGetLastError();
        if (st->gv_count) cudaFree(st->gv_count);
        st->gv_count = nullptr;
        return false;
      }
      st->gv_count_cap = cap;
    }
    a.part = st->gv_part;
    a.counters = st->gv_count;
  }
  const dim3 grid(tiles, a.ksplit);
  if (nr == 1) gemv_launch<1>(a, grid, m->stream);
  else gemv_launch<2>(a, grid, m->stream);
  sr_count_launch(m);
  return true;
}

}  // namespace sr
