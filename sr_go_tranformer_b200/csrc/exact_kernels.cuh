// exact_kernels.cuh -- SR_MODE_EXACT kernels: the reference's operation order
// on CUDA cores (cmd/monolith/monolith.go, cited as M:line).
//
// Every fp32 multiply and add is an explicit __fmul_rn / __fadd_rn, so nvcc never
// contracts them into FMA; fp64 sums that the reference performs sequentially
// are performed sequentially here too.  With the same inputs these kernels give
// the reference's bits, up to last-ulp differences between CUDA's and Go's fp64
// exp/log/cos/sin, which the float32 casts that follow absorb.
#pragma once

#include <float.h>
#include "common.cuh"

namespace sr {

// ---------------------------------------------------------------- metadata --
// Exclusive prefix sum over the 1024 threads of k_meta (one value per thread);
// *total receives the sum.  Uses ws[32] of shared memory.
__device__ __forceinline__ int meta_scan(int v, int* ws, int* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int incl = v;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const int x = __shfl_up_sync(0xffffffffu, incl, off);
    if (lane >= off) incl += x;
  }
  if (lane == 31) ws[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    int w = ws[lane];
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int x = __shfl_up_sync(0xffffffffu, w, off);
      if (lane >= off) w += x;
    }
    ws[lane] = w;  // inclusive totals of warps 0..lane
  }
  __syncthreads();
  const int excl = incl - v + (warp > 0 ? ws[warp - 1] : 0);
  *total = ws[31];
  __syncthreads();  // ws is reused by the next scan
  return excl;
}

// Ragged-batch metadata (M:6361-6375, 6420-6427): per row the session position
// and page-table base; per selected session its last row (compacted head); and
// the fast-mode attention's work lists: every (row, kAttnSplit-position split)
// item (row_item0 / item_rs: where each row's split partials live), the items
// of rows from 1-token chunks (single_rs), and (group of up to 4 consecutive
// rows of a longer chunk, split) pairs (grp_rs), whose rows share K/V reads.
__global__ void __launch_bounds__(1024) k_meta(StepMeta m, int sessions, int rows) {
  __shared__ int ws[32];
  const int r = threadIdx.x;  // rows <= 1024 = blockDim.x: one row per thread
  int ns = 0, nsa = 0, nsb = 0, grp = 0;
  if (r < rows) {
    int lo = 0, hi = sessions - 1;
    while (lo < hi) {
      int mid = (lo + hi + 1) >> 1;
      if (m.tok_off[mid] <= r) lo = mid; else hi = mid - 1;
    }
    const int pos = m.sess_pos[lo] + (r - m.tok_off[lo]);
    m.row_pos[r] = pos;
    m.row_pbase[r] = m.page_off[lo];
    ns = (pos + 1 + kAttnSplit - 1) / kAttnSplit;
    const int len = m.tok_off[lo + 1] - m.tok_off[lo], k = r - m.tok_off[lo];
    if (len == 1) {
      nsa = ns;
    } else if ((k & 3) == 0) {
      grp = min(4, len - k);
      nsb = (pos + grp + kAttnSplit - 1) / kAttnSplit;  // the group's last row reaches pos + grp
    }
  }
  int total;
  const int base = meta_scan(ns, ws, &total);
  const int base_a = meta_scan(nsa, ws, &total);
  const int base_b = meta_scan(nsb, ws, &total);
  if (r < rows) {
    m.row_item0[r] = base;
    for (int s = 0; s < ns; s++) m.item_rs[base + s] = (r << 16) | s;
    for (int s = 0; s < nsa; s++) m.single_rs[base_a + s] = (r << 16) | s;
    for (int s = 0; s < nsb; s++) m.grp_rs[base_b + s] = (r << 16) | ((grp - 1) << 13) | s;
  }
  if (threadIdx.x == 0) {
    int h = 0;
    for (int i = 0; i < sessions; i++) {
      if (m.want[i]) {
        m.head_src[h] = m.tok_off[i + 1] - 1;
        m.head_dst[h] = i;
        h++;
      }
    }
    *m.n_heads = h;
  }
}

// ------------------------------------------------------------ dequant gather --
// Param.copyRow (M:3900-3921): f32 copy, Q8 float32(q)*scale, Q4 nibble*scale.
__device__ __forceinline__ float param_value(const Param& p, int64_t row, int64_t col) {
  int64_t groups = (p.cols + kQBlock - 1) / kQBlock;
  if (p.format == kQ8) {
    const int8_t* v = (const int8_t*)p.values;
    return fmul((float)v[row * p.cols + col], p.scales[row * groups + col / kQBlock]);
  }
  if (p.format == kQ4) {
    const uint8_t* v = (const uint8_t*)p.values;
    uint32_t b = v[row * ((p.cols + 1) / 2) + col / 2];
    float w = (col & 1) ? q4_hi(b) : q4_lo(b);
    return fmul(w, p.scales[row * groups + col / kQBlock]);
  }
  return ((const float*)p.values)[row * p.cols + col];
}

__global__ void k_embed(Param E, const int32_t* __restrict__ tokens, float* __restrict__ X, int d) {
  int r = blockIdx.x;
  int tok = tokens[r];
  for (int j = threadIdx.x; j < d; j += blockDim.x) X[(int64_t)r * d + j] = param_value(E, tok, j);
}

// ------------------------------------------------------------------ RMSNorm --
// rmsInto (M:6182-6194): ss = sequential fp64 sum of exact squares,
// a = float32(1/sqrt(ss/d+eps)), y = (x*a)*w.  One warp per row; lane 0 adds
// the squares in column order.  src_map (optional) gathers input rows.
constexpr int kNormWarps = 4;
constexpr int kNormChunk = 256;
__global__ void __launch_bounds__(kNormWarps * 32)
k_rmsnorm_exact(const float* __restrict__ X, const int32_t* __restrict__ src_map, const float* __restrict__ w,
                float* __restrict__ Y, int rows, int d, double eps) {
  __shared__ double sq[kNormWarps][kNormChunk];
  int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int r = blockIdx.x * kNormWarps + warp;
  if (r >= rows) return;
  int srow = src_map ? src_map[r] : r;
  const float* x = X + (int64_t)srow * d;
  double ss = 0.0;
  for (int c0 = 0; c0 < d; c0 += kNormChunk) {
    int cn = min(kNormChunk, d - c0);
    for (int j = lane; j < cn; j += 32) {
      double v = (double)x[c0 + j];
      sq[warp][j] = dmul(v, v);
    }
    __syncwarp();
    if (lane == 0)
      for (int j = 0; j < cn; j++) ss = dadd(ss, sq[warp][j]);
    __syncwarp();
  }
  ss = __shfl_sync(0xffffffffu, ss, 0);
  float a = (float)__ddiv_rn(1.0, __dsqrt_rn(dadd(__ddiv_rn(ss, (double)d), eps)));
  float* y = Y + (int64_t)r * d;
  for (int j = lane; j < d; j += 32) y[j] = fmul(fmul(x[j], a), w[j]);
}

// ------------------------------------------------------------------- linear --
// Epilogue shared by the exact linears: y = s (+ bias[o]) or resid + s, written
// to output row out_map[r] (compacted LM-head rows) or r.
struct LinearOut {
  float* y;
  int ldy;
  const float* bias;
  const float* resid;  // may alias y (in-place residual add, M:6400/6417)
  const int32_t* out_map;
};
__device__ __forceinline__ void linear_store(const LinearOut& o, int r, int col, float s) {
  int orow = o.out_map ? o.out_map[r] : r;
  float* dst = o.y + (int64_t)orow * o.ldy + col;
  if (o.bias) s = fadd(s, o.bias[col]);
  if (o.resid) s = fadd(o.resid[(int64_t)orow * o.ldy + col], s);
  *dst = s;
}

// Wide fp64 path for one (row, output) (linearQ8WideInto M:4356-4382,
// linearQ4WideInto M:4754-4780).
template <int FMT>
__device__ float wide_dot(const float* x, const Param& W, int o, int in) {
  int groups = (in + kQBlock - 1) / kQBlock;
  double sum = 0.0;
  for (int g = 0; g < groups; g++) {
    double part = 0.0;
    int end = min((g + 1) * kQBlock, in);
    for (int j = g * kQBlock; j < end; j++) {
      double w;
      if (FMT == kQ8) {
        w = (double)((const int8_t*)W.values)[(int64_t)o * in + j];
      } else {
        uint32_t b = ((const uint8_t*)W.values)[(int64_t)o * ((in + 1) / 2) + j / 2];
        w = (double)((j & 1) ? q4_hi(b) : q4_lo(b));
      }
      part = dadd(part, dmul((double)x[j], w));
    }
    sum = dadd(sum, dmul(part, (double)W.scales[(int64_t)o * groups + g]));
  }
  return (float)sum;
}

// Q8/Q4 exact linear (linearQ8Into M:4074-4189, linearQ4Into M:4387-4511).
// CTA tile: OT outputs x RT rows, K in chunks of 4 blocks (256 columns).
// Phase A: thread (o, b) computes the block partial p = (a+b)+(c+d) (+tail)
//          of block b for all RT rows, reusing each dequantised weight.
// Phase B: thread (r, o) folds s += p*scale over the chunk's blocks in order.
template <int FMT, int OT, int RT>
__global__ void __launch_bounds__(OT * 4)
k_linear_q_exact(const float* __restrict__ X, int n, int in, int out, Param W, LinearOut O) {
  constexpr int T = OT * 4;
  constexpr int CB = (FMT == kQ8) ? 256 : 128;  // weight bytes per row per chunk
  constexpr int WS = CB + 4;                    // odd word stride: conflict-free 32-bit reads across rows
  __shared__ __align__(16) uint8_t w_s[OT * WS];
  __shared__ __align__(16) float x_s[RT * 256];
  __shared__ float p_s[RT * 4 * OT];
  __shared__ int wide_s[RT];
  const int tid = threadIdx.x;
  const int o0 = blockIdx.x * OT, r0 = blockIdx.y * RT;
  const int groups = (in + kQBlock - 1) / kQBlock;
  const int64_t row_bytes = (FMT == kQ8) ? (int64_t)in : (int64_t)((in + 1) / 2);
  const bool w_aligned = (row_bytes % 16) == 0 && (((uintptr_t)W.values) % 16) == 0;
  const bool x_aligned = (in % 4) == 0 && (((uintptr_t)X) % 16) == 0;
  if (tid < RT) wide_s[tid] = 0;
  float acc[RT / 4];
#pragma unroll
  for (int k = 0; k < RT / 4; k++) acc[k] = 0.f;
  const int po = tid % OT, pb = tid / OT;  // phase-A mapping
  const int nchunks = (in + 255) / 256;
  for (int c = 0; c < nchunks; c++) {
    __syncthreads();
    // --- stage weights: OT rows x CB bytes
    const int64_t cbyte0 = (int64_t)c * CB;
    for (int idx = tid; idx < OT * (CB / 16); idx += T) {
      int o = idx / (CB / 16), piece = idx % (CB / 16);
      int og = o0 + o;
      uint4 v = make_uint4(0, 0, 0, 0);
      int64_t b0 = cbyte0 + piece * 16;
      if (og < out && b0 < row_bytes) {
        const uint8_t* src = (const uint8_t*)W.values + (int64_t)og * row_bytes + b0;
        if (w_aligned) {
          v = __ldg((const uint4*)src);
        } else {
          uint8_t tmp[16];
          for (int q = 0; q < 16; q++) tmp[q] = (b0 + q < row_bytes) ? src[q] : 0;
          v = *(uint4*)tmp;
        }
      }
      uint32_t* dst = (uint32_t*)(w_s + o * WS + piece * 16);
      dst[0] = v.x;
      dst[1] = v.y;
      dst[2] = v.z;
      dst[3] = v.w;
    }
    // --- stage activations: RT rows x 256 columns; flag wide rows
    const int col0 = c * 256;
    for (int idx = tid; idx < RT * 64; idx += T) {
      int r = idx / 64, q = idx % 64;
      int rg = r0 + r, j = col0 + q * 4;
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (rg < n) {
        const float* src = X + (int64_t)rg * in + j;
        if (x_aligned && j + 4 <= in) {
          v = *(const float4*)src;
        } else {
          if (j < in) v.x = src[0];
          if (j + 1 < in) v.y = src[1];
          if (j + 2 < in) v.z = src[2];
          if (j + 3 < in) v.w = src[3];
        }
        const float lim = wide_limit();
        if (v.x > lim || v.x < -lim || v.y > lim || v.y < -lim || v.z > lim || v.z < -lim || v.w > lim ||
            v.w < -lim)
          atomicOr(&wide_s[r], 1);
      }
      *(float4*)(x_s + r * 256 + q * 4) = v;
    }
    __syncthreads();
    // --- phase A: block partials
    {
      const int g = c * 4 + pb;
      if (g < groups) {
        const int jb = pb * 64;                      // column offset inside the chunk
        const int cnt = min(kQBlock, in - g * kQBlock);
        float A[RT], B[RT], Cc[RT], D[RT];
#pragma unroll
        for (int r = 0; r < RT; r++) A[r] = B[r] = Cc[r] = D[r] = 0.f;
        const int full4 = cnt & ~3;
        for (int j = 0; j < full4; j += 4) {
          float w0, w1, w2, w3;
          if (FMT == kQ8) {
            uint32_t wb = *(const uint32_t*)(w_s + po * WS + jb + j);
            w0 = (float)(int8_t)(wb & 0xff);
            w1 = (float)(int8_t)((wb >> 8) & 0xff);
            w2 = (float)(int8_t)((wb >> 16) & 0xff);
            w3 = (float)(int8_t)(wb >> 24);
          } else {
            uint32_t wb = *(const uint16_t*)(w_s + po * WS + (jb + j) / 2);
            w0 = q4_lo(wb & 0xff);
            w1 = q4_hi(wb & 0xff);
            w2 = q4_lo(wb >> 8);
            w3 = q4_hi(wb >> 8);
          }
#pragma unroll
          for (int r = 0; r < RT; r++) {
            float4 xv = *(const float4*)(x_s + r * 256 + jb + j);
            A[r] = fadd(A[r], fmul(xv.x, w0));
            B[r] = fadd(B[r], fmul(xv.y, w1));
            Cc[r] = fadd(Cc[r], fmul(xv.z, w2));
            D[r] = fadd(D[r], fmul(xv.w, w3));
          }
        }
#pragma unroll
        for (int r = 0; r < RT; r++) {
          float p = fadd(fadd(A[r], B[r]), fadd(Cc[r], D[r]));
          for (int j = full4; j < cnt; j++) {
            float w;
            if (FMT == kQ8) {
              w = (float)(int8_t)w_s[po * WS + jb + j];
            } else {
              uint32_t b = w_s[po * WS + (jb + j) / 2];
              w = (j & 1) ? q4_hi(b) : q4_lo(b);
            }
            p = fadd(p, fmul(x_s[r * 256 + jb + j], w));
          }
          p_s[(r * 4 + pb) * OT + po] = p;
        }
      }
    }
    __syncthreads();
    // --- phase B: ordered fold over the chunk's blocks
    {
      const int o = tid % OT, rq = tid / OT;
      const int og = o0 + o;
      if (og < out) {
#pragma unroll
        for (int k = 0; k < RT / 4; k++) {
          const int r = rq + 4 * k;
          for (int b = 0; b < 4; b++) {
            const int g = c * 4 + b;
            if (g >= groups) break;
            acc[k] = fadd(acc[k], fmul(p_s[(r * 4 + b) * OT + o], W.scales[(int64_t)og * groups + g]));
          }
        }
      }
    }
  }
  __syncthreads();
  const int o = tid % OT, rq = tid / OT;
  const int og = o0 + o;
  if (og >= out) return;
#pragma unroll
  for (int k = 0; k < RT / 4; k++) {
    const int r = rq + 4 * k, rg = r0 + r;
    if (rg >= n) continue;
    float s = acc[k];
    if (wide_s[r]) s = wide_dot<FMT>(X + (int64_t)rg * in, W, og, in);
    linear_store(O, rg, og, s);
  }
}

// FP32 exact linear (linearFP32Range M:3970-4070): one sequential accumulator
// per (row, output) over all columns, for every tile shape.
template <int OT, int RT>
__global__ void __launch_bounds__(OT * 4)
k_linear_f32_exact(const float* __restrict__ X, int n, int in, int out, Param W, LinearOut O) {
  constexpr int T = OT * 4;
  constexpr int KC = 64;
  constexpr int WS = KC + 4;
  __shared__ __align__(16) float w_s[OT * WS];
  __shared__ __align__(16) float x_s[RT * KC];
  const int tid = threadIdx.x;
  const int o0 = blockIdx.x * OT, r0 = blockIdx.y * RT;
  const float* Wv = (const float*)W.values;
  const bool aligned = (in % 4) == 0 && (((uintptr_t)Wv) % 16) == 0 && (((uintptr_t)X) % 16) == 0;
  const int o = tid % OT, rq = tid / OT;
  float acc[RT / 4];
#pragma unroll
  for (int k = 0; k < RT / 4; k++) acc[k] = 0.f;
  for (int c0 = 0; c0 < in; c0 += KC) {
    const int cn = min(KC, in - c0);
    __syncthreads();
    for (int idx = tid; idx < OT * (KC / 4); idx += T) {
      int oo = idx / (KC / 4), q = idx % (KC / 4), j = c0 + q * 4;
      int og = o0 + oo;
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (og < out) {
        const float* src = Wv + (int64_t)og * in + j;
        if (aligned && j + 4 <= in) {
          v = __ldg((const float4*)src);
        } else {
          if (j < in) v.x = src[0];
          if (j + 1 < in) v.y = src[1];
          if (j + 2 < in) v.z = src[2];
          if (j + 3 < in) v.w = src[3];
        }
      }
      *(float4*)(w_s + oo * WS + q * 4) = v;
    }
    for (int idx = tid; idx < RT * (KC / 4); idx += T) {
      int r = idx / (KC / 4), q = idx % (KC / 4), j = c0 + q * 4;
      int rg = r0 + r;
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (rg < n) {
        const float* src = X + (int64_t)rg * in + j;
        if (aligned && j + 4 <= in) {
          v = *(const float4*)src;
        } else {
          if (j < in) v.x = src[0];
          if (j + 1 < in) v.y = src[1];
          if (j + 2 < in) v.z = src[2];
          if (j + 3 < in) v.w = src[3];
        }
      }
      *(float4*)(x_s + r * KC + q * 4) = v;
    }
    __syncthreads();
    const int full4 = cn & ~3;
#pragma unroll
    for (int k = 0; k < RT / 4; k++) {
      const int r = rq + 4 * k;
      float s = acc[k];
      for (int j = 0; j < full4; j += 4) {
        float4 wv = *(const float4*)(w_s + o * WS + j);
        float4 xv = *(const float4*)(x_s + r * KC + j);
        s = fadd(s, fmul(xv.x, wv.x));
        s = fadd(s, fmul(xv.y, wv.y));
        s = fadd(s, fmul(xv.z, wv.z));
        s = fadd(s, fmul(xv.w, wv.w));
      }
      for (int j = full4; j < cn; j++) s = fadd(s, fmul(x_s[r * KC + j], w_s[o * WS + j]));
      acc[k] = s;
    }
  }
  const int og = o0 + o;
  if (og >= out) return;
#pragma unroll
  for (int k = 0; k < RT / 4; k++) {
    const int rg = r0 + rq + 4 * k;
    if (rg < n) linear_store(O, rg, og, acc[k]);
  }
}

// ------------------------------------------------------------ RoPE + KV write --
// Model.rope HF half-split branch (M:5264-5289) on Q and K, then the K/V rows
// are written into the row's page (KVCache.row M:6038-6043, copy M:6393-6395).
__global__ void k_rope_kv_exact(float* __restrict__ Q, const float* __restrict__ K, const float* __restrict__ V,
                                const float* __restrict__ cos_t, const float* __restrict__ sin_t, StepMeta meta,
                                float* __restrict__ pool, ModelDims dm, int layer, int row0) {
  const int r = row0 + blockIdx.x;  // row0: first row of a split step's half (else 0)
  const int pos = meta.row_pos[r];
  const int half = dm.hd / 2;
  const float* ct = cos_t + (int64_t)pos * half;
  const float* st = sin_t + (int64_t)pos * half;
  float* q = Q + (int64_t)r * dm.qd;
  for (int idx = threadIdx.x; idx < dm.heads * half; idx += blockDim.x) {
    int h = idx / half, j = idx % half;
    int i = h * dm.hd + j, z = i + half;
    float c = ct[j], s = st[j], a = q[i], b = q[z];
    q[i] = fsub(fmul(a, c), fmul(b, s));
    q[z] = fadd(fmul(a, s), fmul(b, c));
  }
  const int64_t page = meta.page_ids[meta.row_pbase[r] + pos / dm.page_tokens];
  float* kdst = pool + page * dm.page_elems + (int64_t)layer * 2 * dm.page_tokens * dm.kvd +
                (int64_t)(pos % dm.page_tokens) * dm.kvd;
  float* vdst = kdst + (int64_t)dm.page_tokens * dm.kvd;
  const float* k = K + (int64_t)r * dm.kvd;
  for (int idx = threadIdx.x; idx < dm.kv_heads * half; idx += blockDim.x) {
    int h = idx / half, j = idx % half;
    int i = h * dm.hd + j, z = i + half;
    float c = ct[j], s = st[j], a = k[i], b = k[z];
    kdst[i] = fsub(fmul(a, c), fmul(b, s));
    kdst[z] = fadd(fmul(a, s), fmul(b, c));
  }
  const float* v = V + (int64_t)r * dm.kvd;
  for (int j = threadIdx.x; j < dm.kvd; j += blockDim.x) vdst[j] = v[j];
}

// ---------------------------------------------------------------- attention --
// attend (M:5293-5352) for one (row, KV head): the `group` query heads sharing
// that KV head are processed together so each K/V row is read once per pass.
//   pass 1: scores s = (q.k sequential over hd) * scale, running max in order;
//   pass 2: sum += exp(f64(s) - f64(max)) sequentially in position order;
//   pass 3: p = float32(exp(f64(s) - lse)), out[j] += p*v[j] in position order.
// Scores stay in shared memory when they fit (smem_scores); otherwise each pass
// recomputes them from K with the identical dot order.
constexpr int kAttnTile = 64;
struct AttnArgs {
  const float* Q;
  float* A;
  const float* pool;
  StepMeta meta;
  ModelDims dm;
  int layer;
  float scale;
  int smem_scores;  // 1: all scores resident in smem (stride ls)
  int ls;
};

__device__ __forceinline__ void attn_load_tile(const AttnArgs& a, float* dst, int r, int kh, int t0, int tn,
                                               bool value) {
  const int hd = a.dm.hd, hdp = hd + 4, pt = a.dm.page_tokens;
  const int q4 = hd / 4;
  const int pbase = a.meta.row_pbase[r];
  const int64_t lay = (int64_t)a.layer * 2 * pt * a.dm.kvd + (value ? (int64_t)pt * a.dm.kvd : 0) + (int64_t)kh * hd;
  for (int idx = threadIdx.x; idx < tn * q4; idx += blockDim.x) {
    int s = idx / q4, c = idx % q4, pos = t0 + s;
    int64_t page = a.meta.page_ids[pbase + pos / pt];
    const float4* src = (const float4*)(a.pool + page * a.dm.page_elems + lay + (int64_t)(pos % pt) * a.dm.kvd) + c;
    *(float4*)(dst + s * hdp + 4 * c) = __ldg(src);
  }
}

__device__ __forceinline__ void attn_tile_scores(const AttnArgs& a, const float* q_s, const float* kv_s, float* dst,
                                                 int dstride, int doff, int tn) {
  const int hd = a.dm.hd, hdp = hd + 4, group = a.dm.group;
  for (int idx = threadIdx.x; idx < group * tn; idx += blockDim.x) {
    int g = idx / tn, s = idx % tn;
    const float* qg = q_s + g * hd;
    const float* ks = kv_s + s * hdp;
    float dot = 0.f;
    for (int j = 0; j < hd; j += 4) {
      float4 qv = *(const float4*)(qg + j);
      float4 kv = *(const float4*)(ks + j);
      dot = fadd(dot, fmul(qv.x, kv.x));
      dot = fadd(dot, fmul(qv.y, kv.y));
      dot = fadd(dot, fmul(qv.z, kv.z));
      dot = fadd(dot, fmul(qv.w, kv.w));
    }
    dst[g * dstride + doff + s] = fmul(dot, a.scale);
  }
}

__host__ __device__ inline int attn_align4(int x) { return (x + 3) & ~3; }

// Shared-memory layout (floats unless noted), used by host sizing too.
struct AttnSmem {
  int q, kv, sc, p, ex, mx, sum, lse, total;  // offsets in 4-byte words; ex/sum/lse are doubles
  __host__ __device__ AttnSmem(int group, int hd, int smem_scores, int ls) {
    int o = 0;
    q = o; o += attn_align4(group * hd);
    kv = o; o += attn_align4(kAttnTile * (hd + 4));
    sc = o; o += attn_align4(group * (smem_scores ? ls : kAttnTile));
    p = o; o += attn_align4(group * kAttnTile);
    ex = o; o += attn_align4(2 * group * kAttnTile);
    mx = o; o += attn_align4(group);
    sum = o; o += attn_align4(2 * group);
    lse = o; o += attn_align4(2 * group);
    total = o;
  }
};

__global__ void k_attention_exact(AttnArgs a) {
  extern __shared__ __align__(16) float smem[];
  const int r = blockIdx.x, kh = blockIdx.y;
  const int hd = a.dm.hd, hdp = hd + 4, group = a.dm.group;
  const int L = a.meta.row_pos[r] + 1;
  AttnSmem lay(group, hd, a.smem_scores, a.ls);
  float* q_s = smem + lay.q;
  float* kv_s = smem + lay.kv;
  float* sc_s = smem + lay.sc;
  float* p_s = smem + lay.p;
  double* ex_s = (double*)(smem + lay.ex);
  float* mx_s = smem + lay.mx;
  double* sum_s = (double*)(smem + lay.sum);
  double* lse_s = (double*)(smem + lay.lse);
  const int sstride = a.smem_scores ? a.ls : kAttnTile;
  const float* qrow = a.Q + (int64_t)r * a.dm.qd + (int64_t)kh * group * hd;
  for (int i = threadIdx.x; i < group * hd; i += blockDim.x) q_s[i] = qrow[i];
  if (threadIdx.x < group) {
    mx_s[threadIdx.x] = -FLT_MAX;
    sum_s[threadIdx.x] = 0.0;
  }
  // pass 1: scores and running max
  for (int t0 = 0; t0 < L; t0 += kAttnTile) {
    const int tn = min(kAttnTile, L - t0);
    const int off = a.smem_scores ? t0 : 0;
    __syncthreads();
    attn_load_tile(a, kv_s, r, kh, t0, tn, false);
    __syncthreads();
    attn_tile_scores(a, q_s, kv_s, sc_s, sstride, off, tn);
    __syncthreads();
    if (threadIdx.x < group) {
      float m = mx_s[threadIdx.x];
      const float* sg = sc_s + threadIdx.x * sstride + off;
      for (int s = 0; s < tn; s++)
        if (sg[s] > m) m = sg[s];
      mx_s[threadIdx.x] = m;
    }
  }
  // pass 2: fp64 sum of exp(s - max), sequential in position order
  for (int t0 = 0; t0 < L; t0 += kAttnTile) {
    const int tn = min(kAttnTile, L - t0);
    const int off = a.smem_scores ? t0 : 0;
    __syncthreads();
    if (!a.smem_scores) {
      attn_load_tile(a, kv_s, r, kh, t0, tn, false);
      __syncthreads();
      attn_tile_scores(a, q_s, kv_s, sc_s, sstride, off, tn);
      __syncthreads();
    }
    for (int idx = threadIdx.x; idx < group * tn; idx += blockDim.x) {
      int g = idx / tn, s = idx % tn;
      ex_s[g * kAttnTile + s] = exp(__dsub_rn((double)sc_s[g * sstride + off + s], (double)mx_s[g]));
    }
    __syncthreads();
    if (threadIdx.x < group) {
      double acc = sum_s[threadIdx.x];
      for (int s = 0; s < tn; s++) acc = dadd(acc, ex_s[threadIdx.x * kAttnTile + s]);
      sum_s[threadIdx.x] = acc;
    }
  }
  __syncthreads();
  if (threadIdx.x < group) lse_s[threadIdx.x] = dadd((double)mx_s[threadIdx.x], log(sum_s[threadIdx.x]));
  // pass 3: p = float32(exp(s - lse)); out[j] += p*v[j] in position order
  const int q4 = hd / 4;
  const int pairs = group * q4;
  const bool owner = threadIdx.x < pairs;
  const int pg = owner ? threadIdx.x / q4 : 0, pj = owner ? (threadIdx.x % q4) * 4 : 0;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int t0 = 0; t0 < L; t0 += kAttnTile) {
    const int tn = min(kAttnTile, L - t0);
    const int off = a.smem_scores ? t0 : 0;
    __syncthreads();
    if (!a.smem_scores) {
      attn_load_tile(a, kv_s, r, kh, t0, tn, false);
      __syncthreads();
      attn_tile_scores(a, q_s, kv_s, sc_s, sstride, off, tn);
      __syncthreads();
    }
    for (int idx = threadIdx.x; idx < group * tn; idx += blockDim.x) {
      int g = idx / tn, s = idx % tn;
      p_s[g * kAttnTile + s] = (float)exp(__dsub_rn((double)sc_s[g * sstride + off + s], lse_s[g]));
    }
    __syncthreads();
    attn_load_tile(a, kv_s, r, kh, t0, tn, true);
    __syncthreads();
    if (owner) {
      const float* pp = p_s + pg * kAttnTile;
      for (int s = 0; s < tn; s++) {
        float p = pp[s];
        float4 v = *(const float4*)(kv_s + s * hdp + pj);
        acc.x = fadd(acc.x, fmul(p, v.x));
        acc.y = fadd(acc.y, fmul(p, v.y));
        acc.z = fadd(acc.z, fmul(p, v.z));
        acc.w = fadd(acc.w, fmul(p, v.w));
      }
    }
  }
  if (owner) {
    float* out = a.A + (int64_t)r * a.dm.qd + (int64_t)(kh * group + pg) * hd + pj;
    *(float4*)out = acc;
  }
}

// ------------------------------------------------------------------- SwiGLU --
// h = float32(g/(1+exp(-g))) * u with the division and exp in fp64 (M:6410-6413).
__global__ void k_swiglu_exact(const float* __restrict__ G, const float* __restrict__ U, float* __restrict__ H,
                               int64_t count) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < count; i += (int64_t)gridDim.x * blockDim.x) {
    double g = (double)G[i];
    float s = (float)__ddiv_rn(g, dadd(1.0, exp(-g)));
    H[i] = fmul(s, U[i]);
  }
}

}  // namespace sr
