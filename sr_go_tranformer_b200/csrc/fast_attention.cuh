// fast_attention.cuh -- SR_MODE_FAST paged GQA attention (flash-decoding).
//
// Same mathematics as attend (cmd/monolith/monolith.go:5293-5352), reordered
// for the B200.  Every (row, KV head) context is cut into splits of kFaSplit
// positions, one CTA per split (grid: the step's compact (row, split) item list
// built by k_meta x KV heads, so no CTA is launched past a row's context); the `group` query heads that share a KV head
// read each K/V element once (GQA), keep an online softmax (running max,
// rescaled sum and output) and write the split's (O, m, l); a combine kernel
// merges the splits with their log-sum-exp weights.  Results match the exact
// path within fp32 rounding (tolerance-checked), not bit for bit.
//
// head_dim 128 (Mistral, Qwen): k_attn_warp128 -- each of the 4 warps streams
//   its own sub-split (a quarter of the split) through a private 2-stage ring of
//   8-position tiles (one 512-byte bulk copy per K or V row, issued by the
//   row's lane, completing on the warp's mbarrier) and keeps its own softmax
//   state, synchronising with __syncwarp only; the warps merge once at the
//   end of the split.
// head_dim 64 (SmolLM, Llama-1B): k_attn_tile -- the CTA shares 32-position
//   double-buffered tiles.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <float.h>

#include "common.cuh"
#include "tc_gemm.cuh"  // mbarrier and bulk-copy helpers

namespace sr {

constexpr int kFaThreads = 128;
constexpr int kFaSplit = kAttnSplit;  // positions per CTA

struct FastAttnArgs {
  const float* Q;
  float* A;
  const float* pool;
  StepMeta meta;
  ModelDims dm;
  int layer;
  float scale;
  float* part_o;   // [items][kv_heads][group][hd]
  float* part_ml;  // [items][kv_heads][group][2]
  op16* xh;  // optional: write the output as bf16 hi/lo planes (the next
  op16* xl;  // projection's tensor-core operand) instead of fp32 A
  int* err;           // raised when a bounded wait for a tile expires
  // One half of a split step: its first row and its first entries of the
  // single / group / item lists (all zero for a whole step).  The combine
  // runs over the half's rows and writes the planes from the half's row 0.
  int row0 = 0, single0 = 0, grp0 = 0, item0 = 0;
};

// One fp32 activation as the projection's two bf16 operand terms:
// x ~= hi + lo with |x - hi - lo| <= 2^-17 |x|.
__device__ __forceinline__ void split_op(float x, op16* hi, op16* lo) {
  const __nv_bfloat16 h = __float2bfloat16_rn(x);
  *hi = h;
  *lo = __float2bfloat16_rn(x - __bfloat162float(h));
}

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  unsigned s = (unsigned)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(s), "l"(gmem));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N));
}

__device__ __forceinline__ void fa_write_split(const FastAttnArgs& a, int item_idx, int kh, int G, int HD,
                                               const float* o_smem, const float* ml_smem) {
  const int64_t item = (int64_t)item_idx * a.dm.kv_heads + kh;
  for (int idx = threadIdx.x; idx < G * HD; idx += kFaThreads) a.part_o[item * G * HD + idx] = o_smem[idx];
  if (threadIdx.x < 2 * G) a.part_ml[item * G * 2 + threadIdx.x] = ml_smem[threadIdx.x];
}

// ===================================================== head_dim 128: per warp
constexpr int kWpMT = 8;                 // positions per warp tile
constexpr int kWpSub = kFaSplit / 4;     // positions per warp

template <int G>
struct WarpSmem {
  static constexpr int HD = 128;
  static constexpr int GP = (G + 3) & ~3;
  static constexpr int KV = 2 * 2 * kWpMT * HD;   // [stage][K|V][pos][HD]
  static constexpr int SC = G * kWpMT;            // scores [G][MT]
  static constexpr int PS = kWpMT * GP;           // probabilities [MT][GP]
  static constexpr int PER_WARP = KV + SC + PS;
  static constexpr int TOTAL = 4 * PER_WARP;      // floats, then 4 x 2 mbarriers
  static constexpr size_t BYTES = (size_t)TOTAL * 4 + 4 * 2 * 8;
};

// One 8-position tile of a warp's online-softmax attention for the G query
// heads of a KV head (head_dim 128): scores with 8 lanes per position, the
// softmax state (mreg, lreg: head lane/8 + 4*round, replicated in its 8 lanes)
// and the output (acc[g]: dims 4*lane..4*lane+3) updated in place.  kt / vt:
// the tile's K and V rows in shared memory; tn <= 8 valid positions; sc / ps:
// the warp's score and probability scratch.
template <int G>
__device__ __forceinline__ void warp_tile8(const float* kt, const float* vt, int tn, const float4 (&q)[G][4],
                                           float (&mreg)[(G + 3) / 4], float (&lreg)[(G + 3) / 4], float4 (&acc)[G],
                                           float* sc, float* ps, int lane) {
  constexpr int HD = 128, MT = kWpMT, GP = (G + 3) & ~3;
  constexpr int ROUNDS = (G + 3) / 4;
  // scores: 8 lanes per position, 4 positions per pass, 2 passes
#pragma unroll
  for (int pass = 0; pass < 2; pass++) {
    const int s = pass * 4 + (lane >> 3);
    float part[G];
#pragma unroll
    for (int g = 0; g < G; g++) part[g] = 0.f;
    if (s < tn) {
      const float* kr = kt + s * HD + 4 * (lane & 7);
#pragma unroll
      for (int i = 0; i < 4; i++) {
        const float4 kx = *(const float4*)(kr + 32 * i);
#pragma unroll
        for (int g = 0; g < G; g++) {
          part[g] = fmaf(q[g][i].x, kx.x, part[g]);
          part[g] = fmaf(q[g][i].y, kx.y, part[g]);
          part[g] = fmaf(q[g][i].z, kx.z, part[g]);
          part[g] = fmaf(q[g][i].w, kx.w, part[g]);
        }
      }
    }
    if constexpr (G == 4) {
      // reduce-scatter over the 8 lanes of the position: after the three
      // exchanges lane bits (b0, b1) hold head 2*b0 + b1 (4 shuffles, not 12)
      const bool b0 = lane & 1, b1 = lane & 2;
      float k0 = b0 ? part[2] : part[0], k1 = b0 ? part[3] : part[1];
      const float x0 = b0 ? part[0] : part[2], x1 = b0 ? part[1] : part[3];
      k0 += __shfl_xor_sync(0xffffffffu, x0, 1);
      k1 += __shfl_xor_sync(0xffffffffu, x1, 1);
      float kk = b1 ? k1 : k0;
      kk += __shfl_xor_sync(0xffffffffu, b1 ? k0 : k1, 2);
      kk += __shfl_xor_sync(0xffffffffu, kk, 4);
      if ((lane & 4) == 0) sc[(2 * (int)b0 + (int)b1) * MT + s] = s < tn ? kk : -INFINITY;
    } else if constexpr (G > 4) {
      // 5..8 heads, padded to 8: reduce-scatter over the position's 8 lanes
      // (7 shuffles instead of 3 per head); lane bits (b0, b1, b2) end up
      // holding head 4*b0 + 2*b1 + b2
      float h8[8];
#pragma unroll
      for (int g = 0; g < 8; g++) h8[g] = g < G ? part[g] : 0.f;
      const bool b0 = lane & 1, b1 = lane & 2, b2 = lane & 4;
      float k4[4];
#pragma unroll
      for (int j = 0; j < 4; j++) {
        const float keep = b0 ? h8[4 + j] : h8[j], send = b0 ? h8[j] : h8[4 + j];
        k4[j] = keep + __shfl_xor_sync(0xffffffffu, send, 1);
      }
      float m0 = b1 ? k4[2] : k4[0], m1 = b1 ? k4[3] : k4[1];
      const float s0 = b1 ? k4[0] : k4[2], s1 = b1 ? k4[1] : k4[3];
      m0 += __shfl_xor_sync(0xffffffffu, s0, 2);
      m1 += __shfl_xor_sync(0xffffffffu, s1, 2);
      float kk = b2 ? m1 : m0;
      kk += __shfl_xor_sync(0xffffffffu, b2 ? m0 : m1, 4);
      const int h = 4 * (int)b0 + 2 * (int)b1 + (int)b2;
      if (h < G) sc[h * MT + s] = s < tn ? kk : -INFINITY;
    } else {
#pragma unroll
      for (int off = 1; off < 8; off <<= 1)
#pragma unroll
        for (int g = 0; g < G; g++) part[g] += __shfl_xor_sync(0xffffffffu, part[g], off);
      if ((lane & 7) == 0)
#pragma unroll
        for (int g = 0; g < G; g++) sc[g * MT + s] = s < tn ? part[g] : -INFINITY;
    }
  }
  __syncwarp();
  // online softmax: lane = (head lane/8 + 4*round, position lane%8)
  float alpha[ROUNDS];
#pragma unroll
  for (int k = 0; k < ROUNDS; k++) {
    const int g = (lane >> 3) + 4 * k;
    const float v = g < G ? sc[g * MT + (lane & 7)] : -INFINITY;
    float mt = v;
#pragma unroll
    for (int off = 1; off < 8; off <<= 1) mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, off));
    const float mo = mreg[k];
    const float mn = fmaxf(mo, mt);
    const float p = (v == -INFINITY) ? 0.f : __expf(v - mn);
    float sum = p;
#pragma unroll
    for (int off = 1; off < 8; off <<= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
    const float al = (mo == -INFINITY) ? 0.f : __expf(mo - mn);
    lreg[k] = lreg[k] * al + sum;
    mreg[k] = mn;
    alpha[k] = al;
    if (g < G) ps[(lane & 7) * GP + g] = p;
  }
  __syncwarp();
  // rescale and accumulate P.V: lane owns dims 4*lane..4*lane+3
#pragma unroll
  for (int g = 0; g < G; g++) {
    const float al = __shfl_sync(0xffffffffu, alpha[g / 4], (g % 4) * 8);
    acc[g].x *= al;
    acc[g].y *= al;
    acc[g].z *= al;
    acc[g].w *= al;
  }
  for (int s = 0; s < tn; s++) {
    const float4 v = *(const float4*)(vt + s * HD + 4 * lane);
    const float* pp = ps + s * GP;
#pragma unroll
    for (int g4 = 0; g4 < GP; g4 += 4) {
      const float4 p4 = *(const float4*)(pp + g4);
      const float pv[4] = {p4.x, p4.y, p4.z, p4.w};
#pragma unroll
      for (int j = 0; j < 4; j++) {
        if (g4 + j < G) {
          acc[g4 + j].x = fmaf(pv[j], v.x, acc[g4 + j].x);
          acc[g4 + j].y = fmaf(pv[j], v.y, acc[g4 + j].y);
          acc[g4 + j].z = fmaf(pv[j], v.z, acc[g4 + j].z);
          acc[g4 + j].w = fmaf(pv[j], v.w, acc[g4 + j].w);
        }
      }
    }
  }
}

// grid: the step's single-row items (rows of 1-token chunks) x KV heads
template <int G>
__global__ void __launch_bounds__(kFaThreads) k_attn_warp128(FastAttnArgs a) {
  constexpr int HD = 128, MT = kWpMT;
  constexpr int ROUNDS = (G + 3) / 4;  // softmax passes: 4 heads x 8 positions per pass
  extern __shared__ __align__(16) float fsm[];
  const int rs = a.meta.single_rs[a.single0 + blockIdx.x], kh = blockIdx.y;
  const int r = rs >> 16, split = rs & 0xffff;
  const int L = a.meta.row_pos[r] + 1;
  const int s0 = split * kFaSplit;
  if (s0 >= L) return;
  const int s1 = min(L, s0 + kFaSplit);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  float* wsm = fsm + warp * WarpSmem<G>::PER_WARP;
  float* kv = wsm;                                 // [2][2][MT][HD]
  float* sc = wsm + WarpSmem<G>::KV;               // [G][MT]
  float* ps = sc + WarpSmem<G>::SC;                // [MT][GP]
  uint64_t* bar = (uint64_t*)(fsm + WarpSmem<G>::TOTAL) + warp * 2;  // past the merge area
  const int pbase = a.meta.row_pbase[r];
  const int pt = a.dm.page_tokens;
  const int64_t lay = (int64_t)a.layer * 2 * pt * a.dm.kvd + (int64_t)kh * HD;
  const int64_t vofs = (int64_t)pt * a.dm.kvd;
  const int ws0 = s0 + warp * kWpSub;
  const int ws1 = min(s1, ws0 + kWpSub);
  const int nw = max(0, ws1 - ws0);
  const int ntiles = (nw + MT - 1) / MT;

  // The warp's page ids, one per lane (when its sub-split spans <= 32 pages),
  // so the tile loader never waits on a dependent global load.
  const int pg0 = ws0 / pt;
  const int npg = nw > 0 ? (ws1 - 1) / pt - pg0 + 1 : 0;
  const bool page_regs = npg <= 32;
  const int my_page = (page_regs && lane < npg) ? a.meta.page_ids[pbase + pg0 + lane] : 0;
  if (lane == 0) {
    tc::mbar_init(&bar[0], 1);
    tc::mbar_init(&bar[1], 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncwarp();
  // Tile t -> stage t & 1: lane s copies the K and V rows of position t0 + s.
  auto load_tile = [&](int t) {
    const int st = t & 1;
    float* dst = kv + st * 2 * MT * HD;
    const int t0 = ws0 + t * MT, tn = min(MT, ws1 - t0);
    if (lane == 0) tc::mbar_expect_tx(&bar[st], (uint32_t)tn * 2 * HD * 4);
    __syncwarp();
    const int pos = t0 + min(lane, tn - 1);
    const int pi = pos / pt;
    const int pg = __shfl_sync(0xffffffffu, my_page, (pi - pg0) & 31);
    if (lane < tn) {
      const int64_t page = page_regs ? pg : a.meta.page_ids[pbase + pi];
      const float* krow = a.pool + page * a.dm.page_elems + lay + (int64_t)(pos - pi * pt) * a.dm.kvd;
      tc::bulk_load(dst + lane * HD, krow, HD * 4, &bar[st]);
      tc::bulk_load(dst + (MT + lane) * HD, krow + vofs, HD * 4, &bar[st]);
    }
  };
  if (ntiles > 0) load_tile(0);
  bool ok = true;

  // query slices: lane covers dims 4*(lane%8) + 32*i for the score phase
  float4 q[G][4];
  {
    const float* qrow = a.Q + (int64_t)r * a.dm.qd + (int64_t)kh * G * HD;
    const int jl = lane & 7;
#pragma unroll
    for (int g = 0; g < G; g++)
#pragma unroll
      for (int i = 0; i < 4; i++) {
        const float4 v = *(const float4*)(qrow + g * HD + 4 * jl + 32 * i);
        q[g][i] = make_float4(v.x * a.scale, v.y * a.scale, v.z * a.scale, v.w * a.scale);
      }
  }
  float mreg[ROUNDS], lreg[ROUNDS];  // softmax state of head (lane/8 + 4*round), replicated in its 8 lanes
#pragma unroll
  for (int k = 0; k < ROUNDS; k++) {
    mreg[k] = -INFINITY;
    lreg[k] = 0.f;
  }
  float4 acc[G];  // output dims 4*lane..4*lane+3 of every head
#pragma unroll
  for (int g = 0; g < G; g++) acc[g] = make_float4(0.f, 0.f, 0.f, 0.f);

  for (int t = 0; t < ntiles; t++) {
    __syncwarp();  // the stage about to be refilled has been consumed
    if (t + 1 < ntiles) load_tile(t + 1);
    ok = ok && tc::mbar_wait(&bar[t & 1], (t >> 1) & 1, a.err);  // on expiry: error raised, garbage computed
    const float* kt = kv + (t & 1) * 2 * MT * HD;
    const float* vt = kt + MT * HD;
    const int tn = min(MT, ws1 - (ws0 + t * MT));
    warp_tile8<G>(kt, vt, tn, q, mreg, lreg, acc, sc, ps, lane);
  }
  // merge the 4 warps of the split: O_w, m_w, l_w -> (O, m, l)
  __syncthreads();
  float* mo = fsm;                        // [4][G][HD]
  float* mml = fsm + 4 * G * HD;          // [4][G][2]
#pragma unroll
  for (int g = 0; g < G; g++) *(float4*)(mo + (warp * G + g) * HD + 4 * lane) = acc[g];
#pragma unroll
  for (int k = 0; k < ROUNDS; k++) {
    const int g = (lane >> 3) + 4 * k;
    if ((lane & 7) == 0 && g < G) {
      mml[(warp * G + g) * 2] = mreg[k];
      mml[(warp * G + g) * 2 + 1] = lreg[k];
    }
  }
  __syncthreads();
  float* out = fsm + 4 * G * HD + 8 * G;  // [G][HD] then [G][2]
  for (int idx = tid; idx < G * HD; idx += kFaThreads) {
    const int g = idx / HD;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < 4; w++) M = fmaxf(M, mml[(w * G + g) * 2]);
    float o = 0.f, l = 0.f;
#pragma unroll
    for (int w = 0; w < 4; w++) {
      const float mw = mml[(w * G + g) * 2];
      const float e = (mw == -INFINITY) ? 0.f : __expf(mw - M);
      o += e * mo[(w * G + g) * HD + (idx % HD)];
      l += e * mml[(w * G + g) * 2 + 1];
    }
    out[idx] = o;
    if (idx % HD == 0) {
      out[G * HD + 2 * g] = M;
      out[G * HD + 2 * g + 1] = l;
    }
  }
  __syncthreads();
  fa_write_split(a, a.meta.row_item0[r] + split, kh, G, HD, out, out + G * HD);
}

// ============================================ head_dim 128: rows of a chunk
// Prefill chunks: one CTA per (group of up to 4 consecutive rows of one
// session, split), one warp per row.  The split's K/V rows are loaded once into
// a CTA ring of 16-position tiles that all warps read (a row at position p
// sees positions < p + 1 of the same pages), so the group reads its prefix
// once instead of once per row.  Warp 0's lanes issue the bulk copies; each
// warp releases a stage through the empty barrier; every wait is bounded.
constexpr int kRwTile = 16;
constexpr int kRwStages = 3;
template <int G>
struct RowsSmem {
  static constexpr int HD = 128;
  static constexpr int GP = (G + 3) & ~3;
  static constexpr int KV = kRwStages * 2 * kRwTile * HD;  // [stage][K|V][pos][HD]
  static constexpr int PER_WARP = G * kWpMT + kWpMT * GP;  // scores, probabilities
  static constexpr int TOTAL = KV + 4 * PER_WARP;            // floats, then full and empty barriers
  static constexpr size_t BYTES = (size_t)TOTAL * 4 + 2 * kRwStages * 8;
};

// grid: the step's row groups x KV heads
template <int G>
__global__ void __launch_bounds__(kFaThreads) k_attn_rows128(FastAttnArgs a) {
  constexpr int HD = 128, RT = kRwTile, NS = kRwStages;
  constexpr int ROUNDS = (G + 3) / 4;
  extern __shared__ __align__(16) float fsm[];
  const int gr = a.meta.grp_rs[a.grp0 + blockIdx.x], kh = blockIdx.y;
  const int r0 = gr >> 16, nr = ((gr >> 13) & 7) + 1, split = gr & 0x1fff;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int s0 = split * kFaSplit;
  const int s1 = min(a.meta.row_pos[r0 + nr - 1] + 1, s0 + kFaSplit);  // the group's last row reaches furthest
  const int r = r0 + min(warp, nr - 1);
  const int er = min(s1, a.meta.row_pos[r] + 1);  // this warp's row: positions [s0, er)
  const bool has = warp < nr && er > s0;
  float* kv = fsm;
  float* sc = fsm + RowsSmem<G>::KV + warp * RowsSmem<G>::PER_WARP;
  float* ps = sc + G * kWpMT;
  uint64_t* full = (uint64_t*)(fsm + RowsSmem<G>::TOTAL);
  uint64_t* empty = full + NS;
  const int pbase = a.meta.row_pbase[r0];
  const int pt = a.dm.page_tokens;
  const int64_t lay = (int64_t)a.layer * 2 * pt * a.dm.kvd + (int64_t)kh * HD;
  const int64_t vofs = (int64_t)pt * a.dm.kvd;
  const int ntiles = (s1 - s0 + RT - 1) / RT;
  if (tid == 0) {
    for (int i = 0; i < NS; i++) {
      tc::mbar_init(&full[i], 1);
      tc::mbar_init(&empty[i], 4);  // one arrival per warp
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  // warp 0 holds the split's page ids in lane registers (<= 32 pages)
  const int pg0 = s0 / pt;
  const int npg = (s1 - 1) / pt - pg0 + 1;
  const bool page_regs = npg <= 32;
  const int my_page = (warp == 0 && page_regs && lane < npg) ? a.meta.page_ids[pbase + pg0 + lane] : 0;
  auto load_tile = [&](int t) {  // warp 0 only
    const int st = t % NS;
    float* dst = kv + st * 2 * RT * HD;
    const int t0 = s0 + t * RT, tn = min(RT, s1 - t0);
    if (lane == 0) tc::mbar_expect_tx(&full[st], (uint32_t)tn * 2 * HD * 4);
    __syncwarp();
    const int pos = t0 + min(lane, tn - 1);
    const int pi = pos / pt;
    const int pg = __shfl_sync(0xffffffffu, my_page, (pi - pg0) & 31);
    if (lane < tn) {
      const int64_t page = page_regs ? pg : a.meta.page_ids[pbase + pi];
      const float* krow = a.pool + page * a.dm.page_elems + lay + (int64_t)(pos - pi * pt) * a.dm.kvd;
      tc::bulk_load(dst + lane * HD, krow, HD * 4, &full[st]);
      tc::bulk_load(dst + (RT + lane) * HD, krow + vofs, HD * 4, &full[st]);
    }
  };
  bool ok = true;
  if (warp == 0)
    for (int t = 0; t < min(ntiles, NS - 1); t++) load_tile(t);

  float4 q[G][4];
  {
    const float* qrow = a.Q + (int64_t)r * a.dm.qd + (int64_t)kh * G * HD;
    const int jl = lane & 7;
#pragma unroll
    for (int g = 0; g < G; g++)
#pragma unroll
      for (int i = 0; i < 4; i++) {
        const float4 v = *(const float4*)(qrow + g * HD + 4 * jl + 32 * i);
        q[g][i] = make_float4(v.x * a.scale, v.y * a.scale, v.z * a.scale, v.w * a.scale);
      }
  }
  float mreg[ROUNDS], lreg[ROUNDS];
#pragma unroll
  for (int k = 0; k < ROUNDS; k++) {
    mreg[k] = -INFINITY;
    lreg[k] = 0.f;
  }
  float4 acc[G];
#pragma unroll
  for (int g = 0; g < G; g++) acc[g] = make_float4(0.f, 0.f, 0.f, 0.f);

  for (int t = 0; t < ntiles; t++) {
    if (warp == 0 && t + NS - 1 < ntiles) {
      const int u = t - 1;  // the stage refilled now was read in iteration t - 1 by every warp
      if (u >= 0) ok = ok && tc::mbar_wait(&empty[u % NS], (u / NS) & 1, a.err);
      load_tile(t + NS - 1);
    }
    ok = ok && tc::mbar_wait(&full[t % NS], (t / NS) & 1, a.err);  // on expiry: error raised, garbage computed
    const float* kt = kv + (t % NS) * 2 * RT * HD;
    const float* vt = kt + RT * HD;
    if (has) {
#pragma unroll
      for (int h = 0; h < RT / kWpMT; h++) {
        const int p0 = s0 + t * RT + h * kWpMT;
        const int tn = min(kWpMT, er - p0);
        if (tn > 0) warp_tile8<G>(kt + h * kWpMT * HD, vt + h * kWpMT * HD, tn, q, mreg, lreg, acc, sc, ps, lane);
      }
    }
    __syncwarp();
    if (lane == 0) tc::mbar_arrive(&empty[t % NS]);
  }
  if (has) {  // this row's split partial (O, m, l), same layout as fa_write_split
    const int64_t unit = (int64_t)(a.meta.row_item0[r] + split) * a.dm.kv_heads + kh;
#pragma unroll
    for (int g = 0; g < G; g++) *(float4*)(a.part_o + (unit * G + g) * HD + 4 * lane) = acc[g];
#pragma unroll
    for (int k = 0; k < ROUNDS; k++) {
      const int g = (lane >> 3) + 4 * k;
      if ((lane & 7) == 0 && g < G) {
        a.part_ml[(unit * G + g) * 2] = mreg[k];
        a.part_ml[(unit * G + g) * 2 + 1] = lreg[k];
      }
    }
  }
}

// ============================= head_dim 128, 4 query heads per KV head:
// prefill rows on the tensor cores.  A group's 4 rows x 4 query heads are the
// 16 rows of an mma.m16n8k16 tile: S = Q K^T and O += P V each run as three
// bf16 products of hi/lo splits (Qh Kh + Qh Kl + Ql Kh; Ph Vh + Ph Vl + Pl Vh,
// about 2^-16 relative per product) with fp32 accumulation, and the online
// softmax works on the accumulator fragments (the score fragments of two
// 8-position tiles are the P operand of the 16-position P.V product).  The two
// warps of a CTA take the split's 16-position tiles alternately (so short
// prefixes keep both busy), each through a private 2-stage ring; K/V rows are
// padded to 132 floats so that the fragment loads are (nearly) free of bank
// conflicts.
constexpr int kMmTile = 16;
constexpr int kMmStride = 132;
constexpr int kMmWarps = 2;
struct MmaSmem {
  static constexpr int PER_WARP = 2 * 2 * kMmTile * kMmStride;          // [stage][K|V][pos][132]
  static constexpr int MERGE = kMmWarps * (16 * 128 + 2 * 16);          // per warp: O[16][128], (m, l)[16]
  static constexpr int TOTAL = kMmWarps * PER_WARP > MERGE ? kMmWarps * PER_WARP : MERGE;  // floats, then barriers
  static constexpr size_t BYTES = (size_t)TOTAL * 4 + kMmWarps * 2 * 8;
};

__device__ __forceinline__ void split_bf16x2(float x0, float x1, uint32_t& hi, uint32_t& lo) {
  const __nv_bfloat16 h0 = __float2bfloat16_rn(x0), h1 = __float2bfloat16_rn(x1);
  const __nv_bfloat16 l0 = __float2bfloat16_rn(x0 - __bfloat162float(h0));
  const __nv_bfloat16 l1 = __float2bfloat16_rn(x1 - __bfloat162float(h1));
  hi = (uint32_t)__bfloat16_as_ushort(h0) | ((uint32_t)__bfloat16_as_ushort(h1) << 16);  // lower k in the low half
  lo = (uint32_t)__bfloat16_as_ushort(l0) | ((uint32_t)__bfloat16_as_ushort(l1) << 16);
}
__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// grid: the step's row groups x KV heads (query heads per KV head = 4)
__global__ void __launch_bounds__(kMmWarps * 32) k_attn_mma128(FastAttnArgs a) {
  constexpr int HD = 128, T = kMmTile, ST = kMmStride, G = 4;
  extern __shared__ __align__(16) float fsm[];
  const int gr = a.meta.grp_rs[a.grp0 + blockIdx.x], kh = blockIdx.y;
  const int r0 = gr >> 16, nr = ((gr >> 13) & 7) + 1, split = gr & 0x1fff;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int gid = lane >> 2, tig = lane & 3;
  const int p0 = a.meta.row_pos[r0];  // row k of the group sits at position p0 + k
  const int s0 = split * kFaSplit;
  const int s1 = min(p0 + nr, s0 + kFaSplit);
  const int nall = (s1 - s0 + T - 1) / T;                           // the split's tiles
  const int ntiles = nall > warp ? (nall - warp + kMmWarps - 1) / kMmWarps : 0;  // this warp's: warp, warp+2, ...
  float* kv = fsm + warp * MmaSmem::PER_WARP;
  uint64_t* bar = (uint64_t*)(fsm + MmaSmem::TOTAL) + warp * 2;
  const int pbase = a.meta.row_pbase[r0];
  const int pt = a.dm.page_tokens;
  const int64_t lay = (int64_t)a.layer * 2 * pt * a.dm.kvd + (int64_t)kh * HD;
  const int64_t vofs = (int64_t)pt * a.dm.kvd;
  const int pg0 = s0 / pt;
  const int npg = (s1 - 1) / pt - pg0 + 1;
  const bool page_regs = npg <= 32;
  const int my_page = (page_regs && lane < npg) ? a.meta.page_ids[pbase + pg0 + lane] : 0;
  if (lane == 0) {
    tc::mbar_init(&bar[0], 1);
    tc::mbar_init(&bar[1], 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncwarp();
  auto load_tile = [&](int t) {  // this warp's t-th tile: split tile warp + t * kMmWarps
    const int st = t & 1;
    float* dst = kv + st * 2 * T * ST;
    const int t0 = s0 + (warp + t * kMmWarps) * T, tn = min(T, s1 - t0);
    if (lane == 0) tc::mbar_expect_tx(&bar[st], (uint32_t)tn * 2 * HD * 4);
    __syncwarp();
    const int pos = t0 + min(lane, tn - 1);
    const int pi = pos / pt;
    const int pg = __shfl_sync(0xffffffffu, my_page, (pi - pg0) & 31);
    if (lane < tn) {
      const int64_t page = page_regs ? pg : a.meta.page_ids[pbase + pi];
      const float* krow = a.pool + page * a.dm.page_elems + lay + (int64_t)(pos - pi * pt) * a.dm.kvd;
      tc::bulk_load(dst + lane * ST, krow, HD * 4, &bar[st]);
      tc::bulk_load(dst + (T + lane) * ST, krow + vofs, HD * 4, &bar[st]);
    }
  };
  if (ntiles > 0) load_tile(0);

  // query rows i = 4k + g (row k of the group, head g); this thread's rows gid and gid + 8
  const int k0 = gid >> 2, k1 = (gid + 8) >> 2, g0 = gid & 3;
  const int e0 = k0 < nr ? p0 + k0 + 1 : 0, e1 = k1 < nr ? p0 + k1 + 1 : 0;  // positions < e are visible
  uint32_t qh[8][4], ql[8][4];
  {
    const float* q0 = a.Q + (int64_t)(r0 + min(k0, nr - 1)) * a.dm.qd + (int64_t)(kh * G + g0) * HD;
    const float* q1 = a.Q + (int64_t)(r0 + min(k1, nr - 1)) * a.dm.qd + (int64_t)(kh * G + g0) * HD;
    const float z0 = k0 < nr ? a.scale : 0.f, z1 = k1 < nr ? a.scale : 0.f;
#pragma unroll
    for (int ks = 0; ks < 8; ks++) {
      const int c = ks * 16 + tig * 2;
      const float2 x0 = *(const float2*)(q0 + c), x1 = *(const float2*)(q1 + c);
      const float2 y0 = *(const float2*)(q0 + c + 8), y1 = *(const float2*)(q1 + c + 8);
      split_bf16x2(x0.x * z0, x0.y * z0, qh[ks][0], ql[ks][0]);
      split_bf16x2(x1.x * z1, x1.y * z1, qh[ks][1], ql[ks][1]);
      split_bf16x2(y0.x * z0, y0.y * z0, qh[ks][2], ql[ks][2]);
      split_bf16x2(y1.x * z1, y1.y * z1, qh[ks][3], ql[ks][3]);
    }
  }
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;  // l: this thread's columns only
  float o[16][4];
#pragma unroll
  for (int dn = 0; dn < 16; dn++) o[dn][0] = o[dn][1] = o[dn][2] = o[dn][3] = 0.f;
  bool ok = true;

  for (int t = 0; t < ntiles; t++) {
    __syncwarp();  // the stage about to be refilled has been consumed
    if (t + 1 < ntiles) load_tile(t + 1);
    ok = ok && tc::mbar_wait(&bar[t & 1], (t >> 1) & 1, a.err);  // on expiry: error raised, garbage computed
    float* Kt = kv + (t & 1) * 2 * T * ST;
    float* Vt = Kt + T * ST;
    const int tp0 = s0 + (warp + t * kMmWarps) * T, tn = min(T, s1 - tp0);
    if (tn < T) {  // rows past the tile's end: zero V so that 0-probability columns add exactly nothing
      for (int idx = lane; idx < (T - tn) * HD; idx += 32) Vt[(tn + idx / HD) * ST + idx % HD] = 0.f;
      __syncwarp();
    }
    // S = Q K^T over the tile's two 8-position halves
    float sacc[2][4];
#pragma unroll
    for (int nt = 0; nt < 2; nt++) sacc[nt][0] = sacc[nt][1] = sacc[nt][2] = sacc[nt][3] = 0.f;
#pragma unroll
    for (int ks = 0; ks < 8; ks++) {
#pragma unroll
      for (int nt = 0; nt < 2; nt++) {
        const float* kr = Kt + (nt * 8 + gid) * ST + ks * 16 + tig * 2;
        const float2 x = *(const float2*)kr, y = *(const float2*)(kr + 8);
        uint32_t bh0, bl0, bh1, bl1;
        split_bf16x2(x.x, x.y, bh0, bl0);
        split_bf16x2(y.x, y.y, bh1, bl1);
        mma_bf16_16816(sacc[nt], qh[ks], bh0, bh1);
        mma_bf16_16816(sacc[nt], qh[ks], bl0, bl1);
        mma_bf16_16816(sacc[nt], ql[ks], bh0, bh1);
      }
    }
    // causal mask and online softmax on rows gid (c0, c1) and gid + 8 (c2, c3)
    const int lim0 = min(e0, tp0 + tn), lim1 = min(e1, tp0 + tn);
    float mt0 = -INFINITY, mt1 = -INFINITY;
#pragma unroll
    for (int nt = 0; nt < 2; nt++)
#pragma unroll
      for (int e = 0; e < 2; e++) {
        const int pos = tp0 + nt * 8 + tig * 2 + e;
        sacc[nt][e] = pos < lim0 ? sacc[nt][e] : -INFINITY;
        sacc[nt][2 + e] = pos < lim1 ? sacc[nt][2 + e] : -INFINITY;
        mt0 = fmaxf(mt0, sacc[nt][e]);
        mt1 = fmaxf(mt1, sacc[nt][2 + e]);
      }
#pragma unroll
    for (int off = 1; off < 4; off <<= 1) {
      mt0 = fmaxf(mt0, __shfl_xor_sync(0xffffffffu, mt0, off));
      mt1 = fmaxf(mt1, __shfl_xor_sync(0xffffffffu, mt1, off));
    }
    const float mn0 = fmaxf(m0, mt0), mn1 = fmaxf(m1, mt1);
    const float al0 = (m0 == -INFINITY) ? 0.f : __expf(m0 - mn0);
    const float al1 = (m1 == -INFINITY) ? 0.f : __expf(m1 - mn1);
    m0 = mn0;
    m1 = mn1;
    float pr[2][4];
#pragma unroll
    for (int nt = 0; nt < 2; nt++)
#pragma unroll
      for (int e = 0; e < 2; e++) {
        pr[nt][e] = sacc[nt][e] == -INFINITY ? 0.f : __expf(sacc[nt][e] - mn0);
        pr[nt][2 + e] = sacc[nt][2 + e] == -INFINITY ? 0.f : __expf(sacc[nt][2 + e] - mn1);
      }
    l0 = l0 * al0 + pr[0][0] + pr[0][1] + pr[1][0] + pr[1][1];
    l1 = l1 * al1 + pr[0][2] + pr[0][3] + pr[1][2] + pr[1][3];
#pragma unroll
    for (int dn = 0; dn < 16; dn++) {
      o[dn][0] *= al0;
      o[dn][1] *= al0;
      o[dn][2] *= al1;
      o[dn][3] *= al1;
    }
    // P as the A operand (16 rows x 16 positions), hi/lo
    uint32_t ph[4], pl[4];
    split_bf16x2(pr[0][0], pr[0][1], ph[0], pl[0]);
    split_bf16x2(pr[0][2], pr[0][3], ph[1], pl[1]);
    split_bf16x2(pr[1][0], pr[1][1], ph[2], pl[2]);
    split_bf16x2(pr[1][2], pr[1][3], ph[3], pl[3]);
    // O += P V over the 16 eight-dim slices
#pragma unroll
    for (int dn = 0; dn < 16; dn++) {
      const float* vc = Vt + tig * 2 * ST + dn * 8 + gid;
      uint32_t vh0, vl0, vh1, vl1;
      split_bf16x2(vc[0], vc[ST], vh0, vl0);
      split_bf16x2(vc[8 * ST], vc[9 * ST], vh1, vl1);
      mma_bf16_16816(o[dn], ph, vh0, vh1);
      mma_bf16_16816(o[dn], ph, vl0, vl1);
      mma_bf16_16816(o[dn], pl, vh0, vh1);
    }
  }
#pragma unroll
  for (int off = 1; off < 4; off <<= 1) {
    l0 += __shfl_xor_sync(0xffffffffu, l0, off);
    l1 += __shfl_xor_sync(0xffffffffu, l1, off);
  }
  // merge the warps: O_w[16][128], (m, l)_w[16] -> the rows' split partials
  __syncthreads();
  float* mo = fsm + warp * (16 * HD + 32);
  float* mml = mo + 16 * HD;
#pragma unroll
  for (int dn = 0; dn < 16; dn++) {
    const int c = dn * 8 + tig * 2;
    *(float2*)(mo + gid * HD + c) = make_float2(o[dn][0], o[dn][1]);
    *(float2*)(mo + (gid + 8) * HD + c) = make_float2(o[dn][2], o[dn][3]);
  }
  if (tig == 0) {
    mml[gid * 2] = m0;
    mml[gid * 2 + 1] = l0;
    mml[(gid + 8) * 2] = m1;
    mml[(gid + 8) * 2 + 1] = l1;
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < 16 * HD; idx += kMmWarps * 32) {
    const int i = idx / HD, d = idx % HD, k = i >> 2, g = i & 3;
    if (k >= nr || p0 + k + 1 <= s0) continue;  // no such row, or the row does not reach this split
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kMmWarps; w++) M = fmaxf(M, fsm[w * (16 * HD + 32) + 16 * HD + i * 2]);
    float ov = 0.f, lv = 0.f;
#pragma unroll
    for (int w = 0; w < kMmWarps; w++) {
      const float* base = fsm + w * (16 * HD + 32);
      const float mw = base[16 * HD + i * 2];
      const float ew = (mw == -INFINITY) ? 0.f : __expf(mw - M);
      ov += ew * base[i * HD + d];
      lv += ew * base[16 * HD + i * 2 + 1];
    }
    const int64_t unit = (int64_t)(a.meta.row_item0[r0 + k] + split) * a.dm.kv_heads + kh;
    a.part_o[(unit * G + g) * HD + d] = ov;
    if (d == 0) {
      a.part_ml[(unit * G + g) * 2] = M;
      a.part_ml[(unit * G + g) * 2 + 1] = lv;
    }
  }
}

// ====================================================== head_dim 64: per CTA
constexpr int kFaTile = 32;

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
__global__ void __launch_bounds__(kFaThreads) k_attn_tile(FastAttnArgs a) {
  constexpr int LPP = HD / 16;
  constexpr int PPW = 32 / LPP;
  constexpr int PPAR = kFaThreads / HD;
  constexpr int GP = (G + 3) & ~3;
  extern __shared__ __align__(16) float fsm[];
  float* ks = fsm;                          // [2][kFaTile][HD]
  float* vs = ks + 2 * kFaTile * HD;        // [2][kFaTile][HD]
  float* sc = vs + 2 * kFaTile * HD;        // [G][kFaTile]
  float* ps = sc + G * kFaTile;             // [kFaTile][GP]
  float* alpha_s = ps + kFaTile * GP;       // [GP]
  float* m_s = alpha_s + GP;                // [GP]
  float* l_s = m_s + GP;                    // [GP]
  float* red = fsm;                         // reuses the tiles after the loop

  const int rs = a.meta.item_rs[a.item0 + blockIdx.x], kh = blockIdx.y;
  const int r = rs >> 16, split = rs & 0xffff;
  const int L = a.meta.row_pos[r] + 1;
  const int s0 = split * kFaSplit;
  if (s0 >= L) return;
  const int s1 = min(L, s0 + kFaSplit);
  const int pbase = a.meta.row_pbase[r];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  float4 q[G][4];
  {
    const float* qrow = a.Q + (int64_t)r * a.dm.qd + (int64_t)kh * G * HD;
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
    cp_async_wait<0>();
    __syncthreads();
    if (t + 1 < ntiles) {
      const int n0 = t0 + kFaTile;
      fa_load_tile<HD>(a, ks + ((t + 1) & 1) * kFaTile * HD, vs + ((t + 1) & 1) * kFaTile * HD, pbase, kh, n0,
                       min(kFaTile, s1 - n0));
    }
    cp_async_commit();
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
          float4 kx = *(const float4*)(kr + 4 * LPP * i);
#pragma unroll
          for (int g = 0; g < G; g++)
            part[g] += q[g][i].x * kx.x + q[g][i].y * kx.y + q[g][i].z * kx.z + q[g][i].w * kx.w;
        }
      }
#pragma unroll
      for (int off = 1; off < LPP; off <<= 1)
#pragma unroll
        for (int g = 0; g < G; g++) part[g] += __shfl_xor_sync(0xffffffffu, part[g], off);
      if (jl == 0)
#pragma unroll
        for (int g = 0; g < G; g++) sc[g * kFaTile + s] = s < tn ? part[g] : -INFINITY;
    }
    __syncthreads();
    for (int g = warp; g < G; g += 4) {
      const float v = sc[g * kFaTile + lane];
      float mt = v;
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, off));
      const float mo = m_s[g];
      const float mn = fmaxf(mo, mt);
      const float p = (v == -INFINITY) ? 0.f : __expf(v - mn);
      float sum = p;
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
      ps[lane * GP + g] = p;
      if (lane == 0) {
        const float al = (mo == -INFINITY) ? 0.f : __expf(mo - mn);
        alpha_s[g] = al;
        m_s[g] = mn;
        l_s[g] = l_s[g] * al + sum;
      }
    }
    __syncthreads();
#pragma unroll
    for (int g = 0; g < G; g++) acc[g] *= alpha_s[g];
    for (int s = par; s < tn; s += PPAR) {
      const float v = vt[s * HD + d];
      const float* pp = ps + s * GP;
#pragma unroll
      for (int g = 0; g < G; g++) acc[g] += pp[g] * v;
    }
  }
  cp_async_wait<0>();
  __syncthreads();
  float ml[2 * 8];
#pragma unroll
  for (int g = 0; g < G; g++) {
    ml[2 * g] = m_s[g];
    ml[2 * g + 1] = l_s[g];
  }
#pragma unroll
  for (int g = 0; g < G; g++) red[(par * G + g) * HD + d] = acc[g];
  __syncthreads();
  float* out = fsm + PPAR * G * HD;
  for (int idx = tid; idx < G * HD; idx += kFaThreads) {
    float v = 0.f;
#pragma unroll
    for (int p = 0; p < PPAR; p++) v += red[p * G * HD + idx];
    out[idx] = v;
  }
  if (tid < 2 * G) out[G * HD + tid] = ml[tid];
  __syncthreads();
  fa_write_split(a, a.meta.row_item0[r] + split, kh, G, HD, out, out + G * HD);
}

// Merge the splits of each (row, query head) and write the attention output.
template <int HD>
__global__ void __launch_bounds__(HD) k_attn_combine(FastAttnArgs a) {
  const int r = a.row0 + blockIdx.x, h = blockIdx.y, d = threadIdx.x;
  const int G = a.dm.group, kh = h / G, g = h % G;
  const int L = a.meta.row_pos[r] + 1;
  const int ns = (L + kFaSplit - 1) / kFaSplit;
  const int KVH = a.dm.kv_heads;
  const int64_t base = (int64_t)a.meta.row_item0[r] * KVH + kh;  // split s is unit base + s*KVH
  // one online pass over the splits in order; the loads of 8 splits are issued together
  float M = -INFINITY, den = 0.f, num = 0.f;
  for (int c = 0; c < ns; c += 8) {
    float m8[8], l8[8], o8[8];
#pragma unroll
    for (int k = 0; k < 8; k++) {
      const bool v = c + k < ns;
      const int64_t u = base + (int64_t)(c + k) * KVH;
      m8[k] = v ? a.part_ml[(u * G + g) * 2] : -INFINITY;
      l8[k] = v ? a.part_ml[(u * G + g) * 2 + 1] : 0.f;
      o8[k] = v ? a.part_o[(u * G + g) * HD + d] : 0.f;
    }
    float Mc = M;
#pragma unroll
    for (int k = 0; k < 8; k++) Mc = fmaxf(Mc, m8[k]);
    const float rs = (M == -INFINITY) ? 0.f : __expf(M - Mc);
    den *= rs;
    num *= rs;
#pragma unroll
    for (int k = 0; k < 8; k++) {
      const float w = (m8[k] == -INFINITY) ? 0.f : __expf(m8[k] - Mc);
      den += w * l8[k];
      num += w * o8[k];
    }
    M = Mc;
  }
  const int64_t hd_off = (int64_t)h * HD + d;
  if (a.xh) {
    const int64_t o = (int64_t)blockIdx.x * a.dm.qd + hd_off;  // the planes start at the half's row 0
    split_op(num / den, a.xh + o, a.xl + o);
  } else {
    a.A[(int64_t)r * a.dm.qd + hd_off] = num / den;
  }
}

template <int HD, int G>
inline size_t fa_smem_bytes() {
  if (HD == 128) {
    const size_t merge = (size_t)(4 * G * HD + 8 * G + G * HD + 2 * G);
    static_assert((4 * G * HD + 8 * G + G * HD + 2 * G) <= WarpSmem<G>::TOTAL, "merge area overlaps the mbarriers");
    return WarpSmem<G>::BYTES + 0 * merge;
  }
  constexpr int GP = (G + 3) & ~3;
  constexpr int PPAR = kFaThreads / HD;
  const size_t tiles = (size_t)(4 * kFaTile * HD + G * kFaTile + kFaTile * GP + 3 * GP);
  const size_t merge = (size_t)(PPAR * G * HD + G * HD + 2 * G);
  return std::max(tiles, merge) * 4;
}

}  // namespace sr
