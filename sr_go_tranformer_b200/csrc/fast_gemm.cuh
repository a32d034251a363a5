// fast_gemm.cuh -- host side of the tensor-core projections (tc_gemm.cuh,
// tc_gemm_direct.cuh): the bf16 code cache of every Q8/Q4 matrix (Q|K|V and
// gate|up fused row-wise), TMA descriptors, the stream-K schedule and the
// per-layer entry points.
//
// Code cache (the default): each matrix's codes are also kept as bf16 in tile
// order, 2 bytes per weight (about 1.9x the Q8 payload, 3.8x Q4), so every A
// tile is one bulk copy (k_gemm_q).  Without it (sr_model_set_code_cache(m, 0),
// or when the copy does not fit in device memory) k_gemm_direct reads the
// reference codes through per-parameter TMA maps and widens them in shared
// memory: no extra device memory, more shared-memory traffic, slower.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>

#include <vector>

#include "fast_kernels.cuh"
#include "srstep_internal.h"
#include "tc_gemm.cuh"
#include "tc_gemm2.cuh"
#include "tc_gemm_direct.cuh"

namespace sr {

struct TcMatrix {
  uint8_t* wt = nullptr;  // bf16 code cache in 32 KiB swizzled (256-feature, 64-column) tiles, or null
  CUtensorMap cmap;       // the cache as [tiles * 256][64] bf16 rows, 128-row boxes (k_gemm_q2)
  float* scales = nullptr;
  bool own_scales = false;
  int rows = 0, cols = 0;
  // the reference codes, for k_gemm_direct: up to 3 row-stacked parameters
  int nseg = 0, fmt = kQ8;
  CUtensorMap map[3];
};

struct TcState {
  uint64_t version = ~0ull;
  bool disabled = false;
  bool cache_wanted = true;  // build the bf16 code cache when it fits
  bool cached = false;       // the matrices below carry it
  std::vector<TcMatrix> qkv, o, gateup, down;
  TcMatrix head;
  __nv_bfloat16* xh = nullptr;
  __nv_bfloat16* xl = nullptr;
  // Operand maps for in = dim, hidden, attention width, per plane slot: slot
  // 0 starts at row 0 of the planes (a whole step, or the first half of a
  // split step), slot 1 at row kLaneRows (the second half).
  CUtensorMap xh_d[2], xl_d[2], xh_h[2], xl_h[2], xh_q[2], xl_q[2];
  int xcols = 0;              // row stride bound of the planes: max(dim, hidden, attention width)
  float* partial[2] = {nullptr, nullptr};  // per slot: [sms][2][kN][kMC] stream-K partial tiles
  int sms = 148;
  int pairs = 0;              // SM pairs (2-CTA clusters of k_gemm_q2) that fit at once; 0: pair MMAs off
  int* err = nullptr;
  int* h_err = nullptr;
  bool ran = false;
  std::vector<void*> allocs;
};

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = (EncodeTiledFn)p;
    cudaGetLastError();
  }
  return fn;
}

// 2-D bf16 tensor [rows][cols], box 64 x box_rows, 128-byte swizzle.
inline bool make_map(CUtensorMap* map, void* base, uint64_t cols, uint64_t rows, uint32_t box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn || (cols * 2) % 16 != 0 || ((uintptr_t)base) % 16 != 0) return false;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {cols * 2};
  cuuint32_t box[2] = {64, box_rows};
  cuuint32_t estr[2] = {1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, base, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// The bf16 code cache as [rows][64] (128-byte rows, already in the MMA's
// swizzled order), boxes of 128 rows copied as they are: one CTA's half of a
// 256-feature tile.
inline bool make_cache_map(CUtensorMap* map, void* base, uint64_t rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn || ((uintptr_t)base) % 16 != 0) return false;
  cuuint64_t dims[2] = {(cuuint64_t)tc::kKB, rows};
  cuuint64_t strides[1] = {(cuuint64_t)tc::kKB * 2};
  cuuint32_t box[2] = {(cuuint32_t)tc::kKB, (cuuint32_t)tc::kM};
  cuuint32_t estr[2] = {1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, base, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// The codes of a Q8 / Q4 parameter as stored: uint8 [rows][row bytes], box of
// 64 rows x one 64-column block's bytes (64 for Q8, 32 packed for Q4), no
// swizzle; rows past the end read as zero.
inline bool make_code_map(CUtensorMap* map, const Param& p) {
  EncodeTiledFn fn = encode_fn();
  const uint64_t rb = p.format == kQ8 ? (uint64_t)p.cols : (uint64_t)(p.cols + 1) / 2;
  if (!fn || rb % 16 != 0 || ((uintptr_t)p.values) % 16 != 0) return false;
  cuuint64_t dims[2] = {rb, (cuuint64_t)p.rows};
  cuuint64_t strides[1] = {rb};
  cuuint32_t box[2] = {(cuuint32_t)(p.format == kQ8 ? tc::kKB : tc::kKB / 2), (cuuint32_t)tc::kDirSub};
  cuuint32_t estr[2] = {1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, p.values, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

inline TcState* tc_state(sr_model* m) { return (TcState*)m->tc; }

// (kLaneRows: the second half of a split step has its operand planes from
// that row of the plane buffers on.)
// One half of a split step: its stream, operand-plane slot (0 or 1), the SM
// count of its partition and its first step row.
struct TcLane {
  cudaStream_t s;
  int slot;
  int sms;
  int row0;
};

inline void tc_free(TcState* t) {
  for (void* p : t->allocs) cudaFree(p);
  t->allocs.clear();
  if (t->h_err) cudaFreeHost(t->h_err);
  t->h_err = nullptr;
  t->qkv.clear();
  t->o.clear();
  t->gateup.clear();
  t->down.clear();
  t->partial[0] = t->partial[1] = nullptr;
}

inline bool tc_alloc(TcState* t, void** p, size_t bytes) {
  if (cudaMalloc(p, bytes) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  t->allocs.push_back(*p);
  return true;
}

// One (optionally row-fused) matrix over parameters sharing the input: the
// concatenated block scales, the code maps (k_gemm_direct: same format and
// width, every segment but the last a multiple of 64 rows) and, with cache,
// the bf16 code cache (k_gemm_q).  A false return with dst.wt == nullptr and
// cache set means only the cache did not fit.
inline bool tc_build(sr_model* m, TcState* t, TcMatrix& dst, const std::vector<const Param*>& parts, bool cache) {
  int rows = 0;
  const int cols = parts[0]->cols;
  dst.nseg = (int)parts.size();
  dst.fmt = parts[0]->format;
  for (size_t i = 0; i < parts.size(); i++) {
    const Param* p = parts[i];
    if (p->format == kF32 || p->cols != cols || p->format != dst.fmt) return false;
    if (i + 1 < parts.size() && p->rows % tc::kDirSub) return false;
    if (!make_code_map(&dst.map[i], *p)) return false;
    rows += p->rows;
  }
  for (int i = dst.nseg; i < 3; i++) dst.map[i] = dst.map[0];
  const int groups = (cols + kQBlock - 1) / kQBlock;
  const int mt = (rows + tc::kMC - 1) / tc::kMC;
  dst.rows = rows;
  dst.cols = cols;
  if (parts.size() == 1) {
    dst.scales = parts[0]->scales;
    dst.own_scales = false;
  } else {
    if (!tc_alloc(t, (void**)&dst.scales, (size_t)rows * groups * 4)) return false;
    dst.own_scales = true;
  }
  int r0 = 0;
  for (const Param* p : parts) {
    if (dst.own_scales)
      cudaMemcpyAsync(dst.scales + (int64_t)r0 * groups, p->scales, (size_t)p->rows * groups * 4,
                      cudaMemcpyDeviceToDevice, m->stream);
    r0 += p->rows;
  }
  dst.wt = nullptr;
  if (!cache) return true;
  const size_t bytes = (size_t)mt * groups * tc::kTileA;
  if (!tc_alloc(t, (void**)&dst.wt, bytes)) return false;
  if (!make_cache_map(&dst.cmap, dst.wt, (uint64_t)mt * groups * tc::kMC)) return false;
  cudaMemsetAsync(dst.wt, 0, bytes, m->stream);  // padding rows of the last tile
  r0 = 0;
  for (const Param* p : parts) {
    const int64_t chunks = (int64_t)p->rows * groups * 8;
    tc::k_codes_tiled<<<(int)std::min<int64_t>((chunks + 255) / 256, 148 * 64), 256, 0, m->stream>>>(
        p->values, p->format, p->rows, cols, r0, groups, dst.wt);
    r0 += p->rows;
  }
  return true;
}

// Lazily (re)build the matrices after the weights change.  Returns false when
// the tensor-core path is unavailable (f32 weights, shapes, memory).  The code
// cache is all or nothing: if it does not fit, every matrix reads its codes
// directly.
inline TcState* tc_state_make(sr_model* m) {
  if (!m->tc) {
    TcState* t = new TcState();
    m->tc = t;
    m->fast_free.push_back([t]() {
      tc_free(t);
      delete t;
    });
  }
  return tc_state(m);
}
inline bool tc_build_all(sr_model* m, TcState* t, bool cache) {
  const ModelDims& dm = m->dm;
  const int L = dm.layers;
  t->qkv.assign(L, TcMatrix());
  t->o.assign(L, TcMatrix());
  t->gateup.assign(L, TcMatrix());
  t->down.assign(L, TcMatrix());
  for (int l = 0; l < L; l++) {
    if (m->d.arch == SR_ARCH_GPT2) {  // loadGPT2's layer order: q, k, v at +2..4, o +8, c_fc +12, c_proj +14
      const Param* P = &m->params[4 + 16 * l];
      if (!tc_build(m, t, t->qkv[l], {&P[2], &P[3], &P[4]}, cache) || !tc_build(m, t, t->o[l], {&P[8]}, cache) ||
          !tc_build(m, t, t->gateup[l], {&P[12]}, cache) || !tc_build(m, t, t->down[l], {&P[14]}, cache))
        return false;
      continue;
    }
    const Param* P = &m->params[1 + 9 * l];
    if (!tc_build(m, t, t->qkv[l], {&P[1], &P[2], &P[3]}, cache) || !tc_build(m, t, t->o[l], {&P[4]}, cache) ||
        !tc_build(m, t, t->gateup[l], {&P[6], &P[7]}, cache) || !tc_build(m, t, t->down[l], {&P[8]}, cache))
      return false;
  }
  const Param& head = m->d.tied ? m->params[0] : m->params.back();
  return tc_build(m, t, t->head, {&head}, cache);
}
inline bool tc_prepare(sr_model* m) {
  TcState* t = tc_state_make(m);
  if (t->version == m->weights_version) return !t->disabled;
  tc_free(t);
  t->version = m->weights_version;
  t->disabled = true;
  t->cached = false;
  const ModelDims& dm = m->dm;
  if (m->d.weight_format == SR_FMT_F32 || dm.dim % 8 || dm.hidden % 8 || dm.qd % 8 || !encode_fn()) return false;
  cudaFuncSetAttribute(tc::k_gemm_q, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)tc::kSmemBytes);
  cudaFuncSetAttribute(tc::k_gemm_direct, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)tc::kDirSmemBytes);
  cudaFuncSetAttribute(tc::k_gemm_q2, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)tc::kSmemBytes2);
  bool built = t->cache_wanted && tc_build_all(m, t, true);
  t->cached = built;
  if (!built) {  // without the cache (not wanted, or it did not fit)
    tc_free(t);
    if (!tc_build_all(m, t, false)) {
      tc_free(t);
      return false;
    }
  }
  const int xcols = std::max(std::max(dm.dim, dm.hidden), dm.qd);
  {
    int sms = 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, m->device) != cudaSuccess || sms < 1) {
      cudaGetLastError();
      sms = 148;
    }
    t->sms = sms;
    // how many 2-CTA clusters of k_gemm_q2 can be resident at once
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeClusterDimension;
    attr.val.clusterDim.x = 2;
    attr.val.clusterDim.y = 1;
    attr.val.clusterDim.z = 1;
    cfg.gridDim = dim3(sms / 2 * 2);
    cfg.blockDim = dim3(tc::kThreads);
    cfg.dynamicSmemBytes = tc::kSmemBytes2;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    int clusters = 0;
    if (cudaOccupancyMaxActiveClusters(&clusters, tc::k_gemm_q2, &cfg) != cudaSuccess) {
      cudaGetLastError();
      clusters = 0;
    }
    t->pairs = std::min(clusters, sms / 2);
  }
  if (!tc_alloc(t, (void**)&t->xh, (size_t)kMaxRows * xcols * 2) ||
      !tc_alloc(t, (void**)&t->xl, (size_t)kMaxRows * xcols * 2) || !tc_alloc(t, (void**)&t->err, 16) ||
      !tc_alloc(t, (void**)&t->partial[0], (size_t)t->sms * 2 * tc::kN * tc::kMC * 4) ||
      !tc_alloc(t, (void**)&t->partial[1], (size_t)t->sms * 2 * tc::kN * tc::kMC * 4)) {
    tc_free(t);
    return false;
  }
  cudaMemsetAsync(t->xh, 0, (size_t)kMaxRows * xcols * 2, m->stream);
  cudaMemsetAsync(t->xl, 0, (size_t)kMaxRows * xcols * 2, m->stream);
  cudaMemsetAsync(t->err, 0, 16, m->stream);
  if (cudaMallocHost((void**)&t->h_err, 16) != cudaSuccess) {
    cudaGetLastError();
    tc_free(t);
    return false;
  }
  t->xcols = xcols;
  for (int sl = 0; sl < 2; sl++) {
    const size_t off = (size_t)sl * kLaneRows * xcols;
    const uint64_t rows = sl == 0 ? kMaxRows : kLaneRows;
    if (!make_map(&t->xh_d[sl], t->xh + off, dm.dim, rows, tc::kN) ||
        !make_map(&t->xl_d[sl], t->xl + off, dm.dim, rows, tc::kN) ||
        !make_map(&t->xh_h[sl], t->xh + off, dm.hidden, rows, tc::kN) ||
        !make_map(&t->xl_h[sl], t->xl + off, dm.hidden, rows, tc::kN) ||
        !make_map(&t->xh_q[sl], t->xh + off, dm.qd, rows, tc::kN) ||
        !make_map(&t->xl_q[sl], t->xl + off, dm.qd, rows, tc::kN)) {
      tc_free(t);
      return false;
    }
  }
  if (cudaStreamSynchronize(m->stream) != cudaSuccess) {
    cudaGetLastError();
    tc_free(t);
    return false;
  }
  t->disabled = false;
  return true;
}

// Minimum step rows for the tensor-core path: its time is the same for 1 to 128
// rows, and from 3 rows it beats the decode GEMV (gemv.cuh), which serves the
// 1- and 2-row steps.
constexpr int kTcMinRows = 3;
static_assert(kTcMinRows == gv::kMaxRows + 1, "every fast step has a projection kernel");

inline void tc_split_x(sr_model* m, const float* X, int n, int in) {
  TcState* t = tc_state(m);
  const int64_t total = (int64_t)n * in;
  tc::k_split_bf16<<<(int)std::min<int64_t>((total + 255) / 256, 148 * 16), 256, 0, m->stream>>>(X, n, in, t->xh,
                                                                                                   t->xl);
  sr_count_launch(m);
}

// in_kind: 0 = the residual width (dim), 1 = hidden, 2 = the attention width (qd).
// Stream-K schedule: groups of nt CTAs (one per 128-row tile), or of nt2 SM
// pairs (one per 256-row tile), fill the SMs, each group taking at least
// kSkMinUnits (tile, block) units.
constexpr int kSkMinUnits = 4;
inline bool tc_gemm(sr_model* m, const TcMatrix& W, int in_kind, int n, tc::GemmArgs a, const TcLane* lane = nullptr) {
  TcState* t = tc_state(m);
  const int slot = lane ? lane->slot : 0, sms = lane ? lane->sms : t->sms;
  cudaStream_t stream = lane ? lane->s : m->stream;
  a.n = n;
  a.out = W.rows;
  a.in = W.cols;
  a.groups = (W.cols + kQBlock - 1) / kQBlock;
  a.scales = W.scales;
  a.err = t->err;
  a.mt = (W.rows + tc::kMC - 1) / tc::kMC;
  const int64_t units = (int64_t)a.mt * a.groups;
  a.partial = t->partial[slot];
  const CUtensorMap& xh = in_kind == 1 ? t->xh_h[slot] : (in_kind == 2 ? t->xh_q[slot] : t->xh_d[slot]);
  const CUtensorMap& xl = in_kind == 1 ? t->xl_h[slot] : (in_kind == 2 ? t->xl_q[slot] : t->xl_d[slot]);
  a.wt = W.wt;
  a.fmt = W.fmt;
  // Pairs of SMs (k_gemm_q2) for a whole step of more than one 128-row tile
  // with the code cache: groups of nt2 2-CTA clusters, one per 256-row tile.
  const int nt2 = (n + tc::kN2 - 1) / tc::kN2;
  if (W.wt && !lane && n > tc::kN && t->pairs > 0 && nt2 <= t->pairs &&
      units * t->pairs < ((int64_t)1 << 31)) {
    a.nt = 2 * nt2;  // 128-row tiles, as the partial slots and k_sk_reduce count them
    a.ngroups = (int)std::max<int64_t>(1, std::min<int64_t>(t->pairs / nt2, (units + kSkMinUnits - 1) / kSkMinUnits));
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeClusterDimension;
    attr.val.clusterDim.x = 2;
    attr.val.clusterDim.y = 1;
    attr.val.clusterDim.z = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.ngroups * nt2 * 2);
    cfg.blockDim = dim3(tc::kThreads);
    cfg.dynamicSmemBytes = tc::kSmemBytes2;
    cfg.stream = stream;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    if (cudaLaunchKernelEx(&cfg, tc::k_gemm_q2, W.cmap, xh, xl, a) != cudaSuccess) {
      cudaGetLastError();
      return false;
    }
  } else {
    a.nt = (n + tc::kN - 1) / tc::kN;
    if (a.nt > sms || units * sms >= ((int64_t)1 << 31)) return false;  // 32-bit schedule math
    a.ngroups = (int)std::max<int64_t>(1, std::min<int64_t>(sms / a.nt, (units + kSkMinUnits - 1) / kSkMinUnits));
    if (W.wt)
      tc::k_gemm_q<<<a.ngroups * a.nt, tc::kThreads, tc::kSmemBytes, stream>>>(xh, xl, a);
    else
      tc::k_gemm_direct<<<a.ngroups * a.nt, tc::kDirThreads, tc::kDirSmemBytes, stream>>>(xh, xl, W.map[0],
                                                                                         W.map[1], W.map[2], a);
  }
  sr_count_launch(m);
  // Tiles left in partial slots: every tile when the epilogue needs the
  // residual or the head row map, otherwise only tiles cut by a group boundary.
  bool all = a.out_map != nullptr;
  for (int sg = 0; sg < a.nseg; sg++) all = all || a.seg[sg].resid != nullptr;
  if (all) {
    tc::k_sk_reduce<<<dim3(a.mt * a.nt, tc::kN / tc::kRedBlockRows), tc::kMC, 0, stream>>>(a, 0);
    sr_count_launch(m);
  } else if (a.ngroups > 1) {
    tc::k_sk_reduce<<<dim3((a.ngroups - 1) * a.nt, tc::kN / tc::kRedBlockRows), tc::kMC, 0, stream>>>(a, 1);
    sr_count_launch(m);
  }
  t->ran = true;
  return true;
}

inline tc::Segment seg(int rows, float* y, int ldy, const float* bias, const float* resid) {
  tc::Segment s;
  s.rows = rows;
  s.y = y;
  s.ldy = ldy;
  s.bias = bias;
  s.resid = resid;
  return s;
}

// Whether this step's projections run on the tensor cores (and their inputs
// are therefore produced directly as bf16 hi/lo planes).
inline bool tc_active(sr_model* m, int n) { return n >= kTcMinRows && tc_prepare(m); }
inline __nv_bfloat16* tc_xh(sr_model* m) { return tc_state(m)->xh; }
inline __nv_bfloat16* tc_xl(sr_model* m) { return tc_state(m)->xl; }

// Q|K|V in one GEMM (+ qwen2 biases).  presplit: the producer already wrote
// the operand planes.
// With a lane (one half of a split step), n is the half's row count, the
// operand planes are the lane's slot and the outputs start at row lane->row0.
// Q|K|V with explicit biases (each may be null).
inline bool tc_qkv_bias(sr_model* m, int l, int n, bool presplit, const TcLane* lane, const float* bq,
                        const float* bk, const float* bv) {
  if (n < kTcMinRows || !tc_prepare(m)) return false;
  const ModelDims& dm = m->dm;
  const int64_t r0 = lane ? lane->row0 : 0;
  tc::GemmArgs a{};
  a.nseg = 3;
  a.seg[0] = seg(dm.qd, m->Q + r0 * dm.qd, dm.qd, bq, nullptr);
  a.seg[1] = seg(dm.kvd, m->K + r0 * dm.kvd, dm.kvd, bk, nullptr);
  a.seg[2] = seg(dm.kvd, m->V + r0 * dm.kvd, dm.kvd, bv, nullptr);
  a.out_map = nullptr;
  if (!presplit) tc_split_x(m, m->N, n, dm.dim);
  return tc_gemm(m, tc_state(m)->qkv[l], 0, n, a, lane);
}
inline bool tc_qkv(sr_model* m, int l, int n, bool presplit = false, const TcLane* lane = nullptr) {
  const Param* B = m->d.qkv_bias ? &m->params[2 + 9 * m->dm.layers + 3 * l] : nullptr;
  return tc_qkv_bias(m, l, n, presplit, lane, B ? (const float*)B[0].values : nullptr,
                     B ? (const float*)B[1].values : nullptr, B ? (const float*)B[2].values : nullptr);
}
// GPT-2's c_fc (+ bias) into G, from operand planes a producer already wrote.
inline bool tc_fc(sr_model* m, int l, int n, const float* bias) {
  if (n < kTcMinRows || !tc_prepare(m)) return false;
  const ModelDims& dm = m->dm;
  tc::GemmArgs a{};
  a.nseg = 1;
  a.seg[0] = seg(dm.hidden, m->G, dm.hidden, bias, nullptr);
  a.out_map = nullptr;
  return tc_gemm(m, tc_state(m)->gateup[l], 0, n, a);
}
// gate|up in one GEMM.
inline bool tc_gateup(sr_model* m, int l, int n, bool presplit = false, const TcLane* lane = nullptr) {
  if (n < kTcMinRows || !tc_prepare(m)) return false;
  const ModelDims& dm = m->dm;
  const int64_t r0 = lane ? lane->row0 : 0;
  tc::GemmArgs a{};
  a.nseg = 2;
  a.seg[0] = seg(dm.hidden, m->G + r0 * dm.hidden, dm.hidden, nullptr, nullptr);
  a.seg[1] = seg(dm.hidden, m->U + r0 * dm.hidden, dm.hidden, nullptr, nullptr);
  a.out_map = nullptr;
  if (!presplit) tc_split_x(m, m->N, n, dm.dim);
  return tc_gemm(m, tc_state(m)->gateup[l], 0, n, a, lane);
}
// O / down projection into y (with the residual add y = resid + W x when
// resid is set; tensor-parallel ranks write their partial sum instead).
// (y and resid point at the first output row: the caller offsets them for a lane.)
inline bool tc_proj(sr_model* m, const TcMatrix& W, const float* X, int n, int in_kind, bool presplit, float* y,
                    const float* resid, const TcLane* lane = nullptr, const float* bias = nullptr) {
  const ModelDims& dm = m->dm;
  tc::GemmArgs a{};
  a.nseg = 1;
  a.seg[0] = seg(dm.dim, y, dm.dim, bias, resid);
  a.out_map = nullptr;
  if (!presplit) tc_split_x(m, X, n, in_kind == 1 ? dm.hidden : (in_kind == 2 ? dm.qd : dm.dim));
  return tc_gemm(m, W, in_kind, n, a, lane);
}
inline bool tc_o(sr_model* m, int l, int n, bool presplit, float* y, const float* resid,
                 const TcLane* lane = nullptr, const float* bias = nullptr) {
  if (n < kTcMinRows || !tc_prepare(m)) return false;
  return tc_proj(m, tc_state(m)->o[l], m->A, n, 2, presplit, y, resid, lane, bias);
}
inline bool tc_down(sr_model* m, int l, int n, bool presplit, float* y, const float* resid,
                    const TcLane* lane = nullptr, const float* bias = nullptr) {
  if (n < kTcMinRows || !tc_prepare(m)) return false;
  return tc_proj(m, tc_state(m)->down[l], m->H, n, 1, presplit, y, resid, lane, bias);
}
// The operand planes of slot `slot` (row 0 of a lane's rows).
inline void tc_planes(sr_model* m, int slot, __nv_bfloat16** xh, __nv_bfloat16** xl) {
  TcState* t = tc_state(m);
  const size_t off = (size_t)slot * kLaneRows * t->xcols;
  *xh = t->xh + off;
  *xl = t->xl + off;
}
inline bool tc_head(sr_model* m, int heads, bool presplit = false) {
  if (heads < kTcMinRows || !tc_prepare(m)) return false;
  const ModelDims& dm = m->dm;
  tc::GemmArgs a{};
  a.nseg = 1;
  a.seg[0] = seg(dm.vocab, m->logits, dm.vocab, nullptr, nullptr);
  a.out_map = m->meta.head_dst;
  if (!presplit) tc_split_x(m, m->N, heads, dm.dim);
  return tc_gemm(m, tc_state(m)->head, 0, heads, a);
}

// One matrix parameter on the tensor cores, outside the step (sr_linear in
// fast mode), with the same code source as the step's matrices; its input
// width must be one the operand maps cover (dim, hidden, attention width).
inline bool tc_linear(sr_model* m, const float* X, int n, const Param& W, const LinearOut& O) {
  if (n < kTcMinRows || (W.format != kQ8 && W.format != kQ4) || !tc_prepare(m)) return false;
  const ModelDims& dm = m->dm;
  const int in_kind = W.cols == dm.dim ? 0 : (W.cols == dm.hidden ? 1 : (W.cols == dm.qd ? 2 : -1));
  if (in_kind < 0) return false;
  TcState* t = tc_state(m);
  const size_t before = t->allocs.size();
  TcMatrix M;
  bool ok = tc_build(m, t, M, {&W}, t->cached);
  if (ok) {
    tc::GemmArgs a{};
    a.nseg = 1;
    a.seg[0] = seg(W.rows, O.y, O.ldy, O.bias, O.resid);
    a.out_map = O.out_map;
    tc_split_x(m, X, n, W.cols);
    ok = tc_gemm(m, M, in_kind, n, a);
  }
  if (t->allocs.size() > before) {  // the temporary cache of M
    cudaStreamSynchronize(m->stream);
    for (size_t i = before; i < t->allocs.size(); i++) cudaFree(t->allocs[i]);
    t->allocs.resize(before);
  }
  return ok;
}

// sr_model_set_code_cache: rebuild on the next fast step with or without it.
inline void tc_set_cache(sr_model* m, bool on) {
  TcState* t = tc_state_make(m);
  if (t->cache_wanted != on) {
    t->cache_wanted = on;
    t->version = ~0ull;
  }
}
inline bool tc_cached(sr_model* m) { return m->tc && tc_state(m)->cached && !tc_state(m)->disabled; }

// After the step's stream synchronize: SR_ETIMEOUT if a bounded wait expired.
inline int tc_check(sr_model* m) {
  TcState* t = tc_state(m);
  if (!t || !t->ran) return SR_OK;
  t->ran = false;
  if (cudaMemcpy(t->h_err, t->err, 4, cudaMemcpyDeviceToHost) != cudaSuccess) {
    cudaGetLastError();
    return sr_fail(SR_EDEVICE, "reading the tensor-core error flag failed");
  }
  if (*t->h_err) {
    cudaMemset(t->err, 0, 4);
    return sr_fail(SR_ETIMEOUT, "a tensor-core pipeline wait expired; results of this step are invalid");
  }
  return SR_OK;
}

}  // namespace sr
