// common.cuh -- shared definitions for the sm_100a engine-step kernels.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace sr {

constexpr int kQBlock = 64;          // q8Block: 64 columns per scale (monolith.go:3793)
constexpr int kMaxRows = 1024;       // rows per step (monolith.go:6275)
constexpr int kMaxSessions = 256;    // sessions per step (monolith.go:6248)
constexpr int kAttnSplit = 512;      // positions per split-K attention item (fast mode)

enum ParamFormat { kF32 = 0, kQ8 = 1, kQ4 = 2 };

// Element of the fast path's tensor-core operand planes: an fp32 activation is
// carried as two bf16 terms (hi + lo), and Q8/Q4 codes widen to bf16 exactly.
typedef __nv_bfloat16 op16;

// float32(MaxFloat32 / (2*64*127)): rows with a larger |x| take the fp64 path
// (q8NeedsWideSum, monolith.go:4346-4354).
__host__ __device__ inline float wide_limit() { return 2.0932724e+34f; }

// Exact-mode arithmetic: explicit round-to-nearest operations that nvcc never
// contracts into FMA, matching Go's unfused amd64 code generation.
__device__ __forceinline__ float fmul(float a, float b) { return __fmul_rn(a, b); }
__device__ __forceinline__ float fadd(float a, float b) { return __fadd_rn(a, b); }
__device__ __forceinline__ float fsub(float a, float b) { return __fsub_rn(a, b); }
__device__ __forceinline__ double dmul(double a, double b) { return __dmul_rn(a, b); }
__device__ __forceinline__ double dadd(double a, double b) { return __dadd_rn(a, b); }
__device__ __forceinline__ double dsub(double a, double b) { return __dsub_rn(a, b); }

// q4Pairs (monolith.go:3811-3817): sign-extended low / high nibble of a byte.
__device__ __forceinline__ float q4_lo(uint32_t b) { return (float)((int32_t)(b << 28) >> 28); }
__device__ __forceinline__ float q4_hi(uint32_t b) { return (float)((int32_t)(b << 24) >> 28); }

struct Param {
  int32_t rows, cols, format;
  void* values;   // device
  float* scales;  // device, rows * ceil(cols/64) for q8/q4
};

// One step's per-row metadata, built on the device by the metadata kernel.
struct StepMeta {
  int32_t* tokens;      // [rows]
  int32_t* row_pos;     // [rows]
  int32_t* row_pbase;   // [rows] offset of the row's page table in page_ids
  int32_t* page_ids;    // concatenated page tables
  int32_t* sess_pos;    // [sessions]
  int32_t* tok_off;     // [sessions+1]
  int32_t* page_off;    // [sessions+1]
  uint8_t* want;        // [sessions]
  int32_t* head_src;    // [sessions] compact head row -> step row
  int32_t* head_dst;    // [sessions] compact head row -> session index
  int32_t* n_heads;     // [1]
  int32_t* row_item0;   // [rows] first attention item of the row
  int32_t* item_rs;     // [items] attention item -> (row << 16) | split
  int32_t* single_rs;   // items of rows from 1-token chunks (decode): (row << 16) | split
  int32_t* grp_rs;      // groups of up to 4 consecutive rows of a longer chunk:
                        // (first row << 16) | ((rows - 1) << 13) | split
};

// Per-device model dimensions.  With tensor parallelism, heads, kv_heads,
// hidden, qd (= heads*hd, the attention width) and kvd are this rank's local
// shares; dim (the residual width) and vocab stay whole.
struct ModelDims {
  int32_t vocab, dim, hidden, layers, heads, kv_heads, context, hd, kvd, group, page_tokens;
  int32_t qd, tp_rank, tp_size;
  int64_t page_elems;   // 2 * page_tokens * kvd * layers
};

}  // namespace sr
