// fast_kernels.cuh -- SR_MODE_FAST: fused-multiply-add kernels checked against
// the reference within a stated tolerance.  Entry points return false / fall
// back to the exact kernels for shapes they do not cover.
#pragma once

#include "common.cuh"
#include "exact_kernels.cuh"
#include "srstep_internal.h"

namespace sr {

inline int fast_init(sr_model* m) {
  (void)m;
  return SR_OK;
}

// Returns true when the fast path handled the projection.
inline bool fast_linear(sr_model* m, const float* X, int n, const Param& W, LinearOut O) {
  (void)m, (void)X, (void)n, (void)W, (void)O;
  return false;
}

inline void fast_rmsnorm(sr_model* m, const float* X, const int32_t* src_map, const float* w, float* Y, int rows, int d,
                         double eps) {
  k_rmsnorm_exact<<<(rows + kNormWarps - 1) / kNormWarps, kNormWarps * 32, 0, m->stream>>>(X, src_map, w, Y, rows, d,
                                                                                           eps);
}

void fast_attention_launch(sr_model* m, sr_kvpool* pool, int n, int max_len, int layer);
inline void fast_attention(sr_model* m, sr_kvpool* pool, int n, int max_len, int layer) {
  fast_attention_launch(m, pool, n, max_len, layer);
}

}  // namespace sr
