// sampler.cuh -- device restatement of sampleWithBlocked (monolith.go:7320-7426)
// with the SplitMix64 RNG (monolith.go:1411-1439).  One CTA per session.
//
// Greedy (temperature 0): strict-'>' scan in ascending id order == block
//   arg-max with ties to the lower id; no RNG draw.
// Sampled: repeat penalty in fp64 -> the top_k candidates of the total order
//   (logit desc, id asc), found by an exact radix select over 96-bit keys
//   (ordered fp64 logit, inverted id) -> sorted -> probabilities
//   exp((l-max)/T) summed sequentially in fp64 -> top-p cut -> one
//   RNG.Float64 draw walked down the sorted list.  Identical decisions to the
//   reference's bounded heap / full sort, which keep the same candidates.
#pragma once

#include <float.h>
#include "common.cuh"

namespace sr {

struct SampleSetting {
  double temperature, top_p, penalty;
  int32_t top_k, pad;
};

struct SampleArgs {
  const float* logits;  // [n, V]
  int V, n, blocked;
  const uint8_t* want;
  const SampleSetting* settings;
  const int32_t* hist_off;
  const int32_t* hist;
  uint64_t* rng;
  int32_t* ids;
  int32_t* status;  // 0 ok, 1 nonfinite logit, 2 empty distribution, 3 unsupported
};

constexpr int kSampleThreads = 256;
constexpr int kMaxTopK = 256;

__device__ __forceinline__ uint64_t splitmix_next(uint64_t& state) {
  state += 0x9e3779b97f4a7c15ULL;
  uint64_t z = state;
  z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ULL;
  z = (z ^ (z >> 27)) * 0x94d049bb133111ebULL;
  return z ^ (z >> 31);
}
__device__ __forceinline__ double splitmix_float64(uint64_t& state) {
  return (double)(splitmix_next(state) >> 11) * (1.0 / 9007199254740992.0);
}

// Order-preserving map of a finite double (with -0 folded into +0).
__device__ __forceinline__ uint64_t ord64(double x) {
  if (x == 0.0) x = 0.0;
  uint64_t u = (uint64_t)__double_as_longlong(x);
  return (u >> 63) ? ~u : (u | (1ULL << 63));
}
// Digit d (0..11, most significant first) of the 96-bit key (ord64(x), ~id).
__device__ __forceinline__ uint32_t key_digit(uint64_t hi, uint32_t lo, int d) {
  return d < 8 ? (uint32_t)(hi >> (56 - 8 * d)) & 0xffu : (lo >> (24 - 8 * (d - 8))) & 0xffu;
}
// Compare the first nd digits of a key with the prefix: -1 / 0 / +1.
__device__ __forceinline__ int key_cmp_prefix(uint64_t hi, uint32_t lo, uint64_t phi, uint32_t plo, int nd) {
  if (nd <= 0) return 0;
  if (nd <= 8) {
    int sh = 64 - 8 * nd;
    uint64_t a = sh ? hi >> sh : hi, b = sh ? phi >> sh : phi;
    return a < b ? -1 : (a > b ? 1 : 0);
  }
  if (hi != phi) return hi < phi ? -1 : 1;
  int sh = 32 - 8 * (nd - 8);
  uint32_t a = sh ? lo >> sh : lo, b = sh ? plo >> sh : plo;
  return a < b ? -1 : (a > b ? 1 : 0);
}

__device__ __forceinline__ double penalized(const SampleArgs& a, const uint32_t* seen, bool use_seen, double pen,
                                            const float* lg, int id) {
  double x = (double)lg[id];
  if (use_seen && ((seen[id >> 5] >> (id & 31)) & 1u)) x = x > 0 ? __ddiv_rn(x, pen) : __dmul_rn(x, pen);
  return x;
}

__global__ void __launch_bounds__(kSampleThreads) k_sample(SampleArgs a) {
  extern __shared__ __align__(16) uint32_t seen[];  // ceil(V/32) words
  __shared__ int hist[256];
  __shared__ double cx[kMaxTopK], cprob[kMaxTopK];
  __shared__ int cid[kMaxTopK];
  __shared__ double sx[kMaxTopK];
  __shared__ int sid[kMaxTopK];
  __shared__ uint64_t s_phi;
  __shared__ uint32_t s_plo;
  __shared__ int s_nd, s_kneed, s_done, s_count;
  __shared__ double red_x[kSampleThreads];
  __shared__ int red_id[kSampleThreads];
  const int i = blockIdx.x, tid = threadIdx.x;
  if (!a.want[i]) {
    if (tid == 0) {
      a.ids[i] = -1;
      a.status[i] = 0;
    }
    return;
  }
  const SampleSetting st = a.settings[i];
  const int V = a.V;
  const float* lg = a.logits + (int64_t)i * V;
  const bool use_seen = st.temperature != 0.0 || st.penalty != 1.0;
  const int words = (V + 31) / 32;
  if (use_seen) {
    for (int w = tid; w < words; w += blockDim.x) seen[w] = 0u;
    __syncthreads();
    for (int h = a.hist_off[i] + tid; h < a.hist_off[i + 1]; h += blockDim.x) {
      int id = a.hist[h];
      if (id >= 0 && id < V) atomicOr(&seen[id >> 5], 1u << (id & 31));
    }
  }
  // every logit must be finite (the reference validates even masked ones)
  int bad = 0;
  for (int id = tid; id < V; id += blockDim.x) bad |= !isfinite(lg[id]);
  if (__syncthreads_or(bad)) {
    if (tid == 0) a.status[i] = 1;
    return;
  }
  if (st.temperature == 0.0) {
    double bx = 0.0;
    int bid = -1;
    for (int id = tid; id < V; id += blockDim.x) {
      if (id == a.blocked) continue;
      double x = penalized(a, seen, use_seen, st.penalty, lg, id);
      if (bid < 0 || x > bx) {
        bx = x;
        bid = id;
      }
    }
    red_x[tid] = bx;
    red_id[tid] = bid;
    __syncthreads();
    for (int s = blockDim.x / 2; s > 0; s >>= 1) {
      if (tid < s) {
        int oid = red_id[tid + s];
        double ox = red_x[tid + s];
        int cid0 = red_id[tid];
        if (oid >= 0 && (cid0 < 0 || ox > red_x[tid] || (ox == red_x[tid] && oid < cid0))) {
          red_x[tid] = ox;
          red_id[tid] = oid;
        }
      }
      __syncthreads();
    }
    if (tid == 0) {
      a.ids[i] = red_id[0];
      a.status[i] = red_id[0] < 0 ? 2 : 0;
    }
    return;
  }
  const int eligible = V - ((a.blocked >= 0 && a.blocked < V) ? 1 : 0);
  if (st.top_k <= 0 || st.top_k > kMaxTopK) {
    if (tid == 0) a.status[i] = 3;
    return;
  }
  if (eligible <= 0) {
    if (tid == 0) a.status[i] = 2;
    return;
  }
  const int K = min(st.top_k, eligible);
  // --- radix select of the K-th key, most significant digit first
  if (tid == 0) {
    s_phi = 0;
    s_plo = 0;
    s_nd = 0;
    s_kneed = K;
    s_done = 0;
  }
  __syncthreads();
  for (int d = 0; d < 12; d++) {
    hist[tid] = 0;
    __syncthreads();
    const uint64_t phi = s_phi;
    const uint32_t plo = s_plo;
    const int nd = s_nd;
    for (int id = tid; id < V; id += blockDim.x) {
      if (id == a.blocked) continue;
      uint64_t hi = ord64(penalized(a, seen, use_seen, st.penalty, lg, id));
      uint32_t lo = 0xffffffffu - (uint32_t)id;
      if (key_cmp_prefix(hi, lo, phi, plo, nd) == 0) atomicAdd(&hist[key_digit(hi, lo, d)], 1);
    }
    __syncthreads();
    if (tid == 0) {
      int need = s_kneed, above = 0, b = 255;
      for (; b >= 0; b--) {
        if (above + hist[b] >= need) break;
        above += hist[b];
      }
      need -= above;
      if (d < 8)
        s_phi |= (uint64_t)b << (56 - 8 * d);
      else
        s_plo |= (uint32_t)b << (24 - 8 * (d - 8));
      s_nd = d + 1;
      s_kneed = need;
      if (hist[b] == need) s_done = 1;
    }
    __syncthreads();
    if (s_done) break;
  }
  // --- collect the K candidates (keys >= prefix on the resolved digits)
  if (tid == 0) s_count = 0;
  __syncthreads();
  {
    const uint64_t phi = s_phi;
    const uint32_t plo = s_plo;
    const int nd = s_nd;
    for (int id = tid; id < V; id += blockDim.x) {
      if (id == a.blocked) continue;
      double x = penalized(a, seen, use_seen, st.penalty, lg, id);
      uint64_t hi = ord64(x);
      uint32_t lo = 0xffffffffu - (uint32_t)id;
      if (key_cmp_prefix(hi, lo, phi, plo, nd) >= 0) {
        int slot = atomicAdd(&s_count, 1);
        if (slot < kMaxTopK) {
          cx[slot] = x;
          cid[slot] = id;
        }
      }
    }
  }
  __syncthreads();
  const int cnt = min(s_count, kMaxTopK);
  // --- rank sort by (logit desc, id asc) (candidateBefore, monolith.go:7277-7282)
  for (int t = tid; t < cnt; t += blockDim.x) {
    int rank = 0;
    for (int u = 0; u < cnt; u++) {
      bool before = (cx[u] == cx[t]) ? (cid[u] < cid[t]) : (cx[u] > cx[t]);
      rank += before;
    }
    sx[rank] = cx[t];
    sid[rank] = cid[t];
  }
  __syncthreads();
  if (tid == 0) {
    int count = cnt;
    double total = 0.0, mx = sx[0];
    for (int k = 0; k < count; k++) {
      cprob[k] = exp(__ddiv_rn(__dsub_rn(sx[k], mx), st.temperature));
      total = dadd(total, cprob[k]);
    }
    if (st.top_p < 1.0) {
      double mass = 0.0;
      for (int k = 0; k < count; k++) {
        mass = dadd(mass, cprob[k]);
        if (mass >= __dmul_rn(st.top_p, total)) {
          count = k + 1;
          total = mass;
          break;
        }
      }
    }
    uint64_t state = a.rng[i];
    double draw = __dmul_rn(splitmix_float64(state), total);
    int out = sid[count - 1];
    for (int k = 0; k < count; k++) {
      draw = __dsub_rn(draw, cprob[k]);
      if (draw < 0) {
        out = sid[k];
        break;
      }
    }
    a.rng[i] = state;
    a.ids[i] = out;
    a.status[i] = (cnt == K) ? 0 : 2;
  }
}

}  // namespace sr
