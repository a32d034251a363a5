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
// Sampled with top_k 0 (every candidate) or above kMaxTopK: k_sample_full, one
//   1024-thread CTA per session, sorts every eligible candidate (stable LSD
//   radix sort of the ordered logit, ids in ascending order) in global
//   scratch, then runs the same sequential fp64 sums, cut and walk.
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
  const uint8_t* want;  // null: every session
  const SampleSetting* settings;
  const int32_t* hist_off;
  const int32_t* hist;
  uint64_t* rng;
  int32_t* ids;
  int32_t* status;  // 0 ok, 1 nonfinite logit, 2 empty distribution, 3 unsupported
};

constexpr int kSampleThreads = 1024;  // one CTA per session walks its whole vocabulary
constexpr int kMaxTopK = 256;
constexpr int kSampleFullThreads = 1024;
constexpr int kSampleFullStage = 2048;  // fp64 values staged in shared memory per sequential chunk
constexpr int kSampleWave = 32;         // sessions per k_sample_full launch (bounds the scratch)

// Sampled sessions whose candidate list is the whole eligible vocabulary
// (top_k 0) or longer than the bounded select keeps.
__host__ __device__ inline bool sample_needs_full(const SampleSetting& s) {
  return s.temperature != 0.0 && (s.top_k <= 0 || s.top_k > kMaxTopK);
}
// Scratch bytes per session of k_sample_full: two (key, id) buffers.
__host__ __device__ inline int64_t sample_full_stride(int V) { return ((int64_t)V * 24 + 255) / 256 * 256; }

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
// Inverse of ord64 (a folded -0 comes back as +0, which every later use --
// x - max and the exp of it -- treats alike).
__device__ __forceinline__ double unord64(uint64_t u) {
  return __longlong_as_double((long long)((u >> 63) ? (u & ~(1ULL << 63)) : ~u));
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

// The penalized logit of a value already loaded (penalized() above reads it).
__device__ __forceinline__ double penalized_value(const uint32_t* seen, bool use_seen, double pen, float v, int id) {
  double x = (double)v;
  if (use_seen && ((seen[id >> 5] >> (id & 31)) & 1u)) x = x > 0 ? __ddiv_rn(x, pen) : __dmul_rn(x, pen);
  return x;
}
constexpr int kSampleUnroll = 8;

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
  if (a.want && !a.want[i]) {
    if (tid == 0) {
      a.ids[i] = -1;
      a.status[i] = 0;
    }
    return;
  }
  const SampleSetting st = a.settings[i];
  if (sample_needs_full(st)) return;  // k_sample_full samples this session
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
    if (tid < 256) hist[tid] = 0;
    __syncthreads();
    const uint64_t phi = s_phi;
    const uint32_t plo = s_plo;
    const int nd = s_nd;
    // kSampleUnroll logits per thread are loaded before any is used (the
    // scan is bound by load latency: one CTA walks the whole vocabulary)
    for (int id0 = tid; id0 < V; id0 += blockDim.x * kSampleUnroll) {
      float v[kSampleUnroll];
#pragma unroll
      for (int u = 0; u < kSampleUnroll; u++) {
        const int id = id0 + u * blockDim.x;
        v[u] = id < V ? lg[id] : 0.f;
      }
#pragma unroll
      for (int u = 0; u < kSampleUnroll; u++) {
        const int id = id0 + u * blockDim.x;
        if (id >= V || id == a.blocked) continue;
        uint64_t hi = ord64(penalized_value(seen, use_seen, st.penalty, v[u], id));
        uint32_t lo = 0xffffffffu - (uint32_t)id;
        if (key_cmp_prefix(hi, lo, phi, plo, nd) == 0) atomicAdd(&hist[key_digit(hi, lo, d)], 1);
      }
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
    for (int id0 = tid; id0 < V; id0 += blockDim.x * kSampleUnroll) {
      float v[kSampleUnroll];
#pragma unroll
      for (int u = 0; u < kSampleUnroll; u++) {
        const int id = id0 + u * blockDim.x;
        v[u] = id < V ? lg[id] : 0.f;
      }
#pragma unroll
      for (int u = 0; u < kSampleUnroll; u++) {
        const int id = id0 + u * blockDim.x;
        if (id >= V || id == a.blocked) continue;
        double x = penalized_value(seen, use_seen, st.penalty, v[u], id);
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

// sampleWithBlocked's full-sort branch (M:7367-7426) for top_k 0 or above
// kMaxTopK: one CTA per listed session (list[blockIdx.x]).  scratch holds,
// per CTA (sample_full_stride bytes), two uint64 key buffers and two int32 id
// buffers of V entries each.
//  1. key = ~ord64(penalized logit) for every eligible id, in id order;
//  2. stable LSD radix sort of the keys, 8 bits per pass (a pass whose digit is
//     the same for every key is skipped): ascending keys = descending logits,
//     ties in ascending id -- candidateBefore's total order (M:7277-7282);
//  3. prob[k] = exp((x_k - x_0) / T) for the first K = min(top_k or all, N);
//  4. one thread forms the running sums total += prob[k] in order (staged
//     through shared memory); a top-p cut takes the first k whose running sum
//     reaches top_p * total (the reference's mass loop forms the same sums);
//  5. draw = Float64() * total, subtracted prob by prob in order.
// The dynamic shared memory holds the history bitset (ceil(V/32) words) and
// kSampleFullStage staged doubles.
__global__ void __launch_bounds__(kSampleFullThreads) k_sample_full(SampleArgs a, const int32_t* list,
                                                                     uint8_t* scratch) {
  extern __shared__ __align__(16) uint8_t sfull_sm[];
  const int V = a.V;
  const int words = (V + 31) / 32;
  uint32_t* seen = (uint32_t*)sfull_sm;
  double* stage = (double*)(sfull_sm + ((words * 4 + 15) & ~15));
  __shared__ int wcnt[kSampleFullThreads / 32][256];
  __shared__ int base[256];
  __shared__ int s_skip, s_cut, s_out, s_done;
  __shared__ double s_total, s_draw;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int i = list[blockIdx.x];
  const SampleSetting st = a.settings[i];
  const float* lg = a.logits + (int64_t)i * V;
  uint8_t* sc = scratch + (int64_t)blockIdx.x * sample_full_stride(V);
  uint64_t* keys[2] = {(uint64_t*)sc, (uint64_t*)sc + V};
  int32_t* idv[2] = {(int32_t*)((uint64_t*)sc + 2 * (int64_t)V), (int32_t*)((uint64_t*)sc + 2 * (int64_t)V) + V};

  for (int w = tid; w < words; w += blockDim.x) seen[w] = 0u;
  __syncthreads();
  for (int h = a.hist_off[i] + tid; h < a.hist_off[i + 1]; h += blockDim.x) {
    const int id = a.hist[h];
    if (id >= 0 && id < V) atomicOr(&seen[id >> 5], 1u << (id & 31));
  }
  int bad = 0;
  for (int id = tid; id < V; id += blockDim.x) bad |= !isfinite(lg[id]);
  if (__syncthreads_or(bad)) {
    if (tid == 0) a.status[i] = 1;
    return;
  }
  const bool has_blocked = a.blocked >= 0 && a.blocked < V;
  const int N = V - (has_blocked ? 1 : 0);
  if (N <= 0) {
    if (tid == 0) a.status[i] = 2;
    return;
  }
  // 1. keys in id order (the blocked id leaves no gap)
  for (int id = tid; id < V; id += blockDim.x) {
    if (id == a.blocked) continue;
    const int j = (has_blocked && id > a.blocked) ? id - 1 : id;
    keys[0][j] = ~ord64(penalized(a, seen, true, st.penalty, lg, id));
    idv[0][j] = id;
  }
  __syncthreads();
  // 2. stable LSD radix sort
  int cur = 0;
  for (int pass = 0; pass < 8; pass++) {
    const int shift = 8 * pass;
    if (tid < 256) base[tid] = 0;
    __syncthreads();
    for (int j = tid; j < N; j += blockDim.x) atomicAdd(&base[(int)((keys[cur][j] >> shift) & 255u)], 1);
    __syncthreads();
    if (tid == 0) {
      int skip = 0, run = 0;
      for (int d = 0; d < 256; d++) {
        const int c = base[d];
        skip |= (c == N);
        base[d] = run;
        run += c;
      }
      s_skip = skip;
    }
    __syncthreads();
    if (s_skip) continue;
    for (int t0 = 0; t0 < N; t0 += blockDim.x) {
      for (int k = tid; k < (kSampleFullThreads / 32) * 256; k += blockDim.x) (&wcnt[0][0])[k] = 0;
      __syncthreads();
      const int j = t0 + tid;
      const bool valid = j < N;
      const uint64_t kv = valid ? keys[cur][j] : 0ull;
      const int32_t iv = valid ? idv[cur][j] : 0;
      const int d = valid ? (int)((kv >> shift) & 255u) : 256 + lane;  // idle lanes match no digit
      const unsigned peers = __match_any_sync(0xffffffffu, d);
      const int rank = __popc(peers & ((1u << lane) - 1u));
      if (valid && rank == 0) wcnt[warp][d] = __popc(peers);
      __syncthreads();
      if (tid < 256) {  // digit tid: offsets of each warp's run, in warp order
        int run = base[tid];
        for (int w = 0; w < kSampleFullThreads / 32; w++) {
          const int c = wcnt[w][tid];
          wcnt[w][tid] = run;
          run += c;
        }
        base[tid] = run;
      }
      __syncthreads();
      if (valid) {
        const int p = wcnt[warp][d] + rank;
        keys[cur ^ 1][p] = kv;
        idv[cur ^ 1][p] = iv;
      }
      __syncthreads();
    }
    cur ^= 1;
  }
  const uint64_t* ks = keys[cur];
  const int32_t* is = idv[cur];
  double* prob = (double*)keys[cur ^ 1];
  const int K = (st.top_k > 0 && st.top_k < N) ? st.top_k : N;
  // 3. probabilities
  const double mx = unord64(~ks[0]);
  for (int k = tid; k < K; k += blockDim.x) prob[k] = exp(__ddiv_rn(__dsub_rn(unord64(~ks[k]), mx), st.temperature));
  if (tid == 0) {
    s_total = 0.0;
    s_cut = K;
  }
  __syncthreads();
  // 4. running sums in order; sums[k] reuses the sorted-key buffer
  double* sums = (double*)keys[cur];
  const bool cut = st.top_p < 1.0;
  for (int c0 = 0; c0 < K; c0 += kSampleFullStage) {
    const int cn = min(kSampleFullStage, K - c0);
    for (int k = tid; k < cn; k += blockDim.x) stage[k] = prob[c0 + k];
    __syncthreads();
    if (tid == 0) {
      double t = s_total;
      for (int k = 0; k < cn; k++) {
        t = dadd(t, stage[k]);
        stage[k] = t;
      }
      s_total = t;
    }
    __syncthreads();
    if (cut)
      for (int k = tid; k < cn; k += blockDim.x) sums[c0 + k] = stage[k];
    __syncthreads();
  }
  double total = s_total;
  int count = K;
  if (cut) {
    const double thr = __dmul_rn(st.top_p, total);
    int first = K;
    for (int k = tid; k < K; k += blockDim.x)
      if (sums[k] >= thr) {
        first = k;
        break;
      }
    atomicMin(&s_cut, first);
    __syncthreads();
    if (s_cut < K) {
      count = s_cut + 1;
      total = sums[s_cut];
    }
  }
  // 5. draw and walk
  if (tid == 0) {
    uint64_t state = a.rng[i];
    s_draw = __dmul_rn(splitmix_float64(state), total);
    a.rng[i] = state;
    s_out = is[count - 1];
    s_done = 0;
  }
  __syncthreads();
  for (int c0 = 0; c0 < count; c0 += kSampleFullStage) {
    const int cn = min(kSampleFullStage, count - c0);
    for (int k = tid; k < cn; k += blockDim.x) stage[k] = prob[c0 + k];
    __syncthreads();
    if (tid == 0) {
      double draw = s_draw;
      for (int k = 0; k < cn; k++) {
        draw = __dsub_rn(draw, stage[k]);
        if (draw < 0) {
          s_out = is[c0 + k];
          s_done = 1;
          break;
        }
      }
      s_draw = draw;
    }
    __syncthreads();
    if (s_done) break;
  }
  if (tid == 0) {
    a.ids[i] = s_out;
    a.status[i] = 0;
  }
}

}  // namespace sr
