// srstep_internal.h -- definitions shared by the step library's translation units.
#pragma once

#include <cuda_runtime.h>

#include <functional>
#include <string>
#include <vector>

#include "../../include/srstep.h"
#include "common.cuh"

// Metadata upload layout (int32 words): the host stages exactly this prefix and
// copies it with one cudaMemcpyAsync per step.
constexpr int kOffSessPos = 0;                  // [256]
constexpr int kOffTokOff = 256;                 // [257], padded to 260
constexpr int kOffPageOff = 516;                // [257], padded to 260
constexpr int kOffWant = 776;                   // 256 bytes
constexpr int kOffTokens = 840;                 // [1024]
constexpr int kMetaHeader = 1864;               // page ids follow
constexpr int kMetaComputed = 2 * 1024 + 2 * 256 + 4;
constexpr int64_t kSampleHistCap = 4 << 20;     // history ids staged per sampling call
// Sampler staging layout (host pinned and device copies share it).  Every
// region starts on a 16-byte boundary: the RNG states are 8-byte words.
constexpr size_t sr_align16(size_t x) { return (x + 15) & ~(size_t)15; }
constexpr size_t kSampOffSettings = 0;
constexpr size_t kSampOffHistOff = sr_align16(kSampOffSettings + 256 * 32);
constexpr size_t kSampOffHist = sr_align16(kSampOffHistOff + 257 * 4);
constexpr size_t kSampOffRng = sr_align16(kSampOffHist + (size_t)kSampleHistCap * 4);
constexpr size_t kSampOffIds = sr_align16(kSampOffRng + 256 * 8);
constexpr size_t kSampOffStatus = sr_align16(kSampOffIds + 256 * 4);
constexpr size_t kSampOffList = sr_align16(kSampOffStatus + 256 * 4);  // sessions of the full-vocabulary path
constexpr size_t kSampleStageBytes = sr_align16(kSampOffList + 256 * 4);
static_assert(kSampOffRng % 16 == 0, "RNG states must be 8-byte aligned");

struct BatchInfo {
  int sessions, rows, max_len, heads;
  int64_t pages;
  int attn_items;  // (row, kAttnSplit-position split) pairs of the split-K attention
  int attn_single;  // of those, the items of rows from 1-token chunks
  int attn_groups;  // (group of up to 4 consecutive rows of a longer chunk, split) pairs
  // Rows and attention counts of the first half when the step can run as two
  // halves cut at a session boundary (split_rows == 0: it cannot).
  int split_rows, split_items, split_single, split_groups;
};
// Rows of one half of a split step: at least a tensor-core tile's worth, at
// most half the step's row bound (each half has its own operand planes).
constexpr int kSplitMinRows = 64;
constexpr int kLaneRows = sr::kMaxRows / 2;

// Event-based per-kernel-class timing on the model's stream.
struct Profiler {
  uint32_t mask = 0;
  std::vector<cudaEvent_t> events;
  size_t used = 0;
  std::vector<int> pending;  // class of each recorded (start, end) event pair
  double ms[SR_PROF_CLASSES] = {};
  int64_t launches[SR_PROF_CLASSES] = {};
  int64_t total_launches = 0;
  cudaEvent_t span0 = nullptr, span1 = nullptr;
  bool span_open = false;
  double span_ms = 0;
  int64_t steps = 0;
};

// Where this device's copy of a parameter sits in the full tensor (tensor
// parallelism shards Q/K/V/gate/up by rows and O/down/qkv-bias by columns).
struct Shard {
  int32_t full_rows, full_cols, row0, col0;
};

struct sr_model {
  sr_model_desc d;
  std::vector<Shard> shards;  // parallel to params
  void* nccl_comm = nullptr;
  void* peer = nullptr;  // tensor-parallel peer-memory all-reduce state (tp_peer.cuh)
  int device = 0;
  int mode = SR_MODE_EXACT;
  sr::ModelDims dm;
  std::vector<sr::Param> params;
  std::vector<void*> allocs;
  uint64_t weights_version = 0;
  float* cos_t = nullptr;
  float* sin_t = nullptr;
  float *X = nullptr, *N = nullptr, *Q = nullptr, *K = nullptr, *V = nullptr, *A = nullptr, *T = nullptr;
  float *G = nullptr, *U = nullptr, *H = nullptr, *logits = nullptr;
  int32_t* meta_dev = nullptr;
  sr::StepMeta meta;
  int64_t max_pages_per_session = 0, page_cap = 0, upload_ints = 0;
  void* h_stage = nullptr;
  void* samp_dev = nullptr;
  // k_sample_full scratch (kSampleWave sessions x sample_full_stride(V)) and the
  // logits buffer of sr_sample_logits; both allocated on first use, grow-only
  uint8_t* samp_full = nullptr;
  size_t samp_full_bytes = 0;
  float* samp_logits = nullptr;
  size_t samp_logits_bytes = 0;
  cudaStream_t stream = nullptr;
  int last_sessions = 0;
  std::vector<uint8_t> last_want;
  Profiler prof;
  // fast-mode state (owned by fast_kernels.cuh)
  void* fast = nullptr;
  void* tc = nullptr;  // tensor-core shadows (fast_gemm.cuh)
  void* split = nullptr;       // split-step partitions and streams (srstep.cu), made on first use
  int split_mode = 0;          // sr_model_set_split: fast-mode steps may run as two overlapped halves
  std::vector<std::function<void()>> fast_free;
};

struct sr_kvpool {
  sr_model* m = nullptr;
  int64_t num_pages = 0;
  float* data = nullptr;
  std::vector<int32_t> owner;  // validation scratch: session listing each page (-2: none), reset after use
};

int sr_fail(int code, const std::string& msg);
// Heads of one tensor-parallel rank: query heads [q0, q0 + nq), KV heads
// [g0, g0 + nkv).
struct TpHeads {
  int q0, nq, g0, nkv;
};
bool tp_heads(const sr_model_desc& c, int rank, int size, TpHeads* t);
// Parameter table (hfProfileSpecs order) of one tensor-parallel rank.
int sr_param_table(const sr_model_desc& c, int rank, int size, std::vector<sr::Param>* params,
                   std::vector<Shard>* shards);

// Every kernel launch of a step increments this counter (the benchmark's
// gpu_launches); class scopes below may cover several launches.
inline void sr_count_launch(sr_model* m, int k = 1) { m->prof.total_launches += k; }

// RAII scope around one kernel launch: counts it and, when its class is
// selected, brackets it with a pair of events on the model's stream (or on
// the stream of a split step's half).
struct ProfScope {
  sr_model* m;
  int cls;
  bool timed;
  cudaStream_t s;
  ProfScope(sr_model* m_, int cls_, cudaStream_t s_ = nullptr)
      : m(m_), cls(cls_), timed((m_->prof.mask >> cls_) & 1u), s(s_ ? s_ : m_->stream) {
    if (timed) {
      Profiler& p = m->prof;
      while (p.events.size() < p.used + 2) {
        cudaEvent_t e;
        cudaEventCreate(&e);
        p.events.push_back(e);
      }
      cudaEventRecord(p.events[p.used], s);
    }
  }
  ~ProfScope() {
    Profiler& p = m->prof;
    p.launches[cls]++;
    if (timed) {
      cudaEventRecord(p.events[p.used + 1], s);
      p.used += 2;
      p.pending.push_back(cls);
    }
  }
};
#define SR_LAUNCH(m, cls, ...) \
  do {                         \
    ProfScope ps_((m), (cls)); \
    __VA_ARGS__;               \
  } while (0)
#define SR_LAUNCH_ON(m, cls, stream, ...) \
  do {                                    \
    ProfScope ps_((m), (cls), (stream));  \
    __VA_ARGS__;                          \
  } while (0)
void sr_prof_span_begin(sr_model* m);
void sr_prof_span_end(sr_model* m);
void sr_prof_resolve(sr_model* m);  // after a stream synchronize
int sr_model_alloc(sr_model* m, void** p, size_t bytes);
int sr_validate_batch(const sr_model* m, const sr_kvpool* pool, const sr_batch* b, BatchInfo* info);
int sr_upload_batch(sr_model* m, const sr_batch* b, const BatchInfo& info);
// Optional attention scratch supplied by the caller (the allocation-free step):
// when part_o is set, the step runs exact-order projections and norms and the
// split-K attention with this scratch, and allocates nothing.
struct StepScratch {
  float* part_o = nullptr;
  float* part_ml = nullptr;
};
int sr_step_enqueue(sr_model* m, sr_kvpool* pool, const BatchInfo& info, const volatile int32_t* cancel,
                    const StepScratch* scratch = nullptr);
// Samples sessions 0..n-1 of logits [n x V] (device): the last step's rows
// (all == false: only the sessions the step selected) or every row (all).
int sr_sample_enqueue(sr_model* m, int32_t n, const sr_sampling* settings, const int32_t* history_offsets,
                      const int32_t* history, const uint64_t* rng_state, int32_t blocked, const float* logits,
                      int32_t V, bool all);
int sr_sample_finish(sr_model* m, int32_t n, uint64_t* rng_state, int32_t* ids_out, bool all);
