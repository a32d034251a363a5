// srstep.cu -- C ABI of the engine step (include/srstep.h): model storage,
// KV page pool, step orchestration and the device sampler entry points.
//
// Reference: RyoSpiralArchitect/sr_go_tranformer cmd/monolith/monolith.go (M:line).
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/srstep.h"
#include "common.cuh"
#include "exact_kernels.cuh"
#include "fast_kernels.cuh"
#include "fast_gemm.cuh"
#include "sampler.cuh"
#include "srstep_internal.h"
#include "nccl_dl.h"
#include "tp_peer.cuh"
#include "gpt2_kernels.cuh"

using namespace sr;

// ------------------------------------------------------------------ errors --
static thread_local std::string g_err;
int sr_fail(int code, const std::string& msg) {
  g_err = msg;
  return code;
}
extern "C" const char* sr_last_error(void) { return g_err.c_str(); }
extern "C" const char* sr_version(void) { return "srstep 0.1 sm_100a"; }

#define CK(call)                                                                            \
  do {                                                                                      \
    cudaError_t e_ = (call);                                                                \
    if (e_ != cudaSuccess) return sr_fail(SR_EDEVICE, std::string(#call) + ": " + cudaGetErrorString(e_)); \
  } while (0)

// ------------------------------------------------------------------- model --
static int64_t param_value_bytes(int rows, int cols, int fmt) {
  if (fmt == kQ8) return (int64_t)rows * cols;
  if (fmt == kQ4) return (int64_t)rows * ((cols + 1) / 2);
  return (int64_t)rows * cols * 4;
}
static int64_t param_scale_count(int rows, int cols, int fmt) {
  return fmt == kF32 ? 0 : (int64_t)rows * ((cols + kQBlock - 1) / kQBlock);
}
static int matrix_format(int model_fmt, bool embed_or_head) {
  switch (model_fmt) {
    case SR_FMT_Q8: return kQ8;
    case SR_FMT_Q4: return kQ4;
    case SR_FMT_Q4_MIXED: return embed_or_head ? kQ8 : kQ4;  // hfMatrixFormat (M:572-582)
    default: return kF32;
  }
}

// hfInverseFrequency (M:4961-4977), evaluated on the host at load time.
static float hf_inverse_frequency(const sr_model_desc& c, int hd, int index) {
  float inv = 1.0f / (float)std::pow(c.rope_theta, (double)((float)(2 * index) / (float)hd));
  if (!c.rope_scaling) return inv;
  volatile float two_pi = (float)(2 * M_PI);
  float wave = two_pi / inv;
  float low_wave = (float)((double)c.rope_original_max_positions / c.rope_low_freq_factor);
  float high_wave = (float)((double)c.rope_original_max_positions / c.rope_high_freq_factor);
  float factor = (float)c.rope_factor;
  if (wave > low_wave) return inv / factor;
  if (wave >= high_wave) {
    volatile float smooth = ((float)c.rope_original_max_positions / wave - (float)c.rope_low_freq_factor) /
                            (float)(c.rope_high_freq_factor - c.rope_low_freq_factor);
    volatile float t1 = (1 - smooth) * inv;
    volatile float t2 = t1 / factor;
    volatile float t3 = smooth * inv;
    return t2 + t3;
  }
  return inv;
}

static void peer_close(sr_model* m);
static void free_model(sr_model* m) {
  if (!m) return;
  cudaSetDevice(m->device);
  peer_close(m);
  if (m->nccl_comm) nccl::api().CommDestroy((nccl::Comm)m->nccl_comm);
  for (void* p : m->allocs) cudaFree(p);
  if (m->h_stage) cudaFreeHost(m->h_stage);
  if (m->samp_full) cudaFree(m->samp_full);
  if (m->samp_logits) cudaFree(m->samp_logits);
  if (m->stream) cudaStreamDestroy(m->stream);
  for (auto& f : m->fast_free) f();
  delete m;
}

int sr_model_alloc(sr_model* m, void** p, size_t bytes) {
  cudaError_t e = cudaMalloc(p, bytes ? bytes : 16);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return sr_fail(SR_ENOMEM, "cudaMalloc(" + std::to_string(bytes) + "): " + cudaGetErrorString(e));
  }
  m->allocs.push_back(*p);
  return SR_OK;
}

// Heads of tensor-parallel rank `rank` of `size`: query heads [q0, q0 + nq)
// and KV heads [g0, g0 + nkv).  Either the KV heads divide over the ranks (each
// takes kv_heads/size of them with all their query heads), or each KV head is
// replicated on r = size/kv_heads consecutive ranks that split its `group`
// query heads, the first (group mod r) of them taking one more: Qwen2.5-7B (28
// query / 4 KV heads) on 8 ranks gives rank 2g+0 query heads 7g..7g+3 and rank
// 2g+1 heads 7g+4..7g+6, both holding KV head g.  The o_proj all-reduce then
// still sums every query head's contribution exactly once; the replicated KV
// projection is computed on both ranks of the pair.
bool tp_heads(const sr_model_desc& c, int rank, int size, TpHeads* t) {
  const int G = c.heads / c.kv_heads;
  if (c.kv_heads % size == 0) {
    t->nkv = c.kv_heads / size;
    t->g0 = rank * t->nkv;
    t->nq = t->nkv * G;
    t->q0 = t->g0 * G;
    return true;
  }
  if (size % c.kv_heads) return false;
  const int r = size / c.kv_heads;
  if (G < r) return false;
  const int sub = rank % r, base = G / r, extra = G % r;
  t->nkv = 1;
  t->g0 = rank / r;
  t->nq = base + (sub < extra ? 1 : 0);
  t->q0 = t->g0 * G + sub * base + std::min(sub, extra);
  return true;
}

// Validation shared by the single-GPU and tensor-parallel constructors
// (Config.validateShapeLimits, M:98-118, plus this implementation's limits).
static int validate_desc(const sr_model_desc& c, int tp_size) {
  if (c.vocab < 1 || c.vocab > 262144 || c.dim < 2 || c.dim > 8192 || c.hidden < 1 || c.hidden > 32768 ||
      c.layers < 1 || c.layers > 128 || c.heads < 1 || c.heads > c.dim || c.kv_heads < 1 || c.kv_heads > c.heads ||
      c.context < 1 || c.context > 32768)
    return sr_fail(SR_EINVAL, "invalid model dimensions");
  if (c.dim % c.heads || c.heads % c.kv_heads || (c.dim / c.heads) % 2)
    return sr_fail(SR_EINVAL, "dim must be divisible by heads with an even head dimension; heads must be divisible by kv_heads");
  if (!std::isfinite(c.rope_theta) || c.rope_theta <= 1 || !std::isfinite(c.norm_eps) || c.norm_eps < 1e-12 ||
      c.norm_eps > 1)
    return sr_fail(SR_EINVAL, "invalid RoPE theta or RMS epsilon");
  if (c.weight_format < SR_FMT_F32 || c.weight_format > SR_FMT_Q4_MIXED) return sr_fail(SR_EINVAL, "invalid weight format");
  if (c.page_tokens < 1 || c.page_tokens > 1024) return sr_fail(SR_EINVAL, "page_tokens must be 1..1024");
  const int hd = c.dim / c.heads, group = c.heads / c.kv_heads;
  if (hd % 4) return sr_fail(SR_EUNSUPPORTED, "head_dim must be a multiple of 4 on this device path");
  if (group * hd / 4 > 1024) return sr_fail(SR_EUNSUPPORTED, "query heads per KV head x head_dim exceeds 4096");
  if (c.rope_scaling && (c.rope_low_freq_factor <= 0 || c.rope_high_freq_factor <= c.rope_low_freq_factor))
    return sr_fail(SR_EINVAL, "invalid llama3 rope scaling");
  if (c.arch != SR_ARCH_LLAMA && c.arch != SR_ARCH_GPT2) return sr_fail(SR_EINVAL, "invalid model architecture");
  if (c.arch == SR_ARCH_GPT2) {  // readGPT2Config's profile (M:446-513)
    if (c.kv_heads != c.heads || !c.tied || c.qkv_bias || c.rope_scaling)
      return sr_fail(SR_EINVAL, "GPT-2 needs kv_heads == heads, a tied head, no q/k/v bias flag and no RoPE scaling");
    if (c.positions < c.context || c.positions > 32768)
      return sr_fail(SR_EINVAL, "GPT-2 position table must cover the context (at most 32768 rows)");
    if (tp_size != 1) return sr_fail(SR_EUNSUPPORTED, "the GPT-2 profile runs on one GPU");
  }
  if (tp_size < 1 || tp_size > 64) return sr_fail(SR_EINVAL, "tensor-parallel size must be 1..64");
  if (tp_size > 1) {
    if (c.hidden % tp_size)
      return sr_fail(SR_EUNSUPPORTED, "tensor parallelism needs hidden divisible by the rank count");
    if (c.weight_format != SR_FMT_F32 && (c.hidden / tp_size) % kQBlock)
      return sr_fail(SR_EUNSUPPORTED, "tensor-parallel column shards of quantized matrices must hold whole 64-column blocks");
    for (int r = 0; r < tp_size; r++) {
      TpHeads t;
      if (!tp_heads(c, r, tp_size, &t))
        return sr_fail(SR_EUNSUPPORTED, "tensor parallelism needs kv_heads divisible by the rank count, or the rank "
                                        "count divisible by kv_heads with at least one query head per rank");
      if (c.weight_format != SR_FMT_F32 && (t.nq * hd) % kQBlock)
        return sr_fail(SR_EUNSUPPORTED, "tensor-parallel column shards of quantized matrices must hold whole 64-column blocks");
    }
  }
  return SR_OK;
}

// Parameter table in hfProfileSpecs order (M:407-442) for rank `rank` of
// `size`: Q/K/V/gate/up keep a contiguous block of rows, O/down and the qkv
// biases a contiguous block of columns (the rank's heads from tp_heads, or its
// 1/size of the FFN); everything else is replicated.
int sr_param_table(const sr_model_desc& c, int rank, int size, std::vector<Param>* params,
                   std::vector<Shard>* shards) {
  params->clear();
  shards->clear();
  const int hd = c.dim / c.heads, kd = hd * c.kv_heads;
  TpHeads th{0, c.heads, 0, c.kv_heads};
  if (c.arch != SR_ARCH_GPT2 && !tp_heads(c, rank, size, &th)) return SR_EUNSUPPORTED;
  const int hs = c.hidden / size;
  // kind 0: replicated; 1: rows [lo, lo + n); 2: columns [lo, lo + n)
  auto add = [&](int rows, int cols, bool matrix, bool eh, int kind, int lo = 0, int n = 0) {
    Shard sh{rows, cols, 0, 0};
    Param p;
    p.rows = rows;
    p.cols = cols;
    if (kind == 1) {
      p.rows = n;
      sh.row0 = lo;
    } else if (kind == 2) {
      p.cols = n;
      sh.col0 = lo;
    }
    p.format = matrix ? matrix_format(c.weight_format, eh) : kF32;
    p.values = nullptr;
    p.scales = nullptr;
    params->push_back(p);
    shards->push_back(sh);
  };
  const int L = c.layers, d = c.dim, h = c.hidden;
  if (c.arch == SR_ARCH_GPT2) {  // loadGPT2's parameter order (M:5063-5066, 5114-5122)
    add(c.vocab, d, true, true, 0);
    add(c.positions, d, false, false, 0);
    add(1, d, false, false, 0);
    add(1, d, false, false, 0);
    for (int l = 0; l < L; l++) {
      add(1, d, false, false, 0);
      add(1, d, false, false, 0);
      for (int k = 0; k < 3; k++) add(d, d, true, false, 0);
      for (int k = 0; k < 3; k++) add(1, d, false, false, 0);
      add(d, d, true, false, 0);
      add(1, d, false, false, 0);
      add(1, d, false, false, 0);
      add(1, d, false, false, 0);
      add(h, d, true, false, 0);
      add(1, h, false, false, 0);
      add(d, h, true, false, 0);
      add(1, d, false, false, 0);
    }
    return SR_OK;
  }
  const int q0 = th.q0 * hd, nq = th.nq * hd, k0 = th.g0 * hd, nk = th.nkv * hd;
  add(c.vocab, d, true, true, 0);
  for (int l = 0; l < L; l++) {
    add(1, d, false, false, 0);
    add(d, d, true, false, 1, q0, nq);
    add(kd, d, true, false, 1, k0, nk);
    add(kd, d, true, false, 1, k0, nk);
    add(d, d, true, false, 2, q0, nq);
    add(1, d, false, false, 0);
    add(h, d, true, false, 1, rank * hs, hs);
    add(h, d, true, false, 1, rank * hs, hs);
    add(d, h, true, false, 2, rank * hs, hs);
  }
  add(1, d, false, false, 0);
  if (c.qkv_bias)
    for (int l = 0; l < L; l++) {
      add(1, d, false, false, 2, q0, nq);
      add(1, kd, false, false, 2, k0, nk);
      add(1, kd, false, false, 2, k0, nk);
    }
  if (!c.tied) add(c.vocab, d, true, true, 0);
  return SR_OK;
}

extern "C" int sr_tp_shard(const sr_model_desc* desc, int32_t rank, int32_t size, int32_t index, int32_t* shard) {
  if (!desc || !shard) return sr_fail(SR_EINVAL, "null argument");
  int rc = validate_desc(*desc, size);
  if (rc != SR_OK) return rc;
  if (rank < 0 || rank >= size) return sr_fail(SR_EINVAL, "rank out of range");
  std::vector<Param> ps;
  std::vector<Shard> sh;
  sr_param_table(*desc, rank, size, &ps, &sh);
  if (index < 0 || index >= (int32_t)ps.size()) return sr_fail(SR_EINVAL, "parameter index out of range");
  shard[0] = sh[index].row0;
  shard[1] = ps[index].rows;
  shard[2] = sh[index].col0;
  shard[3] = ps[index].cols;
  return SR_OK;
}

static int model_create(const sr_model_desc* desc, int device, int tp_rank, int tp_size, const void* nccl_id,
                        sr_model** out);

extern "C" int sr_model_create(const sr_model_desc* desc, int device, sr_model** out) {
  return model_create(desc, device, 0, 1, nullptr, out);
}

extern "C" int sr_tp_unique_id(void* id_out) {
  if (!id_out) return sr_fail(SR_EINVAL, "null argument");
  nccl::Api& api = nccl::api();
  if (!api.ok) return sr_fail(SR_EUNSUPPORTED, api.error);
  nccl::UniqueId id;
  int r = api.GetUniqueId(&id);
  if (r != nccl::kSuccess) return sr_fail(SR_EDEVICE, std::string("ncclGetUniqueId: ") + api.GetErrorString(r));
  memcpy(id_out, &id, sizeof(id));
  return SR_OK;
}

extern "C" int sr_model_create_tp(const sr_model_desc* desc, int device, int32_t tp_rank, int32_t tp_size,
                                  const void* nccl_id, sr_model** out) {
  if (tp_size > 1 && !nccl_id) return sr_fail(SR_EINVAL, "tensor parallelism needs the rank-0 NCCL id");
  if (tp_rank < 0 || tp_rank >= tp_size) return sr_fail(SR_EINVAL, "rank out of range");
  return model_create(desc, device, tp_rank, tp_size, nccl_id, out);
}

// ------------------------------------------------- tensor-parallel peer memory --
// One exported allocation per rank: the two all-reduce buffers, the barrier
// slots and the finished-CTA counter, then the LL protocol's two reduce and
// two gather buffers (tp_peer.cuh).  tables (device) holds, once the peers are
// open, every rank's buffer 0, buffer 1, slots, reduce 0, reduce 1, gather 0
// and gather 1 pointers (7 x size).
struct PeerHost {
  uint8_t* base = nullptr;
  size_t buf_bytes = 0, rb_bytes = 0, gb_bytes = 0;
  int protocol = SR_PEER_BARRIER;
  int ll_parity = 0;
  float* buf[2] = {};
  int* slots = nullptr;
  int* counter = nullptr;
  int* err = nullptr;
  void** tables = nullptr;
  std::vector<void*> opened;  // peers' allocations mapped through IPC
  uint32_t epoch = 0;
  int cur = 0;
  bool open = false, ran = false;
};
constexpr size_t kPeerTail = 1024;  // slots (peer::kSlots ints), counter, error flag
static_assert(peer::kSlots * 4 + 64 <= kPeerTail, "peer tail too small");
static_assert(sizeof(cudaIpcMemHandle_t) == SR_TP_PEER_HANDLE_BYTES, "IPC handle size");

static int peer_alloc(sr_model* m, size_t buf_bytes) {
  PeerHost* ph = new PeerHost();
  m->peer = ph;
  ph->buf_bytes = buf_bytes;
  // LL buffers: 16-byte lines of two values (8 bytes per value), every rank's
  // chunk slot of the reduce buffer sized for the largest step
  const int64_t count_max = (int64_t)(buf_bytes / 4), size = m->dm.tp_size;
  const int64_t chunk_max = ((count_max + size - 1) / size + 3) / 4 * 4;
  ph->rb_bytes = (size_t)(size * chunk_max * 8);
  ph->gb_bytes = (size_t)(count_max * 8);
  int rc = sr_model_alloc(m, (void**)&ph->base, 2 * buf_bytes + kPeerTail + 2 * ph->rb_bytes + 2 * ph->gb_bytes);
  if (rc != SR_OK) return rc;
  ph->buf[0] = (float*)ph->base;
  ph->buf[1] = (float*)(ph->base + buf_bytes);
  ph->slots = (int*)(ph->base + 2 * buf_bytes);
  ph->counter = ph->slots + peer::kSlots;
  ph->err = ph->counter + 4;
  if (cudaMemset(ph->base + 2 * buf_bytes, 0, kPeerTail) != cudaSuccess) {
    cudaGetLastError();
    return sr_fail(SR_EDEVICE, "clearing the all-reduce barrier slots failed");
  }
  if (cudaMemset(ph->base + 2 * buf_bytes + kPeerTail, 0, 2 * ph->rb_bytes + 2 * ph->gb_bytes) != cudaSuccess) {
    cudaGetLastError();
    return sr_fail(SR_EDEVICE, "clearing the LL all-reduce buffers failed");
  }
  if ((rc = sr_model_alloc(m, (void**)&ph->tables, (size_t)7 * m->dm.tp_size * sizeof(void*))) != SR_OK) return rc;
  m->T = ph->buf[0];
  return SR_OK;
}

// A last barrier over the peers (bounded) before this rank's memory goes away,
// so that no rank still reads it; then the IPC mappings close.
__global__ void k_peer_barrier(peer::Args a) {
  if (threadIdx.x < a.size) {
    __threadfence_system();
    peer::st_release_sys(a.flags[threadIdx.x] + a.rank, (int)a.epoch);
  }
  peer::wait_all(a, 0);
}
static void peer_close(sr_model* m) {
  PeerHost* ph = (PeerHost*)m->peer;
  if (!ph) return;
  if (ph->open && m->stream) {
    peer::Args a{};
    a.flags = (int* const*)(ph->tables + (size_t)2 * m->dm.tp_size);
    a.err = ph->err;
    a.epoch = ++ph->epoch;
    a.rank = m->dm.tp_rank;
    a.size = m->dm.tp_size;
    cudaMemsetAsync(ph->err, 0, 4, m->stream);
    k_peer_barrier<<<1, 64, 0, m->stream>>>(a);
    cudaStreamSynchronize(m->stream);
    cudaGetLastError();
  }
  for (void* p : ph->opened) cudaIpcCloseMemHandle(p);
  delete ph;
  m->peer = nullptr;
}

extern "C" int sr_tp_peer_handle(sr_model* m, void* handle_out) {
  if (!m || !handle_out) return sr_fail(SR_EINVAL, "null argument");
  PeerHost* ph = (PeerHost*)m->peer;
  if (!ph) return sr_fail(SR_EINVAL, "not a tensor-parallel model");
  CK(cudaSetDevice(m->device));
  cudaIpcMemHandle_t h;
  CK(cudaIpcGetMemHandle(&h, ph->base));
  memcpy(handle_out, &h, sizeof(h));
  return SR_OK;
}

extern "C" int sr_tp_peer_open(sr_model* m, const void* handles) {
  if (!m || !handles) return sr_fail(SR_EINVAL, "null argument");
  PeerHost* ph = (PeerHost*)m->peer;
  if (!ph) return sr_fail(SR_EINVAL, "not a tensor-parallel model");
  if (ph->open) return sr_fail(SR_EINVAL, "peer memory is already open");
  const int size = m->dm.tp_size, rank = m->dm.tp_rank;
  if (size > peer::kMaxRanks) return sr_fail(SR_EUNSUPPORTED, "peer all-reduce supports at most 64 ranks");
  if (m->dm.dim % 4) return sr_fail(SR_EUNSUPPORTED, "peer all-reduce needs a model width divisible by 4");
  CK(cudaSetDevice(m->device));
  std::vector<void*> host((size_t)7 * size);
  for (int q = 0; q < size; q++) {
    uint8_t* b = ph->base;
    if (q != rank) {
      cudaIpcMemHandle_t h;
      memcpy(&h, (const uint8_t*)handles + (size_t)q * SR_TP_PEER_HANDLE_BYTES, sizeof(h));
      void* p = nullptr;
      cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
      if (e != cudaSuccess) {
        cudaGetLastError();
        for (void* o : ph->opened) cudaIpcCloseMemHandle(o);
        ph->opened.clear();
        return sr_fail(SR_EDEVICE, "opening rank " + std::to_string(q) + "'s memory: " + cudaGetErrorString(e));
      }
      ph->opened.push_back(p);
      b = (uint8_t*)p;
    }
    host[q] = b;
    host[size + q] = b + ph->buf_bytes;
    host[2 * size + q] = b + 2 * ph->buf_bytes;
    uint8_t* ll = b + 2 * ph->buf_bytes + kPeerTail;
    host[3 * size + q] = ll;
    host[4 * size + q] = ll + ph->rb_bytes;
    host[5 * size + q] = ll + 2 * ph->rb_bytes;
    host[6 * size + q] = ll + 2 * ph->rb_bytes + ph->gb_bytes;
  }
  CK(cudaMemcpy(ph->tables, host.data(), host.size() * sizeof(void*), cudaMemcpyHostToDevice));
  ph->open = true;
  return SR_OK;
}

extern "C" int sr_tp_peer_set_protocol(sr_model* m, int32_t protocol) {
  if (!m) return sr_fail(SR_EINVAL, "null model");
  PeerHost* ph = (PeerHost*)m->peer;
  if (!ph || !ph->open) return sr_fail(SR_EINVAL, "peer memory is not open (sr_tp_peer_open)");
  if (protocol != SR_PEER_BARRIER && protocol != SR_PEER_LL) return sr_fail(SR_EINVAL, "unknown peer protocol");
  ph->protocol = protocol;
  return SR_OK;
}

// After the step's stream synchronize: SR_ETIMEOUT if an all-reduce barrier
// wait expired (a rank did not take part).
static int tp_check(sr_model* m) {
  PeerHost* ph = (PeerHost*)m->peer;
  if (!ph || !ph->ran) return SR_OK;
  ph->ran = false;
  int h = 0;
  if (cudaMemcpy(&h, ph->err, 4, cudaMemcpyDeviceToHost) != cudaSuccess) {
    cudaGetLastError();
    return sr_fail(SR_EDEVICE, "reading the all-reduce error flag failed");
  }
  if (h) {
    cudaMemset(ph->err, 0, 4);
    return sr_fail(SR_ETIMEOUT, "a tensor-parallel all-reduce barrier expired (a rank did not join the step)");
  }
  return SR_OK;
}

static int model_create(const sr_model_desc* desc, int device, int tp_rank, int tp_size, const void* nccl_id,
                        sr_model** out) {
  if (!desc || !out) return sr_fail(SR_EINVAL, "null argument");
  *out = nullptr;
  const sr_model_desc& c = *desc;
  int rc = validate_desc(c, tp_size);
  if (rc != SR_OK) return rc;
  const int hd = c.dim / c.heads;
  TpHeads th{0, c.heads, 0, c.kv_heads};
  if (c.arch != SR_ARCH_GPT2) tp_heads(c, tp_rank, tp_size, &th);  // validated above
  int ndev = 0;
  CK(cudaGetDeviceCount(&ndev));
  if (device < 0 || device >= ndev) return sr_fail(SR_EINVAL, "invalid device ordinal");
  CK(cudaSetDevice(device));

  sr_model* m = new sr_model();
  m->d = c;
  m->device = device;
  m->mode = SR_MODE_EXACT;
  ModelDims& dm = m->dm;
  dm.vocab = c.vocab;
  dm.dim = c.dim;
  dm.hidden = c.hidden / tp_size;
  dm.layers = c.layers;
  dm.heads = th.nq;
  dm.kv_heads = th.nkv;
  dm.context = c.context;
  dm.hd = hd;
  dm.kvd = hd * dm.kv_heads;
  dm.qd = hd * dm.heads;
  dm.group = th.nq / th.nkv;
  dm.tp_rank = tp_rank;
  dm.tp_size = tp_size;
  dm.page_tokens = c.page_tokens;
  dm.page_elems = 2LL * c.page_tokens * dm.kvd * c.layers;
  sr_param_table(c, tp_rank, tp_size, &m->params, &m->shards);
  const int d = c.dim, kd = dm.kvd, h = dm.hidden;
  if (tp_size > 1) {
    nccl::Api& api = nccl::api();
    if (!api.ok) {
      delete m;
      return sr_fail(SR_EUNSUPPORTED, api.error);
    }
    nccl::UniqueId id;
    memcpy(&id, nccl_id, sizeof(id));
    nccl::Comm comm = nullptr;
    int r = api.CommInitRank(&comm, tp_size, id, tp_rank);
    if (r != nccl::kSuccess) {
      delete m;
      return sr_fail(SR_EDEVICE, std::string("ncclCommInitRank: ") + api.GetErrorString(r));
    }
    m->nccl_comm = comm;
  }

  for (auto& p : m->params) {
    int64_t vb = param_value_bytes(p.rows, p.cols, p.format);
    int64_t sc = param_scale_count(p.rows, p.cols, p.format);
    if ((rc = sr_model_alloc(m, &p.values, (size_t)vb)) != SR_OK) { free_model(m); return rc; }
    if (sc && (rc = sr_model_alloc(m, (void**)&p.scales, (size_t)sc * 4)) != SR_OK) { free_model(m); return rc; }
    cudaMemset(p.values, 0, (size_t)vb);
    if (sc) cudaMemset(p.scales, 0, (size_t)sc * 4);
  }
  // HF RoPE tables (M:5034-5043).
  {
    const int half = hd / 2;
    std::vector<float> cs((size_t)c.context * half), sn((size_t)c.context * half);
    std::vector<float> inv(half);
    for (int j = 0; j < half; j++) inv[j] = hf_inverse_frequency(c, hd, j);
    for (int pos = 0; pos < c.context; pos++)
      for (int j = 0; j < half; j++) {
        volatile float prod = (float)pos * inv[j];
        double angle = (double)prod;
        cs[(size_t)pos * half + j] = (float)std::cos(angle);
        sn[(size_t)pos * half + j] = (float)std::sin(angle);
      }
    if ((rc = sr_model_alloc(m, (void**)&m->cos_t, cs.size() * 4)) != SR_OK ||
        (rc = sr_model_alloc(m, (void**)&m->sin_t, sn.size() * 4)) != SR_OK) {
      free_model(m);
      return rc;
    }
    cudaMemcpy(m->cos_t, cs.data(), cs.size() * 4, cudaMemcpyHostToDevice);
    cudaMemcpy(m->sin_t, sn.data(), sn.size() * 4, cudaMemcpyHostToDevice);
  }
  // Step workspace (decodeWorkspace, M:6064-6096) at the 1024-row bound.
  {
    const int64_t R = kMaxRows;
    float** bufs[] = {&m->X, &m->N, &m->Q, &m->A, &m->T};
    for (float** b : bufs) {
      if (b == &m->T && tp_size > 1) continue;  // the two all-reduce buffers below
      if ((rc = sr_model_alloc(m, (void**)b, (size_t)(R * d * 4))) != SR_OK) { free_model(m); return rc; }
    }
    if (tp_size > 1 && (rc = peer_alloc(m, (size_t)(R * d * 4))) != SR_OK) {
      free_model(m);
      return rc;
    }
    if ((rc = sr_model_alloc(m, (void**)&m->K, (size_t)(R * kd * 4))) != SR_OK ||
        (rc = sr_model_alloc(m, (void**)&m->V, (size_t)(R * kd * 4))) != SR_OK ||
        (rc = sr_model_alloc(m, (void**)&m->G, (size_t)(R * h * 4))) != SR_OK ||
        (rc = sr_model_alloc(m, (void**)&m->U, (size_t)(R * h * 4))) != SR_OK ||
        (rc = sr_model_alloc(m, (void**)&m->H, (size_t)(R * h * 4))) != SR_OK ||
        (rc = sr_model_alloc(m, (void**)&m->logits, (size_t)kMaxSessions * c.vocab * 4)) != SR_OK) {
      free_model(m);
      return rc;
    }
  }
  // Metadata: upload region (host-staged) followed by the device-built region.
  m->max_pages_per_session = (c.context + c.page_tokens - 1) / c.page_tokens;
  m->page_cap = (int64_t)kMaxSessions * m->max_pages_per_session;
  m->upload_ints = kMetaHeader + m->page_cap;
  // computed region: per-row data, head maps, then the attention item table
  // (at most ceil(context / kAttnSplit) items for each of the 1024 rows)
  const int64_t item_cap = (int64_t)kMaxRows * ((c.context + kAttnSplit - 1) / kAttnSplit);
  const int64_t meta_ints = m->upload_ints + kMetaComputed + kMaxRows + 3 * item_cap;
  if ((rc = sr_model_alloc(m, (void**)&m->meta_dev, (size_t)meta_ints * 4)) != SR_OK) { free_model(m); return rc; }
  if (cudaMallocHost(&m->h_stage, (size_t)(m->upload_ints * 4 + kSampleStageBytes)) != cudaSuccess) {
    cudaGetLastError();
    free_model(m);
    return sr_fail(SR_ENOMEM, "cudaMallocHost for the batch staging buffer failed");
  }
  {
    int32_t* b = m->meta_dev;
    StepMeta& s = m->meta;
    s.sess_pos = b + kOffSessPos;
    s.tok_off = b + kOffTokOff;
    s.page_off = b + kOffPageOff;
    s.want = (uint8_t*)(b + kOffWant);
    s.tokens = b + kOffTokens;
    s.page_ids = b + kMetaHeader;
    int32_t* cbase = b + m->upload_ints;
    s.row_pos = cbase;
    s.row_pbase = cbase + kMaxRows;
    s.head_src = cbase + 2 * kMaxRows;
    s.head_dst = cbase + 2 * kMaxRows + kMaxSessions;
    s.n_heads = cbase + 2 * kMaxRows + 2 * kMaxSessions;
    s.row_item0 = cbase + kMetaComputed;
    s.item_rs = cbase + kMetaComputed + kMaxRows;
    s.single_rs = s.item_rs + item_cap;
    s.grp_rs = s.single_rs + item_cap;
  }
  // Sampler device buffers.
  {
    static_assert(sizeof(SampleSetting) == 32, "sampler settings layout");
    if ((rc = sr_model_alloc(m, (void**)&m->samp_dev, kSampleStageBytes)) != SR_OK) { free_model(m); return rc; }
  }
  if (cudaStreamCreateWithFlags(&m->stream, cudaStreamNonBlocking) != cudaSuccess) {
    cudaGetLastError();
    free_model(m);
    return sr_fail(SR_EDEVICE, "cudaStreamCreate failed");
  }
  cudaFuncSetAttribute(k_attention_exact, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
  cudaFuncSetAttribute(k_sample, cudaFuncAttributeMaxDynamicSharedMemorySize, 64 * 1024);
  cudaFuncSetAttribute(k_sample_full, cudaFuncAttributeMaxDynamicSharedMemorySize, 96 * 1024);
  if ((rc = fast_init(m)) != SR_OK) { free_model(m); return rc; }
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    free_model(m);
    return sr_fail(SR_EDEVICE, std::string("model init: ") + cudaGetErrorString(e));
  }
  *out = m;
  return SR_OK;
}

extern "C" int sr_model_destroy(sr_model* m) {
  if (!m) return sr_fail(SR_EINVAL, "null model");
  free_model(m);
  return SR_OK;
}
extern "C" int sr_model_param_count(const sr_model* m, int32_t* count) {
  if (!m || !count) return sr_fail(SR_EINVAL, "null argument");
  *count = (int32_t)m->params.size();
  return SR_OK;
}
extern "C" int sr_model_param_info(const sr_model* m, int32_t index, sr_param_info* out) {
  if (!m || !out) return sr_fail(SR_EINVAL, "null argument");
  if (index < 0 || index >= (int32_t)m->params.size()) return sr_fail(SR_EINVAL, "parameter index out of range");
  const Param& p = m->params[index];
  const Shard& sh = m->shards[index];
  out->rows = sh.full_rows;
  out->cols = sh.full_cols;
  out->format = p.format;
  out->reserved = 0;
  out->value_bytes = param_value_bytes(sh.full_rows, sh.full_cols, p.format);
  out->scale_count = param_scale_count(sh.full_rows, sh.full_cols, p.format);
  return SR_OK;
}

// Copy this rank's shard (rows [row0, row0+rows), columns [col0, col0+cols))
// out of a full host tensor in the reference layout.  Column shards start on
// 64-column blocks, so Q4 bytes and scale blocks split cleanly.
static void extract_shard(const Param& p, const Shard& sh, const void* full_values, const float* full_scales,
                          std::vector<uint8_t>* values, std::vector<float>* scales) {
  const int64_t vb = param_value_bytes(p.rows, p.cols, p.format), sc = param_scale_count(p.rows, p.cols, p.format);
  values->resize((size_t)vb);
  scales->resize((size_t)sc);
  const int64_t full_row_bytes = param_value_bytes(1, sh.full_cols, p.format);
  const int64_t row_bytes = param_value_bytes(1, p.cols, p.format);
  const int64_t col_byte0 = param_value_bytes(1, sh.col0, p.format);
  const int64_t full_groups = (sh.full_cols + kQBlock - 1) / kQBlock, groups = (p.cols + kQBlock - 1) / kQBlock;
  for (int64_t r = 0; r < p.rows; r++) {
    const uint8_t* src = (const uint8_t*)full_values + (sh.row0 + r) * full_row_bytes + col_byte0;
    memcpy(values->data() + r * row_bytes, src, (size_t)row_bytes);
    if (sc)
      memcpy(scales->data() + r * groups, full_scales + (sh.row0 + r) * full_groups + sh.col0 / kQBlock,
             (size_t)groups * 4);
  }
}
extern "C" int sr_model_load_param(sr_model* m, int32_t index, const void* values, size_t value_bytes,
                                   const float* scales, size_t scale_count) {
  if (!m || !values) return sr_fail(SR_EINVAL, "null argument");
  if (index < 0 || index >= (int32_t)m->params.size()) return sr_fail(SR_EINVAL, "parameter index out of range");
  Param& p = m->params[index];
  const Shard& sh = m->shards[index];
  const int64_t fvb = param_value_bytes(sh.full_rows, sh.full_cols, p.format);
  const int64_t fsc = param_scale_count(sh.full_rows, sh.full_cols, p.format);
  if ((int64_t)value_bytes != fvb) return sr_fail(SR_EINVAL, "value byte count does not match the parameter layout");
  if ((int64_t)scale_count != fsc || (fsc && !scales)) return sr_fail(SR_EINVAL, "scale count does not match the parameter layout");
  CK(cudaSetDevice(m->device));
  std::vector<uint8_t> v;
  std::vector<float> sv;
  extract_shard(p, sh, values, scales, &v, &sv);
  CK(cudaMemcpy(p.values, v.data(), v.size(), cudaMemcpyHostToDevice));
  if (!sv.empty()) CK(cudaMemcpy(p.scales, sv.data(), sv.size() * 4, cudaMemcpyHostToDevice));
  m->weights_version++;
  return SR_OK;
}
extern "C" int sr_model_read_param(const sr_model* m, int32_t index, void* values, size_t value_bytes, float* scales,
                                   size_t scale_count) {
  if (!m || !values) return sr_fail(SR_EINVAL, "null argument");
  if (index < 0 || index >= (int32_t)m->params.size()) return sr_fail(SR_EINVAL, "parameter index out of range");
  const Param& p = m->params[index];
  int64_t vb = param_value_bytes(p.rows, p.cols, p.format), sc = param_scale_count(p.rows, p.cols, p.format);
  if ((int64_t)value_bytes != vb) return sr_fail(SR_EINVAL, "value byte count does not match the parameter layout");
  if ((int64_t)scale_count != sc || (sc && !scales)) return sr_fail(SR_EINVAL, "scale count does not match the parameter layout");
  CK(cudaSetDevice(m->device));
  CK(cudaMemcpy(values, p.values, (size_t)vb, cudaMemcpyDeviceToHost));
  if (sc) CK(cudaMemcpy(scales, p.scales, (size_t)sc * 4, cudaMemcpyDeviceToHost));
  return SR_OK;
}

// ------------------------------------------------------------ synthetic init --
// Counter-based SplitMix64: the k-th output (1-based) of a generator seeded with
// `seed` is mix(seed + k*gamma), so element e (two draws per Normal) can be
// generated independently of every other element.
__device__ __forceinline__ uint64_t splitmix_at(uint64_t seed, uint64_t k) {
  uint64_t z = seed + k * 0x9e3779b97f4a7c15ULL;
  z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ULL;
  z = (z ^ (z >> 27)) * 0x94d049bb133111ebULL;
  return z ^ (z >> 31);
}
__device__ __forceinline__ float synth_value(uint64_t seed, uint64_t e, double scale) {
  double u1 = (double)(splitmix_at(seed, 2 * e + 1) >> 11) * (1.0 / 9007199254740992.0);
  double u2 = (double)(splitmix_at(seed, 2 * e + 2) >> 11) * (1.0 / 9007199254740992.0);
  double nrm = sqrt(__dmul_rn(-2.0, log(__dsub_rn(1.0, u1)))) * cos(__dmul_rn(2 * M_PI, u2));
  return (float)__dmul_rn(nrm, scale);
}
// One thread per (row, 64-column block): generate, then quantize with the
// reference's block quantizer (readParam M:857-880, lowBitScale M:3877-3891).
// (row0, col0, full_cols) place the local shard in the full tensor, so every
// rank generates exactly its part of the same model.
__global__ void k_init_param(Param p, uint64_t seed, uint64_t e0, double scale, int norm, const float* src, int row0,
                             int col0, int full_cols) {
  const int64_t groups = (p.cols + kQBlock - 1) / kQBlock;
  const int64_t total = (int64_t)p.rows * groups;
  for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = t / groups, g = t % groups;
    const int j0 = (int)(g * kQBlock), j1 = min(j0 + kQBlock, p.cols);
    float v[kQBlock];
    float amax = 0.f;
    for (int j = j0; j < j1; j++) {
      float x = src ? src[row * p.cols + j]
                    : (norm ? 1.0f
                            : synth_value(seed, e0 + (uint64_t)((row0 + row) * (int64_t)full_cols + col0 + j), scale));
      v[j - j0] = x;
      amax = fmaxf(amax, fabsf(x));
    }
    if (p.format == kF32) {
      for (int j = j0; j < j1; j++) ((float*)p.values)[row * p.cols + j] = v[j - j0];
      continue;
    }
    const double levels = p.format == kQ4 ? 7.0 : 127.0;
    float sc = 0.f;
    if (amax != 0.f) {
      sc = (float)__ddiv_rn((double)amax, levels);
      if (sc == 0.f) {
        sc = 1.40129846e-45f;
      } else if (sc > 1.40129846e-45f && __dmul_rn((double)sc, levels) > (double)amax) {
        sc = nextafterf(sc, 0.f);
      }
    }
    p.scales[row * groups + g] = sc;
    for (int j = j0; j < j1; j++) {
      double q = 0.0;
      if (sc != 0.f) q = fmin(levels, fmax(-levels, round(__ddiv_rn((double)v[j - j0], (double)sc))));
      if (p.format == kQ8) {
        ((int8_t*)p.values)[row * p.cols + j] = (int8_t)q;
      } else {
        uint8_t* b = (uint8_t*)p.values + row * ((p.cols + 1) / 2) + j / 2;
        uint8_t nib = (uint8_t)((int)q & 15);
        // Each thread owns whole 64-column blocks, i.e. whole bytes.
        *b = (j & 1) ? (uint8_t)((*b & 0x0f) | (nib << 4)) : (uint8_t)((*b & 0xf0) | nib);
      }
    }
  }
}

extern "C" int sr_model_init_synthetic(sr_model* m, uint64_t seed, double scale) {
  if (!m) return sr_fail(SR_EINVAL, "null model");
  if (m->d.arch == SR_ARCH_GPT2) return sr_fail(SR_EUNSUPPORTED, "no synthetic initialisation for the GPT-2 profile");
  CK(cudaSetDevice(m->device));
  const int L = m->d.layers;
  uint64_t e0 = 0;
  for (size_t i = 0; i < m->params.size(); i++) {
    Param& p = m->params[i];
    bool norm = (i >= 1 && i < (size_t)(1 + 9 * L) && ((i - 1) % 9 == 0 || (i - 1) % 9 == 5)) || i == (size_t)(1 + 9 * L);
    if (p.format == kQ4) CK(cudaMemsetAsync(p.values, 0, (size_t)param_value_bytes(p.rows, p.cols, p.format), m->stream));
    int64_t work = (int64_t)p.rows * ((p.cols + kQBlock - 1) / kQBlock);
    int blocks = (int)std::min<int64_t>((work + 255) / 256, 148 * 32);
    const Shard& sh = m->shards[i];
    k_init_param<<<blocks, 256, 0, m->stream>>>(p, seed, e0, scale, norm ? 1 : 0, nullptr, sh.row0, sh.col0,
                                                 sh.full_cols);
    CK(cudaGetLastError());
    if (!norm) e0 += (uint64_t)sh.full_rows * sh.full_cols;
  }
  CK(cudaStreamSynchronize(m->stream));
  m->weights_version++;
  return SR_OK;
}

extern "C" int sr_model_load_param_f32(sr_model* m, int32_t index, const float* values, size_t count) {
  if (!m || !values) return sr_fail(SR_EINVAL, "null argument");
  if (index < 0 || index >= (int32_t)m->params.size()) return sr_fail(SR_EINVAL, "parameter index out of range");
  Param& p = m->params[index];
  const Shard& sh = m->shards[index];
  if ((int64_t)count != (int64_t)sh.full_rows * sh.full_cols)
    return sr_fail(SR_EINVAL, "value count does not match rows*cols");
  CK(cudaSetDevice(m->device));
  // this rank's rows/columns of the full fp32 tensor
  Param fp = p;
  fp.format = kF32;
  std::vector<uint8_t> local;
  std::vector<float> unused;
  extract_shard(fp, sh, values, nullptr, &local, &unused);
  const size_t lcount = (size_t)p.rows * p.cols;
  float* tmp = nullptr;
  cudaError_t e = cudaMalloc((void**)&tmp, lcount * 4);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return sr_fail(SR_ENOMEM, "staging allocation for a parameter failed");
  }
  e = cudaMemcpy(tmp, local.data(), lcount * 4, cudaMemcpyHostToDevice);
  if (e == cudaSuccess && p.format == kQ4)
    e = cudaMemset(p.values, 0, (size_t)param_value_bytes(p.rows, p.cols, p.format));
  if (e == cudaSuccess) {
    int64_t work = (int64_t)p.rows * ((p.cols + kQBlock - 1) / kQBlock);
    int blocks = (int)std::min<int64_t>((work + 255) / 256, 148 * 32);
    k_init_param<<<blocks, 256, 0, 0>>>(p, 0, 0, 0.0, 0, tmp, 0, 0, p.cols);
    e = cudaGetLastError();
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
  }
  cudaFree(tmp);
  if (e != cudaSuccess) return sr_fail(SR_EDEVICE, std::string("parameter upload: ") + cudaGetErrorString(e));
  m->weights_version++;
  return SR_OK;
}

extern "C" int sr_model_set_mode(sr_model* m, int32_t mode) {
  if (!m) return sr_fail(SR_EINVAL, "null model");
  if (mode != SR_MODE_EXACT && mode != SR_MODE_FAST) return sr_fail(SR_EINVAL, "invalid mode");
  m->mode = mode;
  return SR_OK;
}

extern "C" int sr_model_set_code_cache(sr_model* m, int32_t enabled) {
  if (!m) return sr_fail(SR_EINVAL, "null model");
  CK(cudaSetDevice(m->device));
  tc_set_cache(m, enabled != 0);
  return SR_OK;
}
extern "C" int sr_model_code_cache(sr_model* m, int32_t* cached) {
  if (!m || !cached) return sr_fail(SR_EINVAL, "null argument");
  CK(cudaSetDevice(m->device));
  tc_prepare(m);
  *cached = tc_cached(m) ? 1 : 0;
  return SR_OK;
}

// ----------------------------------------------------------------- KV pool --
extern "C" int sr_kvpool_create(sr_model* m, int64_t num_pages, sr_kvpool** out) {
  if (!m || !out) return sr_fail(SR_EINVAL, "null argument");
  *out = nullptr;
  if (num_pages < 1 || num_pages > (int64_t)INT32_MAX) return sr_fail(SR_EINVAL, "num_pages must be 1..2^31-1");
  CK(cudaSetDevice(m->device));
  sr_kvpool* p = new sr_kvpool();
  p->m = m;
  p->num_pages = num_pages;
  size_t bytes = (size_t)num_pages * (size_t)m->dm.page_elems * 4;
  cudaError_t e = cudaMalloc((void**)&p->data, bytes);
  if (e != cudaSuccess) {
    cudaGetLastError();
    delete p;
    return sr_fail(SR_ENOMEM, "KV pool allocation of " + std::to_string(bytes) + " bytes failed");
  }
  e = cudaMemset(p->data, 0, bytes);
  if (e != cudaSuccess) {
    cudaFree(p->data);
    delete p;
    return sr_fail(SR_EDEVICE, std::string("cudaMemset: ") + cudaGetErrorString(e));
  }
  *out = p;
  return SR_OK;
}
extern "C" int sr_kvpool_destroy(sr_kvpool* p) {
  if (!p) return sr_fail(SR_EINVAL, "null pool");
  cudaSetDevice(p->m->device);
  cudaFree(p->data);
  delete p;
  return SR_OK;
}
extern "C" int sr_kvpool_read_row(const sr_kvpool* p, int64_t page, int32_t layer, int32_t slot, float* k_out,
                                  float* v_out) {
  if (!p || !k_out || !v_out) return sr_fail(SR_EINVAL, "null argument");
  const ModelDims& dm = p->m->dm;
  if (page < 0 || page >= p->num_pages || layer < 0 || layer >= dm.layers || slot < 0 || slot >= dm.page_tokens)
    return sr_fail(SR_EINVAL, "page, layer or slot out of range");
  CK(cudaSetDevice(p->m->device));
  const float* base = p->data + page * dm.page_elems + (int64_t)layer * 2 * dm.page_tokens * dm.kvd +
                      (int64_t)slot * dm.kvd;
  CK(cudaMemcpy(k_out, base, (size_t)dm.kvd * 4, cudaMemcpyDeviceToHost));
  CK(cudaMemcpy(v_out, base + (int64_t)dm.page_tokens * dm.kvd, (size_t)dm.kvd * 4, cudaMemcpyDeviceToHost));
  return SR_OK;
}
// copyKVPrefixRows (M:5907-5914): the first `rows` slots of every layer's K and
// V planes.  grid (2*layers planes, chunks); float4 when the plane stride and
// the copied length allow it.
__global__ void k_copy_rows(float* __restrict__ dst, const float* __restrict__ src, int64_t plane_elems,
                            int64_t copy_elems) {
  const int64_t base = (int64_t)blockIdx.x * plane_elems;
  const int64_t step = (int64_t)gridDim.y * blockDim.x;
  if ((plane_elems & 3) == 0 && (copy_elems & 3) == 0) {
    const float4* s = (const float4*)(src + base);
    float4* d = (float4*)(dst + base);
    for (int64_t i = blockIdx.y * (int64_t)blockDim.x + threadIdx.x; i < copy_elems / 4; i += step) d[i] = s[i];
  } else {
    for (int64_t i = blockIdx.y * (int64_t)blockDim.x + threadIdx.x; i < copy_elems; i += step)
      dst[base + i] = src[base + i];
  }
}
extern "C" int sr_kvpool_copy_rows(sr_kvpool* p, int64_t dst_page, int64_t src_page, int32_t rows) {
  if (!p) return sr_fail(SR_EINVAL, "null pool");
  const ModelDims& dm = p->m->dm;
  if (dst_page < 0 || dst_page >= p->num_pages || src_page < 0 || src_page >= p->num_pages)
    return sr_fail(SR_EINVAL, "page id out of range");
  if (rows < 0 || rows > dm.page_tokens) return sr_fail(SR_EINVAL, "rows must be 0..page_tokens");
  if (rows == 0 || dst_page == src_page) return SR_OK;
  CK(cudaSetDevice(p->m->device));
  const int64_t plane = (int64_t)dm.page_tokens * dm.kvd, copy = (int64_t)rows * dm.kvd;
  const int chunks = (int)std::min<int64_t>(32, (copy / 4 + 1023) / 1024 + 1);
  k_copy_rows<<<dim3(2 * dm.layers, chunks), 256, 0, p->m->stream>>>(p->data + dst_page * dm.page_elems,
                                                                       p->data + src_page * dm.page_elems, plane,
                                                                       copy);
  CK(cudaGetLastError());
  return SR_OK;
}
__global__ void k_fill_pool(float* data, int64_t count, uint64_t seed, float scale) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < count; i += (int64_t)gridDim.x * blockDim.x) {
    uint64_t z = seed + (uint64_t)(i + 1) * 0x9e3779b97f4a7c15ULL;
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ULL;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebULL;
    z ^= z >> 31;
    data[i] = scale * ((float)(z >> 40) * (1.0f / 16777216.0f) * 2.0f - 1.0f);
  }
}
extern "C" int sr_kvpool_fill_synthetic(sr_kvpool* p, uint64_t seed, float scale) {
  if (!p) return sr_fail(SR_EINVAL, "null pool");
  CK(cudaSetDevice(p->m->device));
  int64_t count = p->num_pages * p->m->dm.page_elems;
  k_fill_pool<<<148 * 16, 256, 0, p->m->stream>>>(p->data, count, seed, scale);
  CK(cudaGetLastError());
  CK(cudaStreamSynchronize(p->m->stream));
  return SR_OK;
}

// --------------------------------------------------------------------- step --
// Host validation mirroring prefillSelected (M:6246-6339): completes before any
// device state changes.
int sr_validate_batch(const sr_model* m, const sr_kvpool* pool, const sr_batch* b, BatchInfo* info) {
  if (!b) return sr_fail(SR_EINVAL, "null batch");
  const sr_model_desc& c = m->d;
  const int S = b->n_sessions;
  if (S < 1 || S > kMaxSessions) return sr_fail(SR_EINVAL, "invalid prefill batch (1..256 sessions)");
  if (!b->pos || !b->token_offsets || !b->tokens || !b->page_offsets || !b->page_ids)
    return sr_fail(SR_EINVAL, "null batch array");
  if (b->token_offsets[0] != 0 || b->page_offsets[0] != 0) return sr_fail(SR_EINVAL, "offsets must start at 0");
  const int pt = c.page_tokens;
  int64_t n = 0, max_end = 0, heads = 0, items = 0, single = 0, groups = 0;
  int64_t pre[kMaxSessions + 1][4];  // rows, items, single, groups before session i
  for (int i = 0; i < S; i++) {
    pre[i][0] = n, pre[i][1] = items, pre[i][2] = single, pre[i][3] = groups;
    int64_t len = (int64_t)b->token_offsets[i + 1] - b->token_offsets[i];
    if (len < 1 || len > kMaxRows - n)
      return sr_fail(SR_EINVAL, "prefill requires nonempty chunks totaling at most 1024 tokens");
    int64_t pos = b->pos[i];
    if (pos < 0 || pos > c.context || len > c.context - pos)
      return sr_fail(SR_EINVAL, "KV cache context exhausted or invalid position");
    for (int64_t j = b->token_offsets[i]; j < b->token_offsets[i + 1]; j++)
      if (b->tokens[j] < 0 || b->tokens[j] >= c.vocab) return sr_fail(SR_EINVAL, "token outside vocabulary");
    int64_t np = (int64_t)b->page_offsets[i + 1] - b->page_offsets[i];
    int64_t need = (pos + len + pt - 1) / pt;
    if (np < need || np > m->max_pages_per_session) return sr_fail(SR_EINVAL, "invalid KV page coverage");
    for (int64_t j = b->page_offsets[i]; j < b->page_offsets[i + 1]; j++)
      if (b->page_ids[j] < 0 || b->page_ids[j] >= pool->num_pages) return sr_fail(SR_EINVAL, "invalid KV page id");
    for (int64_t L = pos + 1; L <= pos + len; L++) items += (L + kAttnSplit - 1) / kAttnSplit;
    if (len == 1)
      single += (pos + 1 + kAttnSplit - 1) / kAttnSplit;
    else
      for (int64_t k = 0; k < len; k += 4) groups += (pos + k + std::min<int64_t>(4, len - k) + kAttnSplit - 1) / kAttnSplit;
    n += len;
    max_end = std::max(max_end, pos + len);
    heads += (!b->want_logits || b->want_logits[i]) ? 1 : 0;
  }
  // A page this step writes must belong to exactly one session (the reference
  // rejects duplicate caches, M:6264-6266; shared prefix pages are read-only).
  // pool->owner is indexed by page id (ids were range-checked above).
  {
    std::vector<int32_t>& owner = const_cast<sr_kvpool*>(pool)->owner;
    if ((int64_t)owner.size() != pool->num_pages) owner.assign((size_t)pool->num_pages, -2);
    const int64_t np_all = b->page_offsets[S];
    for (int i = 0; i < S; i++)
      for (int64_t j = b->page_offsets[i]; j < b->page_offsets[i + 1]; j++) {
        int32_t& o = owner[b->page_ids[j]];
        if (o == -2) o = i;
        else if (o != i) o = -1;  // listed by several sessions
      }
    const char* err = nullptr;
    for (int i = 0; i < S && !err; i++) {
      int64_t len = (int64_t)b->token_offsets[i + 1] - b->token_offsets[i];
      int64_t first = b->pos[i] / pt, last = (b->pos[i] + len - 1) / pt;
      for (int64_t pg = first; pg <= last && !err; pg++) {
        int32_t id = b->page_ids[b->page_offsets[i] + pg];
        if (owner[id] != i) err = "a written KV page is shared with another session";
        for (int64_t q = b->page_offsets[i]; q < b->page_offsets[i] + pg && !err; q++)
          if (b->page_ids[q] == id) err = "duplicate page in one session's page table";
      }
    }
    for (int64_t j = 0; j < np_all; j++) owner[b->page_ids[j]] = -2;  // leave the scratch clear
    if (err) return sr_fail(SR_EINVAL, err);
  }
  // resizeInferenceArrays bound (M:6149-6174) with maxActivationElements (M:50),
  // counting one attention lane.
  {
    const int64_t d = c.dim, kd = m->dm.kvd, hid = c.hidden;
    int64_t stride = std::min<int64_t>(c.context, ((max_end + 31) / 32) * 32);
    int64_t required = n * (5 * d + 2 * kd + 3 * hid) + 2 * (int64_t)S * c.vocab + stride;
    if (required > 128LL * 1024 * 1024)
      return sr_fail(SR_EINVAL, "inference workspace budget exceeded; reduce prefill tokens or batch size");
  }
  info->sessions = S;
  info->rows = (int)n;
  info->max_len = (int)max_end;
  info->heads = (int)heads;
  info->pages = b->page_offsets[S];
  info->attn_items = (int)items;
  info->attn_single = (int)single;
  info->attn_groups = (int)groups;
  // Split point for a step run as two halves: the session boundary closest to
  // half the rows with both halves between kSplitMinRows and kLaneRows rows.
  info->split_rows = info->split_items = info->split_single = info->split_groups = 0;
  {
    int best = -1;
    int64_t best_d = 0;
    for (int i = 1; i < S; i++) {
      const int64_t a = pre[i][0], bh = n - a;
      if (a < kSplitMinRows || bh < kSplitMinRows || a > kLaneRows || bh > kLaneRows) continue;
      const int64_t dd = a > n - a ? 2 * a - n : n - 2 * a;
      if (best < 0 || dd < best_d) best = i, best_d = dd;
    }
    if (best > 0) {
      info->split_rows = (int)pre[best][0];
      info->split_items = (int)pre[best][1];
      info->split_single = (int)pre[best][2];
      info->split_groups = (int)pre[best][3];
    }
  }
  return SR_OK;
}

int sr_upload_batch(sr_model* m, const sr_batch* b, const BatchInfo& info) {
  int32_t* h = (int32_t*)m->h_stage;
  const int S = info.sessions;
  memset(h, 0, (size_t)kMetaHeader * 4);
  memcpy(h + kOffSessPos, b->pos, (size_t)S * 4);
  memcpy(h + kOffTokOff, b->token_offsets, (size_t)(S + 1) * 4);
  memcpy(h + kOffPageOff, b->page_offsets, (size_t)(S + 1) * 4);
  uint8_t* want = (uint8_t*)(h + kOffWant);
  for (int i = 0; i < S; i++) want[i] = (!b->want_logits || b->want_logits[i]) ? 1 : 0;
  memcpy(h + kOffTokens, b->tokens, (size_t)info.rows * 4);
  memcpy(h + kMetaHeader, b->page_ids, (size_t)info.pages * 4);
  m->last_want.assign(want, want + S);
  m->last_sessions = S;
  CK(cudaMemcpyAsync(m->meta_dev, h, (size_t)(kMetaHeader + info.pages) * 4, cudaMemcpyHostToDevice, m->stream));
  return SR_OK;
}

static void launch_linear_exact(sr_model* m, const float* X, int n, const Param& W, LinearOut O) {
  const int in = W.cols, out = W.rows;
  cudaStream_t s = m->stream;
  auto grid = [&](int ot, int rt) { return dim3((out + ot - 1) / ot, (n + rt - 1) / rt); };
  int choice;  // 0: (32,4)  1: (32,8)  2: (64,8)
  if (n <= 4) choice = 0;
  else if ((int64_t)((out + 63) / 64) * ((n + 7) / 8) >= 2 * 148) choice = 2;
  else choice = 1;
  if (W.format == kF32) {
    if (choice == 0) k_linear_f32_exact<32, 4><<<grid(32, 4), 128, 0, s>>>(X, n, in, out, W, O);
    else if (choice == 1) k_linear_f32_exact<32, 8><<<grid(32, 8), 128, 0, s>>>(X, n, in, out, W, O);
    else k_linear_f32_exact<64, 8><<<grid(64, 8), 256, 0, s>>>(X, n, in, out, W, O);
  } else if (W.format == kQ8) {
    if (choice == 0) k_linear_q_exact<kQ8, 32, 4><<<grid(32, 4), 128, 0, s>>>(X, n, in, out, W, O);
    else if (choice == 1) k_linear_q_exact<kQ8, 32, 8><<<grid(32, 8), 128, 0, s>>>(X, n, in, out, W, O);
    else k_linear_q_exact<kQ8, 64, 8><<<grid(64, 8), 256, 0, s>>>(X, n, in, out, W, O);
  } else {
    if (choice == 0) k_linear_q_exact<kQ4, 32, 4><<<grid(32, 4), 128, 0, s>>>(X, n, in, out, W, O);
    else if (choice == 1) k_linear_q_exact<kQ4, 32, 8><<<grid(32, 8), 128, 0, s>>>(X, n, in, out, W, O);
    else k_linear_q_exact<kQ4, 64, 8><<<grid(64, 8), 256, 0, s>>>(X, n, in, out, W, O);
  }
}
static bool fast_attention(sr_model* m, sr_kvpool* pool, int n, const BatchInfo& info, int layer,
                           op16* xh, op16* xl);
void sr_launch_linear(sr_model* m, const float* X, int n, const Param& W, LinearOut O, int cls = SR_PROF_LINEAR) {
  ProfScope ps(m, cls);
  if (m->mode == SR_MODE_FAST && fast_linear(m, X, n, W, O)) return;
  launch_linear_exact(m, X, n, W, O);
  sr_count_launch(m);
}

static void launch_attention_exact(sr_model* m, sr_kvpool* pool, int n, int max_len, int layer) {
  const ModelDims& dm = m->dm;
  AttnArgs a;
  a.Q = m->Q;
  a.A = m->A;
  a.pool = pool->data;
  a.meta = m->meta;
  a.dm = dm;
  a.layer = layer;
  a.scale = (float)(1.0 / std::sqrt((double)dm.hd));
  a.ls = attn_align4(max_len);
  AttnSmem with_scores(dm.group, dm.hd, 1, a.ls);
  a.smem_scores = with_scores.total * 4 <= 160 * 1024 ? 1 : 0;
  AttnSmem lay(dm.group, dm.hd, a.smem_scores, a.ls);
  int threads = std::max(128, ((dm.group * dm.hd / 4 + 31) / 32) * 32);
  k_attention_exact<<<dim3(n, dm.kv_heads), threads, (size_t)lay.total * 4, m->stream>>>(a);
  sr_count_launch(m);
}

// The exchange after o_proj and down_proj of the tensor-parallel step: every
// rank's partial T is summed in place over NCCL.  The residual add X += T is
// then folded into the next fast-mode RMSNorm (k_rmsnorm_fast with T), or done
// by k_add_inplace where no norm follows directly.
__global__ void k_add_inplace(float* __restrict__ X, const float* __restrict__ T, int64_t count) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < count; i += (int64_t)gridDim.x * blockDim.x)
    X[i] += T[i];
}
// An all-reduced sum as its consumer reads it: a plain buffer, or the LL
// protocol's gather buffer of this rank with the all-reduce's epoch.
struct TpSum {
  const float* plain = nullptr;
  const uint4* ll = nullptr;
  uint32_t epoch = 0;
  explicit operator bool() const { return plain || ll; }
};

// Sums the ranks' partials in m->T (over peer memory once sr_tp_peer_open has
// run, else NCCL), sets *sum to where the sums are and points m->T at the
// other buffer for the next row-parallel projection.
static int tp_allreduce(sr_model* m, int n, TpSum* sum) {
  PeerHost* ph = (PeerHost*)m->peer;
  const int64_t count = (int64_t)n * m->dm.dim;
  float* T = m->T;
  *sum = TpSum();
  if (ph->open && ph->protocol == SR_PEER_LL) {
    const int size = m->dm.tp_size, par = ph->ll_parity;
    peer::LLArgs a;
    a.part = T;
    a.rb = (uint4* const*)(ph->tables + (size_t)(3 + par) * size);
    a.gb = (uint4* const*)(ph->tables + (size_t)(5 + par) * size);
    a.err = ph->err;
    a.count = count;
    a.chunk = ((count + size - 1) / size + 3) / 4 * 4;
    a.epoch = ++ph->epoch;
    a.rank = m->dm.tp_rank;
    a.size = size;
    const int grid = (int)std::min<int64_t>(std::max<int64_t>((a.chunk / 2 + peer::kThreads - 1) / peer::kThreads, 1),
                                            148 * 2);
    peer::k_peer_ll<<<grid, peer::kThreads, 0, m->stream>>>(a);
    sr_count_launch(m);
    ph->ran = true;
    sum->ll = (const uint4*)(ph->base + 2 * ph->buf_bytes + kPeerTail + 2 * ph->rb_bytes + (size_t)par * ph->gb_bytes);
    sum->epoch = a.epoch;
    ph->ll_parity ^= 1;
  } else if (ph->open) {
    peer::Args a;
    a.bufs = (float* const*)(ph->tables + (size_t)ph->cur * m->dm.tp_size);
    a.flags = (int* const*)(ph->tables + (size_t)2 * m->dm.tp_size);
    a.counter = ph->counter;
    a.err = ph->err;
    a.count = count;
    a.chunk = ((count + m->dm.tp_size - 1) / m->dm.tp_size + 3) / 4 * 4;
    a.epoch = ++ph->epoch;
    a.rank = m->dm.tp_rank;
    a.size = m->dm.tp_size;
    const int rb = (int)std::min<int64_t>(std::max<int64_t>((a.chunk / 4 + peer::kThreads - 1) / peer::kThreads, 1),
                                          148 * 2);
    const int gb = (int)std::min<int64_t>(std::max<int64_t>((count / 4 + peer::kThreads - 1) / peer::kThreads, 1),
                                          148 * 4);
    peer::k_peer_reduce<<<rb, peer::kThreads, 0, m->stream>>>(a);
    peer::k_peer_gather<<<gb, peer::kThreads, 0, m->stream>>>(a);
    sr_count_launch(m, 2);
    ph->ran = true;
    sum->plain = T;
  } else {
    nccl::Api& api = nccl::api();
    const int r = api.AllReduce(T, T, (size_t)count, nccl::kFloat32, nccl::kSum, (nccl::Comm)m->nccl_comm, m->stream);
    if (r != nccl::kSuccess) return sr_fail(SR_EDEVICE, std::string("ncclAllReduce: ") + api.GetErrorString(r));
    sum->plain = T;
  }
  ph->cur ^= 1;
  m->T = ph->buf[ph->cur];
  return SR_OK;
}
static void tp_add(sr_model* m, int n, const TpSum& t) {
  const int64_t count = (int64_t)n * m->dm.dim;
  if (t.ll)
    peer::k_add_ll<<<(int)std::min<int64_t>((count / 2 + 255) / 256, 148 * 8), 256, 0, m->stream>>>(
        m->X, t.ll, t.epoch, ((PeerHost*)m->peer)->err, count);
  else
    k_add_inplace<<<(int)std::min<int64_t>((count + 255) / 256, 148 * 8), 256, 0, m->stream>>>(m->X, t.plain, count);
  sr_count_launch(m);
}

// The GPT-2 profile's step (prefillSelected's GPT-2 branches, M:6369-6371,
// 6389, 6403-6408), exact order on every kernel: embedding + position row,
// then per layer LayerNorm, Q/K/V with bias, K/V write without RoPE,
// attention, O with bias + residual, LayerNorm, c_fc with bias, GELU-tanh,
// c_proj with bias + residual; the selected head is LayerNorm + tied wte.
// The GPT-2 profile in SR_MODE_FAST: the same steps as gpt2_step_enqueue
// with the fast kernels -- LayerNorm and GELU in fp32 with fp64 statistics
// (k_layernorm_fast, k_gelu_fast) writing the next projection's bf16 hi/lo
// operand planes, the projections with their biases (and residuals) on the
// tensor cores from 3 rows (the decode GEMV or, for f32 weights, the exact
// kernels below that), split-K attention where the head dimension is 64 or
// 128.  Matches the exact step within the fast-mode tolerance.
static int gpt2_fast_step_enqueue(sr_model* m, sr_kvpool* pool, const BatchInfo& info,
                                  const volatile int32_t* cancel) {
  const ModelDims& dm = m->dm;
  const int n = info.rows, d = dm.dim, L = dm.layers;
  const double eps = m->d.norm_eps;
  cudaStream_t s = m->stream;
  auto fv = [&](int i) { return (const float*)m->params[i].values; };
  sr_prof_span_begin(m);
  SR_LAUNCH(m, SR_PROF_META, k_meta<<<1, 1024, 0, s>>>(m->meta, info.sessions, n));
  SR_LAUNCH(m, SR_PROF_EMBED, k_embed<<<n, 256, 0, s>>>(m->params[0], m->meta.tokens, m->X, d);
            k_add_position<<<n, 256, 0, s>>>(m->X, fv(1), m->meta, d));
  sr_count_launch(m, 3);
  const bool tc = tc_active(m, n);
  op16* xh = tc ? tc_xh(m) : nullptr;
  op16* xl = tc ? tc_xl(m) : nullptr;
  const int64_t hcnt = (int64_t)n * dm.hidden;
  const int gelu_blocks = (int)std::min<int64_t>((hcnt + 255) / 256, 148 * 16);
  const char* tc_fail = "tensor-core projection could not run (scratch allocation failed)";
  for (int l = 0; l < L; l++) {
    if (cancel && *cancel) {
      sr_prof_span_end(m);
      cudaStreamSynchronize(s);
      sr_prof_resolve(m);
      return sr_fail(SR_ECANCELED, "step canceled between layers");
    }
    const int b = 4 + 16 * l;
    const Param* P = &m->params[b];
    LinearOut o;
    o.resid = nullptr;
    o.out_map = nullptr;
    SR_LAUNCH(m, SR_PROF_NORM,
              k_layernorm_fast<<<n, 128, 0, s>>>(m->X, nullptr, fv(b), fv(b + 1), m->N, n, d, eps, xh, xl));
    bool done;
    SR_LAUNCH(m, SR_PROF_LINEAR, done = tc && tc_qkv_bias(m, l, n, true, nullptr, fv(b + 5), fv(b + 6), fv(b + 7)));
    if (tc && !done) return sr_fail(SR_ENOMEM, tc_fail);
    if (!done) {
      float* qkv[3] = {m->Q, m->K, m->V};
      for (int k = 0; k < 3; k++) {
        o.y = qkv[k];
        o.ldy = d;
        o.bias = fv(b + 5 + k);
        sr_launch_linear(m, m->N, n, P[2 + k], o);
      }
    }
    SR_LAUNCH(m, SR_PROF_ROPE_KV, k_kv_write_exact<<<n, 128, 0, s>>>(m->K, m->V, m->meta, pool->data, dm, l));
    sr_count_launch(m, 3);  // norm, kv write, second norm
    bool a_split = false;   // the attention wrote the O projection's operand planes
    SR_LAUNCH(m, SR_PROF_ATTENTION, a_split = fast_attention(m, pool, n, info, l, xh, xl));
    SR_LAUNCH(m, SR_PROF_LINEAR, done = tc && tc_o(m, l, n, a_split, m->X, m->X, nullptr, fv(b + 9)));
    if (tc && !done) return sr_fail(SR_ENOMEM, tc_fail);
    if (!done) {
      o.y = m->X;  // X += O(a) + bias (M:6398-6400)
      o.ldy = d;
      o.bias = fv(b + 9);
      o.resid = m->X;
      sr_launch_linear(m, m->A, n, P[8], o);
    }
    SR_LAUNCH(m, SR_PROF_NORM,
              k_layernorm_fast<<<n, 128, 0, s>>>(m->X, nullptr, fv(b + 10), fv(b + 11), m->N, n, d, eps, xh, xl));
    SR_LAUNCH(m, SR_PROF_LINEAR, done = tc && tc_fc(m, l, n, fv(b + 13)));
    if (tc && !done) return sr_fail(SR_ENOMEM, tc_fail);
    if (!done) {
      o.y = m->G;
      o.ldy = dm.hidden;
      o.bias = fv(b + 13);
      o.resid = nullptr;
      sr_launch_linear(m, m->N, n, P[12], o);
    }
    SR_LAUNCH(m, SR_PROF_SWIGLU, k_gelu_fast<<<gelu_blocks, 256, 0, s>>>(m->G, m->H, xh, xl, hcnt));
    sr_count_launch(m);
    SR_LAUNCH(m, SR_PROF_LINEAR, done = tc && tc_down(m, l, n, true, m->X, m->X, nullptr, fv(b + 15)));
    if (tc && !done) return sr_fail(SR_ENOMEM, tc_fail);
    if (!done) {
      o.y = m->X;  // X += c_proj(h) + bias (M:6415-6417)
      o.ldy = d;
      o.bias = fv(b + 15);
      o.resid = m->X;
      sr_launch_linear(m, m->H, n, P[14], o);
    }
  }
  CK(cudaMemsetAsync(m->logits, 0, (size_t)info.sessions * dm.vocab * 4, s));
  if (info.heads > 0) {
    const bool tc_h = tc_active(m, info.heads);
    SR_LAUNCH(m, SR_PROF_HEAD,
              k_layernorm_fast<<<info.heads, 128, 0, s>>>(m->X, m->meta.head_src, fv(2), fv(3), m->N, info.heads, d,
                                                          eps, tc_h ? tc_xh(m) : nullptr, tc_h ? tc_xl(m) : nullptr));
    sr_count_launch(m);
    LinearOut o;
    o.y = m->logits;
    o.ldy = dm.vocab;
    o.bias = nullptr;
    o.resid = nullptr;
    o.out_map = m->meta.head_dst;
    bool done;
    SR_LAUNCH(m, SR_PROF_HEAD, done = tc_h && tc_head(m, info.heads, true));
    if (tc_h && !done) return sr_fail(SR_ENOMEM, "tensor-core LM head could not run (scratch allocation failed)");
    if (!done) sr_launch_linear(m, m->N, info.heads, m->params[0], o, SR_PROF_HEAD);
  }
  CK(cudaGetLastError());
  return SR_OK;
}

static int gpt2_step_enqueue(sr_model* m, sr_kvpool* pool, const BatchInfo& info, const volatile int32_t* cancel) {
  const ModelDims& dm = m->dm;
  if (m->mode == SR_MODE_FAST) return gpt2_fast_step_enqueue(m, pool, info, cancel);
  const int n = info.rows, d = dm.dim, L = dm.layers;
  const double eps = m->d.norm_eps;
  cudaStream_t s = m->stream;
  auto fv = [&](int i) { return (const float*)m->params[i].values; };
  sr_prof_span_begin(m);
  SR_LAUNCH(m, SR_PROF_META, k_meta<<<1, 1024, 0, s>>>(m->meta, info.sessions, n));
  SR_LAUNCH(m, SR_PROF_EMBED, k_embed<<<n, 256, 0, s>>>(m->params[0], m->meta.tokens, m->X, d);
            k_add_position<<<n, 256, 0, s>>>(m->X, fv(1), m->meta, d));
  sr_count_launch(m, 3);
  const int norm_blocks = (n + kNormWarps - 1) / kNormWarps;
  for (int l = 0; l < L; l++) {
    if (cancel && *cancel) {
      sr_prof_span_end(m);
      cudaStreamSynchronize(s);
      sr_prof_resolve(m);
      return sr_fail(SR_ECANCELED, "step canceled between layers");
    }
    const int b = 4 + 16 * l;
    const Param* P = &m->params[b];
    SR_LAUNCH(m, SR_PROF_NORM,
              k_layernorm_exact<<<norm_blocks, kNormWarps * 32, 0, s>>>(m->X, nullptr, fv(b), fv(b + 1), m->N, n, d,
                                                                          eps));
    LinearOut o;
    o.resid = nullptr;
    o.out_map = nullptr;
    float* qkv[3] = {m->Q, m->K, m->V};
    for (int k = 0; k < 3; k++) {
      o.y = qkv[k];
      o.ldy = d;
      o.bias = fv(b + 5 + k);  // addBias after the projection (M:6384-6386)
      SR_LAUNCH(m, SR_PROF_LINEAR, launch_linear_exact(m, m->N, n, P[2 + k], o));
    }
    SR_LAUNCH(m, SR_PROF_ROPE_KV,
              k_kv_write_exact<<<n, 128, 0, s>>>(m->K, m->V, m->meta, pool->data, dm, l));
    sr_count_launch(m, 5);  // norm, q, k, v, kv write
    SR_LAUNCH(m, SR_PROF_ATTENTION, launch_attention_exact(m, pool, n, info.max_len, l));
    o.y = m->X;  // Tmp = O(a) + bias; X += Tmp (M:6398-6400)
    o.ldy = d;
    o.bias = fv(b + 9);
    o.resid = m->X;
    SR_LAUNCH(m, SR_PROF_LINEAR, launch_linear_exact(m, m->A, n, P[8], o));
    SR_LAUNCH(m, SR_PROF_NORM,
              k_layernorm_exact<<<norm_blocks, kNormWarps * 32, 0, s>>>(m->X, nullptr, fv(b + 10), fv(b + 11), m->N, n,
                                                                          d, eps));
    o.y = m->G;
    o.ldy = dm.hidden;
    o.bias = fv(b + 13);
    o.resid = nullptr;
    SR_LAUNCH(m, SR_PROF_LINEAR, launch_linear_exact(m, m->N, n, P[12], o));
    const int64_t cnt = (int64_t)n * dm.hidden;
    SR_LAUNCH(m, SR_PROF_SWIGLU,
              k_gelu_exact<<<(int)std::min<int64_t>((cnt + 255) / 256, 148 * 16), 256, 0, s>>>(m->G, m->H, cnt));
    o.y = m->X;  // X += c_proj(h) + bias (M:6415-6417)
    o.ldy = d;
    o.bias = fv(b + 15);
    o.resid = m->X;
    SR_LAUNCH(m, SR_PROF_LINEAR, launch_linear_exact(m, m->H, n, P[14], o));
    sr_count_launch(m, 5);  // o, norm, c_fc, gelu, c_proj
  }
  CK(cudaMemsetAsync(m->logits, 0, (size_t)info.sessions * dm.vocab * 4, s));
  if (info.heads > 0) {
    const int hb = (info.heads + kNormWarps - 1) / kNormWarps;
    SR_LAUNCH(m, SR_PROF_HEAD,
              k_layernorm_exact<<<hb, kNormWarps * 32, 0, s>>>(m->X, m->meta.head_src, fv(2), fv(3), m->N, info.heads,
                                                               d, eps));
    LinearOut o;
    o.y = m->logits;
    o.ldy = dm.vocab;
    o.bias = nullptr;
    o.resid = nullptr;
    o.out_map = m->meta.head_dst;
    SR_LAUNCH(m, SR_PROF_HEAD, launch_linear_exact(m, m->N, info.heads, m->params[0], o));
    sr_count_launch(m, 2);
  }
  CK(cudaGetLastError());
  return SR_OK;
}

// ------------------------------------------------------------- split steps --
// A fast-mode step whose rows can be cut at a session boundary into two
// halves of 64..512 rows runs as two halves on two SM partitions of the GPU
// (CUDA green contexts, 72 and 76 SMs on a B200), each with its own stream.
// Per layer a half is HBM-bound in its attention (it streams its sessions' KV
// pages) and tensor-bound in its four projections; the two halves' attentions
// alternate (events), so one half's projections run while the other half's
// attention has the HBM to itself.  The halves share the weights, the KV pool
// (disjoint pages) and the model buffers (disjoint rows); each has its own
// operand planes, stream-K scratch and attention item range.  The step's
// results per row are the same arithmetic as the unsplit fast step except the
// stream-K cut of each projection (the partition's SM count changes which
// block ranges are summed first).  Off by default (sr_model_set_split): on the
// Mistral-7B step one half's attention on 72 SMs reaches only 45% of the HBM
// bandwidth (the kernel is bound by instruction issue per SM as much as by
// HBM), so two alternating half-speed attentions take as long as the whole
// step's and the split step is slower (10.55 against 7.96 ms per 8 layers).
namespace {

struct SplitState {
  bool ok = false;
  CUgreenCtx g[2] = {nullptr, nullptr};
  cudaStream_t s[2] = {nullptr, nullptr};
  int sms[2] = {0, 0};
  cudaEvent_t fork = nullptr, join[2] = {nullptr, nullptr}, attn[2] = {nullptr, nullptr};
  decltype(&cuStreamDestroy) stream_destroy = nullptr;
  decltype(&cuGreenCtxDestroy) ctx_destroy = nullptr;
};

template <typename F>
bool driver_fn(const char* name, F* out) {
  void* p = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPoint(name, &p, cudaEnableDefault, &q) != cudaSuccess || q != cudaDriverEntryPointSuccess ||
      !p) {
    cudaGetLastError();
    return false;
  }
  *out = (F)p;
  return true;
}

void split_free(SplitState* sp) {
  for (int i = 0; i < 2; i++) {
    if (sp->s[i] && sp->stream_destroy) sp->stream_destroy((CUstream)sp->s[i]);
    if (sp->join[i]) cudaEventDestroy(sp->join[i]);
    if (sp->attn[i]) cudaEventDestroy(sp->attn[i]);
    if (sp->g[i] && sp->ctx_destroy) sp->ctx_destroy(sp->g[i]);
  }
  if (sp->fork) cudaEventDestroy(sp->fork);
  delete sp;
}

// The partitions and streams, made on the first split step (with the model's
// device current).  Returns null when the device or driver cannot partition.
SplitState* split_state(sr_model* m) {
  if (m->split) {
    SplitState* sp = (SplitState*)m->split;
    return sp->ok ? sp : nullptr;
  }
  SplitState* sp = new SplitState();
  m->split = sp;
  m->fast_free.push_back([sp]() { split_free(sp); });
  decltype(&cuDeviceGet) device_get;
  decltype(&cuDeviceGetDevResource) get_resource;
  decltype(&cuDevSmResourceSplitByCount) split_by_count;
  decltype(&cuDevResourceGenerateDesc) generate_desc;
  decltype(&cuGreenCtxCreate) ctx_create;
  decltype(&cuGreenCtxStreamCreate) stream_create;
  if (!driver_fn("cuDeviceGet", &device_get) || !driver_fn("cuDeviceGetDevResource", &get_resource) ||
      !driver_fn("cuDevSmResourceSplitByCount", &split_by_count) ||
      !driver_fn("cuDevResourceGenerateDesc", &generate_desc) || !driver_fn("cuGreenCtxCreate", &ctx_create) ||
      !driver_fn("cuGreenCtxStreamCreate", &stream_create) || !driver_fn("cuStreamDestroy", &sp->stream_destroy) ||
      !driver_fn("cuGreenCtxDestroy", &sp->ctx_destroy))
    return nullptr;
  CUdevice dev;
  CUdevResource all, groups[2], rest;
  unsigned ng = 2;
  if (device_get(&dev, m->device) != CUDA_SUCCESS || get_resource(dev, &all, CU_DEV_RESOURCE_TYPE_SM) != CUDA_SUCCESS)
    return nullptr;
  // two equal groups in the partition granularity (8 SMs), the rest to the second
  const unsigned half = all.sm.smCount / 2 / 8 * 8;
  if (half < 16 || split_by_count(groups, &ng, &all, &rest, 0, half) != CUDA_SUCCESS || ng != 2) return nullptr;
  CUdevResource second[2] = {groups[1], rest};
  CUdevResourceDesc desc[2];
  if (generate_desc(&desc[0], &groups[0], 1) != CUDA_SUCCESS ||
      generate_desc(&desc[1], second, rest.sm.smCount ? 2 : 1) != CUDA_SUCCESS)
    return nullptr;
  sp->sms[0] = (int)groups[0].sm.smCount;
  sp->sms[1] = (int)(groups[1].sm.smCount + rest.sm.smCount);
  for (int i = 0; i < 2; i++) {
    CUstream cs = nullptr;
    if (ctx_create(&sp->g[i], desc[i], dev, CU_GREEN_CTX_DEFAULT_STREAM) != CUDA_SUCCESS ||
        stream_create(&cs, sp->g[i], CU_STREAM_NON_BLOCKING, 0) != CUDA_SUCCESS)
      return nullptr;
    sp->s[i] = (cudaStream_t)cs;
    if (cudaEventCreateWithFlags(&sp->join[i], cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&sp->attn[i], cudaEventDisableTiming) != cudaSuccess)
      return nullptr;
  }
  if (cudaEventCreateWithFlags(&sp->fork, cudaEventDisableTiming) != cudaSuccess) return nullptr;
  cudaGetLastError();
  sp->ok = true;
  return sp;
}

}  // namespace

extern "C" int sr_model_set_split(sr_model* m, int32_t enabled) {
  if (!m) return sr_fail(SR_EINVAL, "null model");
  if (enabled != 0 && enabled != 1) return sr_fail(SR_EINVAL, "enabled must be 0 or 1");
  m->split_mode = enabled;
  return SR_OK;
}

// The layers of a split step (fast mode, tensor-core projections, one GPU).
// Returns SR_EUNSUPPORTED before enqueueing anything when the step cannot be
// split (the caller then runs the whole-step layers).
static int split_layers(sr_model* m, sr_kvpool* pool, const BatchInfo& info, const volatile int32_t* cancel) {
  const ModelDims& dm = m->dm;
  if (!m->split_mode || info.split_rows == 0 || dm.tp_size > 1 || !fast_attention_supported(dm))
    return SR_EUNSUPPORTED;
  SplitState* sp = split_state(m);
  if (!sp || !fa_reserve(m, info.attn_items)) return SR_EUNSUPPORTED;
  const int n = info.rows, d = dm.dim, L = dm.layers;
  const double eps = m->d.norm_eps;
  struct Half {
    int r0, rows;
    FaWork work, base;
    TcLane lane;
    FaLane fa;
    op16 *xh, *xl;
  } h[2];
  const FaWork a_work{info.split_items, info.split_single, info.split_groups};
  for (int i = 0; i < 2; i++) {
    Half& x = h[i];
    x.r0 = i == 0 ? 0 : info.split_rows;
    x.rows = i == 0 ? info.split_rows : n - info.split_rows;
    x.base = i == 0 ? FaWork{0, 0, 0} : a_work;
    x.work = i == 0 ? a_work
                    : FaWork{info.attn_items - a_work.items, info.attn_single - a_work.single,
                             info.attn_groups - a_work.groups};
    x.lane = TcLane{sp->s[i], i, sp->sms[i], x.r0};
    x.fa = FaLane{sp->s[i], x.r0, x.base};
    tc_planes(m, i, &x.xh, &x.xl);
  }
  CK(cudaEventRecord(sp->fork, m->stream));
  for (int i = 0; i < 2; i++) CK(cudaStreamWaitEvent(sp->s[i], sp->fork, 0));
  auto join = [&]() {
    for (int i = 0; i < 2; i++) {
      cudaEventRecord(sp->join[i], sp->s[i]);
      cudaStreamWaitEvent(m->stream, sp->join[i], 0);
    }
  };
  for (int l = 0; l < L; l++) {
    if (cancel && *cancel) {
      join();
      sr_prof_span_end(m);
      cudaStreamSynchronize(m->stream);
      sr_prof_resolve(m);
      return sr_fail(SR_ECANCELED, "step canceled between layers");
    }
    const Param* P = &m->params[1 + 9 * l];
    for (int i = 0; i < 2; i++) {
      const Half& x = h[i];
      cudaStream_t s = sp->s[i];
      float* X = m->X + (int64_t)x.r0 * d;
      float* N = m->N + (int64_t)x.r0 * d;
      bool ok = true;
      SR_LAUNCH_ON(m, SR_PROF_NORM, s,
                   fast_rmsnorm(m, X, nullptr, (const float*)P[0].values, N, x.rows, d, eps, x.xh, x.xl, nullptr,
                                nullptr, 0, nullptr, s));
      SR_LAUNCH_ON(m, SR_PROF_LINEAR, s, ok = tc_qkv(m, l, x.rows, true, &x.lane));
      SR_LAUNCH_ON(m, SR_PROF_ROPE_KV, s,
                   k_rope_kv_exact<<<x.rows, 128, 0, s>>>(m->Q, m->K, m->V, m->cos_t, m->sin_t, m->meta, pool->data,
                                                          dm, l, x.r0));
      sr_count_launch(m, 3);  // two norms and RoPE/KV of this half-layer
      // the halves' attentions alternate: half 1 after half 0's of this layer,
      // half 0 after half 1's of the previous layer
      if (i == 1) CK(cudaStreamWaitEvent(s, sp->attn[0], 0));
      else if (l > 0) CK(cudaStreamWaitEvent(s, sp->attn[1], 0));
      SR_LAUNCH_ON(m, SR_PROF_ATTENTION, s,
                   ok = ok && fast_attention_try(m, pool->data, x.rows, x.work, l, x.xh, x.xl, &x.fa));
      CK(cudaEventRecord(sp->attn[i], s));
      SR_LAUNCH_ON(m, SR_PROF_LINEAR, s, ok = ok && tc_o(m, l, x.rows, true, X, X, &x.lane));
      SR_LAUNCH_ON(m, SR_PROF_NORM, s,
                   fast_rmsnorm(m, X, nullptr, (const float*)P[5].values, N, x.rows, d, eps, x.xh, x.xl, nullptr,
                                nullptr, 0, nullptr, s));
      SR_LAUNCH_ON(m, SR_PROF_LINEAR, s, ok = ok && tc_gateup(m, l, x.rows, true, &x.lane));
      const int64_t cnt = (int64_t)x.rows * dm.hidden;
      const int sw_blocks = (int)std::min<int64_t>((cnt + 255) / 256, 148 * 16);
      SR_LAUNCH_ON(m, SR_PROF_SWIGLU, s,
                   k_swiglu_split<<<sw_blocks, 256, 0, s>>>(m->G + (int64_t)x.r0 * dm.hidden,
                                                            m->U + (int64_t)x.r0 * dm.hidden, x.xh, x.xl, cnt));
      sr_count_launch(m);
      SR_LAUNCH_ON(m, SR_PROF_LINEAR, s, ok = ok && tc_down(m, l, x.rows, true, X, X, &x.lane));
      if (!ok) {
        join();
        return sr_fail(SR_ENOMEM, "split step: a projection or the attention could not run (scratch allocation failed)");
      }
    }
  }
  join();
  CK(cudaGetLastError());
  return SR_OK;
}

int sr_step_enqueue(sr_model* m, sr_kvpool* pool, const BatchInfo& info, const volatile int32_t* cancel,
                    const StepScratch* scratch) {
  if (m->d.arch == SR_ARCH_GPT2) return gpt2_step_enqueue(m, pool, info, cancel);
  const ModelDims& dm = m->dm;
  const int n = info.rows, d = dm.dim, kd = dm.kvd, L = dm.layers;
  const double eps = m->d.norm_eps;
  cudaStream_t s = m->stream;
  sr_prof_span_begin(m);
  SR_LAUNCH(m, SR_PROF_META, k_meta<<<1, 1024, 0, s>>>(m->meta, info.sessions, n));
  SR_LAUNCH(m, SR_PROF_EMBED, k_embed<<<n, 256, 0, s>>>(m->params[0], m->meta.tokens, m->X, d));
  sr_count_launch(m, 2);
  const int norm_blocks = (n + kNormWarps - 1) / kNormWarps;
  const bool fixed_scratch = scratch && scratch->part_o;
  const bool fast = m->mode == SR_MODE_FAST && !fixed_scratch;
  // Tensor-core projections: every producer writes the next projection's bf16
  // hi/lo operand planes directly (no fp32 round trip, no split kernel).
  const bool tc = fast && tc_active(m, n);
  const bool tp = dm.tp_size > 1;
  int rc = SR_OK;
  op16* xh = tc ? tc_xh(m) : nullptr;
  op16* xl = tc ? tc_xl(m) : nullptr;
  TpSum pending;  // tensor parallel: an all-reduced sum still to be added to X
  int* tp_err = m->peer ? ((PeerHost*)m->peer)->err : nullptr;
  bool split = false;
  if (tc && !tp) {
    rc = split_layers(m, pool, info, cancel);
    if (rc != SR_OK && rc != SR_EUNSUPPORTED) return rc;
    split = rc == SR_OK;
    rc = SR_OK;
  }
  for (int l = 0; l < (split ? 0 : L); l++) {
    if (cancel && *cancel) {
      sr_prof_span_end(m);
      cudaStreamSynchronize(s);
      sr_prof_resolve(m);
      return sr_fail(SR_ECANCELED, "step canceled between layers");
    }
    const Param* P = &m->params[1 + 9 * l];
    const Param* B = m->d.qkv_bias ? &m->params[2 + 9 * L + 3 * l] : nullptr;
    LinearOut o;
    o.ldy = 0;
    o.resid = nullptr;
    o.out_map = nullptr;
    if (pending && !fast) tp_add(m, n, pending);
    SR_LAUNCH(m, SR_PROF_NORM,
              if (fast) fast_rmsnorm(m, m->X, nullptr, (const float*)P[0].values, m->N, n, d, eps, xh, xl,
                                     pending.plain, pending.ll, pending.epoch, tp_err);
              else k_rmsnorm_exact<<<norm_blocks, kNormWarps * 32, 0, s>>>(m->X, nullptr, (const float*)P[0].values, m->N, n, d, eps));
    pending = TpSum();
    bool done;
    SR_LAUNCH(m, SR_PROF_LINEAR, done = tc && tc_qkv(m, l, n, true));
    if (tc && !done) return sr_fail(SR_ENOMEM, "tensor-core projection could not run (scratch allocation failed)");
    if (!done && fast) {  // decode GEMV: Q|K|V in one launch
      const Param* w3[3] = {&P[1], &P[2], &P[3]};
      LinearOut o3[3] = {o, o, o};
      o3[0].y = m->Q; o3[0].ldy = dm.qd; o3[0].bias = B ? (const float*)B[0].values : nullptr;
      o3[1].y = m->K; o3[1].ldy = kd; o3[1].bias = B ? (const float*)B[1].values : nullptr;
      o3[2].y = m->V; o3[2].ldy = kd; o3[2].bias = B ? (const float*)B[2].values : nullptr;
      SR_LAUNCH(m, SR_PROF_LINEAR, done = gemv_run(m, m->N, n, w3, o3, 3));
    }
    if (!done) {
      o.y = m->Q; o.ldy = dm.qd; o.bias = B ? (const float*)B[0].values : nullptr;
      sr_launch_linear(m, m->N, n, P[1], o);
      o.y = m->K; o.ldy = kd; o.bias = B ? (const float*)B[1].values : nullptr;
      sr_launch_linear(m, m->N, n, P[2], o);
      o.y = m->V; o.ldy = kd; o.bias = B ? (const float*)B[2].values : nullptr;
      sr_launch_linear(m, m->N, n, P[3], o);
    }
    SR_LAUNCH(m, SR_PROF_ROPE_KV,
              k_rope_kv_exact<<<n, 128, 0, s>>>(m->Q, m->K, m->V, m->cos_t, m->sin_t, m->meta, pool->data, dm, l, 0));
    sr_count_launch(m, 3);  // two norms and RoPE/KV of this layer
    bool a_split = false;   // attention wrote the O projection's operand planes
    SR_LAUNCH(m, SR_PROF_ATTENTION,
              if (fixed_scratch) fast_attention_run(m, pool->data, n, FaWork{info.attn_items, info.attn_single, info.attn_groups}, l, scratch->part_o, scratch->part_ml);
              else if (fast) a_split = fast_attention(m, pool, n, info, l, xh, xl);
              else launch_attention_exact(m, pool, n, info.max_len, l));
    // O projection: X += O(a); a tensor-parallel rank writes its partial sum to
    // T, which the ranks all-reduce before the residual add.
    float* oy = tp ? m->T : m->X;
    const float* ores = tp ? nullptr : m->X;
    o.y = oy; o.ldy = d; o.bias = nullptr; o.resid = ores;
    SR_LAUNCH(m, SR_PROF_LINEAR, done = tc && tc_o(m, l, n, a_split, oy, ores));
    if (tc && !done) return sr_fail(SR_ENOMEM, "tensor-core projection could not run (scratch allocation failed)");
    if (!done) sr_launch_linear(m, m->A, n, P[4], o);
    TpSum tsum;
    if (tp) {
      if ((rc = tp_allreduce(m, n, &tsum)) != SR_OK) return rc;
      if (!fast) tp_add(m, n, tsum);
    }
    SR_LAUNCH(m, SR_PROF_NORM,
              if (fast) fast_rmsnorm(m, m->X, nullptr, (const float*)P[5].values, m->N, n, d, eps, xh, xl,
                                     tsum.plain, tsum.ll, tsum.epoch, tp_err);
              else k_rmsnorm_exact<<<norm_blocks, kNormWarps * 32, 0, s>>>(m->X, nullptr, (const float*)P[5].values, m->N, n, d, eps));
    o.resid = nullptr;
    SR_LAUNCH(m, SR_PROF_LINEAR, done = tc && tc_gateup(m, l, n, true));
    if (tc && !done) return sr_fail(SR_ENOMEM, "tensor-core projection could not run (scratch allocation failed)");
    if (!done && fast) {  // decode GEMV: gate|up in one launch
      const Param* w2[2] = {&P[6], &P[7]};
      LinearOut o2[2] = {o, o};
      o2[0].y = m->G; o2[0].ldy = dm.hidden; o2[0].bias = nullptr;
      o2[1].y = m->U; o2[1].ldy = dm.hidden; o2[1].bias = nullptr;
      SR_LAUNCH(m, SR_PROF_LINEAR, done = gemv_run(m, m->N, n, w2, o2, 2));
    }
    if (!done) {
      o.y = m->G; o.ldy = dm.hidden;
      sr_launch_linear(m, m->N, n, P[6], o);
      o.y = m->U;
      sr_launch_linear(m, m->N, n, P[7], o);
    }
    int64_t cnt = (int64_t)n * dm.hidden;
    const int sw_blocks = (int)std::min<int64_t>((cnt + 255) / 256, 148 * 16);
    SR_LAUNCH(m, SR_PROF_SWIGLU,
              if (tc) k_swiglu_split<<<sw_blocks, 256, 0, s>>>(m->G, m->U, xh, xl, cnt);
              else k_swiglu_exact<<<sw_blocks, 256, 0, s>>>(m->G, m->U, m->H, cnt));
    sr_count_launch(m);
    oy = tp ? m->T : m->X;  // the all-reduce above moved m->T to the other buffer
    o.y = oy; o.ldy = d; o.resid = ores;
    SR_LAUNCH(m, SR_PROF_LINEAR, done = tc && tc_down(m, l, n, true, oy, ores));
    if (tc && !done) return sr_fail(SR_ENOMEM, "tensor-core projection could not run (scratch allocation failed)");
    if (!done) sr_launch_linear(m, m->H, n, P[8], o);
    if (tp && (rc = tp_allreduce(m, n, &pending)) != SR_OK) return rc;
  }
  if (pending) tp_add(m, n, pending);  // the final norm below gathers the head rows: a plain add
  // Selected head (M:6420-6448): gather last rows, final norm, LM head into
  // the session's logits row; unselected rows are zero.
  CK(cudaMemsetAsync(m->logits, 0, (size_t)info.sessions * dm.vocab * 4, s));
  if (info.heads > 0) {
    const Param& F = m->params[1 + 9 * L];
    const int hb = (info.heads + kNormWarps - 1) / kNormWarps;
    const bool tc_h = fast && tc_active(m, info.heads);
    sr_count_launch(m);
    SR_LAUNCH(m, SR_PROF_HEAD,
              if (fast) fast_rmsnorm(m, m->X, m->meta.head_src, (const float*)F.values, m->N, info.heads, d, eps,
                                     tc_h ? tc_xh(m) : nullptr, tc_h ? tc_xl(m) : nullptr);
              else k_rmsnorm_exact<<<hb, kNormWarps * 32, 0, s>>>(m->X, m->meta.head_src, (const float*)F.values, m->N, info.heads, d, eps));
    const Param& head = m->d.tied ? m->params[0] : m->params.back();
    LinearOut o;
    o.y = m->logits;
    o.ldy = dm.vocab;
    o.bias = nullptr;
    o.resid = nullptr;
    o.out_map = m->meta.head_dst;
    bool done;
    SR_LAUNCH(m, SR_PROF_HEAD, done = tc_h && tc_head(m, info.heads, true));
    if (tc_h && !done) return sr_fail(SR_ENOMEM, "tensor-core LM head could not run (scratch allocation failed)");
    if (!done) sr_launch_linear(m, m->N, info.heads, head, o, SR_PROF_HEAD);
  }
  CK(cudaGetLastError());
  return SR_OK;
}

extern "C" int sr_step(sr_model* m, sr_kvpool* pool, const sr_batch* batch, float* logits_host,
                       const volatile int32_t* cancel) {
  if (!m || !pool || !batch) return sr_fail(SR_EINVAL, "null argument");
  if (pool->m != m) return sr_fail(SR_EINVAL, "KV pool belongs to another model");
  BatchInfo info;
  int rc = sr_validate_batch(m, pool, batch, &info);
  if (rc != SR_OK) return rc;
  CK(cudaSetDevice(m->device));
  if (cancel && *cancel) return sr_fail(SR_ECANCELED, "step canceled before it started");
  if ((rc = sr_upload_batch(m, batch, info)) != SR_OK) return rc;
  if ((rc = sr_step_enqueue(m, pool, info, cancel)) != SR_OK) return rc;
  sr_prof_span_end(m);
  if (logits_host)
    CK(cudaMemcpyAsync(logits_host, m->logits, (size_t)info.sessions * m->dm.vocab * 4, cudaMemcpyDeviceToHost,
                       m->stream));
  CK(cudaStreamSynchronize(m->stream));
  sr_prof_resolve(m);
  if (int rc = fast_check(m)) return rc;
  if (int rc = tp_check(m)) return rc;
  return tc_check(m);
}

// linearIntoWithExecutor (M:3942-3968) for one loaded matrix: Y = X W^T in
// the model's mode (exact: the reference's reduction order).  Host buffers;
// the device copies are allocated per call (a diagnostic path).
extern "C" int sr_linear(sr_model* m, int32_t index, int32_t rows, const float* x, float* y) {
  if (!m || !x || !y) return sr_fail(SR_EINVAL, "null argument");
  if (index < 0 || index >= (int32_t)m->params.size()) return sr_fail(SR_EINVAL, "parameter index out of range");
  const Param& W = m->params[index];
  if (W.rows < 1 || W.cols < 1 || (W.format == kF32 && W.rows == 1))
    return sr_fail(SR_EINVAL, "parameter is not a matrix");
  if (rows < 1 || rows > kMaxRows) return sr_fail(SR_EINVAL, "rows must be 1..1024");
  CK(cudaSetDevice(m->device));
  const size_t xb = (size_t)rows * W.cols * 4, yb = (size_t)rows * W.rows * 4;
  float *xd = nullptr, *yd = nullptr;
  if (cudaMalloc((void**)&xd, xb) != cudaSuccess || cudaMalloc((void**)&yd, yb) != cudaSuccess) {
    cudaGetLastError();
    if (xd) cudaFree(xd);
    return sr_fail(SR_ENOMEM, "linear buffers");
  }
  cudaError_t e = cudaMemcpyAsync(xd, x, xb, cudaMemcpyHostToDevice, m->stream);
  if (e == cudaSuccess) {
    LinearOut o;
    o.y = yd;
    o.ldy = W.rows;
    o.bias = nullptr;
    o.resid = nullptr;
    o.out_map = nullptr;
    sr_launch_linear(m, xd, rows, W, o);
    e = cudaGetLastError();
  }
  if (e == cudaSuccess) e = cudaMemcpyAsync(y, yd, yb, cudaMemcpyDeviceToHost, m->stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(m->stream);
  cudaFree(xd);
  cudaFree(yd);
  if (e != cudaSuccess) return sr_fail(SR_EDEVICE, std::string("linear: ") + cudaGetErrorString(e));
  sr_prof_resolve(m);
  return SR_OK;
}

extern "C" int sr_step_logits(sr_model* m, const float** device_logits) {
  if (!m || !device_logits) return sr_fail(SR_EINVAL, "null argument");
  *device_logits = m->logits;
  return SR_OK;
}

// ------------------------------------------------------------------ sampler --
// Grow-only device buffer owned by the model (freed with it).
static int grow_buffer(sr_model* m, void** p, size_t* have, size_t need, const char* what) {
  if (*have >= need) return SR_OK;
  if (*p) cudaFree(*p);
  *p = nullptr;
  *have = 0;
  cudaError_t e = cudaMalloc(p, need);
  if (e != cudaSuccess) {
    cudaGetLastError();
    *p = nullptr;
    return sr_fail(SR_ENOMEM, std::string(what) + ": cudaMalloc(" + std::to_string(need) + ") failed");
  }
  *have = need;
  return SR_OK;
}

int sr_sample_enqueue(sr_model* m, int32_t n, const sr_sampling* settings, const int32_t* history_offsets,
                      const int32_t* history, const uint64_t* rng_state, int32_t blocked, const float* logits,
                      int32_t V, bool all) {
  if (!all && n != m->last_sessions) return sr_fail(SR_EINVAL, "session count differs from the last step");
  if (n < 1 || n > kMaxSessions) return sr_fail(SR_EINVAL, "sampling needs 1..256 sessions");
  if (!settings || !history_offsets || !rng_state) return sr_fail(SR_EINVAL, "null argument");
  if (history_offsets[0] != 0) return sr_fail(SR_EINVAL, "history offsets must start at 0");
  const int64_t nh = history_offsets[n];
  if (nh < 0 || nh > kSampleHistCap) return sr_fail(SR_EINVAL, "history exceeds the device staging capacity");
  if (nh > 0 && !history) return sr_fail(SR_EINVAL, "null history");
  int32_t* list = (int32_t*)((uint8_t*)m->h_stage + m->upload_ints * 4 + kSampOffList);
  int n_full = 0;
  for (int i = 0; i < n; i++) {
    if (history_offsets[i + 1] < history_offsets[i]) return sr_fail(SR_EINVAL, "history offsets must be nondecreasing");
    if (!all && !m->last_want[i]) continue;
    const sr_sampling& s = settings[i];
    if (!std::isfinite(s.temperature) || s.temperature < 0 || s.temperature > 100 || !std::isfinite(s.top_p) ||
        s.top_p <= 0 || s.top_p > 1 || !std::isfinite(s.repeat_penalty) || s.repeat_penalty < 1 ||
        s.repeat_penalty > 100 || s.top_k < 0)
      return sr_fail(SR_EINVAL, "invalid sampling settings");  // Sampling.Validate (M:7264-7269)
    if (s.temperature != 0 && (s.top_k == 0 || s.top_k > kMaxTopK)) list[n_full++] = i;
  }
  if (n_full) {
    const size_t need = (size_t)std::min(n_full, kSampleWave) * (size_t)sample_full_stride(V);
    int rc = grow_buffer(m, (void**)&m->samp_full, &m->samp_full_bytes, need, "full-vocabulary sampler scratch");
    if (rc != SR_OK) return rc;
  }
  // Staging: settings | hist_off | hist | rng | ids | status | list
  uint8_t* h = (uint8_t*)m->h_stage + m->upload_ints * 4;
  SampleSetting* hs = (SampleSetting*)h;
  for (int i = 0; i < n; i++) {
    hs[i].temperature = settings[i].temperature;
    hs[i].top_p = settings[i].top_p;
    hs[i].penalty = settings[i].repeat_penalty;
    hs[i].top_k = settings[i].top_k;
    hs[i].pad = 0;
  }
  const size_t off_hoff = kSampOffHistOff, off_hist = kSampOffHist, off_rng = kSampOffRng, off_ids = kSampOffIds,
               off_status = kSampOffStatus;
  memcpy(h + off_hoff, history_offsets, (size_t)(n + 1) * 4);
  if (nh) memcpy(h + off_hist, history, (size_t)nh * 4);
  memcpy(h + off_rng, rng_state, (size_t)n * 8);
  uint8_t* dv = (uint8_t*)m->samp_dev;
  CK(cudaMemcpyAsync(dv, h, (size_t)n * sizeof(SampleSetting), cudaMemcpyHostToDevice, m->stream));
  CK(cudaMemcpyAsync(dv + off_hoff, h + off_hoff, (size_t)(n + 1) * 4, cudaMemcpyHostToDevice, m->stream));
  if (nh) CK(cudaMemcpyAsync(dv + off_hist, h + off_hist, (size_t)nh * 4, cudaMemcpyHostToDevice, m->stream));
  CK(cudaMemcpyAsync(dv + off_rng, h + off_rng, (size_t)n * 8, cudaMemcpyHostToDevice, m->stream));
  if (n_full)
    CK(cudaMemcpyAsync(dv + kSampOffList, h + kSampOffList, (size_t)n_full * 4, cudaMemcpyHostToDevice, m->stream));
  SampleArgs a;
  a.logits = logits;
  a.V = V;
  a.n = n;
  a.blocked = blocked;
  a.want = all ? nullptr : m->meta.want;
  a.settings = (const SampleSetting*)dv;
  a.hist_off = (const int32_t*)(dv + off_hoff);
  a.hist = (const int32_t*)(dv + off_hist);
  a.rng = (uint64_t*)(dv + off_rng);
  a.ids = (int32_t*)(dv + off_ids);
  a.status = (int32_t*)(dv + off_status);
  size_t smem = (size_t)((V + 31) / 32) * 4;
  SR_LAUNCH(m, SR_PROF_SAMPLE, k_sample<<<n, kSampleThreads, smem, m->stream>>>(a));
  sr_count_launch(m);
  CK(cudaGetLastError());
  if (n_full) {
    const size_t fsmem = (((size_t)(V + 31) / 32) * 4 + 15) / 16 * 16 + (size_t)kSampleFullStage * 8;
    for (int w0 = 0; w0 < n_full; w0 += kSampleWave) {
      const int wn = std::min(kSampleWave, n_full - w0);
      SR_LAUNCH(m, SR_PROF_SAMPLE,
                k_sample_full<<<wn, kSampleFullThreads, fsmem, m->stream>>>(
                    a, (const int32_t*)(dv + kSampOffList) + w0, m->samp_full));
      sr_count_launch(m);
      CK(cudaGetLastError());
    }
  }
  sr_prof_span_end(m);
  // results: rng | ids | status are contiguous -> one copy back
  CK(cudaMemcpyAsync(h + off_rng, dv + off_rng, off_status + (size_t)kMaxSessions * 4 - off_rng, cudaMemcpyDeviceToHost,
                     m->stream));
  return SR_OK;
}

int sr_sample_finish(sr_model* m, int32_t n, uint64_t* rng_state, int32_t* ids_out, bool all) {
  CK(cudaStreamSynchronize(m->stream));
  sr_prof_resolve(m);
  if (int rc = fast_check(m)) return rc;
  if (int rc = tp_check(m)) return rc;
  if (int rc = tc_check(m)) return rc;
  uint8_t* h = (uint8_t*)m->h_stage + m->upload_ints * 4;
  const size_t off_rng = kSampOffRng, off_ids = kSampOffIds, off_status = kSampOffStatus;
  const int32_t* ids = (const int32_t*)(h + off_ids);
  const int32_t* status = (const int32_t*)(h + off_status);
  memcpy(ids_out, ids, (size_t)n * 4);
  for (int i = 0; i < n; i++) {
    if (!all && !m->last_want[i]) continue;
    if (status[i] == 1) return sr_fail(SR_EINVAL, "nonfinite sampling logit (session " + std::to_string(i) + ")");
    if (status[i] == 2) return sr_fail(SR_EINVAL, "empty sampling distribution (session " + std::to_string(i) + ")");
    if (status[i] == 3) return sr_fail(SR_EUNSUPPORTED, "unsupported sampling settings (session " + std::to_string(i) + ")");
  }
  memcpy(rng_state, h + off_rng, (size_t)n * 8);
  return SR_OK;
}

extern "C" int sr_sample(sr_model* m, int32_t n_sessions, const sr_sampling* settings, const int32_t* history_offsets,
                         const int32_t* history, uint64_t* rng_state, int32_t blocked, int32_t* ids_out) {
  if (!m || !ids_out || !rng_state) return sr_fail(SR_EINVAL, "null argument");
  CK(cudaSetDevice(m->device));
  sr_prof_span_begin(m);
  int rc = sr_sample_enqueue(m, n_sessions, settings, history_offsets, history, rng_state, blocked, m->logits,
                             m->dm.vocab, false);
  if (rc != SR_OK) return rc;
  return sr_sample_finish(m, n_sessions, rng_state, ids_out, false);
}

extern "C" int sr_sample_logits(sr_model* m, int32_t n_sessions, int32_t vocab, const float* logits,
                                const sr_sampling* settings, const int32_t* history_offsets, const int32_t* history,
                                uint64_t* rng_state, int32_t blocked, int32_t* ids_out) {
  if (!m || !logits || !ids_out || !rng_state) return sr_fail(SR_EINVAL, "null argument");
  if (vocab < 1 || vocab > 262144) return sr_fail(SR_EINVAL, "empty sampling distribution or vocabulary above 262144");
  if (n_sessions < 1 || n_sessions > kMaxSessions) return sr_fail(SR_EINVAL, "sampling needs 1..256 sessions");
  CK(cudaSetDevice(m->device));
  const size_t bytes = (size_t)n_sessions * vocab * 4;
  int rc = grow_buffer(m, (void**)&m->samp_logits, &m->samp_logits_bytes, bytes, "sampling logits buffer");
  if (rc != SR_OK) return rc;
  CK(cudaMemcpyAsync(m->samp_logits, logits, bytes, cudaMemcpyHostToDevice, m->stream));
  sr_prof_span_begin(m);
  rc = sr_sample_enqueue(m, n_sessions, settings, history_offsets, history, rng_state, blocked, m->samp_logits, vocab,
                         true);
  if (rc != SR_OK) {
    sr_prof_span_end(m);
    cudaStreamSynchronize(m->stream);
    sr_prof_resolve(m);
    return rc;
  }
  return sr_sample_finish(m, n_sessions, rng_state, ids_out, true);
}

extern "C" int sr_step_sample(sr_model* m, sr_kvpool* pool, const sr_batch* batch, const sr_sampling* settings,
                              const int32_t* history_offsets, const int32_t* history, uint64_t* rng_state,
                              int32_t blocked, int32_t* ids_out) {
  if (!m || !pool || !batch || !ids_out || !rng_state) return sr_fail(SR_EINVAL, "null argument");
  if (pool->m != m) return sr_fail(SR_EINVAL, "KV pool belongs to another model");
  BatchInfo info;
  int rc = sr_validate_batch(m, pool, batch, &info);
  if (rc != SR_OK) return rc;
  CK(cudaSetDevice(m->device));
  if ((rc = sr_upload_batch(m, batch, info)) != SR_OK) return rc;
  if ((rc = sr_step_enqueue(m, pool, info, nullptr)) != SR_OK) return rc;
  if ((rc = sr_sample_enqueue(m, batch->n_sessions, settings, history_offsets, history, rng_state, blocked, m->logits,
                              m->dm.vocab, false)) != SR_OK) {
    sr_prof_span_end(m);
    cudaStreamSynchronize(m->stream);
    sr_prof_resolve(m);
    return rc;
  }
  return sr_sample_finish(m, batch->n_sessions, rng_state, ids_out, false);
}

// Fast-mode attention: split-K kernels when the shape is covered (returns true
// when they also wrote xh/xl, if given), else the exact kernel into fp32 A.
static bool fast_attention(sr_model* m, sr_kvpool* pool, int n, const BatchInfo& info, int layer,
                           op16* xh, op16* xl) {
  if (fast_attention_try(m, pool->data, n, FaWork{info.attn_items, info.attn_single, info.attn_groups}, layer, xh, xl))
    return xh != nullptr;
  launch_attention_exact(m, pool, n, info.max_len, layer);
  return false;
}

// Per-call fast projection hook: the decode GEMV for steps of a few rows
// (gemv.cuh), the tensor-core GEMM (fast_gemm.cuh) from kTcMinRows rows; the
// step calls the fused tensor-core entry points directly, and shapes neither
// covers run the exact kernels.
bool sr::fast_linear(sr_model* m, const float* X, int n, const Param& W, LinearOut O) {
  const Param* w = &W;
  return gemv_run(m, X, n, &w, &O, 1) || tc_linear(m, X, n, W, O);
}

// ---------------------------------------------------------------- profiling --
void sr_prof_span_begin(sr_model* m) {
  Profiler& p = m->prof;
  if (!p.span0) {
    cudaEventCreate(&p.span0);
    cudaEventCreate(&p.span1);
  }
  if (!p.span_open) {
    cudaEventRecord(p.span0, m->stream);
    p.span_open = true;
  }
}
void sr_prof_span_end(sr_model* m) {
  Profiler& p = m->prof;
  if (p.span_open) cudaEventRecord(p.span1, m->stream);
}
void sr_prof_resolve(sr_model* m) {
  Profiler& p = m->prof;
  for (size_t i = 0; i < p.pending.size(); i++) {
    float t = 0.f;
    if (cudaEventElapsedTime(&t, p.events[2 * i], p.events[2 * i + 1]) == cudaSuccess) p.ms[p.pending[i]] += t;
  }
  p.pending.clear();
  p.used = 0;
  if (p.span_open) {
    float t = 0.f;
    if (cudaEventElapsedTime(&t, p.span0, p.span1) == cudaSuccess) {
      p.span_ms += t;
      p.steps++;
    }
    p.span_open = false;
  }
  cudaGetLastError();
}
extern "C" int sr_profile_set(sr_model* m, uint32_t class_mask) {
  if (!m) return sr_fail(SR_EINVAL, "null model");
  m->prof.mask = class_mask & ((1u << SR_PROF_CLASSES) - 1);
  return SR_OK;
}
extern "C" int sr_profile_read(sr_model* m, double* ms, int64_t* launches, double* span_ms, int64_t* steps,
                               int64_t* total_launches, int32_t reset) {
  if (!m) return sr_fail(SR_EINVAL, "null model");
  Profiler& p = m->prof;
  for (int i = 0; i < SR_PROF_CLASSES; i++) {
    if (ms) ms[i] = p.ms[i];
    if (launches) launches[i] = p.launches[i];
  }
  if (span_ms) *span_ms = p.span_ms;
  if (steps) *steps = p.steps;
  if (total_launches) *total_launches = p.total_launches;
  if (reset) {
    for (int i = 0; i < SR_PROF_CLASSES; i++) {
      p.ms[i] = 0;
      p.launches[i] = 0;
    }
    p.span_ms = 0;
    p.steps = 0;
    p.total_launches = 0;
  }
  return SR_OK;
}
extern "C" int sr_model_stream(sr_model* m, void** stream) {
  if (!m || !stream) return sr_fail(SR_EINVAL, "null argument");
  *stream = (void*)m->stream;
  return SR_OK;
}

// --------------------------------------------------------- allocation-free step --
// sr_step_noalloc serves callers that must not allocate device memory while
// they serve: an engine that sized its KV page pool to fill nearly all of HBM
// up front (the reference plans its page budget before admitting anything),
// or an embedding runtime that owns every device allocation itself.  Its only
// scratch -- the split-K attention partials (unnormalised outputs and the
// (max, sum) pair of every row x KV head x split of kAttnSplit positions) -- lives in this
// file-scope device array, which every GPU that loads the library holds until
// the process exits.  All calls on a device share it and it keeps the last
// call's contents; nothing in it needs to start at zero, because each call
// writes every slot it later reads.  Calls that overlap on the GPU (other
// streams, other threads, other models on the same device) race on it.
constexpr size_t kNoAllocScratchBytes = 16u << 20;  // 16 MiB per device
static __device__ __align__(256) float g_noalloc_scratch[kNoAllocScratchBytes / sizeof(float)];

static std::mutex g_noalloc_mu;
static float* g_noalloc_ptr[256];  // device address of g_noalloc_scratch, per device ordinal

// The first call on each device resolves the array's device address with that
// device current (host code must not use the symbol itself as an address).
static int noalloc_scratch(int device, float** out) {
  if (device < 0 || device >= 256) return sr_fail(SR_EINVAL, "device ordinal out of range for the static scratch");
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (!g_noalloc_ptr[device]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p)
      return sr_fail(SR_EDEVICE, std::string("cudaGetSymbolAddress(static attention scratch): ") +
                                     cudaGetErrorString(e));
    g_noalloc_ptr[device] = (float*)p;
  }
  *out = g_noalloc_ptr[device];
  return SR_OK;
}

extern "C" int sr_step_noalloc(sr_model* m, sr_kvpool* pool, const sr_batch* batch, float* logits_host) {
  if (!m || !pool || !batch) return sr_fail(SR_EINVAL, "null argument");
  if (pool->m != m) return sr_fail(SR_EINVAL, "KV pool belongs to another model");
  BatchInfo info;
  int rc = sr_validate_batch(m, pool, batch, &info);
  if (rc != SR_OK) return rc;
  if (m->d.arch == SR_ARCH_GPT2) return sr_fail(SR_EUNSUPPORTED, "the allocation-free step runs the RMSNorm profiles");
  if (!fast_attention_supported(m->dm))
    return sr_fail(SR_EUNSUPPORTED, "the allocation-free step needs head_dim 64 or 128 and at most 8 query heads per KV head");
  if (m->dm.tp_size > 1)
    return sr_fail(SR_EUNSUPPORTED, "the allocation-free step runs on single-GPU models (NCCL may allocate)");
  size_t items = 0;
  const size_t floats = fa_scratch_floats(m->dm, info.attn_items, &items);
  if (floats * sizeof(float) > kNoAllocScratchBytes)
    return sr_fail(SR_EINVAL, "batch needs " + std::to_string(floats * sizeof(float)) +
                                  " bytes of attention scratch; the allocation-free step holds " +
                                  std::to_string(kNoAllocScratchBytes) +
                                  " (16 MiB): use fewer rows or shorter contexts, or sr_step");
  CK(cudaSetDevice(m->device));
  float* base = nullptr;
  if ((rc = noalloc_scratch(m->device, &base)) != SR_OK) return rc;
  StepScratch sc;
  sc.part_o = base;
  sc.part_ml = base + items * m->dm.group * m->dm.hd;
  if ((rc = sr_upload_batch(m, batch, info)) != SR_OK) return rc;
  if ((rc = sr_step_enqueue(m, pool, info, nullptr, &sc)) != SR_OK) return rc;
  sr_prof_span_end(m);
  if (logits_host)
    CK(cudaMemcpyAsync(logits_host, m->logits, (size_t)info.sessions * m->dm.vocab * 4, cudaMemcpyDeviceToHost,
                       m->stream));
  CK(cudaStreamSynchronize(m->stream));
  sr_prof_resolve(m);
  return fast_check(m);
}
