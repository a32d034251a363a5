/*
 * srstep.h -- C ABI of the B200 engine step (libsrstep.so).
 *
 * This is the drop-in boundary for the continuous-batching prefill/decode step
 * of RyoSpiralArchitect/sr_go_tranformer's Go engine.  Every entry point uses
 * plain C types (pointers, fixed-width integers, sizes) so that the reference's
 * Go engine can bind it through cgo; no C++ or torch types cross it.
 *
 * Conventions shared by every call:
 *   - Return value: SR_OK (0) or one of the SR_E* codes below.  On any error
 *     sr_last_error() returns a NUL-terminated message for the calling thread.
 *   - Validation completes before any device state is mutated: an SR_EINVAL
 *     step leaves every KV page untouched (reference contract,
 *     cmd/monolith/prefill_test.go:91).
 *   - One caller at a time per sr_model (the reference's single engine actor,
 *     cmd/monolith/monolith.go:3704-3708, 6209-6213).  Weights are read-only
 *     after loading; a model may serve several pools.
 *   - Host pointers passed in are only read during the call (they may be
 *     ordinary or pinned memory); the call returns after its device work has
 *     completed unless the entry point says otherwise.
 */
#ifndef SRSTEP_H
#define SRSTEP_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---------------------------------------------------------------- status */
enum {
    SR_OK = 0,
    SR_EINVAL = 1,    /* invalid argument or batch; nothing mutated */
    SR_ECANCELED = 2, /* cancel flag observed between layers; positions not committed */
    SR_ENOMEM = 3,    /* device allocation failed */
    SR_ETIMEOUT = 4,  /* a bounded device or collective wait expired */
    SR_EDEVICE = 5,   /* CUDA error; the message names the failing call */
    SR_EUNSUPPORTED = 6
};

/* Weight formats (cmd/monolith/monolith.go:566-582, validHFWeightFormat /
 * hfMatrixFormat): q4-mixed stores embedding and LM head as Q8, others Q4. */
enum { SR_FMT_F32 = 0, SR_FMT_Q8 = 1, SR_FMT_Q4 = 2, SR_FMT_Q4_MIXED = 3 };
/* Per-parameter storage of one tensor. */
enum { SR_PARAM_F32 = 0, SR_PARAM_Q8 = 1, SR_PARAM_Q4 = 2 };

/* Arithmetic mode of the step.
 * SR_MODE_EXACT reproduces the reference's fp32/fp64 operation order
 *   (sequential fp32 dots, 4-strided Q8/Q4 partials per 64-block, fp64 norm,
 *   softmax and SwiGLU sums) on CUDA cores, without FMA contraction.
 * SR_MODE_FAST uses fused multiply-adds, split-K attention and, for the Q8/Q4
 *   projections, a decode GEMV on CUDA cores for steps of 1 or 2 rows and
 *   tcgen05 tensor cores from 3; it matches the reference within a stated
 *   tolerance. */
enum { SR_MODE_EXACT = 0, SR_MODE_FAST = 1 };

/* Model description: Config (cmd/monolith/monolith.go:56-66) plus the HF
 * switches the step reads (hfConfig, :134-150; readHFConfig, :253-385). */
typedef struct sr_model_desc {
    int32_t vocab, dim, hidden, layers, heads, kv_heads, context;
    double rope_theta, norm_eps;
    int32_t tied;          /* 1: LM head is the token embedding (:6440-6443) */
    int32_t qkv_bias;      /* 1: qwen2 q/k/v biases (:5022-5029) */
    int32_t weight_format; /* SR_FMT_* */
    int32_t page_tokens;   /* KV positions per page; the reference uses 32 (:5846) */
    int32_t rope_scaling;  /* 1: llama3 frequency scaling (:4961-4977) */
    double rope_factor, rope_low_freq_factor, rope_high_freq_factor;
    int32_t rope_original_max_positions;
    /* SR_ARCH_GPT2: GPT-2 profile (loadGPT2 :5052-5165): absolute position
     * table of `positions` rows (>= context), affine LayerNorm (norm_eps is
     * layer_norm_epsilon), biases on every projection, GELU-tanh MLP (`hidden`
     * = n_inner), tied head, kv_heads == heads, no RoPE.  Parameters follow
     * loadGPT2's order with [out, in] matrices: wte, wpe, ln_f.weight,
     * ln_f.bias, then per layer ln_1 w/b, q, k, v, q/k/v biases, o, o bias, ln_2
     * w/b, c_fc, c_fc bias, c_proj, c_proj bias.  Exact or fast mode, one GPU. */
    int32_t arch;          /* SR_ARCH_LLAMA (0) or SR_ARCH_GPT2 (1) */
    int32_t positions;     /* GPT-2 position-table rows (n_positions) */
} sr_model_desc;
#define SR_ARCH_LLAMA 0
#define SR_ARCH_GPT2 1

typedef struct sr_param_info {
    int32_t rows, cols, format; /* SR_PARAM_* */
    int32_t reserved;
    int64_t value_bytes; /* f32: rows*cols*4; q8: rows*cols; q4: rows*ceil(cols/2) */
    int64_t scale_count; /* q8/q4: rows*ceil(cols/64); f32: 0 */
} sr_param_info;

typedef struct sr_model sr_model;
typedef struct sr_kvpool sr_kvpool;

/* Ragged step batch, structure of arrays.  Session i owns step rows
 * token_offsets[i] .. token_offsets[i+1]-1 (its chunk) starting at committed
 * position pos[i] (KVCache.Pos), and pages page_ids[page_offsets[i] ..
 * page_offsets[i+1]) in position order (KVCache.Pages).  want_logits may be
 * NULL (all sessions).  Mirrors prefillSelected's arguments (caches, chunks,
 * wantLogits), cmd/monolith/monolith.go:6245. */
typedef struct sr_batch {
    int32_t n_sessions;
    const int32_t *pos;
    const int32_t *token_offsets; /* n_sessions + 1 entries, [0] == 0 */
    const int32_t *tokens;
    const int32_t *page_offsets; /* n_sessions + 1 entries, [0] == 0 */
    const int32_t *page_ids;
    const uint8_t *want_logits;
} sr_batch;

/* Sampling settings per session: Sampling (cmd/monolith/monolith.go:7253-7260). */
typedef struct sr_sampling {
    double temperature; /* 0 = greedy */
    int32_t top_k;      /* 0 = no top-k */
    int32_t reserved;
    double top_p;
    double repeat_penalty;
} sr_sampling;

const char *sr_last_error(void);
const char *sr_version(void);

/* ---------------------------------------------------------------- model */
/* Replaces loadHFModelFormatKV's storage allocation (:4985-5050).  Allocates
 * device storage for every parameter in hfProfileSpecs order (:407-442), the
 * RoPE tables (:5034-5043) and the step workspace (decodeWorkspace,
 * :6064-6096; bounded by maxActivationElements, :50). */
int sr_model_create(const sr_model_desc *desc, int device, sr_model **out);
/* Tensor-parallel rank `tp_rank` of `tp_size` (Megatron-style sharding of the
 * reference model; the reference itself has no multi-GPU path): Q/K/V and
 * gate/up keep a contiguous block of output rows (whole heads / FFN columns),
 * o_proj and down_proj the matching block of input columns, the KV pool holds
 * only this rank's KV heads, and embedding, norms and LM head are replicated.
 * The step all-reduces (fp32 sum; NCCL, or peer memory after
 * sr_tp_peer_open) after o_proj and down_proj.  nccl_id is
 * the 128-byte id from sr_tp_unique_id on rank 0, shared with every rank;
 * creation blocks until all ranks have joined.  Heads: kv_heads divisible by
 * tp_size (each rank takes kv_heads/tp_size KV heads with all their query
 * heads), or tp_size divisible by kv_heads with r = tp_size/kv_heads <= the
 * query heads per KV head: each KV head is then replicated on r consecutive
 * ranks that split its query heads, the first (group mod r) taking one more
 * (Qwen2.5-7B, 28/4 heads, on 8 ranks: 4 and 3 query heads of one KV head).
 * Requires hidden divisible by tp_size and, for quantized weights, column
 * shards of whole 64-column blocks.  Parameters are still loaded as full
 * tensors. */
int sr_model_create_tp(const sr_model_desc *desc, int device, int32_t tp_rank, int32_t tp_size, const void *nccl_id,
                       sr_model **out);
/* 128-byte NCCL unique id for sr_model_create_tp (call on rank 0). */
int sr_tp_unique_id(void *id_out);
/* Host-only: rows [shard[0], shard[0]+shard[1]) and columns [shard[2],
 * shard[2]+shard[3]) of parameter `index` that rank `rank` of `size` holds. */
int sr_tp_shard(const sr_model_desc *desc, int32_t rank, int32_t size, int32_t index, int32_t *shard);
/* All-reduce over NVLink peer memory (no counterpart in the reference, which
 * runs on one CPU process).  By default a tensor-parallel step all-reduces the
 * o_proj / down_proj partial sums with NCCL.  After every rank has called
 * sr_tp_peer_open with all ranks' handles (rank order, SR_TP_PEER_HANDLE_BYTES
 * each, exchanged by the caller like the NCCL id), it uses two kernels of plain
 * peer loads and stores over CUDA IPC mappings instead: each rank sums one
 * chunk of the array in rank order and gathers the others, so every rank holds
 * bit-identical sums.  Barrier waits are bounded; a rank that does not join a
 * step makes the others' step return SR_ETIMEOUT.  sr_model_destroy runs a
 * last bounded barrier, so all ranks must destroy their models. */
#define SR_TP_PEER_HANDLE_BYTES 64
int sr_tp_peer_handle(sr_model *m, void *handle_out);
int sr_tp_peer_open(sr_model *m, const void *handles);
/* Protocol of the peer-memory all-reduce (after sr_tp_peer_open; every rank
 * the same):
 *   SR_PEER_BARRIER  two kernels, reduce-scatter then gather, with a flag
 *                    barrier before each (the default);
 *   SR_PEER_LL       one kernel: every 16-byte line carries two values and
 *                    the all-reduce's epoch twice, each chunk is pushed to its
 *                    owner, summed there in rank order as its lines arrive and
 *                    pushed to every rank; the next RMSNorm (or the residual
 *                    add) waits on the lines it reads.  Same sums, bit for bit,
 *                    as SR_PEER_BARRIER.  Not yet run on a GPU. */
#define SR_PEER_BARRIER 0
#define SR_PEER_LL 1
int sr_tp_peer_set_protocol(sr_model *m, int32_t protocol);
int sr_model_destroy(sr_model *m);
int sr_model_param_count(const sr_model *m, int32_t *count);
int sr_model_param_info(const sr_model *m, int32_t index, sr_param_info *out);
/* Upload one parameter in the reference's storage layout, verbatim (Param,
 * :3784-3850): f32 [rows,cols]; q8 int8 [rows,cols] + f32 scales
 * [rows,ceil(cols/64)]; q4 packed nibbles (low first) [rows,ceil(cols/2)] +
 * scales.  `values` and `scales` are host pointers. */
int sr_model_load_param(sr_model *m, int32_t index, const void *values, size_t value_bytes, const float *scales,
                        size_t scale_count);
/* Upload one parameter as fp32 [rows,cols] and store it in the parameter's
 * format, quantising on the device with the reference's streaming block
 * quantizer (readParam, :857-880; lowBitScale, :3877-3891; q8Value, :3893).
 * This is the path of loadHFModelFormatKV for f32/q8/q4/q4-mixed models. */
int sr_model_load_param_f32(sr_model *m, int32_t index, const float *values, size_t count);
/* Read one parameter back (same layout; a tensor-parallel rank returns its
 * shard, whose extent sr_tp_shard gives), for verification. */
int sr_model_read_param(const sr_model *m, int32_t index, void *values, size_t value_bytes, float *scales,
                        size_t scale_count);
/* Synthetic random init on the device (no reference counterpart beyond
 * NewModel(c, seed), :5195-5199): every matrix and bias element e, counted in
 * hfProfileSpecs order, is float32(Normal()*scale) where Normal() uses the
 * SplitMix64 outputs number 2e+1 and 2e+2 of a generator seeded with `seed`
 * (RNG.Normal, :1437-1439); norms are 1; matrices are then quantized with the
 * reference's block quantizer (readParam, :857-880). */
int sr_model_init_synthetic(sr_model *m, uint64_t seed, double scale);
/* Select SR_MODE_EXACT (default) or SR_MODE_FAST for subsequent steps. */
int sr_model_set_mode(sr_model *m, int32_t mode);
/* Fast-mode code cache (no counterpart in the reference, which reads the
 * codes as stored).  enabled = 1 (the default): the tensor-core projections
 * also keep every Q8/Q4 matrix's codes as bf16 in tile order, 2 bytes per
 * weight (about 1.9x the Q8 payload, 3.8x Q4), built on the first fast step
 * of 32+ rows; each weight tile is then one bulk copy.  enabled = 0, or when
 * the copy does not fit in device memory: the projections read the reference
 * codes as stored and widen them to bf16 in shared memory, which uses no
 * extra device memory but more shared-memory bandwidth (slower).  Results are
 * identical either way.  sr_model_code_cache reports whether the cache is in
 * use (building it if enabled). */
int sr_model_set_code_cache(sr_model *m, int32_t enabled);
int sr_model_code_cache(sr_model *m, int32_t *cached);
/* Split steps (no counterpart in the reference, which runs on CPU cores):
 * with enabled = 1, a SR_MODE_FAST step on one GPU whose rows can
 * be cut at a session boundary into two halves of 64..512 rows runs as those
 * two halves on two SM partitions of the GPU (CUDA green contexts, made on the
 * first such step), so that one half's projections run while the other half's
 * attention reads its KV pages.  Per-row results equal the unsplit fast step's
 * within the fast-mode tolerance (the projections' partial sums are grouped
 * differently).  0 (the default) runs every step whole. */
int sr_model_set_split(sr_model *m, int32_t enabled);

/* ---------------------------------------------------------------- KV pool */
/* Device page pool holding num_pages pages of 2*page_tokens*kvDim*layers fp32
 * values each; page layout [layer][K plane | V plane] (KVCache.row,
 * :6038-6043).  Page ids are chosen by the caller (the engine's LIFO pagePool,
 * :5854-5866, stays on the host). */
int sr_kvpool_create(sr_model *m, int64_t num_pages, sr_kvpool **out);
int sr_kvpool_destroy(sr_kvpool *p);
/* Copy one K and one V row (kvDim floats each) of (page, layer, slot) to host. */
int sr_kvpool_read_row(const sr_kvpool *p, int64_t page, int32_t layer, int32_t slot, float *k_out, float *v_out);
/* Copy the first `rows` token slots (0..page_tokens) of every layer's K and V
 * planes of page src_page into page dst_page: copyKVPrefixRows (:5907-5914),
 * the device half of the prefix cache's restore and capture (:5881-5952).
 * Enqueued on the model's stream, so it is ordered with the steps around it;
 * the pages may not overlap a step's writes in flight on another stream. */
int sr_kvpool_copy_rows(sr_kvpool *p, int64_t dst_page, int64_t src_page, int32_t rows);
/* Fill every page with deterministic pseudo-random values (benchmark state). */
int sr_kvpool_fill_synthetic(sr_kvpool *p, uint64_t seed, float scale);

/* ---------------------------------------------------------------- step */
/* One engine step: replaces Model.prefillSelected (:6245-6456).  Validates the
 * batch (1..256 sessions, >=1 token per chunk, <=1024 rows, tokens in
 * [0,vocab), pos+len <= context, pages covering pos+len), then runs every layer
 * and writes logits [n_sessions x vocab] fp32 (unselected rows zeroed) into the
 * model's device buffer, borrowed until the next step (:6236-6237).
 * logits_host may be NULL; when set, the logits are copied there.  cancel may
 * be NULL; when *cancel becomes nonzero between layers the step stops with
 * SR_ECANCELED (future KV rows may be written; positions are never committed
 * here: the caller commits Pos += len on SR_OK, :6452-6454). */
int sr_step(sr_model *m, sr_kvpool *pool, const sr_batch *batch, float *logits_host, const volatile int32_t *cancel);
/* Allocation-free variant of sr_step for callers that cannot allocate device
 * memory while serving (for example an engine that reserved nearly all of HBM
 * for its KV page pool up front).  No counterpart in the reference.  Same
 * arguments, validation and outputs as sr_step (without the cancel flag); the
 * projections and norms run in the exact order, attention runs as split-K
 * flash-decoding whose partial results use a 16 MiB scratch array compiled into
 * the library (resident on every GPU that loads it).  Row r of the batch
 * attends to c_r = pos + (r's index in its chunk) + 1 positions, cut into
 * splits of 512 positions; a batch whose scratch,
 *   sum over rows of ceil(c_r / 512) x kv_heads x group x (head_dim + 2)
 * floats, exceeds 16 MiB is rejected with SR_EINVAL; head_dim must be 64 or
 * 128 and at most 8 query heads may share a KV head (SR_EUNSUPPORTED
 * otherwise).  The first
 * call on each device resolves the array's address; make it before any stream
 * capture.  Calls that overlap on one device race on the shared array.  Never
 * calls cudaMalloc or cudaFree. */
int sr_step_noalloc(sr_model *m, sr_kvpool *pool, const sr_batch *batch, float *logits_host);
/* One projection of a loaded matrix parameter: y[rows x out] = x[rows x in]
 * W^T, as linearIntoWithExecutor computes it (:3942-3968) -- FP32 sequential
 * dots, Q8/Q4 4-strided partials per 64-column block (:4074-4780) in
 * SR_MODE_EXACT, the step's fast kernels in SR_MODE_FAST.  x and y are host
 * fp32 arrays, rows 1..1024.  For kernel-level parity checks and diagnostics
 * (allocates its device copies per call). */
int sr_linear(sr_model *m, int32_t index, int32_t rows, const float *x, float *y);
/* Device pointer of the last step's logits [n_sessions x vocab]. */
int sr_step_logits(sr_model *m, const float **device_logits);

/* Sample one token per session from the last step's logits on the device:
 * sampleWithBlocked (:7320-7426) with the SplitMix64 RNG (:1411-1439).
 * history: per session the prompt+output ids (history_offsets[n+1]).
 * rng_state: per session, advanced exactly as RNG.Float64 does (one draw per
 * sampled, non-greedy token).  blocked: id never sampled (-1 for HF models).
 * Every setting Sampling.Validate accepts (:7264-7269) is supported: top_k 0
 * (every candidate) and top_k above 256 sort the whole eligible vocabulary on
 * the device (scratch of 24 bytes per vocabulary entry for up to 32 sessions,
 * allocated on first use).  ids_out[i] receives the token; a nonfinite logit
 * or empty distribution returns SR_EINVAL naming the session. */
int sr_sample(sr_model *m, int32_t n_sessions, const sr_sampling *settings, const int32_t *history_offsets,
              const int32_t *history, uint64_t *rng_state, int32_t blocked, int32_t *ids_out);
/* sampleWithBlocked(logits, history, s, rng, blocked) (:7320) over logits the
 * caller passes: host fp32 [n_sessions x vocab] (vocab 1..262144), every
 * session sampled, the rest as sr_sample.  The model's last-step logits are
 * left as they were (the rows go to a separate device buffer, allocated on
 * first use). */
int sr_sample_logits(sr_model *m, int32_t n_sessions, int32_t vocab, const float *logits, const sr_sampling *settings,
                     const int32_t *history_offsets, const int32_t *history, uint64_t *rng_state, int32_t blocked,
                     int32_t *ids_out);

/* Step + sample in one call (one host round trip per engine tick). */
int sr_step_sample(sr_model *m, sr_kvpool *pool, const sr_batch *batch, const sr_sampling *settings,
                   const int32_t *history_offsets, const int32_t *history, uint64_t *rng_state, int32_t blocked,
                   int32_t *ids_out);

/* ---------------------------------------------------------------- profiling */
/* Kernel classes timed with CUDA events on the model's stream (no reference
 * counterpart; the reference traces regions with runtime/trace, :6380, :8392). */
enum {
    SR_PROF_META = 0, SR_PROF_EMBED, SR_PROF_NORM, SR_PROF_LINEAR, SR_PROF_ROPE_KV, SR_PROF_ATTENTION,
    SR_PROF_SWIGLU, SR_PROF_HEAD, SR_PROF_SAMPLE, SR_PROF_CLASSES
};
/* Time every launch of the classes in class_mask (bit i = class i); 0 = off.
 * Step spans (first to last kernel of each step) and launch counts are always
 * recorded. */
int sr_profile_set(sr_model *m, uint32_t class_mask);
/* Accumulated milliseconds and launches per class (arrays of SR_PROF_CLASSES),
 * summed step spans, step count and total kernel launches; reset clears them. */
int sr_profile_read(sr_model *m, double *ms, int64_t *launches, double *span_ms, int64_t *steps,
                    int64_t *total_launches, int32_t reset);
/* The cudaStream_t every step of this model runs on (for external events). */
int sr_model_stream(sr_model *m, void **stream);

/* ---------------------------------------------------------------- host engine */
/* C++ restatement of the reference's Engine actor loop (:7629-8476) over this
 * step: request queue, page-reserving admission (:8325-8366), scheduleTokens
 * (:8180-8210), the LIFO page pool (:5854-5866, :6023-6062), sampling and
 * finishing.  Used where no Go engine drives the step (tests, benchmarks). */
typedef struct sr_engine sr_engine;
typedef struct sr_engine_config {
    int32_t max_batch;           /* 1..256 */
    int32_t token_budget;        /* max_batch..1024 */
    int32_t prefill_chunk;       /* 1..1024 */
    int32_t mixed_prefill_chunk; /* 1..1024 */
    int64_t cache_bytes;         /* KV budget; pool Limit = cache_bytes / page bytes */
    int32_t eos_id;              /* -1: no EOS */
    int32_t blocked_id;          /* -1 for HF models */
    /* Prefix cache (EngineConfig.PrefixCacheBytes / PrefixCacheTail, :7639-7640):
     * bytes carved out of cache_bytes for the one-entry prefix snapshot (0 = off;
     * pool Limit = (cache_bytes - prefix_cache_bytes) / page bytes), and whether
     * matching tokens inside a partial page are reused too. */
    int64_t prefix_cache_bytes;
    int32_t prefix_cache_tail;
    int32_t reserved;
} sr_engine_config;
typedef struct sr_request {
    const int32_t *ids;
    int32_t n_ids;
    int32_t max_tokens;
    sr_sampling sampling;
    uint64_t seed;
} sr_request;
typedef struct sr_engine_stats {
    int64_t submitted, completed, rejected, failed, active, queued;
    int64_t input_tokens, generated_tokens, ticks, peak_tick_tokens;
    int64_t pool_limit, pool_reserved, pool_allocated;
    /* EngineStats.PrefixHits / PrefixTokens / PrefixBytes (:8231-8234, :8357-8360);
     * pool_allocated includes the prefix snapshot's pages, as Allocated does. */
    int64_t prefix_hits, prefix_tokens, prefix_bytes;
} sr_engine_stats;

int sr_engine_create(sr_model *m, const sr_engine_config *c, sr_engine **out);
int sr_engine_destroy(sr_engine *e);
/* Queue a request (enqueue, :8071-8148).  Returns SR_EINVAL if it can never fit
 * the pool ("request exceeds total KV cache budget", :8097-8100). */
int sr_engine_submit(sr_engine *e, const sr_request *r, int64_t *request_id);
/* Run one actor tick (admit, schedule, step, sample, finish).  *rows receives
 * the step's row count (0 when idle). */
int sr_engine_tick(sr_engine *e, int32_t *rows);
/* Pop one finished request: ids and count (up to cap), finish reason
 * (0 length, 1 eos, 2 error, 3 rejected/busy).  Returns SR_OK with
 * *request_id = -1 when none is finished. */
int sr_engine_poll(sr_engine *e, int64_t *request_id, int32_t *out_ids, int32_t cap, int32_t *n_out,
                   int32_t *reason);
int sr_engine_stats_get(const sr_engine *e, sr_engine_stats *s);
/* Medians (ms) of the time to first token (submit to first sampled token) and
 * of the gaps between a request's consecutive tokens, over everything this
 * engine has produced so far: firstTokenLatency / tokenGap (:8441-8447). */
int sr_engine_latency(const sr_engine *e, double *ttft_p50_ms, double *itl_p50_ms, int64_t *n_ttft,
                      int64_t *n_itl);
/* Last tick's schedule: counts[i] rows for session i (up to cap), pages owned. */
int sr_engine_last_schedule(const sr_engine *e, int32_t *counts, int32_t cap, int32_t *n_sessions);
/* Page table of active session i in admission order (up to cap ids). */
int sr_engine_session_pages(const sr_engine *e, int32_t i, int32_t *pages, int32_t cap, int32_t *n_pages);
/* Drop the prefix snapshot (the engine's clearPrefix, :8236-8241): sessions
 * admitted before the call never capture into it again.  Like the reference,
 * which takes the request only while no session is active, the clear is applied
 * at once when the engine is idle and otherwise at the start of the first tick
 * that finds it idle.  Snapshot pages stay in device memory while a session
 * borrows them (prefixSnapshot.clear, :5915-5921). */
int sr_engine_clear_prefix(sr_engine *e);

/* ---------------------------------------------------------------- text */
/* Streaming detokenization (incrementalText, :7649-7780, and the Mistral
 * PushToken, :2132-2161): feed each sampled token's piece (the tokenizer's
 * bytes for that id) and receive the text that is final so far, so that the
 * concatenated deltas equal the whole-string decode even when a piece ends
 * inside a UTF-8 sequence, a byte-fallback run or a cleanup pattern.  Host
 * only; needs no GPU.  Flags mirror newTextDecoder (:7662-7668):
 *   0                 plain decoder (strings.ToValidUTF8 across pieces);
 *   SR_TEXT_HF        HF ByteLevel lossy UTF-8 (pushHF, :7737-7780);
 *   SR_TEXT_CLEANUP   with SR_TEXT_HF: Transformers' cleanup cascade (:7672-7701);
 *   SR_TEXT_MISTRAL   byte-fallback runs decode atomically and the first text
 *                     loses one leading space; `fallback` flags the vocab's
 *                     <0xNN> ids (vocab entries). */
#define SR_TEXT_HF 1
#define SR_TEXT_CLEANUP 2
#define SR_TEXT_MISTRAL 4
typedef struct sr_text_decoder sr_text_decoder;
int sr_text_decoder_create(int32_t flags, const uint8_t *fallback, int32_t vocab, sr_text_decoder **out);
int sr_text_decoder_destroy(sr_text_decoder *d);
/* incrementalText.Push of n bytes (final: end of the stream).  Up to cap bytes of
 * text (whole characters) go to out, *n_out receives their count and *queued
 * (may be NULL) how many bytes still wait; call again with n = 0 to drain. */
int sr_text_decoder_push(sr_text_decoder *d, const uint8_t *bytes, int64_t n, int32_t final, char *out,
                         int64_t cap, int64_t *n_out, int64_t *queued);
/* PushToken (:2132-2161) for token `id` with its piece; other decoders treat it
 * as sr_text_decoder_push of the piece. */
int sr_text_decoder_push_token(sr_text_decoder *d, int32_t id, const uint8_t *piece, int64_t n, int32_t final,
                               char *out, int64_t cap, int64_t *n_out, int64_t *queued);

/* The engine's token events (TokenEvent, :7643-7647, sent at :8451-8462): with
 * the tokenizer's pieces table (bytes of every id concatenated, offsets[vocab+1])
 * and the decoder flags, every sampled token yields an event holding its id and
 * the text it completes (PushToken, final on the request's last token).  Set
 * only while no session is active; vocab 0 turns events off (the default).
 * The queue is unbounded: the reference's slow-consumer cut-off (:8460-8462)
 * is the caller's policy. */
int sr_engine_set_pieces(sr_engine *e, const uint8_t *pieces, const int64_t *offsets, int32_t vocab, int32_t flags,
                         const uint8_t *fallback);
/* Pop the oldest token event: request id (-1 when none), token id, the text
 * (*n_text bytes into text; if cap is smaller, SR_EINVAL with *n_text set and
 * the event kept), and whether it was the request's last token. */
int sr_engine_poll_token(sr_engine *e, int64_t *request_id, int32_t *token_id, char *text, int32_t cap,
                         int32_t *n_text, int32_t *final);

#ifdef __cplusplus
}
#endif
#endif
