/*
 * srref.h -- CPU restatement ("oracle") of the reference engine step.
 *
 * TEST INFRASTRUCTURE ONLY.  This library restates, in plain C, the arithmetic
 * of RyoSpiralArchitect/sr_go_tranformer's Go inference step
 * (cmd/monolith/monolith.go, "M:" below) with the reference's exact operation
 * order.  Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline /
 * reference arm may load it, and only as the checker or as the timed CPU
 * baseline.  The product library (libsrstep.so) never links or calls it.
 *
 * Floating-point mode: the oracle is compiled with -ffp-contract=off, i.e. it
 * reproduces Go's default amd64 code generation, which never fuses x*y+z into
 * an FMA.  (Go on arm64 fuses; that variant is not the parity target.)
 * Transcendentals (exp, log, pow, cos, sin, sqrt in fp64) come from libm; they
 * can differ from Go's math package in the last fp64 ulp, which the float32
 * casts that follow almost always absorb.
 *
 * Parity pin: tests/test_oracle_golden.py checks this oracle against the
 * reference's own Transformers golden fixtures (testdata/hf-{llama,llama3,
 * qwen2,mistral}/.../reference.json) at the reference's 2e-5 tolerance
 * (cmd/monolith/hf_inference_test.go:32-130).
 */
#ifndef SRREF_H
#define SRREF_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum { OR_F32 = 0, OR_Q8 = 1, OR_Q4 = 2 };
enum { OR_MODEL_F32 = 0, OR_MODEL_Q8 = 1, OR_MODEL_Q4 = 2, OR_MODEL_Q4_MIXED = 3 };

/* Mirrors Config (M:56-66) plus the HF switches the step reads. */
typedef struct or_config {
    int32_t vocab, dim, hidden, layers, heads, kv_heads, context;
    double rope_theta, norm_eps;
    int32_t tied;          /* 1: LM head = token embedding (M:6440-6443) */
    int32_t qkv_bias;      /* qwen2 q/k/v biases (M:5022-5029) */
    int32_t weight_format; /* OR_MODEL_* (M:566-582) */
    int32_t page_tokens;   /* 32 in the reference (M:5846) */
    /* llama3 RoPE scaling (M:126-132, M:4961-4977); rope_scaling=0 disables. */
    int32_t rope_scaling;
    double rope_factor, rope_low, rope_high;
    int32_t rope_original;
    /* GPT-2 profile (loadGPT2 M:5052-5165, step branches M:6369-6371, 6389,
     * 6403-6408): absolute positions (wpe, `positions` rows), affine LayerNorm,
     * biases on every projection, GELU-tanh MLP, tied head, no RoPE.
     * Parameters, in loadGPT2's order: wte, wpe, ln_f.weight, ln_f.bias, then
     * per layer ln_1.weight, ln_1.bias, q, k, v, q bias, k bias, v bias, o, o
     * bias, ln_2.weight, ln_2.bias, c_fc, c_fc bias, c_proj, c_proj bias, with
     * every matrix [out, in] (the transposed HF Conv1D). */
    int32_t gpt2;
    int32_t positions;
} or_config;

typedef struct or_param_info {
    int32_t rows, cols, format; /* OR_F32 / OR_Q8 / OR_Q4 */
    int64_t value_bytes;        /* f32: rows*cols*4; q8: rows*cols; q4: rows*ceil(cols/2) */
    int64_t scale_count;        /* rows*ceil(cols/64) for q8/q4, else 0 */
} or_param_info;

typedef struct or_model or_model;

/* ---- SplitMix64 RNG (M:1411-1439) ---- */
uint64_t or_rng_uint64(uint64_t *state);
double or_rng_float64(uint64_t *state);
int64_t or_rng_intn(uint64_t *state, int64_t n);
double or_rng_normal(uint64_t *state);
/* dst[i] = float32(rng.Normal() * scale), in order (M:5212-5219). */
void or_fill_normal(uint64_t *state, float *dst, int64_t count, double scale);

/* ---- quantizer contract (M:857-880, M:3819-3898) ---- */
float or_low_bit_scale(float amax, double levels);
int8_t or_q8_value(float v, float scale);
void or_quantize(const float *src, int64_t rows, int64_t cols, int format, void *values, float *scales);
/* Row gather / dequantisation (Param.copyRow, M:3900-3921). */
void or_copy_row(const void *values, const float *scales, int format, int64_t cols, int64_t row, float *dst);

/* ---- kernels (one call = the reference kernel over n rows) ---- */
/* Y[n,out] = X[n,in] W^T with the reference's per-row order (M:3942-4780). */
void or_linear(float *y, const float *x, int64_t n, int format, const void *values, const float *scales,
               int64_t out, int64_t in, int threads);
/* rmsInto (M:6182-6194). */
void or_rmsnorm(float *y, const float *x, const float *w, int64_t n, int64_t d, double eps);
/* layerNormInto (M:5167-5185). */
void or_layernorm(float *y, const float *x, const float *w, const float *b, int64_t n, int64_t d, double eps);
/* GPT-2's gelu_new (M:6405-6407): float32(0.5x(1+tanh(sqrt(2/pi)(x+0.044715x^3)))) in fp64. */
float or_gelu_tanh(float v);
/* attend (M:5293-5352) over `length` positions given K/V rows by pointer table. */
double or_attend(const float *q, float *out, float *scores, int64_t hd, int64_t length, const float *const *krows,
                 const float *const *vrows);

/* ---- model / step ---- */
or_model *or_model_new(const or_config *c);
void or_model_free(or_model *m);
int32_t or_model_param_count(const or_model *m);
int or_model_param_info(const or_model *m, int32_t index, or_param_info *out);
int or_model_set_param(or_model *m, int32_t index, const void *values, const float *scales);
/* Generate every parameter from one SplitMix64 stream in hfProfileSpecs order:
 * matrices and biases ~ float32(Normal()*scale), norms = 1, then quantize. */
int or_model_init_synthetic(or_model *m, uint64_t seed, double scale);
/* Same values as or_model_init_synthetic, generated in parallel: the k-th
 * SplitMix64 output of a stream seeded with `seed` is mix(seed + k*gamma), so
 * element e (draws 2e+1, 2e+2) is computed independently of the others. */
int or_model_init_synthetic_mt(or_model *m, uint64_t seed, double scale, int threads);
int or_model_get_param(const or_model *m, int32_t index, void *values, float *scales);
const float *or_model_rope_cos(const or_model *m);
const float *or_model_rope_sin(const or_model *m);
int64_t or_page_elements(const or_model *m);

/* One prefillSelected call (M:6245-6456).  `pool` holds num_pages pages of
 * or_page_elements floats, layout per page [layer][K plane pt x kvDim | V plane
 * pt x kvDim] (M:6038-6043).  Session i owns rows token_offsets[i] ..
 * token_offsets[i+1]-1 starting at position pos[i]; its page table is
 * page_ids[page_offsets[i] .. page_offsets[i+1]).  want_logits may be NULL.
 * logits: sessions x vocab (unselected rows zeroed).  Returns 0 or an error
 * code (1 = invalid input; nothing written). */
int or_step(or_model *m, float *pool, int64_t num_pages, int32_t sessions, const int32_t *pos,
            const int32_t *token_offsets, const int32_t *tokens, const int32_t *page_offsets,
            const int32_t *page_ids, const uint8_t *want_logits, float *logits, int threads);

/* ---- sampler (M:7253-7426) ---- */
typedef struct or_sampling {
    int32_t max_tokens;
    double temperature;
    int32_t top_k;
    double top_p;
    double repeat_penalty;
    uint64_t seed;
} or_sampling;
/* Returns 0 and *out_id, or 1 (nonfinite logit) / 2 (empty distribution). */
int or_sample(const float *logits, int32_t vocab, const int32_t *history, int32_t nhist, const or_sampling *s,
              uint64_t *rng_state, int32_t blocked, int32_t *out_id);

/* ---- scheduler (M:8180-8210) ---- */
/* remaining[i] = len(IDs) - Cursor; decoding sessions have remaining == 0. */
int32_t or_schedule_tokens(int32_t n, const int32_t *remaining, int32_t *counts, int32_t budget, int32_t chunk,
                           int32_t mixed_chunk, int32_t start);

#ifdef __cplusplus
}
#endif
#endif
