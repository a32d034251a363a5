/*
 * srref.c -- CPU oracle: restatement of the reference engine step in C.
 *
 * TEST INFRASTRUCTURE ONLY (see srref.h).  Each function cites the Go code in
 * cmd/monolith/monolith.go ("M:line") whose arithmetic it restates.  Build with
 * -ffp-contract=off (oracle/Makefile) so that every x*y+z rounds twice, as Go's
 * default amd64 code generation does.
 */
#define _GNU_SOURCE
#include "srref.h"

#include <float.h>
#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

#define Q8_BLOCK 64

/* ------------------------------------------------------------------ RNG -- */
/* SplitMix64 (M:1411-1422). */
uint64_t or_rng_uint64(uint64_t *state) {
    *state += 0x9e3779b97f4a7c15ULL;
    uint64_t z = *state;
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ULL;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebULL;
    return z ^ (z >> 31);
}
/* M:1423 */
double or_rng_float64(uint64_t *state) { return (double)(or_rng_uint64(state) >> 11) * (1.0 / 9007199254740992.0); }
/* M:1424-1436 (rejection threshold = (-bound) % bound). */
int64_t or_rng_intn(uint64_t *state, int64_t n) {
    if (n <= 0) return -1;
    uint64_t bound = (uint64_t)n;
    uint64_t threshold = (0 - bound) % bound;
    for (;;) {
        uint64_t x = or_rng_uint64(state);
        if (x >= threshold) return (int64_t)(x % bound);
    }
}
/* M:1437-1439: Go evaluates the Log operand's draw before the Cos operand's. */
double or_rng_normal(uint64_t *state) {
    double u1 = or_rng_float64(state);
    double u2 = or_rng_float64(state);
    return sqrt(-2 * log(1 - u1)) * cos(2 * M_PI * u2);
}
void or_fill_normal(uint64_t *state, float *dst, int64_t count, double scale) {
    for (int64_t i = 0; i < count; i++) dst[i] = (float)(or_rng_normal(state) * scale);
}

/* ------------------------------------------------------------ quantizer -- */
/* lowBitScale (M:3877-3891). */
float or_low_bit_scale(float amax, double levels) {
    if (amax == 0) return 0;
    float scale = (float)((double)amax / levels);
    if (scale == 0) return FLT_TRUE_MIN;
    if (scale > FLT_TRUE_MIN && (double)scale * levels > (double)amax) scale = nextafterf(scale, 0);
    return scale;
}
/* q8Value (M:3893-3898); Go's math.Round rounds half away from zero (C round). */
int8_t or_q8_value(float v, float scale) {
    if (scale == 0) return 0;
    double r = round((double)v / (double)scale);
    if (r > 127) r = 127;
    if (r < -127) r = -127;
    return (int8_t)r;
}
static int8_t q4_value(float v, float scale) { /* putQuantized Q4 branch (M:3840-3846) */
    if (scale == 0) return 0;
    double r = round((double)v / (double)scale);
    if (r > 7) r = 7;
    if (r < -7) r = -7;
    return (int8_t)r;
}
/* q4Weights.put (M:3819-3822): two signed nibbles per byte, low nibble first. */
static void q4_put(uint8_t *values, int64_t cols, int64_t row, int64_t col, int8_t v) {
    int64_t i = row * ((cols + 1) / 2) + col / 2;
    unsigned shift = (unsigned)(col % 2) * 4;
    values[i] = (uint8_t)((values[i] & ~(15u << shift)) | (((uint8_t)v & 15u) << shift));
}
/* q4Pairs (M:3811-3817): sign-extended low / high nibble. */
static inline float q4_nibble(uint8_t b, int hi) {
    return hi ? (float)(((int8_t)b) >> 4) : (float)(((int8_t)(uint8_t)(b << 4)) >> 4);
}
/* readParam streaming quantizer (M:857-880): per (row, 64-column block) amax,
 * scale, then round(v/scale) clamped. */
void or_quantize(const float *src, int64_t rows, int64_t cols, int format, void *values, float *scales) {
    int64_t groups = (cols + Q8_BLOCK - 1) / Q8_BLOCK;
    if (format == OR_Q4) memset(values, 0, (size_t)(rows * ((cols + 1) / 2)));
    for (int64_t r = 0; r < rows; r++) {
        for (int64_t g = 0; g < groups; g++) {
            int64_t lo = g * Q8_BLOCK, hi = lo + Q8_BLOCK < cols ? lo + Q8_BLOCK : cols;
            float amax = 0;
            for (int64_t j = lo; j < hi; j++) {
                float a = (float)fabs((double)src[r * cols + j]);
                amax = a > amax ? a : amax; /* Go max(): NaN propagation is irrelevant for finite weights */
            }
            float scale = format == OR_Q4 ? or_low_bit_scale(amax, 7) : or_low_bit_scale(amax, 127);
            scales[r * groups + g] = scale;
            for (int64_t j = lo; j < hi; j++) {
                if (format == OR_Q4)
                    q4_put((uint8_t *)values, cols, r, j, q4_value(src[r * cols + j], scale));
                else
                    ((int8_t *)values)[r * cols + j] = or_q8_value(src[r * cols + j], scale);
            }
        }
    }
}
/* Param.copyRow (M:3900-3921). */
void or_copy_row(const void *values, const float *scales, int format, int64_t cols, int64_t row, float *dst) {
    int64_t groups = (cols + Q8_BLOCK - 1) / Q8_BLOCK;
    if (format == OR_Q4) {
        const uint8_t *wr = (const uint8_t *)values + row * ((cols + 1) / 2);
        for (int64_t j = 0; j < cols; j++) dst[j] = q4_nibble(wr[j / 2], (int)(j % 2)) * scales[row * groups + j / Q8_BLOCK];
    } else if (format == OR_Q8) {
        const int8_t *wr = (const int8_t *)values + row * cols;
        for (int64_t j = 0; j < cols; j++) dst[j] = (float)wr[j] * scales[row * groups + j / Q8_BLOCK];
    } else {
        memcpy(dst, (const float *)values + row * cols, (size_t)cols * 4);
    }
}

/* -------------------------------------------------------- parallel-for -- */
typedef struct {
    void (*fn)(void *, int64_t, int64_t);
    void *arg;
    int64_t lo, hi;
} pf_job;
static void *pf_run(void *p) {
    pf_job *j = (pf_job *)p;
    j->fn(j->arg, j->lo, j->hi);
    return NULL;
}
/* Partitioning never changes results: every output owns its whole reduction. */
static void parallel_for(int64_t tasks, int threads, void (*fn)(void *, int64_t, int64_t), void *arg) {
    if (threads > 64) threads = 64;
    if (threads <= 1 || tasks < 2) {
        fn(arg, 0, tasks);
        return;
    }
    if (threads > tasks) threads = (int)tasks;
    pthread_t th[64];
    pf_job jobs[64];
    for (int t = 0; t < threads; t++) {
        jobs[t].fn = fn;
        jobs[t].arg = arg;
        jobs[t].lo = tasks * t / threads;
        jobs[t].hi = tasks * (t + 1) / threads;
        if (t > 0) pthread_create(&th[t], NULL, pf_run, &jobs[t]);
    }
    pf_run(&jobs[0]);
    for (int t = 1; t < threads; t++) pthread_join(th[t], NULL);
}

/* --------------------------------------------------------------- linear -- */
/* q8NeedsWideSum limit: float32(MaxFloat32 / (2*64*127)) (M:4346-4354). */
static float wide_limit(void) {
    union { uint32_t u; float f; } c = {0x78810204u};
    return c.f;
}
static int row_needs_wide(const float *x, int64_t in) {
    float lim = wide_limit();
    for (int64_t j = 0; j < in; j++)
        if (x[j] > lim || x[j] < -lim) return 1;
    return 0;
}

typedef struct {
    float *y;
    const float *x;
    int64_t n, out, in;
    int format;
    const void *values;
    const float *scales;
    const uint8_t *wide;
} linear_job;

/* FP32: one sequential accumulator per output for every tile shape
 * (linearFP32Range, M:3970-4070). */
static float dot_f32(const float *x, const float *w, int64_t in) {
    float s = 0;
    for (int64_t j = 0; j < in; j++) s += x[j] * w[j];
    return s;
}
/* Q8: per 64-block four strided partials, (a+b)+(c+d), tail, s += p*scale
 * (linearQ8Into, M:4074-4189; dotQ8PairBlock64, M:4194-4342). */
static float dot_q8(const float *x, const int8_t *w, const float *scales, int64_t in) {
    int64_t groups = (in + Q8_BLOCK - 1) / Q8_BLOCK;
    float s = 0;
    for (int64_t g = 0; g < groups; g++) {
        float a = 0, b = 0, c = 0, d = 0;
        int64_t j = g * Q8_BLOCK, end = j + Q8_BLOCK < in ? j + Q8_BLOCK : in;
        for (; j + 4 <= end; j += 4) {
            a += x[j] * (float)w[j];
            b += x[j + 1] * (float)w[j + 1];
            c += x[j + 2] * (float)w[j + 2];
            d += x[j + 3] * (float)w[j + 3];
        }
        float p = (a + b) + (c + d);
        for (; j < end; j++) p += x[j] * (float)w[j];
        s += p * scales[g];
    }
    return s;
}
/* Q4: identical order with values decoded from packed nibbles (linearQ4Into,
 * M:4387-4511; dotQ4PairBlock64 / dotQ4Block64, M:4517-4752). */
static float dot_q4(const float *x, const uint8_t *w, const float *scales, int64_t in) {
    int64_t groups = (in + Q8_BLOCK - 1) / Q8_BLOCK;
    float s = 0;
    for (int64_t g = 0; g < groups; g++) {
        float a = 0, b = 0, c = 0, d = 0;
        int64_t j = g * Q8_BLOCK, end = j + Q8_BLOCK < in ? j + Q8_BLOCK : in;
        for (; j + 4 <= end; j += 4) {
            a += x[j] * q4_nibble(w[j / 2], 0);
            b += x[j + 1] * q4_nibble(w[j / 2], 1);
            c += x[j + 2] * q4_nibble(w[j / 2 + 1], 0);
            d += x[j + 3] * q4_nibble(w[j / 2 + 1], 1);
        }
        float p = (a + b) + (c + d);
        for (; j < end; j++) p += x[j] * q4_nibble(w[j / 2], (int)(j % 2));
        s += p * scales[g];
    }
    return s;
}
/* Wide fp64 fallback for rows with |x| > limit (linearQ8WideInto M:4356-4382,
 * linearQ4WideInto M:4754-4780). */
static float dot_wide(const float *x, int format, const void *wrow, const float *scales, int64_t in) {
    int64_t groups = (in + Q8_BLOCK - 1) / Q8_BLOCK;
    double sum = 0;
    for (int64_t g = 0; g < groups; g++) {
        double part = 0;
        int64_t end = (g + 1) * Q8_BLOCK < in ? (g + 1) * Q8_BLOCK : in;
        for (int64_t j = g * Q8_BLOCK; j < end; j++) {
            double w = format == OR_Q4 ? (double)q4_nibble(((const uint8_t *)wrow)[j / 2], (int)(j % 2))
                                       : (double)((const int8_t *)wrow)[j];
            part += (double)x[j] * w;
        }
        sum += part * (double)scales[g];
    }
    return (float)sum;
}
static void linear_range(void *arg, int64_t lo, int64_t hi) {
    linear_job *J = (linear_job *)arg;
    int64_t in = J->in, groups = (in + Q8_BLOCK - 1) / Q8_BLOCK;
    for (int64_t o = lo; o < hi; o++) {
        for (int64_t r = 0; r < J->n; r++) {
            const float *x = J->x + r * in;
            float v;
            if (J->format == OR_F32) {
                v = dot_f32(x, (const float *)J->values + o * in, in);
            } else if (J->format == OR_Q8) {
                const int8_t *w = (const int8_t *)J->values + o * in;
                v = J->wide[r] ? dot_wide(x, OR_Q8, w, J->scales + o * groups, in) : dot_q8(x, w, J->scales + o * groups, in);
            } else {
                const uint8_t *w = (const uint8_t *)J->values + o * ((in + 1) / 2);
                v = J->wide[r] ? dot_wide(x, OR_Q4, w, J->scales + o * groups, in) : dot_q4(x, w, J->scales + o * groups, in);
            }
            J->y[r * J->out + o] = v;
        }
    }
}
/* linearIntoWithExecutor (M:3942-3968): the wide path is selected per row
 * (M:4359-4365), so a neighbouring extreme row never changes another row. */
void or_linear(float *y, const float *x, int64_t n, int format, const void *values, const float *scales, int64_t out,
               int64_t in, int threads) {
    uint8_t *wide = (uint8_t *)calloc((size_t)(n > 0 ? n : 1), 1);
    if (format != OR_F32)
        for (int64_t r = 0; r < n; r++) wide[r] = (uint8_t)row_needs_wide(x + r * in, in);
    linear_job J = {y, x, n, out, in, format, values, scales, wide};
    parallel_for(out, threads, linear_range, &J);
    free(wide);
}

/* rmsInto (M:6182-6194). */
void or_rmsnorm(float *y, const float *x, const float *w, int64_t n, int64_t d, double eps) {
    for (int64_t r = 0; r < n; r++) {
        double ss = 0;
        for (int64_t j = 0; j < d; j++) ss += (double)x[r * d + j] * (double)x[r * d + j];
        float a = (float)(1 / sqrt(ss / (double)d + eps));
        for (int64_t j = 0; j < d; j++) y[r * d + j] = x[r * d + j] * a * w[j];
    }
}

/* layerNormInto (M:5167-5185): fp64 mean and variance in element order, then
 * float32((x - mean) * inv) * w + b in float32. */
void or_layernorm(float *y, const float *x, const float *w, const float *b, int64_t n, int64_t d, double eps) {
    for (int64_t r = 0; r < n; r++) {
        const float *xr = x + r * d;
        double mean = 0, variance = 0;
        for (int64_t j = 0; j < d; j++) mean += (double)xr[j];
        mean /= (double)d;
        for (int64_t j = 0; j < d; j++) {
            double z = (double)xr[j] - mean;
            variance += z * z;
        }
        double inv = 1 / sqrt(variance / (double)d + eps);
        for (int64_t j = 0; j < d; j++) y[r * d + j] = (float)(((double)xr[j] - mean) * inv) * w[j] + b[j];
    }
}

/* gelu_new as the reference writes it (M:6405-6407), left to right in fp64.
 * The constant is the double nearest 2/pi (Go folds 2/math.Pi exactly; here
 * 2.0/M_PI rounds to the same double). */
float or_gelu_tanh(float v) {
    double x = (double)v;
    return (float)(0.5 * x * (1 + tanh(sqrt(0x1.45f306dc9c883p-1) * (x + 0.044715 * x * x * x))));
}

/* attend (M:5293-5352). */
double or_attend(const float *q, float *out, float *scores, int64_t hd, int64_t length, const float *const *krows,
                 const float *const *vrows) {
    float scale = (float)(1 / sqrt((double)hd));
    float max_score = -FLT_MAX;
    for (int64_t j = 0; j < hd; j++) out[j] = 0;
    for (int64_t s = 0; s < length; s++) {
        const float *k = krows[s];
        float dot = 0;
        for (int64_t j = 0; j < hd; j++) dot += q[j] * k[j];
        scores[s] = dot * scale;
        if (scores[s] > max_score) max_score = scores[s];
    }
    double sum = 0;
    for (int64_t s = 0; s < length; s++) sum += exp((double)scores[s] - (double)max_score);
    double lse = (double)max_score + log(sum);
    for (int64_t s = 0; s < length; s++) {
        float p = (float)exp((double)scores[s] - lse);
        const float *v = vrows[s];
        for (int64_t j = 0; j < hd; j++) out[j] += p * v[j];
    }
    return lse;
}

/* ---------------------------------------------------------------- model -- */
typedef struct {
    int32_t rows, cols, format;
    void *values;
    float *scales;
} or_param;

struct or_model {
    or_config c;
    int32_t nparams;
    or_param *params;
    float *cos_t, *sin_t;
};

static int param_format(const or_config *c, int matrix, int is_embed_or_head) {
    if (!matrix) return OR_F32;
    switch (c->weight_format) {
    case OR_MODEL_Q8: return OR_Q8;
    case OR_MODEL_Q4: return OR_Q4;
    case OR_MODEL_Q4_MIXED: return is_embed_or_head ? OR_Q8 : OR_Q4; /* hfMatrixFormat (M:572-582) */
    default: return OR_F32;
    }
}
static int64_t value_bytes(int32_t rows, int32_t cols, int format) {
    if (format == OR_Q8) return (int64_t)rows * cols;
    if (format == OR_Q4) return (int64_t)rows * ((cols + 1) / 2);
    return (int64_t)rows * cols * 4;
}
static int64_t scale_count(int32_t rows, int32_t cols, int format) {
    return format == OR_F32 ? 0 : (int64_t)rows * ((cols + Q8_BLOCK - 1) / Q8_BLOCK);
}

/* hfInverseFrequency (M:4961-4977). */
static float hf_inverse_frequency(const or_config *c, int hd, int index) {
    float inv = 1.0f / (float)pow(c->rope_theta, (double)((float)(2 * index) / (float)hd));
    if (!c->rope_scaling) return inv;
    float wave = (float)(2 * M_PI) / inv;
    float low_wave = (float)((double)c->rope_original / c->rope_low);
    float high_wave = (float)((double)c->rope_original / c->rope_high);
    float factor = (float)c->rope_factor;
    if (wave > low_wave) return inv / factor;
    if (wave >= high_wave) {
        float smooth = ((float)c->rope_original / wave - (float)c->rope_low) / (float)(c->rope_high - c->rope_low);
        return (1 - smooth) * inv / factor + smooth * inv;
    }
    return inv;
}

or_model *or_model_new(const or_config *c) {
    if (c->dim < 2 || c->heads < 1 || c->kv_heads < 1 || c->dim % c->heads || c->heads % c->kv_heads ||
        (c->dim / c->heads) % 2 || c->layers < 1 || c->vocab < 1 || c->hidden < 1 || c->context < 1 ||
        c->page_tokens < 1)
        return NULL;
    if (c->gpt2 && (c->kv_heads != c->heads || !c->tied || c->qkv_bias || c->positions < c->context)) return NULL;
    or_model *m = (or_model *)calloc(1, sizeof(or_model));
    m->c = *c;
    int32_t L = c->layers, d = c->dim, kd = c->dim / c->heads * c->kv_heads, h = c->hidden;
    m->nparams = c->gpt2 ? 4 + 16 * L : 1 + 9 * L + 1 + (c->qkv_bias ? 3 * L : 0) + (c->tied ? 0 : 1);
    m->params = (or_param *)calloc((size_t)m->nparams, sizeof(or_param));
    int32_t i = 0;
#define P(R, C, MAT, EH)                                                                                               \
    do {                                                                                                               \
        m->params[i].rows = (R);                                                                                       \
        m->params[i].cols = (C);                                                                                       \
        m->params[i].format = param_format(c, (MAT), (EH));                                                            \
        i++;                                                                                                           \
    } while (0)
    if (c->gpt2) { /* loadGPT2's parameter order (M:5063-5066, 5114-5122) */
        P(c->vocab, d, 1, 1);
        P(c->positions, d, 0, 0);
        P(1, d, 0, 0);
        P(1, d, 0, 0);
        for (int32_t l = 0; l < L; l++) {
            P(1, d, 0, 0);
            P(1, d, 0, 0);
            P(d, d, 1, 0);
            P(d, d, 1, 0);
            P(d, d, 1, 0);
            P(1, d, 0, 0);
            P(1, d, 0, 0);
            P(1, d, 0, 0);
            P(d, d, 1, 0);
            P(1, d, 0, 0);
            P(1, d, 0, 0);
            P(1, d, 0, 0);
            P(h, d, 1, 0);
            P(1, h, 0, 0);
            P(d, h, 1, 0);
            P(1, d, 0, 0);
        }
    } else {
    P(c->vocab, d, 1, 1); /* hfTensorSpecs order (M:407-423) */
    for (int32_t l = 0; l < L; l++) {
        P(1, d, 0, 0);
        P(d, d, 1, 0);
        P(kd, d, 1, 0);
        P(kd, d, 1, 0);
        P(d, d, 1, 0);
        P(1, d, 0, 0);
        P(h, d, 1, 0);
        P(h, d, 1, 0);
        P(d, h, 1, 0);
    }
    P(1, d, 0, 0);
    if (c->qkv_bias)
        for (int32_t l = 0; l < L; l++) {
            P(1, d, 0, 0);
            P(1, kd, 0, 0);
            P(1, kd, 0, 0);
        }
    if (!c->tied) P(c->vocab, d, 1, 1);
    }
#undef P
    for (i = 0; i < m->nparams; i++) {
        or_param *p = &m->params[i];
        p->values = calloc((size_t)value_bytes(p->rows, p->cols, p->format), 1);
        int64_t sc = scale_count(p->rows, p->cols, p->format);
        p->scales = sc ? (float *)calloc((size_t)sc, 4) : NULL;
    }
    int hd = d / c->heads;
    m->cos_t = (float *)malloc((size_t)c->context * (hd / 2) * 4);
    m->sin_t = (float *)malloc((size_t)c->context * (hd / 2) * 4);
    for (int32_t pos = 0; pos < c->context; pos++) /* HF RoPE tables (M:5034-5043) */
        for (int j = 0; j < hd / 2; j++) {
            float inv = hf_inverse_frequency(c, hd, j);
            double angle = (double)((float)pos * inv);
            m->cos_t[(int64_t)pos * (hd / 2) + j] = (float)cos(angle);
            m->sin_t[(int64_t)pos * (hd / 2) + j] = (float)sin(angle);
        }
    return m;
}
void or_model_free(or_model *m) {
    if (!m) return;
    for (int32_t i = 0; i < m->nparams; i++) {
        free(m->params[i].values);
        free(m->params[i].scales);
    }
    free(m->params);
    free(m->cos_t);
    free(m->sin_t);
    free(m);
}
int32_t or_model_param_count(const or_model *m) { return m->nparams; }
int or_model_param_info(const or_model *m, int32_t index, or_param_info *out) {
    if (index < 0 || index >= m->nparams) return 1;
    const or_param *p = &m->params[index];
    out->rows = p->rows;
    out->cols = p->cols;
    out->format = p->format;
    out->value_bytes = value_bytes(p->rows, p->cols, p->format);
    out->scale_count = scale_count(p->rows, p->cols, p->format);
    return 0;
}
int or_model_set_param(or_model *m, int32_t index, const void *values, const float *scales) {
    if (index < 0 || index >= m->nparams) return 1;
    or_param *p = &m->params[index];
    memcpy(p->values, values, (size_t)value_bytes(p->rows, p->cols, p->format));
    if (p->scales) memcpy(p->scales, scales, (size_t)scale_count(p->rows, p->cols, p->format) * 4);
    return 0;
}
int or_model_get_param(const or_model *m, int32_t index, void *values, float *scales) {
    if (index < 0 || index >= m->nparams) return 1;
    const or_param *p = &m->params[index];
    memcpy(values, p->values, (size_t)value_bytes(p->rows, p->cols, p->format));
    if (p->scales && scales) memcpy(scales, p->scales, (size_t)scale_count(p->rows, p->cols, p->format) * 4);
    return 0;
}
/* One SplitMix64 stream over every matrix and bias element in hfProfileSpecs
 * order; norms are 1 (native convention M:5212-5219 with HF semantics). */
int or_model_init_synthetic(or_model *m, uint64_t seed, double scale) {
    if (m->c.gpt2) return 1; /* no native initialisation for the GPT-2 profile */
    uint64_t state = seed;
    int32_t L = m->c.layers;
    for (int32_t i = 0; i < m->nparams; i++) {
        or_param *p = &m->params[i];
        int is_norm = (i >= 1 && i < 1 + 9 * L && ((i - 1) % 9 == 0 || (i - 1) % 9 == 5)) || i == 1 + 9 * L;
        int64_t count = (int64_t)p->rows * p->cols;
        float *tmp = (float *)malloc((size_t)count * 4);
        if (is_norm)
            for (int64_t j = 0; j < count; j++) tmp[j] = 1;
        else
            or_fill_normal(&state, tmp, count, scale);
        if (p->format == OR_F32)
            memcpy(p->values, tmp, (size_t)count * 4);
        else
            or_quantize(tmp, p->rows, p->cols, p->format, p->values, p->scales);
        free(tmp);
    }
    return 0;
}
static uint64_t splitmix_at(uint64_t seed, uint64_t k) {
    uint64_t z = seed + k * 0x9e3779b97f4a7c15ULL;
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ULL;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebULL;
    return z ^ (z >> 31);
}
typedef struct {
    or_param *p;
    uint64_t seed, e0;
    double scale;
} synth_job;
static void synth_rows(void *arg, int64_t lo, int64_t hi) {
    synth_job *J = (synth_job *)arg;
    or_param *p = J->p;
    int64_t cols = p->cols;
    float *tmp = (float *)malloc((size_t)cols * 4);
    for (int64_t r = lo; r < hi; r++) {
        for (int64_t j = 0; j < cols; j++) {
            uint64_t e = J->e0 + (uint64_t)(r * cols + j);
            double u1 = (double)(splitmix_at(J->seed, 2 * e + 1) >> 11) * (1.0 / 9007199254740992.0);
            double u2 = (double)(splitmix_at(J->seed, 2 * e + 2) >> 11) * (1.0 / 9007199254740992.0);
            tmp[j] = (float)(sqrt(-2 * log(1 - u1)) * cos(2 * M_PI * u2) * J->scale);
        }
        if (p->format == OR_F32)
            memcpy((float *)p->values + r * cols, tmp, (size_t)cols * 4);
        else if (p->format == OR_Q8)
            or_quantize(tmp, 1, cols, OR_Q8, (int8_t *)p->values + r * cols, p->scales + r * ((cols + 63) / 64));
        else
            or_quantize(tmp, 1, cols, OR_Q4, (uint8_t *)p->values + r * ((cols + 1) / 2),
                        p->scales + r * ((cols + 63) / 64));
    }
    free(tmp);
}
int or_model_init_synthetic_mt(or_model *m, uint64_t seed, double scale, int threads) {
    if (m->c.gpt2) return 1;
    int32_t L = m->c.layers;
    uint64_t e0 = 0;
    for (int32_t i = 0; i < m->nparams; i++) {
        or_param *p = &m->params[i];
        int is_norm = (i >= 1 && i < 1 + 9 * L && ((i - 1) % 9 == 0 || (i - 1) % 9 == 5)) || i == 1 + 9 * L;
        int64_t count = (int64_t)p->rows * p->cols;
        if (is_norm) {
            for (int64_t j = 0; j < count; j++) ((float *)p->values)[j] = 1;
            continue;
        }
        synth_job J = {p, seed, e0, scale};
        parallel_for(p->rows, threads, synth_rows, &J);
        e0 += (uint64_t)count;
    }
    return 0;
}
const float *or_model_rope_cos(const or_model *m) { return m->cos_t; }
const float *or_model_rope_sin(const or_model *m) { return m->sin_t; }
int64_t or_page_elements(const or_model *m) {
    int64_t kd = (int64_t)m->c.dim / m->c.heads * m->c.kv_heads;
    return 2 * (int64_t)m->c.page_tokens * kd * m->c.layers;
}

/* ----------------------------------------------------------------- step -- */
static void linear_p(float *y, const float *x, int64_t n, const or_param *p, int threads) {
    or_linear(y, x, n, p->format, p->values, p->scales, p->rows, p->cols, threads);
}
/* Model.rope HF half-split branch (M:5264-5289). */
static void rope_row(const or_model *m, float *x, int heads, int64_t pos) {
    int hd = m->c.dim / m->c.heads;
    for (int h = 0; h < heads; h++)
        for (int j = 0; j < hd / 2; j++) {
            int64_t i = (int64_t)h * hd + j, z = i + hd / 2, ri = pos * (hd / 2) + j;
            float c = m->cos_t[ri], s = m->sin_t[ri];
            float a = x[i], b = x[z];
            x[i] = a * c - b * s;
            x[z] = a * s + b * c;
        }
}

typedef struct {
    const or_model *m;
    float *pool;
    const int64_t *row_page_base; /* per row: page table start into page_ids */
    const int32_t *page_ids;
    const int32_t *positions;
    const float *Q;
    float *A;
    float *scores; /* per thread scratch */
    int64_t stride;
    int layer, rows;
    const float **kr, **vr; /* per thread row tables */
} attn_job;
typedef struct {
    attn_job *J;
    int64_t threads;
} attn_outer;
static void attn_tasks(attn_job *J, int64_t lane, int64_t tlo, int64_t thi) {
    const or_config *c = &J->m->c;
    int hd = c->dim / c->heads, group = c->heads / c->kv_heads, pt = c->page_tokens;
    int64_t kd = (int64_t)hd * c->kv_heads, pe = or_page_elements(J->m), d = c->dim;
    float *scores = J->scores + lane * J->stride;
    const float **kr = J->kr + lane * J->stride, **vr = J->vr + lane * J->stride;
    for (int64_t task = tlo; task < thi; task++) {
        int64_t i = task / c->heads, h = task % c->heads, kh = h / group;
        int64_t length = (int64_t)J->positions[i] + 1;
        for (int64_t s = 0; s < length; s++) {
            int64_t page = J->page_ids[J->row_page_base[i] + s / pt];
            int64_t base = page * pe + (int64_t)J->layer * 2 * pt * kd + (s % pt) * kd + kh * hd;
            kr[s] = J->pool + base;
            vr[s] = J->pool + base + (int64_t)pt * kd;
        }
        or_attend(J->Q + i * d + h * hd, J->A + i * d + h * hd, scores, hd, length, kr, vr);
    }
}
static void attn_lane(void *arg, int64_t lo, int64_t hi) {
    attn_outer *O = (attn_outer *)arg;
    int64_t tasks = (int64_t)O->J->rows * O->J->m->c.heads;
    for (int64_t lane = lo; lane < hi; lane++)
        attn_tasks(O->J, lane, tasks * lane / O->threads, tasks * (lane + 1) / O->threads);
}

int or_step(or_model *m, float *pool, int64_t num_pages, int32_t sessions, const int32_t *pos,
            const int32_t *token_offsets, const int32_t *tokens, const int32_t *page_offsets,
            const int32_t *page_ids, const uint8_t *want_logits, float *logits, int threads) {
    const or_config *c = &m->c;
    /* Validation before any mutation (M:6246-6339). */
    if (sessions < 1 || sessions > 256) return 1;
    int64_t n = 0;
    if (token_offsets[0] != 0 || page_offsets[0] != 0) return 1;
    for (int32_t i = 0; i < sessions; i++) {
        int64_t len = (int64_t)token_offsets[i + 1] - token_offsets[i];
        if (len < 1 || len > 1024 - n) return 1;
        if (pos[i] < 0 || pos[i] > c->context || len > c->context - pos[i]) return 1;
        for (int64_t j = token_offsets[i]; j < token_offsets[i + 1]; j++)
            if (tokens[j] < 0 || tokens[j] >= c->vocab) return 1;
        int64_t end = pos[i] + len, need = (end + c->page_tokens - 1) / c->page_tokens;
        if ((int64_t)page_offsets[i + 1] - page_offsets[i] < need) return 1;
        for (int64_t j = page_offsets[i]; j < page_offsets[i + 1]; j++)
            if (page_ids[j] < 0 || page_ids[j] >= num_pages) return 1;
        n += len;
    }
    const int32_t L = c->layers, d = c->dim, H = c->heads, Hkv = c->kv_heads, hd = d / H, pt = c->page_tokens;
    const int64_t kd = (int64_t)hd * Hkv, hid = c->hidden, V = c->vocab, pe = or_page_elements(m);
    float *X = (float *)calloc((size_t)(n * d), 4), *N = (float *)calloc((size_t)(n * d), 4);
    float *Q = (float *)calloc((size_t)(n * d), 4), *K = (float *)calloc((size_t)(n * kd), 4);
    float *Vv = (float *)calloc((size_t)(n * kd), 4), *A = (float *)calloc((size_t)(n * d), 4);
    float *T = (float *)calloc((size_t)(n * d), 4), *G = (float *)calloc((size_t)(n * hid), 4);
    float *U = (float *)calloc((size_t)(n * hid), 4), *Hh = (float *)calloc((size_t)(n * hid), 4);
    int32_t *positions = (int32_t *)calloc((size_t)n, 4);
    int64_t *row_page_base = (int64_t *)calloc((size_t)n, 8);
    int32_t *last_rows = (int32_t *)calloc((size_t)sessions, 4);
    int32_t max_pos = 0;
    /* Row metadata + embedding gather (M:6361-6375). */
    int64_t r = 0;
    for (int32_t i = 0; i < sessions; i++) {
        for (int64_t j = token_offsets[i]; j < token_offsets[i + 1]; j++) {
            positions[r] = pos[i] + (int32_t)(j - token_offsets[i]);
            row_page_base[r] = page_offsets[i];
            if (positions[r] + 1 > max_pos) max_pos = positions[r] + 1;
            const or_param *E = &m->params[0];
            or_copy_row(E->values, E->scales, E->format, d, tokens[j], X + r * d);
            if (c->gpt2) { /* absolute position row (M:6369-6371) */
                const float *wpe = (const float *)m->params[1].values + (int64_t)positions[r] * d;
                for (int32_t e = 0; e < d; e++) X[r * d + e] += wpe[e];
            }
            r++;
        }
        last_rows[i] = (int32_t)(r - 1);
    }
    int lanes = threads > 1 ? threads : 1;
    int64_t stride = max_pos;
    float *scores = (float *)malloc((size_t)(lanes * stride) * 4);
    const float **kr = (const float **)malloc((size_t)(lanes * stride) * sizeof(float *));
    const float **vr = (const float **)malloc((size_t)(lanes * stride) * sizeof(float *));
#define FV(p) ((const float *)(p).values)
    for (int32_t l = 0; l < L; l++) { /* layer loop (M:6376-6419) */
        const or_param *P = &m->params[1 + 9 * l];
        const or_param *G2 = &m->params[4 + 16 * l]; /* GPT-2 block (loadGPT2 order) */
        const or_param *wq = c->gpt2 ? &G2[2] : &P[1], *wk = c->gpt2 ? &G2[3] : &P[2], *wv = c->gpt2 ? &G2[4] : &P[3];
        if (c->gpt2)
            or_layernorm(N, X, FV(G2[0]), FV(G2[1]), n, d, c->norm_eps);
        else
            or_rmsnorm(N, X, FV(P[0]), n, d, c->norm_eps);
        linear_p(Q, N, n, wq, threads);
        linear_p(K, N, n, wk, threads);
        linear_p(Vv, N, n, wv, threads);
        if (c->qkv_bias || c->gpt2) { /* addBias (M:3933-3940) */
            const or_param *B = c->gpt2 ? &G2[5] : &m->params[2 + 9 * L + 3 * l];
            for (int64_t e = 0; e < n * d; e++) Q[e] += FV(B[0])[e % d];
            for (int64_t e = 0; e < n * kd; e++) K[e] += FV(B[1])[e % kd];
            for (int64_t e = 0; e < n * kd; e++) Vv[e] += FV(B[2])[e % kd];
        }
        for (int64_t i = 0; i < n; i++) { /* RoPE + KV write (M:6384-6396) */
            if (!c->gpt2) {
                rope_row(m, Q + i * d, H, positions[i]);
                rope_row(m, K + i * kd, Hkv, positions[i]);
            }
            int64_t page = page_ids[row_page_base[i] + positions[i] / pt];
            int64_t base = page * pe + (int64_t)l * 2 * pt * kd + (int64_t)(positions[i] % pt) * kd;
            memcpy(pool + base, K + i * kd, (size_t)kd * 4);
            memcpy(pool + base + (int64_t)pt * kd, Vv + i * kd, (size_t)kd * 4);
        }
        attn_job J;
        memset(&J, 0, sizeof J);
        J.m = m;
        J.pool = pool;
        J.row_page_base = row_page_base;
        J.page_ids = page_ids;
        J.positions = positions;
        J.Q = Q;
        J.A = A;
        J.scores = scores;
        J.stride = stride;
        J.layer = l;
        J.rows = (int)n;
        J.kr = kr;
        J.vr = vr;
        attn_outer O = {&J, lanes};
        parallel_for(lanes, lanes, attn_lane, &O);
        if (c->gpt2) { /* O projection + bias + residual, LayerNorm, c_fc + bias, GELU (M:6398-6408) */
            linear_p(T, A, n, &G2[8], threads);
            for (int64_t e = 0; e < n * d; e++) T[e] += FV(G2[9])[e % d];
            for (int64_t e = 0; e < n * d; e++) X[e] += T[e];
            or_layernorm(N, X, FV(G2[10]), FV(G2[11]), n, d, c->norm_eps);
            linear_p(G, N, n, &G2[12], threads);
            for (int64_t e = 0; e < n * hid; e++) G[e] += FV(G2[13])[e % hid];
            for (int64_t e = 0; e < n * hid; e++) Hh[e] = or_gelu_tanh(G[e]);
            linear_p(T, Hh, n, &G2[14], threads); /* c_proj + bias + residual (M:6415-6417) */
            for (int64_t e = 0; e < n * d; e++) T[e] += FV(G2[15])[e % d];
            for (int64_t e = 0; e < n * d; e++) X[e] += T[e];
            continue;
        }
        linear_p(T, A, n, &P[4], threads); /* O projection + residual (M:6398-6400) */
        for (int64_t e = 0; e < n * d; e++) X[e] += T[e];
        or_rmsnorm(N, X, FV(P[5]), n, d, c->norm_eps);
        linear_p(G, N, n, &P[6], threads);
        linear_p(U, N, n, &P[7], threads);
        for (int64_t e = 0; e < n * hid; e++) /* SwiGLU (M:6410-6413) */
            Hh[e] = (float)((double)G[e] / (1 + exp(-(double)G[e]))) * U[e];
        linear_p(T, Hh, n, &P[8], threads);
        for (int64_t e = 0; e < n * d; e++) X[e] += T[e];
    }
    /* Selected head (M:6420-6448). */
    int64_t heads = 0;
    for (int32_t i = 0; i < sessions; i++)
        if (!want_logits || want_logits[i]) {
            memcpy(T + heads * d, X + (int64_t)last_rows[i] * d, (size_t)d * 4);
            heads++;
        }
    float *compact = heads ? (float *)malloc((size_t)(heads * V) * 4) : NULL;
    if (heads) {
        if (c->gpt2)
            or_layernorm(N, T, FV(m->params[2]), FV(m->params[3]), heads, d, c->norm_eps);
        else
            or_rmsnorm(N, T, FV(m->params[1 + 9 * L]), heads, d, c->norm_eps);
        const or_param *head = c->tied ? &m->params[0] : &m->params[m->nparams - 1];
        linear_p(compact, N, heads, head, threads);
    }
    int64_t hsel = 0;
    for (int32_t i = 0; i < sessions; i++) {
        if (!want_logits || want_logits[i]) {
            memcpy(logits + (int64_t)i * V, compact + hsel * V, (size_t)V * 4);
            hsel++;
        } else {
            memset(logits + (int64_t)i * V, 0, (size_t)V * 4);
        }
    }
#undef FV
    free(compact);
    free(X), free(N), free(Q), free(K), free(Vv), free(A), free(T), free(G), free(U), free(Hh);
    free(positions), free(row_page_base), free(last_rows), free(scores), free(kr), free(vr);
    return 0;
}

/* -------------------------------------------------------------- sampler -- */
typedef struct {
    int32_t id;
    double logit, prob;
} cand;
/* candidateBefore (M:7277-7282). */
static int cand_cmp(const void *pa, const void *pb) {
    const cand *a = (const cand *)pa, *b = (const cand *)pb;
    if (a->logit == b->logit) return a->id < b->id ? -1 : (a->id > b->id);
    return a->logit > b->logit ? -1 : 1;
}
static int finite_f(float v) { return isfinite(v); }
static int in_history(const int32_t *history, int32_t nhist, int32_t id) {
    for (int32_t k = 0; k < nhist; k++)
        if (history[k] == id) return 1;
    return 0;
}
/* sampleWithBlocked (M:7320-7426).  The bounded heap (M:7286-7315) retains
 * exactly the first top_k of the total (logit desc, id asc) order, so a full
 * sort followed by truncation gives the same candidates in the same order. */
int or_sample(const float *logits, int32_t vocab, const int32_t *history, int32_t nhist, const or_sampling *s,
              uint64_t *rng_state, int32_t blocked, int32_t *out_id) {
    if (vocab <= 0) return 2;
    uint8_t *seen = NULL;
    if (s->temperature != 0 || s->repeat_penalty != 1) {
        seen = (uint8_t *)calloc((size_t)vocab, 1);
        for (int32_t k = 0; k < nhist; k++)
            if (history[k] >= 0 && history[k] < vocab) seen[history[k]] = 1;
    }
    (void)in_history;
    if (s->temperature == 0) {
        int32_t best = -1;
        double best_logit = 0;
        for (int32_t id = 0; id < vocab; id++) {
            if (!finite_f(logits[id])) {
                free(seen);
                return 1;
            }
            if (id == blocked) continue;
            double x = (double)logits[id];
            if (seen && seen[id]) x = x > 0 ? x / s->repeat_penalty : x * s->repeat_penalty;
            if (best < 0 || x > best_logit) {
                best = id;
                best_logit = x;
            }
        }
        free(seen);
        if (best < 0) return 2;
        *out_id = best;
        return 0;
    }
    cand *cs = (cand *)malloc((size_t)vocab * sizeof(cand));
    int32_t count = 0;
    for (int32_t id = 0; id < vocab; id++) {
        if (!finite_f(logits[id])) {
            free(cs);
            free(seen);
            return 1;
        }
        if (id == blocked) continue;
        double x = (double)logits[id];
        if (seen && seen[id]) x = x > 0 ? x / s->repeat_penalty : x * s->repeat_penalty;
        cs[count].id = id;
        cs[count].logit = x;
        cs[count].prob = 0;
        count++;
    }
    free(seen);
    if (count == 0) {
        free(cs);
        return 2;
    }
    qsort(cs, (size_t)count, sizeof(cand), cand_cmp);
    if (s->top_k > 0 && s->top_k < count) count = s->top_k;
    double total = 0, max_logit = cs[0].logit;
    for (int32_t i = 0; i < count; i++) {
        cs[i].prob = exp((cs[i].logit - max_logit) / s->temperature);
        total += cs[i].prob;
    }
    if (s->top_p < 1) {
        double mass = 0;
        for (int32_t i = 0; i < count; i++) {
            mass += cs[i].prob;
            if (mass >= s->top_p * total) {
                count = i + 1;
                total = mass;
                break;
            }
        }
    }
    double draw = or_rng_float64(rng_state) * total;
    int32_t id = cs[count - 1].id;
    for (int32_t i = 0; i < count; i++) {
        draw -= cs[i].prob;
        if (draw < 0) {
            id = cs[i].id;
            break;
        }
    }
    free(cs);
    *out_id = id;
    return 0;
}

/* ------------------------------------------------------------ scheduler -- */
/* scheduleTokens (M:8180-8210). */
int32_t or_schedule_tokens(int32_t n, const int32_t *remaining, int32_t *counts, int32_t budget, int32_t chunk,
                           int32_t mixed_chunk, int32_t start) {
    for (int32_t i = 0; i < n; i++)
        if (remaining[i] == 0) {
            chunk = chunk < mixed_chunk ? chunk : mixed_chunk;
            break;
        }
    int32_t total = n;
    for (int32_t i = 0; i < n; i++) counts[i] = 1;
    while (total < budget) {
        int progress = 0;
        for (int32_t j = 0; j < n; j++) {
            int32_t i = (start + j) % n;
            int32_t lim = chunk < remaining[i] ? chunk : remaining[i];
            if (counts[i] < lim) {
                counts[i]++;
                total++;
                progress = 1;
                if (total == budget) break;
            }
        }
        if (!progress) break;
    }
    return total;
}
