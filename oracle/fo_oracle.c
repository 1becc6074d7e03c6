/*
 * fo_oracle.c -- CPU restatement of falcon-ocr-cpu's attention hot path.
 *
 * TEST INFRASTRUCTURE ONLY: the checker the CUDA product is compared with
 * (tests/, __graft_entry__.smoke(), bench.py's cpu_baseline and reference
 * arm).  Nothing in falcon-ocr-cpu_b200/ links or calls it.
 *
 * Parity status: the reference is a Rust crate and no Rust toolchain exists
 * here, so it cannot be run.  This file is pinned against the reference's own
 * tests instead: the 5-token image/sink known answer and the sink = -inf
 * identity (src/kernels/tests.rs:283-309), the extreme-logit cases (:311-345),
 * the dense f64 tolerance table (:250-281), the static/BF16 f64 bounds
 * (prefill64/static_shift/tests.rs:374-394, prefill64/bf16.rs:851-926), the
 * Q8/Q16 bound, chunking bound, NaN propagation, pair refusal and the
 * ties-to-even code table (src/quant/kv/tests.rs).  tests/golden/ holds
 * those inputs and expected outputs; tests/test_oracle_golden.py checks them.
 *
 * Build: oracle/Makefile (gcc -O3 -ffp-contract=off -fopenmp).  Contraction
 * is off so every multiply-add below is the one the reference performs:
 * fmaf() where the reference fuses, separate * and + where it does not.
 */
#include "fo_oracle.h"

#include <float.h>
#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define HD 64          /* head_dim of every fixed-width kernel */
#define QUERY_TILE 32  /* prefill64.rs:58 */
#define KEY_TILE 128   /* prefill64.rs:60 */
#define DEC_TILE 128   /* src/quant/kv.rs:64 */
#define RECORD 160     /* src/quant/kv.rs:55 */
#define TAIL_RECORD 128 /* src/quant/kv.rs:60 */
#define MAX_CHUNKS 4   /* src/quant/kv.rs:66 */
#define MAX_ROWS 8     /* src/quant/kv.rs:68 */

static const float NEG_INF = -INFINITY;

void fo_or_set_threads(int threads) {
#ifdef _OPENMP
    if (threads > 0) omp_set_num_threads(threads);
#else
    (void)threads;
#endif
}

int fo_or_max_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

static inline float from_bits(uint32_t u) {
    float f;
    memcpy(&f, &u, 4);
    return f;
}
static inline uint32_t to_bits(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    return u;
}

/* ------------------------------------------------------------------ */
/* codec: src/quant/kv/codec.rs                                         */
/* ------------------------------------------------------------------ */

/* codec.rs:37-44: smallest BF16 at or above a positive finite scale, 0 or NaN. */
uint16_t fo_or_bf16_up(float scale) {
    if (isnan(scale)) return 0x7FC0;
    uint32_t bits = to_bits(scale);
    uint16_t high = (uint16_t)(bits >> 16);
    return (bits & 0xFFFF) ? (uint16_t)(high + 1) : high;
}

/* codec.rs:48-50 */
float fo_or_bf16_f32(uint16_t bits) { return from_bits((uint32_t)bits << 16); }

/* half::bf16::from_f32 / vcvtneps2bf16: round to nearest even, NaN kept quiet
 * (prefill64/bf16.rs:190-223 rounds every operand and probability this way). */
uint16_t fo_or_bf16_rne(float x) {
    uint32_t u = to_bits(x);
    if ((u & 0x7FFFFFFFu) > 0x7F800000u) return (uint16_t)((u >> 16) | 0x40);
    u += 0x7FFFu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

static inline float bf16_round(float x) { return fo_or_bf16_f32(fo_or_bf16_rne(x)); }

static float absmax(const float *values, int64_t n) {
    float m = 0.0f;
    for (int64_t i = 0; i < n; i++) m = fmaxf(m, fabsf(values[i])); /* Rust f32::max ignores NaN */
    return m;
}

/* codec.rs:11-21 */
float fo_or_q8_scale(const float *values, int64_t n) {
    float max = absmax(values, n);
    if (max == 0.0f) return 0.0f;
    float s = (float)((double)max / 127.0);
    float tiny = from_bits(1);
    return s > tiny ? s : tiny;
}

/* codec.rs:25-32 */
float fo_or_q16_scale(const float *values, int64_t n) {
    float max = absmax(values, n);
    if (max == 0.0f) return 0.0f;
    float s = (float)((double)max / 32767.0);
    float tiny = from_bits(1);
    return s > tiny ? s : tiny;
}

/* codec.rs:60-63: clamp, then the 1.5*2^52 shift rounds ties to even. */
double fo_or_round_clamped(double x, double limit) {
    if (isnan(x)) return x;
    const double SHIFT = 6755399441055744.0;
    double c = x < -limit ? -limit : (x > limit ? limit : x);
    volatile double t = c + SHIFT; /* keep the two roundings separate */
    return t - SHIFT;
}

/* Rust `f64 as iN`: saturating, NaN -> 0. */
static inline int64_t rust_as_int(double x) {
    if (isnan(x)) return 0;
    return (int64_t)x;
}

/* codec.rs:77-83 */
int8_t fo_or_q8_code(float value, float scale) {
    if (scale == 0.0f) return 0;
    return (int8_t)rust_as_int(fo_or_round_clamped((double)value / (double)scale, 127.0));
}

/* codec.rs:67-73 */
int16_t fo_or_q16_code(float value, float scale) {
    if (scale == 0.0f) return 0;
    return (int16_t)rust_as_int(fo_or_round_clamped((double)value / (double)scale, 32767.0));
}

/* ------------------------------------------------------------------ */
/* exp: src/kernels/exp.rs:232-277 (the reference's published constants) */
/* ------------------------------------------------------------------ */
static const float EXP_LOG2E = 1.44269504088896340736f; /* std::f32::consts::LOG2_E */
static const float EXP_LN2_HI = 0.6933594f;
static const float EXP_LN2_LO = -2.1219444e-4f;
static const float EXP_P[6] = {1.9875691e-4f, 1.3981999e-3f, 8.333452e-3f, 4.1665796e-2f, 0.16666665f, 0.5f};
static const float EXP_MIN = -87.0f;
static const float EXP_MAX = 88.376f;

float fo_or_exp_poly_unchecked(float x) {
    float n = rintf(x * EXP_LOG2E); /* round_ties_even (default rounding mode) */
    float r = fmaf(n, -EXP_LN2_HI, x);
    r = fmaf(n, -EXP_LN2_LO, r);
    float p = EXP_P[0];
    for (int i = 1; i < 6; i++) p = fmaf(p, r, EXP_P[i]);
    float rr = r * r;
    float y = fmaf(p, rr, r) + 1.0f;
    int32_t e = (int32_t)n + 127;
    return y * from_bits((uint32_t)e << 23);
}

float fo_or_exp_poly(float x) {
    if (isnan(x)) return x;
    if (x < EXP_MIN) return 0.0f;
    if (x > EXP_MAX) return INFINITY;
    return fo_or_exp_poly_unchecked(x);
}

static inline float exp_sel(float x, int fast) { return fast ? fo_or_exp_poly(x) : expf(x); }

/* bf16/static_shift.rs:36-38, 322-336: 2^t with the degree-3 minimax 2^f. */
static const float EXP2_C[4] = {0.99992806f, 0.69326097f, 0.24261113f, 0.05517167f};
static inline float exp2_static(float t) {
    float n = rintf(t);
    float f = t - n;
    float p = EXP2_C[3];
    p = fmaf(p, f, EXP2_C[2]);
    p = fmaf(p, f, EXP2_C[1]);
    p = fmaf(p, f, EXP2_C[0]);
    return ldexpf(p, (int)n); /* vscalefps: exact while |t| < 126 */
}

/* ------------------------------------------------------------------ */
/* Geometry (src/kernels/attention/mod.rs:35-76)                        */
/* ------------------------------------------------------------------ */
typedef struct {
    int64_t query_offset, image_start, image_end;
} geometry_t;

static inline int in_image(const geometry_t *g, int64_t p) { return p >= g->image_start && p < g->image_end; }
static inline int64_t visible_end(const geometry_t *g, int64_t absolute) {
    return in_image(g, absolute) ? g->image_end : absolute + 1;
}
static inline int masked(const geometry_t *g, int64_t absolute, int64_t key) {
    return key > absolute && !(in_image(g, absolute) && in_image(g, key));
}

/* The compact KV view (mod.rs:84-157). */
typedef struct {
    const float *prefix_k, *generated_k, *v;
    int64_t prefix_len, total_len, n_heads, n_kv_heads, head_dim;
} compact_t;

static inline const float *key_at(const compact_t *kv, int64_t position, int64_t head) {
    if (position < kv->prefix_len) return kv->prefix_k + (position * kv->n_heads + head) * kv->head_dim;
    int64_t repeat = kv->n_heads / kv->n_kv_heads;
    return kv->generated_k + ((position - kv->prefix_len) * kv->n_kv_heads + head / repeat) * kv->head_dim;
}
static inline const float *value_at(const compact_t *kv, int64_t position, int64_t kv_head) {
    return kv->v + (position * kv->n_kv_heads + kv_head) * kv->head_dim;
}

/* ------------------------------------------------------------------ */
/* dense f64 reference: src/kernels/tests.rs:204-248                    */
/* ------------------------------------------------------------------ */
void fo_or_attention_f64(const float *q, const float *prefix_k, const float *generated_k, const float *v,
                         int64_t query_len, int64_t prefix_len, int64_t total_len, int64_t n_heads,
                         int64_t n_kv_heads, int64_t head_dim, int64_t query_offset, int64_t image_start,
                         int64_t image_end, const float *sinks, int bf16_operands, double *out) {
    compact_t kv = {prefix_k, generated_k, v, prefix_len, total_len, n_heads, n_kv_heads, head_dim};
    geometry_t g = {query_offset, image_start, image_end};
    int64_t repeat = n_heads / n_kv_heads;
#pragma omp parallel for schedule(dynamic)
    for (int64_t qh = 0; qh < query_len * n_heads; qh++) {
        int64_t query = qh / n_heads, head = qh % n_heads, kv_head = head / repeat;
        int64_t absolute = query_offset + query;
        double *scores = (double *)malloc(sizeof(double) * (size_t)(total_len > 0 ? total_len : 1));
        const float *qv = q + qh * head_dim;
        double sink = (double)sinks[head];
        double max = sink;
        for (int64_t key = 0; key < total_len; key++) {
            if (masked(&g, absolute, key)) {
                scores[key] = -INFINITY;
                continue;
            }
            const float *kr = key_at(&kv, key, head);
            double s = 0.0;
            for (int64_t d = 0; d < head_dim; d++) {
                double a = bf16_operands ? bf16_round(qv[d]) : qv[d];
                double b = bf16_operands ? bf16_round(kr[d]) : kr[d];
                s += a * b;
            }
            scores[key] = s / sqrt((double)head_dim);
            if (scores[key] > max) max = scores[key];
        }
        double denom = exp(sink - max);
        for (int64_t key = 0; key < total_len; key++) denom += exp(scores[key] - max);
        for (int64_t d = 0; d < head_dim; d++) {
            double sum = 0.0;
            for (int64_t key = 0; key < total_len; key++) {
                if (scores[key] == -INFINITY) continue;
                double val = value_at(&kv, key, kv_head)[d];
                if (bf16_operands) val = bf16_round((float)val);
                sum += exp(scores[key] - max) / denom * val;
            }
            out[qh * head_dim + d] = sum;
        }
        free(scores);
    }
}

/* ------------------------------------------------------------------ */
/* dot / axpy in the AVX2 order: src/simd.rs:743-776, 920-940          */
/* ------------------------------------------------------------------ */
static float dot_ref(const float *a, const float *b, int64_t n) {
    float acc[4][8] = {{0}};
    int64_t i = 0;
    for (; i + 32 <= n; i += 32)
        for (int j = 0; j < 4; j++)
            for (int l = 0; l < 8; l++) acc[j][l] = fmaf(a[i + 8 * j + l], b[i + 8 * j + l], acc[j][l]);
    float s[8];
    for (int l = 0; l < 8; l++) s[l] = (acc[0][l] + acc[1][l]) + (acc[2][l] + acc[3][l]);
    for (; i + 8 <= n; i += 8)
        for (int l = 0; l < 8; l++) s[l] = fmaf(a[i + l], b[i + l], s[l]);
    /* Simd::sum: ((v0+v4) + (v1+v5)) + ((v2+v6) + (v3+v7)) (simd.rs:76-80) */
    float total = ((s[0] + s[4]) + (s[1] + s[5])) + ((s[2] + s[6]) + (s[3] + s[7]));
    for (; i < n; i++) total += a[i] * b[i];
    return total;
}

static void axpy_ref(float a, const float *x, float *y, int64_t n) {
    int64_t i = 0;
    for (; i + 8 <= n; i += 8)
        for (int l = 0; l < 8; l++) y[i + l] = fmaf(a, x[i + l], y[i + l]);
    for (; i < n; i++) y[i] += a * x[i];
}

/* ------------------------------------------------------------------ */
/* online head: src/kernels/attention/online.rs:89-169                  */
/* ------------------------------------------------------------------ */
void fo_or_attention_online(const float *q, const float *prefix_k, const float *generated_k, const float *v,
                            int64_t query_len, int64_t prefix_len, int64_t total_len, int64_t n_heads,
                            int64_t n_kv_heads, int64_t head_dim, int64_t query_offset, int64_t image_start,
                            int64_t image_end, const float *sinks, int exp_fast, float *output) {
    compact_t kv = {prefix_k, generated_k, v, prefix_len, total_len, n_heads, n_kv_heads, head_dim};
    geometry_t g = {query_offset, image_start, image_end};
    const float scale = 1.0f / sqrtf((float)head_dim); /* (head_dim as f32).sqrt().recip() */
    int64_t repeat = n_heads / n_kv_heads;
#pragma omp parallel for schedule(dynamic)
    for (int64_t qh = 0; qh < query_len * n_heads; qh++) {
        int64_t query = qh / n_heads, head = qh % n_heads, kv_head = head / repeat;
        int64_t absolute = query_offset + query;
        int64_t vend = visible_end(&g, absolute);
        const float *qvec = q + qh * head_dim;
        float *out = output + qh * head_dim;
        for (int64_t d = 0; d < head_dim; d++) out[d] = 0.0f;
        float running_max = NEG_INF, denominator = 0.0f;
        float logits[DEC_TILE];
        for (int64_t start = 0; start < vend; start += DEC_TILE) {
            int64_t len = vend - start < DEC_TILE ? vend - start : DEC_TILE;
            float block_max = NEG_INF;
            for (int64_t j = 0; j < len; j++) {
                logits[j] = dot_ref(qvec, key_at(&kv, start + j, head), head_dim) * scale;
                block_max = fmaxf(block_max, logits[j]);
            }
            float new_max = fmaxf(running_max, block_max);
            float rescale = running_max == NEG_INF ? 0.0f : expf(running_max - new_max);
            for (int64_t d = 0; d < head_dim; d++) out[d] *= rescale;
            denominator *= rescale;
            for (int64_t j = 0; j < len; j++) logits[j] = exp_sel(logits[j] - new_max, exp_fast);
            for (int64_t j = 0; j < len; j++) {
                denominator += logits[j];
                axpy_ref(logits[j], value_at(&kv, start + j, kv_head), out, head_dim);
            }
            running_max = new_max;
        }
        float logsumexp = running_max + logf(denominator);
        float sink_scale = 1.0f / (1.0f + expf(sinks[head] - logsumexp));
        for (int64_t d = 0; d < head_dim; d++) out[d] = (out[d] / denominator) * sink_scale;
    }
}

/* ------------------------------------------------------------------ */
/* prefill tiles: src/kernels/attention/prefill64.rs                    */
/* ------------------------------------------------------------------ */
typedef struct {
    int64_t query_width, kv_width, query_offset, image_start, image_end;
    float scale;
} shape_t;

/* span.rs:9-20 */
static void tile_span(const shape_t *s, int64_t first_query, int64_t queries, int64_t *first_absolute,
                      int64_t *vend, int *all_image) {
    int64_t fa = s->query_offset + first_query;
    int64_t la = fa + queries - 1;
    int intersects = fa < s->image_end && la >= s->image_start;
    int64_t ve = la + 1;
    if (intersects && s->image_end > ve) ve = s->image_end;
    *first_absolute = fa;
    *vend = ve;
    *all_image = fa >= s->image_start && la < s->image_end;
}

/* prefill64.rs:549-567 */
static void mask_lanes(const shape_t *s, int64_t first_absolute, int64_t queries, int64_t key_start,
                       int64_t keys, float *st) {
    for (int64_t r = 0; r < queries; r++) {
        int64_t absolute = first_absolute + r;
        int image_query = absolute >= s->image_start && absolute < s->image_end;
        for (int64_t j = 0; j < keys; j++) {
            int64_t key = key_start + j;
            if (key > absolute && !(image_query && key >= s->image_start && key < s->image_end))
                st[j * QUERY_TILE + r] = NEG_INF;
        }
    }
}

/* x86 maxps(a, b): b when either is NaN (simd.rs:108-113) */
static inline float maxps(float a, float b) { return a > b ? a : b; }

/* prefill64.rs:574-652: per-lane online softmax, probabilities over st. */
static void softmax_lanes(int64_t queries, int64_t keys, float *st, float *maxima, float *denominators,
                          float *out, int64_t out_stride, int exp_fast) {
    for (int64_t r = 0; r < queries; r++) {
        float block_max = NEG_INF;
        for (int64_t j = 0; j < keys; j++) block_max = maxps(st[j * QUERY_TILE + r], block_max);
        float old_max = maxima[r];
        float new_max = maxps(block_max, old_max);
        int skip = new_max == NEG_INF;
        int first = old_max == NEG_INF;
        float rescale = exp_sel(old_max - new_max, exp_fast);
        if (first) rescale = 0.0f;
        if (skip) rescale = 1.0f;
        if (!skip && rescale != 1.0f) {
            float *row = out + r * out_stride;
            for (int d = 0; d < HD; d++) row[d] *= rescale;
        }
        float denominator = denominators[r] * rescale;
        for (int64_t j = 0; j < keys; j++) {
            float p = skip ? 0.0f : exp_sel(st[j * QUERY_TILE + r] - new_max, exp_fast);
            denominator = denominator + p;
            st[j * QUERY_TILE + r] = p;
        }
        denominators[r] = denominator;
        maxima[r] = skip ? old_max : new_max;
    }
}

/* static_shift.rs:135-161 */
static void exp_lanes_static(int64_t queries, int64_t keys, int all_image, float *st, float *denominators) {
    for (int64_t r = 0; r < queries; r++) {
        float sum = denominators[r];
        for (int64_t j = 0; j < keys; j++) {
            float score = st[j * QUERY_TILE + r];
            float p = fo_or_exp_poly_unchecked(score);
            if (!all_image && score == NEG_INF) p = 0.0f;
            sum = sum + p;
            st[j * QUERY_TILE + r] = p;
        }
        denominators[r] = sum;
    }
}

/* prefill64.rs:487-545: st[key][query] = scale * (FMA chain over d from +0) */
static void qk_lanes(const float *qt, const float *k, int64_t k_stride, int64_t keys, float scale, float *st) {
    for (int64_t j = 0; j < keys; j++) {
        const float *kr = k + j * k_stride;
        float acc[QUERY_TILE];
        for (int r = 0; r < QUERY_TILE; r++) acc[r] = 0.0f;
        for (int d = 0; d < HD; d++) {
            float kd = kr[d];
#pragma omp simd
            for (int r = 0; r < QUERY_TILE; r++) acc[r] = fmaf(qt[d * QUERY_TILE + r], kd, acc[r]);
        }
        for (int r = 0; r < QUERY_TILE; r++) st[j * QUERY_TILE + r] = scale * acc[r];
    }
}

/* prefill64.rs:657-715: out[q][d] = (FMA chain over keys from +0) + out */
static void pv_lanes(const float *st, int64_t queries, int64_t keys, const float *v, int64_t v_stride,
                     float *out, int64_t out_stride) {
    for (int64_t r = 0; r < queries; r++) {
        float acc[HD];
        for (int d = 0; d < HD; d++) acc[d] = 0.0f;
        for (int64_t j = 0; j < keys; j++) {
            float p = st[j * QUERY_TILE + r];
            const float *vr = v + j * v_stride;
#pragma omp simd
            for (int d = 0; d < HD; d++) acc[d] = fmaf(vr[d], p, acc[d]);
        }
        float *row = out + r * out_stride;
        for (int d = 0; d < HD; d++) row[d] = acc[d] + row[d];
    }
}

/* prefill64.rs:328-480 for a pure prefix (total == prefix). */
static void tile_head_f32(const float *q, const float *k, const float *v, const shape_t *s, int64_t tile,
                          int64_t queries, int64_t head, int64_t kv_head, const float *sinks, float *output,
                          int softmax_static, int exp_fast) {
    int64_t first_query = tile * QUERY_TILE, first_absolute, vend;
    int all_image;
    tile_span(s, first_query, queries, &first_absolute, &vend, &all_image);
    float qt[HD * QUERY_TILE];
    memset(qt, 0, sizeof qt);
    for (int64_t r = 0; r < queries; r++) {
        const float *row = q + (first_query + r) * s->query_width + head * HD;
        for (int d = 0; d < HD; d++) qt[d * QUERY_TILE + r] = row[d];
    }
    float maxima[QUERY_TILE], denominators[QUERY_TILE];
    for (int r = 0; r < QUERY_TILE; r++) {
        maxima[r] = NEG_INF;
        denominators[r] = 0.0f;
    }
    float *out = output + first_query * s->query_width + head * HD;
    for (int64_t r = 0; r < queries; r++) memset(out + r * s->query_width, 0, HD * sizeof(float));
    float st[KEY_TILE * QUERY_TILE];
    for (int64_t key_start = 0; key_start < vend; key_start += KEY_TILE) {
        int64_t keys = vend - key_start < KEY_TILE ? vend - key_start : KEY_TILE;
        const float *krows = k + key_start * s->query_width + head * HD;
        const float *vrows = v + key_start * s->kv_width + kv_head * HD;
        qk_lanes(qt, krows, s->query_width, keys, s->scale, st);
        if (!all_image) mask_lanes(s, first_absolute, queries, key_start, keys, st);
        if (softmax_static)
            exp_lanes_static(queries, keys, all_image, st, denominators);
        else
            softmax_lanes(queries, keys, st, maxima, denominators, out, s->query_width, exp_fast);
        pv_lanes(st, queries, keys, vrows, s->kv_width, out, s->query_width);
    }
    for (int64_t r = 0; r < queries; r++) {
        float *row = out + r * s->query_width;
        float lse = softmax_static ? logf(denominators[r]) : maxima[r] + logf(denominators[r]);
        float sink_scale = 1.0f / (1.0f + expf(sinks[head] - lse));
        for (int d = 0; d < HD; d++) row[d] = (row[d] / denominators[r]) * sink_scale;
    }
}

/* prefill64.rs:179-214: KV group by KV group, tasks (tile, pair). */
void fo_or_prefill64(const float *q, const float *k, const float *v, int64_t query_len, int64_t n_heads,
                     int64_t n_kv_heads, int64_t query_offset, int64_t image_start, int64_t image_end,
                     const float *sinks, int softmax_static, int exp_fast, float *out) {
    shape_t s = {n_heads * HD, n_kv_heads * HD, query_offset, image_start, image_end, 0.125f};
    int64_t repeat = n_heads / n_kv_heads;
    int64_t tiles = (query_len + QUERY_TILE - 1) / QUERY_TILE;
    for (int64_t kv_head = 0; kv_head < n_kv_heads; kv_head++) {
#pragma omp parallel for schedule(dynamic)
        for (int64_t task = 0; task < tiles * repeat; task++) {
            int64_t tile = task / repeat, pair = task % repeat;
            int64_t head = kv_head * repeat + pair;
            int64_t queries = query_len - tile * QUERY_TILE < QUERY_TILE ? query_len - tile * QUERY_TILE : QUERY_TILE;
            tile_head_f32(q, k, v, &s, tile, queries, head, kv_head, sinks, out, softmax_static, exp_fast);
        }
    }
}

/* ------------------------------------------------------------------ */
/* BF16 prefill tiles: prefill64/bf16.rs, prefill64/bf16/static_shift.rs */
/* ------------------------------------------------------------------ */

/* prefill64.rs:65-73: gemm's main microkernel path */
static inline int main_path(int64_t queries, int64_t keys) {
    return queries * keys > 16 * 16 && keys >= 3 && queries >= 2;
}

/* vdpbf16ps per element pair: acc += a_odd*b_odd; acc += a_even*b_even.
 * BF16 products are exact in FP32, so each step is one FMA rounding. */
static inline float dp_pair(float acc, float a_even, float a_odd, float b_even, float b_odd) {
    acc = fmaf(a_odd, b_odd, acc);
    return fmaf(a_even, b_even, acc);
}

/* bf16.rs:565-595: scale * (dpbf16 chain over the 32 pairs) */
static void qk_lanes_bf16(const float *qb /* [64][32] */, const float *kb /* [keys][64] */, int64_t keys,
                          float scale, float *st) {
    for (int64_t j = 0; j < keys; j++) {
        const float *kr = kb + j * HD;
        float acc[QUERY_TILE];
        for (int r = 0; r < QUERY_TILE; r++) acc[r] = 0.0f;
        for (int p = 0; p < HD / 2; p++) {
            float ke = kr[2 * p], ko = kr[2 * p + 1];
#pragma omp simd
            for (int r = 0; r < QUERY_TILE; r++)
                acc[r] = dp_pair(acc[r], qb[(2 * p) * QUERY_TILE + r], qb[(2 * p + 1) * QUERY_TILE + r], ke, ko);
        }
        for (int r = 0; r < QUERY_TILE; r++) st[j * QUERY_TILE + r] = scale * acc[r];
    }
}

/* bf16.rs:600-660: out += dpbf16 chain over key pairs (odd key of a short
 * last pair is a zero probability). pb holds BF16-rounded probabilities. */
static void pv_lanes_bf16(const float *pb /* [keys_padded][32] */, int64_t queries, int64_t keys,
                          const float *vb /* [keys_padded][64] */, float *out, int64_t out_stride) {
    int64_t key_pairs = (keys + 1) / 2;
    for (int64_t r = 0; r < queries; r++) {
        float acc[HD];
        for (int d = 0; d < HD; d++) acc[d] = 0.0f;
        for (int64_t kp = 0; kp < key_pairs; kp++) {
            float pe = pb[(2 * kp) * QUERY_TILE + r];
            float po = 2 * kp + 1 < keys ? pb[(2 * kp + 1) * QUERY_TILE + r] : 0.0f;
            const float *ve = vb + (2 * kp) * HD, *vo = vb + (2 * kp + 1) * HD;
#pragma omp simd
            for (int d = 0; d < HD; d++) acc[d] = dp_pair(acc[d], pe, po, ve[d], vo[d]);
        }
        float *row = out + r * out_stride;
        for (int d = 0; d < HD; d++) row[d] = acc[d] + row[d];
    }
}

/* prefill64.rs:887-982 restated for the short tiles of the online BF16
 * kernel: FP32 operands, the same mask and per-row online softmax. */
static void short_tile_f32(const float *q, const float *k, const float *v, const shape_t *s, int64_t first_query,
                           int64_t first_absolute, int64_t queries, int64_t key_start, int64_t keys, int64_t head,
                           int64_t kv_head, float *maxima, float *denominators, float *out) {
    float st[KEY_TILE * QUERY_TILE];
    float qt[HD * QUERY_TILE];
    memset(qt, 0, sizeof qt);
    for (int64_t r = 0; r < queries; r++)
        for (int d = 0; d < HD; d++) qt[d * QUERY_TILE + r] = q[(first_query + r) * s->query_width + head * HD + d];
    qk_lanes(qt, k + key_start * s->query_width + head * HD, s->query_width, keys, s->scale, st);
    mask_lanes(s, first_absolute, queries, key_start, keys, st);
    softmax_lanes(queries, keys, st, maxima, denominators, out, s->query_width, 0);
    pv_lanes(st, queries, keys, v + key_start * s->kv_width + kv_head * HD, s->kv_width, out, s->query_width);
}

static void tile_head_bf16(const float *q, const float *k, const float *v, const float *kb_head /* [T][64] */,
                           const float *vb_head /* [T+1][64] */, const shape_t *s, int64_t tile, int64_t queries,
                           int64_t head, int64_t kv_head, const float *sinks, float *output, int softmax_static,
                           int exp_fast) {
    int64_t first_query = tile * QUERY_TILE, first_absolute, vend;
    int all_image;
    tile_span(s, first_query, queries, &first_absolute, &vend, &all_image);
    float qb[HD * QUERY_TILE];
    memset(qb, 0, sizeof qb);
    for (int64_t r = 0; r < queries; r++)
        for (int d = 0; d < HD; d++)
            qb[d * QUERY_TILE + r] = bf16_round(q[(first_query + r) * s->query_width + head * HD + d]);
    float maxima[QUERY_TILE], denominators[QUERY_TILE];
    for (int r = 0; r < QUERY_TILE; r++) {
        maxima[r] = NEG_INF;
        denominators[r] = 0.0f;
    }
    float *out = output + first_query * s->query_width + head * HD;
    for (int64_t r = 0; r < queries; r++) memset(out + r * s->query_width, 0, HD * sizeof(float));
    float st[(KEY_TILE + 1) * QUERY_TILE];
    const float exponent_scale = EXP_LOG2E * s->scale; /* bf16/static_shift.rs:177-179 */
    for (int64_t key_start = 0; key_start < vend; key_start += KEY_TILE) {
        int64_t keys = vend - key_start < KEY_TILE ? vend - key_start : KEY_TILE;
        const float *kb = kb_head + key_start * HD;
        const float *vb = vb_head + key_start * HD;
        if (softmax_static) {
            /* bf16/static_shift.rs:263-311: p = 2^(scale*log2e*acc), masked
             * lanes +0, rounded to BF16; denominators sum rounded p. */
            qk_lanes_bf16(qb, kb, keys, 1.0f, st);
            for (int64_t r = 0; r < queries; r++) {
                int64_t absolute = first_absolute + r;
                float sum = denominators[r];
                for (int64_t j = 0; j < keys; j++) {
                    int visible = all_image || !masked(&(geometry_t){s->query_offset, s->image_start, s->image_end},
                                                       absolute, key_start + j);
                    float p = visible ? exp2_static(exponent_scale * st[j * QUERY_TILE + r]) : 0.0f;
                    p = bf16_round(p);
                    sum = sum + p;
                    st[j * QUERY_TILE + r] = p;
                }
                denominators[r] = sum;
            }
            pv_lanes_bf16(st, queries, keys, vb, out, s->query_width);
        } else if (main_path(queries, keys)) {
            qk_lanes_bf16(qb, kb, keys, s->scale, st);
            if (!all_image) mask_lanes(s, first_absolute, queries, key_start, keys, st);
            /* bf16.rs:327-356: the fused (fast) and separate softmaxes both
             * sum unrounded probabilities, then round them for PV. */
            softmax_lanes(queries, keys, st, maxima, denominators, out, s->query_width, exp_fast);
            for (int64_t j = 0; j < keys; j++)
                for (int64_t r = 0; r < queries; r++) st[j * QUERY_TILE + r] = bf16_round(st[j * QUERY_TILE + r]);
            pv_lanes_bf16(st, queries, keys, vb, out, s->query_width);
        } else {
            short_tile_f32(q, k, v, s, first_query, first_absolute, queries, key_start, keys, head, kv_head, maxima,
                           denominators, out);
        }
    }
    for (int64_t r = 0; r < queries; r++) {
        float *row = out + r * s->query_width;
        float lse = softmax_static ? logf(denominators[r]) : maxima[r] + logf(denominators[r]);
        float sink_scale = 1.0f / (1.0f + expf(sinks[head] - lse));
        for (int d = 0; d < HD; d++) row[d] = (row[d] / denominators[r]) * sink_scale;
    }
}

/* bf16.rs:78-178 */
void fo_or_prefill_bf16(const float *q, const float *k, const float *v, int64_t query_len, int64_t n_heads,
                        int64_t n_kv_heads, int64_t image_start, int64_t image_end, const float *sinks,
                        int softmax_static, int exp_fast, float *out) {
    shape_t s = {n_heads * HD, n_kv_heads * HD, 0, image_start, image_end, 0.125f};
    int64_t total = query_len;
    /* BF16 copies, head-major with one zero row past the end for the odd key
     * of a short last pair (bf16.rs:126-137 zero-fills the missing odd row). */
    float *kb = (float *)calloc((size_t)(n_heads * (total + 1) * HD), sizeof(float));
    float *vb = (float *)calloc((size_t)(n_kv_heads * (total + 1) * HD), sizeof(float));
#pragma omp parallel for
    for (int64_t t = 0; t < total; t++) {
        for (int64_t h = 0; h < n_heads; h++)
            for (int d = 0; d < HD; d++) kb[(h * (total + 1) + t) * HD + d] = bf16_round(k[(t * n_heads + h) * HD + d]);
        for (int64_t g = 0; g < n_kv_heads; g++)
            for (int d = 0; d < HD; d++)
                vb[(g * (total + 1) + t) * HD + d] = bf16_round(v[(t * n_kv_heads + g) * HD + d]);
    }
    int64_t repeat = n_heads / n_kv_heads;
    int64_t tiles = (query_len + QUERY_TILE - 1) / QUERY_TILE;
    for (int64_t kv_head = 0; kv_head < n_kv_heads; kv_head++) {
#pragma omp parallel for schedule(dynamic)
        for (int64_t task = 0; task < tiles * repeat; task++) {
            int64_t tile = task / repeat, pair = task % repeat;
            int64_t head = kv_head * repeat + pair;
            int64_t queries = query_len - tile * QUERY_TILE < QUERY_TILE ? query_len - tile * QUERY_TILE : QUERY_TILE;
            tile_head_bf16(q, k, v, kb + head * (total + 1) * HD, vb + kv_head * (total + 1) * HD, &s, tile, queries,
                           head, kv_head, sinks, out, softmax_static, exp_fast);
        }
    }
    free(kb);
    free(vb);
}

/* ------------------------------------------------------------------ */
/* rotation of 32-value blocks: src/quant/rotation.rs                   */
/* ------------------------------------------------------------------ */
/* SplitMix64's output function (rotation.rs:36-40). */
static uint64_t splitmix64_mix(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
    return z ^ (z >> 31);
}

/* rotation.rs:42-61: the low 32 bits of the SplitMix64 outputs for states
 * SEED + (kind + 1) * GAMMA, SEED = "KVROTATE" read big-endian. */
uint32_t fo_or_rotation_signs(int kind) {
    const uint64_t seed = 0x4b56524f54415445ull; /* 'K' 'V' 'R' 'O' 'T' 'A' 'T' 'E' */
    const uint64_t gamma = 0x9e3779b97f4a7c15ull;
    return (uint32_t)splitmix64_mix(seed + (uint64_t)(kind + 1) * gamma);
}

/* rotation.rs:71-84: five stages of FP32 butterflies, half = 1, 2, .., 16;
 * x[i] = a + b, x[i + half] = a - b. */
void fo_or_fwht32(float *x) {
    for (int half = 1; half < 32; half *= 2)
        for (int start = 0; start < 32; start += 2 * half)
            for (int i = start; i < start + half; i++) {
                const float a = x[i], b = x[i + half];
                x[i] = a + b;
                x[i + half] = a - b;
            }
}

/* rotation.rs:87-92: sign-bit flips (exact, NaN included). */
static void flip32(float *x, uint32_t signs) {
    for (int i = 0; i < 32; i++) {
        uint32_t u;
        memcpy(&u, &x[i], 4);
        u ^= ((signs >> i) & 1u) << 31;
        memcpy(&x[i], &u, 4);
    }
}

static void scale32(float *x) {
    for (int i = 0; i < 32; i++) x[i] *= 1.0f / 32.0f;
}

void fo_or_rotate(float *x, int kind) {
    flip32(x, fo_or_rotation_signs(kind));
    fo_or_fwht32(x);
}

void fo_or_rotate_query(float *x, int kind) {
    fo_or_rotate(x, kind);
    scale32(x);
}

void fo_or_unrotate(float *x, int kind) {
    fo_or_fwht32(x);
    flip32(x, fo_or_rotation_signs(kind));
    scale32(x);
}

/* Block kinds of a prefix record [T | S | S | V0 | V1] and of a tail record
 * [T | S | V0 | V1] (kv.rs:72-81). */
static const int RECORD_KINDS[5] = {0, 1, 1, 2, 3};
static const int TAIL_KINDS[4] = {0, 1, 2, 3};

static int all_finite_block(const float *x) {
    for (int i = 0; i < 32; i++)
        if (!isfinite(x[i])) return 0;
    return 1;
}

/* ---- Q4 codec (codec.rs:87-129) ---- */
static float q4_scale(const float *values) {
    float max = absmax(values, 32);
    if (max == 0.0f) return 0.0f;
    float s = (float)((double)max / 7.0);
    float tiny = from_bits(1);
    return s > tiny ? s : tiny;
}

/* codec.rs:98-104 */
static int8_t q4_code(float value, float scale) {
    if (scale == 0.0f) return 0;
    return (int8_t)rust_as_int(fo_or_round_clamped((double)value / (double)scale, 7.0));
}

/* codec.rs:110-122 */
uint16_t fo_or_q4_block(const float *values, uint8_t *codes) {
    const uint16_t stored = fo_or_bf16_up(all_finite_block(values) ? q4_scale(values) : NAN);
    const float scale = fo_or_bf16_f32(stored);
    for (int i = 0; i < 16; i++)
        codes[i] = (uint8_t)(((uint8_t)q4_code(values[2 * i], scale) & 0x0F) |
                             ((uint8_t)q4_code(values[2 * i + 1], scale) << 4));
    return stored;
}

/* codec.rs:127-129: the signed nibble (high 0: bits 0..4, 1: bits 4..8). */
int8_t fo_or_nibble(uint8_t byte, int high) {
    return (int8_t)((int8_t)(uint8_t)(byte << (4 - 4 * high)) >> 4);
}

/* ------------------------------------------------------------------ */
/* split cache: src/quant/kv.rs, src/quant/kv/decode.rs                 */
/* ------------------------------------------------------------------ */
static inline int all_finite(const float *x, int64_t n) {
    for (int64_t i = 0; i < n; i++)
        if (!isfinite(x[i])) return 0;
    return 1;
}

/* Encode one block of 32 values into `format` at element `at`
 * (kv.rs:318-331, 345-358 for the prefix; 471-501 for the tail). */
static int encode_block(const float *values, int format, void *codes, uint16_t *scales, int64_t at,
                        int nonfinite_to_nan) {
    switch (format) {
    case FO_OR_F32:
        memcpy((float *)codes + at, values, 32 * sizeof(float));
        return FO_OR_OK;
    case FO_OR_BF16:
        for (int i = 0; i < 32; i++) ((uint16_t *)codes)[at + i] = fo_or_bf16_rne(values[i]);
        return FO_OR_OK;
    case FO_OR_Q8:
    case FO_OR_Q16: {
        int q8 = format == FO_OR_Q8;
        float raw = (nonfinite_to_nan && !all_finite(values, 32)) ? NAN
                    : (q8 ? fo_or_q8_scale(values, 32) : fo_or_q16_scale(values, 32));
        uint16_t stored = fo_or_bf16_up(raw);
        scales[at / 32] = stored;
        float scale = fo_or_bf16_f32(stored);
        for (int i = 0; i < 32; i++) {
            if (q8) {
                int8_t c = fo_or_q8_code(values[i], scale);
                ((int8_t *)codes)[at + i] = c;
                if (!nonfinite_to_nan && !isfinite((float)c * scale)) return FO_OR_ERR_OVERFLOW;
            } else {
                int16_t c = fo_or_q16_code(values[i], scale);
                ((int16_t *)codes)[at + i] = c;
                if (!nonfinite_to_nan && !isfinite((float)c * scale)) return FO_OR_ERR_OVERFLOW;
            }
        }
        return FO_OR_OK;
    }
    case FO_OR_Q4: {
        /* kv.rs:374-385 (prefix: codes at most 7, so 7 * scale bounds them)
         * and kv.rs:503-508 (tail: a non-finite block gets a NaN scale) */
        float block[32];
        memcpy(block, values, sizeof block);
        if (!nonfinite_to_nan && !all_finite_block(block)) return FO_OR_ERR_NONFINITE;
        scales[at / 32] = fo_or_q4_block(block, (uint8_t *)codes + at / 2);
        if (!nonfinite_to_nan && !isfinite(7.0f * fo_or_bf16_f32(scales[at / 32]))) return FO_OR_ERR_OVERFLOW;
        return FO_OR_OK;
    }
    }
    return FO_OR_ERR_SHAPE;
}

/* kv.rs:239-418 (unrotated storages) */
int fo_or_kv_seal(const float *k, const float *v, int64_t prefix_len, int64_t capacity, int64_t heads,
                  int64_t groups, int64_t head_dim, int format, void *codes, uint16_t *scales) {
    if (!(head_dim == 64 && heads == 2 * groups && groups <= 8 && groups > 0)) return FO_OR_ERR_SHAPE;
    if (!(prefix_len > 0 && capacity >= prefix_len)) return FO_OR_ERR_CAPACITY;
    /* kv.rs:265-278: temporal halves bit-identical inside every pair */
    for (int64_t t = 0; t < prefix_len; t++)
        for (int64_t g = 0; g < groups; g++) {
            const float *a = k + (t * heads + 2 * g) * 64;
            if (memcmp(a, a + 64, 32 * sizeof(float)) != 0) return FO_OR_ERR_PAIR;
        }
    int status = FO_OR_OK;
    int64_t count = groups * prefix_len;
#pragma omp parallel for reduction(max : status)
    for (int64_t record = 0; record < count; record++) {
        int64_t g = record / prefix_len, t = record % prefix_len;
        const float *a = k + (t * heads + 2 * g) * 64, *b = a + 64;
        const float *val = v + (t * groups + g) * 64;
        float dst[RECORD];
        memcpy(dst, a, 32 * sizeof(float));           /* T   0..32  */
        memcpy(dst + 32, a + 32, 32 * sizeof(float)); /* S0 32..64  */
        memcpy(dst + 64, b + 32, 32 * sizeof(float)); /* S1 64..96  */
        memcpy(dst + 96, val, 64 * sizeof(float));    /* V  96..160 */
        if (!all_finite(dst, RECORD)) {
            status = status > FO_OR_ERR_NONFINITE ? status : FO_OR_ERR_NONFINITE;
            continue;
        }
        /* kv.rs:289-293: rotated storage rotates every block after the pair
         * check (which saw the unrotated keys) and refuses an overflow */
        if (format & FO_OR_ROTATED) {
            for (int blk = 0; blk < RECORD / 32; blk++) fo_or_rotate(dst + 32 * blk, RECORD_KINDS[blk]);
            if (!all_finite(dst, RECORD)) {
                status = status > FO_OR_ERR_ROTATED ? status : FO_OR_ERR_ROTATED;
                continue;
            }
        }
        for (int blk = 0; blk < RECORD / 32; blk++) {
            int e = encode_block(dst + 32 * blk, format & ~FO_OR_ROTATED, codes, scales, record * RECORD + 32 * blk, 0);
            if (e > status) status = e;
        }
    }
    return status;
}

/* kv.rs:456-513 (push_unique): one generated position, keys/values [G][64]. */
void fo_or_kv_push(const float *k_unique, const float *v_unique, int64_t groups, int format, int64_t tail_capacity,
                   int64_t index, void *tail_codes, uint16_t *tail_scales) {
    for (int64_t g = 0; g < groups; g++) {
        float values[TAIL_RECORD];
        memcpy(values, k_unique + g * 64, 64 * sizeof(float));
        memcpy(values + 64, v_unique + g * 64, 64 * sizeof(float));
        int64_t record = g * tail_capacity + index;
        if (format & FO_OR_ROTATED) /* kv.rs:466-468 */
            for (int blk = 0; blk < TAIL_RECORD / 32; blk++) fo_or_rotate(values + 32 * blk, TAIL_KINDS[blk]);
        for (int blk = 0; blk < TAIL_RECORD / 32; blk++)
            encode_block(values + 32 * blk, format & ~FO_OR_ROTATED, tail_codes, tail_scales,
                         record * TAIL_RECORD + 32 * blk, 1);
    }
}

/* kv.rs:209-219 */
float fo_or_kv_value(const void *codes, const uint16_t *scales, int format, int64_t width, int64_t record,
                     int64_t offset) {
    int64_t at = record * width + offset;
    switch (format & ~FO_OR_ROTATED) {
    case FO_OR_Q4: return (float)fo_or_nibble(((const uint8_t *)codes)[at / 2], (int)(at % 2)) * fo_or_bf16_f32(scales[at / 32]);
    case FO_OR_F32: return ((const float *)codes)[at];
    case FO_OR_BF16: return fo_or_bf16_f32(((const uint16_t *)codes)[at]);
    case FO_OR_Q8: return (float)((const int8_t *)codes)[at] * fo_or_bf16_f32(scales[at / 32]);
    case FO_OR_Q16: return (float)((const int16_t *)codes)[at] * fo_or_bf16_f32(scales[at / 32]);
    }
    return NAN;
}

typedef struct {
    float out[2][64];
    float max[2];
    float denominator[2];
} partial_t;

typedef struct {
    const void *codes, *tail_codes;
    const uint16_t *scales, *tail_scales;
    int format;
    int64_t prefix_len, tail_capacity;
} store_t;

/* One record's key for both heads and its value (decode.rs:88-98, 246-299). */
static void load_key_value(const store_t *st, int64_t group, int64_t key, float k0[64], float k1[64], float val[64]) {
    if (key < st->prefix_len) {
        int64_t rec = group * st->prefix_len + key;
        for (int d = 0; d < 32; d++) {
            float t = fo_or_kv_value(st->codes, st->scales, st->format, RECORD, rec, d);
            k0[d] = t;
            k1[d] = t;
            k0[32 + d] = fo_or_kv_value(st->codes, st->scales, st->format, RECORD, rec, 32 + d);
            k1[32 + d] = fo_or_kv_value(st->codes, st->scales, st->format, RECORD, rec, 64 + d);
        }
        if (val)
            for (int d = 0; d < 64; d++) val[d] = fo_or_kv_value(st->codes, st->scales, st->format, RECORD, rec, 96 + d);
    } else {
        int64_t rec = group * st->tail_capacity + (key - st->prefix_len);
        for (int d = 0; d < 64; d++) {
            float kk = fo_or_kv_value(st->tail_codes, st->tail_scales, st->format, TAIL_RECORD, rec, d);
            k0[d] = kk;
            k1[d] = kk;
        }
        if (val)
            for (int d = 0; d < 64; d++)
                val[d] = fo_or_kv_value(st->tail_codes, st->tail_scales, st->format, TAIL_RECORD, rec, 64 + d);
    }
}

/* decode.rs:305-367: both heads of one group over [start, end). */
static void pair_span(const store_t *st, int64_t group, int64_t start, int64_t end, const float *q0, const float *q1,
                      int fast_exp, partial_t *part) {
    const float scale = 0.125f;
    memset(part->out, 0, sizeof part->out);
    float max[2] = {NEG_INF, NEG_INF}, den[2] = {0.0f, 0.0f};
    float logits[2][DEC_TILE];
    float k0[64], k1[64], val[64];
    while (start < end) {
        int64_t len = end - start < DEC_TILE ? end - start : DEC_TILE;
        float block_max[2] = {NEG_INF, NEG_INF};
        for (int64_t j = 0; j < len; j++) {
            load_key_value(st, group, start + j, k0, k1, NULL);
            logits[0][j] = dot_ref(q0, k0, 64) * scale;
            block_max[0] = fmaxf(block_max[0], logits[0][j]);
            logits[1][j] = dot_ref(q1, k1, 64) * scale;
            block_max[1] = fmaxf(block_max[1], logits[1][j]);
        }
        float new_max[2];
        for (int h = 0; h < 2; h++) {
            new_max[h] = fmaxf(max[h], block_max[h]);
            float rescale = max[h] == NEG_INF ? 0.0f : expf(max[h] - new_max[h]);
            for (int d = 0; d < 64; d++) part->out[h][d] *= rescale;
            den[h] *= rescale;
        }
        for (int h = 0; h < 2; h++)
            for (int64_t j = 0; j < len; j++) logits[h][j] = exp_sel(logits[h][j] - new_max[h], fast_exp);
        for (int64_t j = 0; j < len; j++) {
            float p0 = logits[0][j], p1 = logits[1][j];
            den[0] += p0;
            den[1] += p1;
            load_key_value(st, group, start + j, k0, k1, val);
            for (int d = 0; d < 64; d++) {
                part->out[0][d] = fmaf(p0, val[d], part->out[0][d]);
                part->out[1][d] = fmaf(p1, val[d], part->out[1][d]);
            }
        }
        max[0] = new_max[0];
        max[1] = new_max[1];
        start += len;
    }
    part->max[0] = max[0];
    part->max[1] = max[1];
    part->denominator[0] = den[0];
    part->denominator[1] = den[1];
}

/* kv.rs:775-813 */
static void merge_parts(const partial_t *parts, int64_t groups, int64_t chunks, const float *sinks, float *output) {
    for (int64_t g = 0; g < groups; g++) {
        const partial_t *gp = parts + g * chunks;
        for (int pair = 0; pair < 2; pair++) {
            int64_t h = 2 * g + pair;
            float *out = output + h * 64;
            float max, den;
            if (chunks == 1) {
                memcpy(out, gp[0].out[pair], 64 * sizeof(float));
                max = gp[0].max[pair];
                den = gp[0].denominator[pair];
            } else {
                max = NEG_INF;
                for (int64_t c = 0; c < chunks; c++) max = fmaxf(max, gp[c].max[pair]);
                den = 0.0f;
                memset(out, 0, 64 * sizeof(float));
                for (int64_t c = 0; c < chunks; c++) {
                    if (gp[c].max[pair] == NEG_INF) continue;
                    float factor = expf(gp[c].max[pair] - max);
                    den = fmaf(gp[c].denominator[pair], factor, den);
                    for (int d = 0; d < 64; d++) out[d] = fmaf(gp[c].out[pair][d], factor, out[d]);
                }
            }
            float lse = max + logf(den);
            float sink = 1.0f / (1.0f + expf(sinks[h] - lse));
            for (int d = 0; d < 64; d++) out[d] = (out[d] / den) * sink;
        }
    }
}

/* kv.rs:685-771 at one length: (group, chunk) tasks, then merge. */
static void decode_one(const store_t *st, int64_t total_len, int64_t heads, int64_t groups, const float *q,
                       const float *sinks, int64_t chunk_request, int fast_exp, float *out) {
    int64_t tiles = (total_len + DEC_TILE - 1) / DEC_TILE;
    int64_t chunks = chunk_request < 1 ? 1 : (chunk_request > MAX_CHUNKS ? MAX_CHUNKS : chunk_request);
    if (chunks > tiles) chunks = tiles;
    if (chunks < 1) chunks = 1;
    int64_t per_chunk = (tiles + chunks - 1) / chunks;
    partial_t parts[8 * MAX_CHUNKS];
#pragma omp parallel for schedule(static)
    for (int64_t index = 0; index < groups * chunks; index++) {
        int64_t g = index / chunks, c = index % chunks;
        int64_t start = c * per_chunk * DEC_TILE, end = (c + 1) * per_chunk * DEC_TILE;
        if (start > total_len) start = total_len;
        if (end > total_len) end = total_len;
        pair_span(st, g, start, end, q + 2 * g * 64, q + (2 * g + 1) * 64, fast_exp, &parts[index]);
    }
    (void)heads;
    merge_parts(parts, groups, chunks, sinks, out);
}

void fo_or_kv_decode_rows(const void *codes, const uint16_t *scales, const void *tail_codes,
                          const uint16_t *tail_scales, int format, int64_t prefix_len, int64_t tail_capacity,
                          int64_t tail_len, int64_t heads, int64_t groups, const float *q, int64_t rows,
                          const float *sinks, int64_t chunks, int fast_exp, float *out) {
    store_t st = {codes, tail_codes, scales, tail_scales, format, prefix_len, tail_capacity};
    int64_t last = prefix_len + tail_len;
    int64_t width = heads * 64;
    const int rotated = (format & FO_OR_ROTATED) != 0;
    float *qr = rotated ? (float *)malloc((size_t)width * sizeof(float)) : NULL;
    for (int64_t r = 0; r < rows; r++) {
        const float *qq = q + r * width;
        if (rotated) {
            /* kv.rs:83-96, 578-589: every head's query halves rotated
             * (rotate_query), the output's value halves un-rotated */
            memcpy(qr, qq, (size_t)width * sizeof(float));
            for (int64_t h = 0; h < heads; h++) {
                fo_or_rotate_query(qr + h * 64, 0);
                fo_or_rotate_query(qr + h * 64 + 32, 1);
            }
            qq = qr;
        }
        decode_one(&st, last + 1 + r - rows, heads, groups, qq, sinks, chunks, fast_exp, out + r * width);
        if (rotated)
            for (int64_t h = 0; h < heads; h++) {
                fo_or_unrotate(out + r * width + h * 64, 2);
                fo_or_unrotate(out + r * width + h * 64 + 32, 3);
            }
    }
    free(qr);
}

/* ------------------------------------------------------- fused QKV rows */
/* sum_squares_pairwise on one 32-value leaf (src/kernels/mod.rs:535-555):
 * squares, then partial[i] += partial[i + w] for w = 16, 8, 4, 2, 1. */
static float sum_squares_leaf32(const float *x) {
    float p[32];
    for (int i = 0; i < 32; i++) p[i] = x[i] * x[i];
    for (int w = 16; w >= 1; w >>= 1)
        for (int i = 0; i < w; i++) p[i] = p[i] + p[i + w];
    return p[0];
}

/* rms_norm_row (width 64: the tree splits at 32, mod.rs:537-541) and the
 * rotation of one head (fused.rs:104-113). */
static void norm_rope_head(const float *x, const float *rope, float *out) {
    const float sum = sum_squares_leaf32(x) + sum_squares_leaf32(x + 32);
    const float scale = 1.0f / sqrtf(sum / 64.0f + FLT_EPSILON);
    float y[64];
    for (int d = 0; d < 64; d++) y[d] = x[d] * scale;
    for (int p = 0; p < 32; p++) {
        const float c = rope[2 * p], s = rope[2 * p + 1], a = y[2 * p], b = y[2 * p + 1];
        out[2 * p] = a * c - b * s;
        out[2 * p + 1] = a * s + b * c;
    }
}

void fo_or_qkv_rows(const float *qkv, const float *rope, int64_t rows, int64_t heads, int64_t groups, float *q,
                    float *k, float *v) {
    const int64_t qdim = heads * 64, kdim = groups * 64, width = qdim + 2 * kdim, group = heads / groups;
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; r++) {
        const float *src = qkv + r * width;
        for (int64_t h = 0; h < heads; h++) {
            const float *f = rope + (r * heads + h) * 64;
            norm_rope_head(src + h * 64, f, q + (r * heads + h) * 64);
            norm_rope_head(src + qdim + (h / group) * 64, f, k + (r * heads + h) * 64);
        }
        memcpy(v + r * kdim, src + qdim + kdim, (size_t)kdim * sizeof(float));
    }
}

/* ------------------------------------------------------------------ */
/* draft-head KV: src/draft_head.rs (DraftState's Kv::Q8 and attend)    */
/* ------------------------------------------------------------------ */
#define DRAFT_KV_WIDTH 512 /* draft_head.rs:41: KV_HEADS * HEAD_DIM */

/* draft_head.rs:213-220: int8 codes with one absmax scale per 64 values,
 * (v * (127 / max)).round() clamped to +-127 (NaN codes 0). */
float fo_or_draft_quantize_row(const float *x, int8_t *codes) {
    float max = absmax(x, 64);
    const float inverse = max > 0.0f ? 127.0f / max : 0.0f;
    for (int i = 0; i < 64; i++) {
        float r = roundf(x[i] * inverse); /* Rust f32::round: half away from zero */
        r = r < -127.0f ? -127.0f : (r > 127.0f ? 127.0f : r);
        codes[i] = (int8_t)rust_as_int((double)r);
    }
    return max / 127.0f;
}

/* draft_head.rs:194-210 (Kv::Q8 push): rows [rows][512] keys and values into
 * group-major codes [8][capacity][64] and scales [8][capacity], at `len`. */
void fo_or_draft_push(const float *keys, const float *values, int64_t rows, int64_t capacity, int64_t len,
                      int8_t *key_codes, float *key_scales, int8_t *value_codes, float *value_scales) {
    for (int64_t r = 0; r < rows; r++)
        for (int g = 0; g < 8; g++) {
            const int64_t row = g * capacity + len + r;
            key_scales[row] = fo_or_draft_quantize_row(keys + r * DRAFT_KV_WIDTH + g * 64, key_codes + row * 64);
            value_scales[row] =
                fo_or_draft_quantize_row(values + r * DRAFT_KV_WIDTH + g * 64, value_codes + row * 64);
        }
}

/* attend (draft_head.rs:548-627) with group_q8 (:706-759) for the int8
 * rows: per KV group, both heads' scores over verified rows
 * [max(0, bases - window), bases) (window 0: all of them), each a dot times
 * key_scale / 8, then the FP32 chain rows' dots / 8; max, exp (exp_poly,
 * the vector kernels' exp), sum; out = (sum_t p_t * value_scale_t * v_t +
 * sum_r p_r * chain_v_r) * (1 / sum). */
void fo_or_draft_attend(const int8_t *key_codes, const float *key_scales, const int8_t *value_codes,
                        const float *value_scales, int64_t capacity, const float *q, int64_t bases, int64_t window,
                        const float *chain_keys, const float *chain_values, int64_t chain, float *out) {
    const int64_t start = window == 0 ? 0 : (bases > window ? bases - window : 0);
    const int64_t n = bases - start, total = n + chain;
    float *s = (float *)malloc((size_t)(2 * total + 1) * sizeof(float));
    for (int g = 0; g < 8; g++) {
        const float *q0 = q + 2 * g * 64, *q1 = q0 + 64;
        float *s0 = s, *s1 = s + total;
        for (int64_t t = 0; t < n; t++) {
            const int64_t row = g * capacity + start + t;
            float d0 = 0.0f, d1 = 0.0f;
            for (int d = 0; d < 64; d++) {
                d0 = fmaf(q0[d], (float)key_codes[row * 64 + d], d0);
                d1 = fmaf(q1[d], (float)key_codes[row * 64 + d], d1);
            }
            const float f = key_scales[row] * 0.125f;
            s0[t] = d0 * f;
            s1[t] = d1 * f;
        }
        for (int64_t r = 0; r < chain; r++) {
            const float *k = chain_keys + r * DRAFT_KV_WIDTH + g * 64;
            float d0 = 0.0f, d1 = 0.0f;
            for (int d = 0; d < 64; d++) {
                d0 = fmaf(q0[d], k[d], d0);
                d1 = fmaf(q1[d], k[d], d1);
            }
            s0[n + r] = d0 * 0.125f;
            s1[n + r] = d1 * 0.125f;
        }
        float m0 = NEG_INF, m1 = NEG_INF;
        for (int64_t t = 0; t < total; t++) {
            m0 = fmaxf(m0, s0[t]);
            m1 = fmaxf(m1, s1[t]);
        }
        float sum0 = 0.0f, sum1 = 0.0f;
        for (int64_t t = 0; t < total; t++) {
            s0[t] = fo_or_exp_poly(s0[t] - m0);
            s1[t] = fo_or_exp_poly(s1[t] - m1);
            sum0 += s0[t];
            sum1 += s1[t];
        }
        float o0[64] = {0}, o1[64] = {0};
        for (int64_t t = 0; t < n; t++) {
            const int64_t row = g * capacity + start + t;
            const float f = value_scales[row], p0 = s0[t] * f, p1 = s1[t] * f;
            for (int d = 0; d < 64; d++) {
                const float v = (float)value_codes[row * 64 + d];
                o0[d] = fmaf(p0, v, o0[d]);
                o1[d] = fmaf(p1, v, o1[d]);
            }
        }
        for (int64_t r = 0; r < chain; r++) {
            const float *v = chain_values + r * DRAFT_KV_WIDTH + g * 64;
            for (int d = 0; d < 64; d++) {
                o0[d] = fmaf(s0[n + r], v[d], o0[d]);
                o1[d] = fmaf(s1[n + r], v[d], o1[d]);
            }
        }
        const float i0 = 1.0f / sum0, i1 = 1.0f / sum1;
        for (int d = 0; d < 64; d++) {
            out[2 * g * 64 + d] = o0[d] * i0;
            out[(2 * g + 1) * 64 + d] = o1[d] * i1;
        }
    }
    free(s);
}
