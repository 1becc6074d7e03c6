/*
 * fo_cpu_simd.c -- the CPU baseline of the benchmark: the reference's
 * production CPU kernels for this path, restated in C with the same x86
 * vector instructions (AVX-512F/BW/BF16 and AVX2/FMA intrinsics).
 *
 * Benchmark and test infrastructure only: bench.py's reference arm and its
 * cpu_baseline leg time these functions, and tests check them against the
 * scalar restatement (fo_oracle.c).  The product never links this file.
 *
 * Restated (paths relative to the reference project):
 *   fo_cpu_prefill_bf16_static
 *       prefill64::bf16::compact_prefill with the static-shift tiles, the
 *       fast mode's default prefill: Bf16Kv::Convert (bf16.rs:108-137,
 *       pair_rows 203-217), the task loop (bf16.rs:150-178), and
 *       bf16/static_shift.rs:106-336 (Visibility, qk_exp_lanes, Block::keys,
 *       exp2_lanes) with pv_lanes / pv_rows (bf16.rs:610-660).
 *   fo_cpu_decode_rows_f32
 *       SplitPrefix::attention_decode_rows over F32 records
 *       (kv.rs:856-972): one task per (group, chunk) with the reference's
 *       chunk partition, pair_rows (kv/decode.rs:551-677; decode_key,
 *       qk2_decoded, pv_decoded with the 8-lane AVX2 instantiation) and the
 *       chunk merge with the sink (kv.rs:775-813).  The exp is the platform
 *       expf, which the reference's vector exp equals bit for bit.
 * Threads: OpenMP; the caller sets the count (fo_cpu_set_threads).
 */
#include <immintrin.h>
#include <math.h>
#include <omp.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define HD 64
#define PAIRS 32
#define QUERY_TILE 32
#define KEY_TILE 128
#define DEC_TILE 128
#define SUB 32
#define RECORD 160
#define TAIL_RECORD 128
#define MAX_ROWS 8
#define MAX_CHUNKS 4

void fo_cpu_set_threads(int threads) {
    if (threads > 0) omp_set_num_threads(threads);
}

int fo_cpu_max_threads(void) { return omp_get_max_threads(); }

/* 1 when the host runs the AVX-512 BF16 prefill (the reference's
 * attention_prefill_bf16 requires AVX512-BF16, and the static shift AVX512BW,
 * mod.rs:330-346 and bf16.rs:148). */
int fo_cpu_has_bf16(void) {
    __builtin_cpu_init();
    return __builtin_cpu_supports("avx512f") && __builtin_cpu_supports("avx512bw") &&
           __builtin_cpu_supports("avx512bf16");
}

int fo_cpu_has_avx2(void) {
    __builtin_cpu_init();
    return __builtin_cpu_supports("avx2") && __builtin_cpu_supports("fma");
}

/* ------------------------------------------------------------------ */
/* BF16 static-shift prefill                                           */
/* ------------------------------------------------------------------ */
#define BF16_TARGET __attribute__((target("avx512f,avx512bw,avx512bf16,avx2,fma")))
#define INLINE static inline __attribute__((always_inline))

/* Minimax coefficients of 2^f on [-1/2, 1/2] (bf16/static_shift.rs:36-38). */
static const float EXP2_C[4] = {0.99992806f, 0.69326097f, 0.24261113f, 0.05517167f};
static const float LOG2E = 1.44269504088896340736f;

typedef struct {
    int64_t first_absolute;
    uint32_t image_lanes;
    int64_t image_start, image_end;
    int all;
} visibility_t;

/* span.rs:9-20 */
static void tile_span(int64_t first_query, int64_t queries, int64_t image_start, int64_t image_end,
                      int64_t *first_absolute, int64_t *visible_end, int *all_image) {
    int64_t first = first_query, last = first + queries - 1;
    int intersects = first < image_end && last >= image_start;
    *first_absolute = first;
    *visible_end = intersects ? (last + 1 > image_end ? last + 1 : image_end) : last + 1;
    *all_image = first >= image_start && last < image_end;
}

/* Visibility::lanes (bf16/static_shift.rs:79-96): bit r = query row r sees key. */
INLINE uint32_t vis_lanes(const visibility_t *v, int64_t key) {
    if (v->all) return 0xFFFFFFFFu;
    uint32_t causal;
    if (key <= v->first_absolute) {
        causal = 0xFFFFFFFFu;
    } else {
        int64_t late = key - v->first_absolute;
        causal = late >= 32 ? 0u : (0xFFFFFFFFu << late);
    }
    if (key >= v->image_start && key < v->image_end) causal |= v->image_lanes;
    return causal;
}

/* exp2_lanes (bf16/static_shift.rs:322-336). */
BF16_TARGET INLINE __m512 exp2_lanes(__m512 t, __mmask16 visible) {
    __m512 n = _mm512_roundscale_ps(t, _MM_FROUND_TO_NEAREST_INT | _MM_FROUND_NO_EXC);
    __m512 f = _mm512_sub_ps(t, n);
    __m512 p = _mm512_set1_ps(EXP2_C[3]);
    p = _mm512_fmadd_ps(p, f, _mm512_set1_ps(EXP2_C[2]));
    p = _mm512_fmadd_ps(p, f, _mm512_set1_ps(EXP2_C[1]));
    p = _mm512_fmadd_ps(p, f, _mm512_set1_ps(EXP2_C[0]));
    return _mm512_maskz_scalef_ps(visible, p, n);
}

BF16_TARGET INLINE __m512bh as_bh(__m512i x) { return (__m512bh)x; }

/* Block::keys (bf16/static_shift.rs:263-311) for N keys from tile row `key`
 * and V query vectors: the dpbf16 chain over the 32 pairs, then per key
 * pair the exp, the BF16 pairs and the denominators of the rounded values. */
BF16_TARGET INLINE void block_keys(const uint32_t *qp, const uint32_t *kp, int key, const int N, const int V,
                                   int64_t key_start, __m512 scale, __m512i interleave, const visibility_t *vis,
                                   __m512 *sums, uint32_t *pairs) {
    __m512 acc[8][2];
    for (int n = 0; n < N; n++)
        for (int v = 0; v < V; v++) acc[n][v] = _mm512_setzero_ps();
    for (int p = 0; p < PAIRS; p++) {
        __m512i q[2];
        for (int v = 0; v < V; v++) q[v] = _mm512_loadu_si512((const void *)(qp + p * QUERY_TILE + 16 * v));
        for (int n = 0; n < N; n++) {
            __m512i kv = _mm512_set1_epi32((int)kp[(key + n) * PAIRS + p]);
            for (int v = 0; v < V; v++) acc[n][v] = _mm512_dpbf16_ps(acc[n][v], as_bh(q[v]), as_bh(kv));
        }
    }
    const __m512i hi_mask = _mm512_set1_epi32((int)0xFFFF0000u);
    for (int n = 0; n < N; n += 2) {
        uint32_t even_lanes = vis_lanes(vis, key_start + key + n);
        uint32_t odd_lanes = n + 1 < N ? vis_lanes(vis, key_start + key + n + 1) : 0u;
        for (int v = 0; v < V; v++) {
            __m512 even = exp2_lanes(_mm512_mul_ps(scale, acc[n][v]), (__mmask16)(even_lanes >> (16 * v)));
            __m512 odd = n + 1 < N ? exp2_lanes(_mm512_mul_ps(scale, acc[n + 1][v]), (__mmask16)(odd_lanes >> (16 * v)))
                                   : _mm512_setzero_ps();
            __m512i halves = (__m512i)_mm512_cvtne2ps_pbh(odd, even);
            __m512i pair = _mm512_permutexvar_epi16(interleave, halves);
            _mm512_storeu_si512((void *)(pairs + (key + n) / 2 * QUERY_TILE + 16 * v), pair);
            __m512 e = _mm512_castsi512_ps(_mm512_slli_epi32(pair, 16));
            __m512 o = _mm512_castsi512_ps(_mm512_and_si512(pair, hi_mask));
            sums[v] = _mm512_add_ps(_mm512_add_ps(sums[v], e), o);
        }
    }
}

/* Block::tile: all keys of the tile, eight at a time. */
BF16_TARGET static void qk_exp_tile(const uint32_t *qp, const uint32_t *kp, int keys, const int V, int64_t key_start,
                                    __m512 scale, __m512i interleave, const visibility_t *vis, float *denominators,
                                    uint32_t *pairs) {
    __m512 sums[2];
    for (int v = 0; v < V; v++) sums[v] = _mm512_loadu_ps(denominators + 16 * v);
    int key = 0;
    if (V == 2) {
        for (; key + 8 <= keys; key += 8) block_keys(qp, kp, key, 8, 2, key_start, scale, interleave, vis, sums, pairs);
        switch (keys - key) {
        case 7: block_keys(qp, kp, key, 7, 2, key_start, scale, interleave, vis, sums, pairs); break;
        case 6: block_keys(qp, kp, key, 6, 2, key_start, scale, interleave, vis, sums, pairs); break;
        case 5: block_keys(qp, kp, key, 5, 2, key_start, scale, interleave, vis, sums, pairs); break;
        case 4: block_keys(qp, kp, key, 4, 2, key_start, scale, interleave, vis, sums, pairs); break;
        case 3: block_keys(qp, kp, key, 3, 2, key_start, scale, interleave, vis, sums, pairs); break;
        case 2: block_keys(qp, kp, key, 2, 2, key_start, scale, interleave, vis, sums, pairs); break;
        case 1: block_keys(qp, kp, key, 1, 2, key_start, scale, interleave, vis, sums, pairs); break;
        default: break;
        }
    } else {
        for (; key + 8 <= keys; key += 8) block_keys(qp, kp, key, 8, 1, key_start, scale, interleave, vis, sums, pairs);
        switch (keys - key) {
        case 7: block_keys(qp, kp, key, 7, 1, key_start, scale, interleave, vis, sums, pairs); break;
        case 6: block_keys(qp, kp, key, 6, 1, key_start, scale, interleave, vis, sums, pairs); break;
        case 5: block_keys(qp, kp, key, 5, 1, key_start, scale, interleave, vis, sums, pairs); break;
        case 4: block_keys(qp, kp, key, 4, 1, key_start, scale, interleave, vis, sums, pairs); break;
        case 3: block_keys(qp, kp, key, 3, 1, key_start, scale, interleave, vis, sums, pairs); break;
        case 2: block_keys(qp, kp, key, 2, 1, key_start, scale, interleave, vis, sums, pairs); break;
        case 1: block_keys(qp, kp, key, 1, 1, key_start, scale, interleave, vis, sums, pairs); break;
        default: break;
        }
    }
    for (int v = 0; v < V; v++) _mm512_storeu_ps(denominators + 16 * v, sums[v]);
}

/* pv_rows (bf16.rs:628-660): R query rows by the whole 64-wide row. */
BF16_TARGET INLINE void pv_rows(const uint32_t *pairs, int row, const int R, int key_pairs, const uint32_t *values,
                                float *out, int64_t out_stride) {
    __m512 acc[6][4];
    for (int r = 0; r < R; r++)
        for (int c = 0; c < 4; c++) acc[r][c] = _mm512_setzero_ps();
    for (int kp = 0; kp < key_pairs; kp++) {
        const uint32_t *vr = values + kp * HD;
        __m512i v[4];
        for (int c = 0; c < 4; c++) v[c] = _mm512_loadu_si512((const void *)(vr + 16 * c));
        const uint32_t *p = pairs + kp * QUERY_TILE + row;
        for (int r = 0; r < R; r++) {
            __m512i pv = _mm512_set1_epi32((int)p[r]);
            for (int c = 0; c < 4; c++) acc[r][c] = _mm512_dpbf16_ps(acc[r][c], as_bh(v[c]), as_bh(pv));
        }
    }
    for (int r = 0; r < R; r++) {
        float *dst = out + (int64_t)(row + r) * out_stride;
        for (int c = 0; c < 4; c++) _mm512_storeu_ps(dst + 16 * c, _mm512_add_ps(acc[r][c], _mm512_loadu_ps(dst + 16 * c)));
    }
}

/* pv_lanes (bf16.rs:610-626): rows six at a time. */
BF16_TARGET static void pv_lanes(const uint32_t *pairs, int queries, int key_pairs, const uint32_t *values, float *out,
                                 int64_t out_stride) {
    int row = 0;
    while (row < queries) {
        int rows = queries - row < 6 ? queries - row : 6;
        switch (rows) {
        case 6: pv_rows(pairs, row, 6, key_pairs, values, out, out_stride); break;
        case 5: pv_rows(pairs, row, 5, key_pairs, values, out, out_stride); break;
        case 4: pv_rows(pairs, row, 4, key_pairs, values, out, out_stride); break;
        case 3: pv_rows(pairs, row, 3, key_pairs, values, out, out_stride); break;
        case 2: pv_rows(pairs, row, 2, key_pairs, values, out, out_stride); break;
        default: pv_rows(pairs, row, 1, key_pairs, values, out, out_stride); break;
        }
        row += rows;
    }
}

/* 16-bit RNE BF16 bits of x, the conversion of vcvtneps2bf16 (as
 * half::bf16::from_f32 in query_pairs, bf16.rs:263-276). */
static inline uint32_t bf16_bits(float x) {
    uint32_t u;
    memcpy(&u, &x, 4);
    if ((u & 0x7FFFFFFFu) > 0x7F800000u) return ((u >> 16) | 0x40u) & 0xFFFFu;
    return ((u + 0x7FFFu + ((u >> 16) & 1u)) >> 16) & 0xFFFFu;
}

/* static_shift::tile_head (bf16/static_shift.rs:106-172). */
BF16_TARGET static void tile_head_static(const float *q, const uint32_t *keys, const uint32_t *values, int64_t tile,
                                         int64_t queries, int64_t head, int64_t query_width, int64_t image_start,
                                         int64_t image_end, const float *sinks, float *output) {
    int64_t first_query = tile * QUERY_TILE, first_absolute, visible_end;
    int all;
    tile_span(first_query, queries, image_start, image_end, &first_absolute, &visible_end, &all);
    visibility_t vis = {first_absolute, 0u, image_start, image_end, all};
    for (int r = 0; r < QUERY_TILE; r++)
        if (first_absolute + r >= image_start && first_absolute + r < image_end) vis.image_lanes |= 1u << r;
    uint32_t qp[PAIRS * QUERY_TILE];
    memset(qp, 0, sizeof qp);
    for (int64_t r = 0; r < queries; r++) {
        const float *row = q + (first_query + r) * query_width + head * HD;
        for (int p = 0; p < PAIRS; p++) qp[p * QUERY_TILE + r] = bf16_bits(row[2 * p]) | bf16_bits(row[2 * p + 1]) << 16;
    }
    float *out = output + first_query * query_width + head * HD;
    for (int64_t r = 0; r < queries; r++) memset(out + r * query_width, 0, HD * sizeof(float));
    float denominators[QUERY_TILE];
    memset(denominators, 0, sizeof denominators);
    uint32_t pairs[KEY_TILE / 2 * QUERY_TILE];
    static const uint16_t INTERLEAVE[32] = {0, 16, 1, 17, 2, 18, 3, 19, 4, 20, 5, 21, 6, 22, 7, 23,
                                            8, 24, 9, 25, 10, 26, 11, 27, 12, 28, 13, 29, 14, 30, 15, 31};
    const __m512i interleave = _mm512_loadu_si512((const void *)INTERLEAVE);
    const __m512 scale = _mm512_set1_ps(LOG2E * 0.125f); /* exponent_scale, static_shift.rs:177-179 */
    const int V = queries > 16 ? 2 : 1;
    for (int64_t key_start = 0; key_start < visible_end; key_start += KEY_TILE) {
        int nk = (int)(visible_end - key_start < KEY_TILE ? visible_end - key_start : KEY_TILE);
        qk_exp_tile(qp, keys + key_start * PAIRS, nk, V, key_start, scale, interleave, &vis, denominators, pairs);
        pv_lanes(pairs, (int)queries, (nk + 1) / 2, values + key_start / 2 * HD, out, query_width);
    }
    for (int64_t r = 0; r < queries; r++) {
        float *row = out + r * query_width;
        float lse = logf(denominators[r]);
        float sink_scale = 1.0f / (1.0f + expf(sinks[head] - lse));
        for (int d = 0; d < HD; d++) row[d] = (row[d] / denominators[r]) * sink_scale;
    }
}

/* to_bf16 (bf16.rs:191-201): 64 values to BF16 (RNE). */
BF16_TARGET INLINE void to_bf16(const float *src, uint16_t *dst) {
    for (int c = 0; c < HD; c += 32) {
        __m512 lo = _mm512_loadu_ps(src + c), hi = _mm512_loadu_ps(src + c + 16);
        _mm512_storeu_si512((void *)(dst + c), (__m512i)_mm512_cvtne2ps_pbh(hi, lo));
    }
}

BF16_TARGET INLINE __m512i bf16_lanes(__m512 x) {
    return _mm512_cvtepu16_epi32((__m256i)_mm512_cvtneps_pbh(x));
}

/* compact_prefill (bf16.rs:78-178) with Bf16Kv::Convert and the static
 * shift.  Returns -1 (nothing written) when the host lacks AVX512-BF16. */
BF16_TARGET int fo_cpu_prefill_bf16_static(const float *q, const float *k, const float *v, int64_t total,
                                           int64_t n_heads, int64_t n_kv_heads, int64_t image_start,
                                           int64_t image_end, const float *sinks, float *out) {
    if (!fo_cpu_has_bf16()) return -1;
    const int64_t qw = n_heads * HD, kvw = n_kv_heads * HD, pairs = (total + 1) / 2;
    uint32_t *keys = (uint32_t *)aligned_alloc(64, (size_t)(n_heads * total * PAIRS * 4 + 64));
    uint32_t *vals = (uint32_t *)aligned_alloc(64, (size_t)(n_kv_heads * pairs * HD * 4 + 64));
    if (!keys || !vals) {
        free(keys);
        free(vals);
        return -2;
    }
#pragma omp parallel for schedule(static)
    for (int64_t head = 0; head < n_heads; head++)
        for (int64_t t = 0; t < total; t++)
            to_bf16(k + t * qw + head * HD, (uint16_t *)(keys + (head * total + t) * PAIRS));
#pragma omp parallel for schedule(static)
    for (int64_t kvh = 0; kvh < n_kv_heads; kvh++)
        for (int64_t p = 0; p < pairs; p++) {
            const float *even = v + 2 * p * kvw + kvh * HD;
            const float *odd = 2 * p + 1 < total ? v + (2 * p + 1) * kvw + kvh * HD : NULL;
            uint32_t *dst = vals + (kvh * pairs + p) * HD;
            for (int c = 0; c < 4; c++) {
                __m512i lo = bf16_lanes(_mm512_loadu_ps(even + 16 * c));
                __m512i hi = odd ? _mm512_slli_epi32(bf16_lanes(_mm512_loadu_ps(odd + 16 * c)), 16)
                                 : _mm512_setzero_si512();
                _mm512_storeu_si512((void *)(dst + 16 * c), _mm512_or_si512(lo, hi));
            }
        }
    const int64_t repeat = n_heads / n_kv_heads, tiles = (total + QUERY_TILE - 1) / QUERY_TILE;
    for (int64_t kvh = 0; kvh < n_kv_heads; kvh++) {
#pragma omp parallel for schedule(dynamic, 1)
        for (int64_t task = 0; task < tiles * repeat; task++) {
            int64_t tile = task / repeat, head = kvh * repeat + task % repeat;
            int64_t queries = total - tile * QUERY_TILE < QUERY_TILE ? total - tile * QUERY_TILE : QUERY_TILE;
            tile_head_static(q, keys + head * total * PAIRS, vals + kvh * pairs * HD, tile, queries, head, qw,
                             image_start, image_end, sinks, out);
        }
    }
    free(keys);
    free(vals);
    return 0;
}

/* ------------------------------------------------------------------ */
/* Split-cache verify decode over F32 records (AVX2 / FMA)             */
/* ------------------------------------------------------------------ */
#define AVX2_TARGET __attribute__((target("avx2,fma")))

typedef struct {
    float out[2][64];
    float max[2];
    float den[2];
} partial_t;

/* Avx2::sum (simd.rs:366-373): ((v0+v4) + (v1+v5)) + ((v2+v6) + (v3+v7)). */
AVX2_TARGET INLINE float sum8(__m256 v) {
    __m128 halves = _mm_add_ps(_mm256_castps256_ps128(v), _mm256_extractf128_ps(v, 1));
    __m128 pairs = _mm_hadd_ps(halves, halves);
    return _mm_cvtss_f32(_mm_hadd_ps(pairs, pairs));
}

typedef struct {
    const float *codes, *tail;       /* prefix [G][prefix_stride][160], tail [G][tail_stride][128] */
    int64_t prefix_len, prefix_stride, tail_stride;
} f32_store_t;

/* pair_rows (kv/decode.rs:551-677) for n rows of one group over spans that
 * start at `start` and end at ends[r], F32 records. */
AVX2_TARGET static void pair_rows_f32(const f32_store_t *st, int64_t g, int64_t start, const int64_t *ends, int n,
                                      const float *const *q0, const float *const *q1, partial_t *parts) {
    float max[MAX_ROWS][2], den[MAX_ROWS][2];
    float logits[MAX_ROWS][2][DEC_TILE];
    float keys[SUB * 96] __attribute__((aligned(32)));
    float values[SUB * 64] __attribute__((aligned(32)));
    int64_t end = start;
    for (int r = 0; r < n; r++) {
        max[r][0] = max[r][1] = -INFINITY;
        den[r][0] = den[r][1] = 0.0f;
        memset(parts[r].out, 0, sizeof parts[r].out);
        if (ends[r] > end) end = ends[r];
    }
    const float scale = 0.125f;
    while (start < end) {
        int lens[MAX_ROWS], len = 0;
        for (int r = 0; r < n; r++) {
            lens[r] = ends[r] > start ? (int)(ends[r] - start < DEC_TILE ? ends[r] - start : DEC_TILE) : 0;
            if (lens[r] > len) len = lens[r];
        }
        float block_max[MAX_ROWS][2];
        for (int r = 0; r < n; r++) block_max[r][0] = block_max[r][1] = -INFINITY;
        for (int sub = 0; sub < len; sub += SUB) {
            int width = len - sub < SUB ? len - sub : SUB;
            /* decode_key: [T 32 | S0 32 | S1 32] per key */
            for (int j = 0; j < width; j++) {
                int64_t key = start + sub + j;
                float *dst = keys + j * 96;
                if (key < st->prefix_len) {
                    const float *rec = st->codes + (g * st->prefix_stride + key) * RECORD;
                    memcpy(dst, rec, 96 * sizeof(float));
                } else {
                    const float *rec = st->tail + (g * st->tail_stride + (key - st->prefix_len)) * TAIL_RECORD;
                    memcpy(dst, rec, 64 * sizeof(float));
                    memcpy(dst + 64, rec + 32, 32 * sizeof(float));
                }
            }
            for (int r = 0; r < n; r++) {
                int hi = lens[r] < sub + width ? lens[r] : sub + width;
                for (int j = sub; j < hi; j++) {
                    const float *key = keys + (j - sub) * 96;
                    __m256 a[4], b[4];
                    for (int c = 0; c < 4; c++) {
                        __m256 t = _mm256_loadu_ps(key + 8 * c);
                        a[c] = _mm256_mul_ps(_mm256_loadu_ps(q0[r] + 8 * c), t);
                        b[c] = _mm256_mul_ps(_mm256_loadu_ps(q1[r] + 8 * c), t);
                    }
                    for (int c = 0; c < 4; c++) {
                        a[c] = _mm256_fmadd_ps(_mm256_loadu_ps(q0[r] + 32 + 8 * c), _mm256_loadu_ps(key + 32 + 8 * c), a[c]);
                        b[c] = _mm256_fmadd_ps(_mm256_loadu_ps(q1[r] + 32 + 8 * c), _mm256_loadu_ps(key + 64 + 8 * c), b[c]);
                    }
                    float s0 = sum8(_mm256_add_ps(_mm256_add_ps(a[0], a[1]), _mm256_add_ps(a[2], a[3])));
                    float s1 = sum8(_mm256_add_ps(_mm256_add_ps(b[0], b[1]), _mm256_add_ps(b[2], b[3])));
                    logits[r][0][j] = s0 * scale;
                    block_max[r][0] = fmaxf(block_max[r][0], logits[r][0][j]);
                    logits[r][1][j] = s1 * scale;
                    block_max[r][1] = fmaxf(block_max[r][1], logits[r][1][j]);
                }
            }
        }
        float new_max[MAX_ROWS][2];
        for (int r = 0; r < n; r++) {
            if (!lens[r]) continue;
            for (int h = 0; h < 2; h++) {
                new_max[r][h] = fmaxf(max[r][h], block_max[r][h]);
                float rescale = max[r][h] == -INFINITY ? 0.0f : expf(max[r][h] - new_max[r][h]);
                for (int d = 0; d < 64; d++) parts[r].out[h][d] *= rescale;
                den[r][h] *= rescale;
                for (int j = 0; j < lens[r]; j++) logits[r][h][j] = expf(logits[r][h][j] - new_max[r][h]);
            }
        }
        for (int sub = 0; sub < len; sub += SUB) {
            int width = len - sub < SUB ? len - sub : SUB;
            for (int j = 0; j < width; j++) {
                int64_t key = start + sub + j;
                const float *src = key < st->prefix_len
                                       ? st->codes + (g * st->prefix_stride + key) * RECORD + 96
                                       : st->tail + (g * st->tail_stride + (key - st->prefix_len)) * TAIL_RECORD + 64;
                memcpy(values + j * 64, src, 64 * sizeof(float));
            }
            for (int r = 0; r < n; r++) {
                int hi = lens[r] < sub + width ? lens[r] : sub + width;
                if (hi <= sub) continue;
                for (int h = 0; h < 2; h++) {
                    /* pv_decoded: outputs in registers, denominator in key order */
                    __m256 o[8];
                    for (int c = 0; c < 8; c++) o[c] = _mm256_loadu_ps(parts[r].out[h] + 8 * c);
                    float dn = den[r][h];
                    for (int j = sub; j < hi; j++) {
                        float p = logits[r][h][j];
                        dn += p;
                        __m256 f = _mm256_set1_ps(p);
                        const float *vv = values + (j - sub) * 64;
                        for (int c = 0; c < 8; c++) o[c] = _mm256_fmadd_ps(f, _mm256_loadu_ps(vv + 8 * c), o[c]);
                    }
                    den[r][h] = dn;
                    for (int c = 0; c < 8; c++) _mm256_storeu_ps(parts[r].out[h] + 8 * c, o[c]);
                }
            }
        }
        for (int r = 0; r < n; r++)
            if (lens[r]) {
                max[r][0] = new_max[r][0];
                max[r][1] = new_max[r][1];
            }
        start += len;
    }
    for (int r = 0; r < n; r++) {
        parts[r].max[0] = max[r][0];
        parts[r].max[1] = max[r][1];
        parts[r].den[0] = den[r][0];
        parts[r].den[1] = den[r][1];
    }
}

/* SplitPrefix::merge (kv.rs:775-813). */
static void merge(const partial_t *gp, int64_t chunks, const float *sinks, int64_t g, float *output) {
    for (int pair = 0; pair < 2; pair++) {
        int64_t h = 2 * g + pair;
        float *out = output + h * 64;
        float mx, den;
        if (chunks == 1) {
            memcpy(out, gp[0].out[pair], 64 * sizeof(float));
            mx = gp[0].max[pair];
            den = gp[0].den[pair];
        } else {
            mx = -INFINITY;
            for (int64_t c = 0; c < chunks; c++) mx = fmaxf(mx, gp[c].max[pair]);
            den = 0.0f;
            memset(out, 0, 64 * sizeof(float));
            for (int64_t c = 0; c < chunks; c++) {
                if (gp[c].max[pair] == -INFINITY) continue;
                float factor = expf(gp[c].max[pair] - mx);
                den = fmaf(gp[c].den[pair], factor, den);
                for (int d = 0; d < 64; d++) out[d] = fmaf(gp[c].out[pair][d], factor, out[d]);
            }
        }
        float lse = mx + logf(den);
        float sink = 1.0f / (1.0f + expf(sinks[h] - lse));
        for (int d = 0; d < 64; d++) out[d] = (out[d] / den) * sink;
    }
}

/* attention_decode_rows over F32 split records (kv.rs:856-972): rows that
 * share a chunk partition run together, one task per (group, chunk); the
 * default chunk count for F32 records is 1 (kv.rs:188-197).  Returns -1 if
 * the host lacks AVX2/FMA. */
AVX2_TARGET int fo_cpu_decode_rows_f32(const float *codes, const float *tail, int64_t prefix_len,
                                       int64_t prefix_stride, int64_t tail_len, int64_t tail_stride, int64_t groups,
                                       const float *q, int64_t rows, const float *sinks, int64_t chunk_request,
                                       float *output) {
    if (!fo_cpu_has_avx2()) return -1;
    if (rows < 1 || rows > MAX_ROWS || groups > 64) return -2;
    f32_store_t st = {codes, tail, prefix_len, prefix_stride, tail_stride};
    const int64_t width = groups * 2 * 64, last = prefix_len + tail_len;
    int assigned[MAX_ROWS] = {0};
    for (int first = 0; first < rows; first++) {
        if (assigned[first]) continue;
        int64_t t_first = last + 1 + first - rows;
        int64_t tiles = (t_first + DEC_TILE - 1) / DEC_TILE;
        int64_t chunks = chunk_request < 1 ? 1 : (chunk_request > MAX_CHUNKS ? MAX_CHUNKS : chunk_request);
        if (chunks > tiles) chunks = tiles;
        int64_t per_chunk = (tiles + chunks - 1) / chunks;
        int members[MAX_ROWS], n = 0;
        for (int r = first; r < rows; r++) {
            int64_t t = last + 1 + r - rows, tl = (t + DEC_TILE - 1) / DEC_TILE;
            int64_t ch = chunk_request < 1 ? 1 : (chunk_request > MAX_CHUNKS ? MAX_CHUNKS : chunk_request);
            if (ch > tl) ch = tl;
            if (!assigned[r] && ch == chunks && (tl + ch - 1) / ch == per_chunk) {
                assigned[r] = 1;
                members[n++] = r;
            }
        }
        partial_t *parts = (partial_t *)malloc(sizeof(partial_t) * (size_t)(n * groups * chunks));
#pragma omp parallel for schedule(dynamic, 1)
        for (int64_t index = 0; index < groups * chunks; index++) {
            int64_t g = index / chunks, chunk = index % chunks;
            int64_t ends[MAX_ROWS], start = 0;
            const float *q0[MAX_ROWS], *q1[MAX_ROWS];
            int live = 0;
            partial_t local[MAX_ROWS];
            for (int i = 0; i < n; i++) {
                int64_t t = last + 1 + members[i] - rows;
                int64_t s = chunk * per_chunk * DEC_TILE, e = (chunk + 1) * per_chunk * DEC_TILE;
                s = s < t ? s : t;
                e = e < t ? e : t;
                if (s < e) {
                    start = s;
                    live = 1;
                }
                ends[i] = e;
                q0[i] = q + members[i] * width + 2 * g * 64;
                q1[i] = q + members[i] * width + (2 * g + 1) * 64;
            }
            if (!live) {
                for (int i = 0; i < n; i++) {
                    memset(&local[i], 0, sizeof local[i]);
                    local[i].max[0] = local[i].max[1] = -INFINITY;
                }
            } else {
                for (int i = 0; i < n; i++)
                    if (ends[i] < start) ends[i] = start;
                pair_rows_f32(&st, g, start, ends, n, q0, q1, local);
            }
            for (int i = 0; i < n; i++) parts[(i * groups + g) * chunks + chunk] = local[i];
        }
        for (int i = 0; i < n; i++)
            for (int64_t g = 0; g < groups; g++)
                merge(parts + (i * groups + g) * chunks, chunks, sinks, g, output + members[i] * width);
        free(parts);
    }
    return 0;
}
