/*
 * fo_oracle.h -- CPU restatement of falcon-ocr-cpu's attention hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the checker that the CUDA
 * product is compared against; only tests/, __graft_entry__.smoke() and
 * bench.py's cpu_baseline / reference arm may load it.  The product path
 * (falcon-ocr-cpu_b200/) never links or calls it.
 *
 * Every function restates the reference Rust crate's arithmetic (file:line
 * given per function, paths relative to the reference project root).  The
 * reference cannot be compiled here (no Rust toolchain), so this
 * restatement is pinned against the reference's own known-answer tests and
 * f64 tolerance tables (tests/golden/, tests/test_oracle_golden.py).
 */
#ifndef FO_ORACLE_H
#define FO_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- element formats of the split cache (src/quant/kv.rs:120-127) ---- */
#define FO_OR_F32 0
#define FO_OR_Q16 1
#define FO_OR_Q8 2
#define FO_OR_BF16 3 /* new in this build: BF16 records, no scales */
#define FO_OR_Q4 4   /* 4-bit codes -7..7, two per byte (element 2i low), BF16 scale per 32 (kv.rs:109-114) */
/* Flag: every 32-element block stored rotated, H D x (src/quant/rotation.rs,
 * kv.rs:128-152); with F32, Q8 or Q4.  Q8|ROTATED is Kv::Q8Rot and
 * Q4|ROTATED Kv::Q4Rot; rotated F32 and unrotated Q4 are the reference's
 * test storages. */
#define FO_OR_ROTATED 16

/* ---- seal / append status codes (src/quant/kv.rs:248-295) ---- */
#define FO_OR_OK 0
#define FO_OR_ERR_PAIR 1      /* temporal keys differ inside a GQA pair */
#define FO_OR_ERR_NONFINITE 2 /* non-finite K/V value in the prefix */
#define FO_OR_ERR_OVERFLOW 3  /* code * scale overflowed */
#define FO_OR_ERR_SHAPE 4     /* head_dim/heads/groups not Falcon's paired GQA */
#define FO_OR_ERR_CAPACITY 5  /* prefix_len == 0 or capacity < prefix_len */
#define FO_OR_ERR_ROTATED 6   /* a rotated block is no longer finite (kv.rs:290-293) */

/* Randomized Hadamard rotation of 32-value blocks (src/quant/rotation.rs).
 * kind: 0 temporal key half, 1 spatial key half, 2 value 0..32, 3 value
 * 32..64.  signs(kind) is D's bit pattern (bit i set: element i negated). */
uint32_t fo_or_rotation_signs(int kind);
void fo_or_fwht32(float *x);                    /* x <- H x, Sylvester order */
void fo_or_rotate(float *x, int kind);          /* x <- H D x (stored form) */
void fo_or_rotate_query(float *x, int kind);    /* x <- 2^-5 H D x */
void fo_or_unrotate(float *x, int kind);        /* x <- 2^-5 D H x */
/* Q4 codec (codec.rs:87-129): the block's BF16 scale bits; codes packed. */
uint16_t fo_or_q4_block(const float *values, uint8_t *codes);
int8_t fo_or_nibble(uint8_t byte, int high);

/* codec (src/quant/kv/codec.rs) */
uint16_t fo_or_bf16_up(float scale);
float fo_or_bf16_f32(uint16_t bits);
uint16_t fo_or_bf16_rne(float x);
float fo_or_q8_scale(const float *values, int64_t n);
float fo_or_q16_scale(const float *values, int64_t n);
double fo_or_round_clamped(double x, double limit);
int8_t fo_or_q8_code(float value, float scale);
int16_t fo_or_q16_code(float value, float scale);

/* exp definitions (src/kernels/exp.rs:232-277) */
float fo_or_exp_poly(float x);
float fo_or_exp_poly_unchecked(float x);

/* Dense f64 attention over a compact cache, sink folded into the
 * denominator (src/kernels/tests.rs:204-248).  bf16_operands rounds q, k, v
 * to BF16 first (src/kernels/attention/prefill64/bf16.rs:847-916). */
void fo_or_attention_f64(const float *q, const float *prefix_k, const float *generated_k, const float *v,
                         int64_t query_len, int64_t prefix_len, int64_t total_len, int64_t n_heads,
                         int64_t n_kv_heads, int64_t head_dim, int64_t query_offset, int64_t image_start,
                         int64_t image_end, const float *sinks, int bf16_operands, double *out);

/* The online-softmax head for every layout and head width
 * (src/kernels/attention/online.rs:89-169). exp_fast selects exp_poly. */
void fo_or_attention_online(const float *q, const float *prefix_k, const float *generated_k, const float *v,
                            int64_t query_len, int64_t prefix_len, int64_t total_len, int64_t n_heads,
                            int64_t n_kv_heads, int64_t head_dim, int64_t query_offset, int64_t image_start,
                            int64_t image_end, const float *sinks, int exp_fast, float *out);

/* FP32 prefill tiles for head_dim 64 over a pure prefix
 * (src/kernels/attention/prefill64.rs:179-715, static_shift.rs:129-161).
 * softmax_static: 0 online, 1 static shift.  exp_fast: online exp_poly. */
void fo_or_prefill64(const float *q, const float *k, const float *v, int64_t query_len, int64_t n_heads,
                     int64_t n_kv_heads, int64_t query_offset, int64_t image_start, int64_t image_end,
                     const float *sinks, int softmax_static, int exp_fast, float *out);

/* BF16 prefill tiles (src/kernels/attention/prefill64/bf16.rs:78-660,
 * bf16/static_shift.rs:106-340).  softmax_static: 0 online (exp_fast picks
 * the fused exp_poly softmax), 1 static shift. */
void fo_or_prefill_bf16(const float *q, const float *k, const float *v, int64_t query_len, int64_t n_heads,
                        int64_t n_kv_heads, int64_t image_start, int64_t image_end, const float *sinks,
                        int softmax_static, int exp_fast, float *out);

/* Split cache (src/quant/kv.rs).  Records are group-major [G][P][160]
 * (`[T 32 | S(2g) 32 | S(2g+1) 32 | V 64]`), scales [G][P][5] BF16 bits;
 * tails [G][tail_capacity][128] (`[K 64 | V 64]`), scales [G][cap][4]. */
int fo_or_kv_seal(const float *k, const float *v, int64_t prefix_len, int64_t capacity, int64_t heads,
                  int64_t groups, int64_t head_dim, int format, void *codes, uint16_t *scales);
void fo_or_kv_push(const float *k_unique, const float *v_unique, int64_t groups, int format,
                   int64_t tail_capacity, int64_t index, void *tail_codes, uint16_t *tail_scales);
/* Element `offset` of record `record`, decoded (src/quant/kv.rs:209-219). */
float fo_or_kv_value(const void *codes, const uint16_t *scales, int format, int64_t width, int64_t record,
                     int64_t offset);
/* attention_decode_rows / attention_decode (src/quant/kv.rs:565-972).
 * rows 1..8; row r sees prefix_len + tail_len - rows + 1 + r positions. */
void fo_or_kv_decode_rows(const void *codes, const uint16_t *scales, const void *tail_codes,
                          const uint16_t *tail_scales, int format, int64_t prefix_len, int64_t tail_capacity,
                          int64_t tail_len, int64_t heads, int64_t groups, const float *q, int64_t rows,
                          const float *sinks, int64_t chunks, int fast_exp, float *out);

/* The fused QKV rows (src/model/fused.rs:96-116 `fused_row`, the same
 * arithmetic as src/model/rope.rs:15-85 `split_norm_rope`): per row, query
 * head h and key head h (KV head h / (heads / groups) of the projection) get
 * rms_norm_row (width 64, eps f32::EPSILON, no weight; the pairwise sum of
 * squares of src/kernels/mod.rs:509-555) and the pairwise rotation by
 * rope[row][h][pair] = {cos, sin} (a*cos - b*sin, a*sin + b*cos, unfused);
 * v is copied.  qkv [rows][heads*64 + 2*groups*64], rope [rows][heads][32][2];
 * q, k [rows][heads][64], v [rows][groups][64]. */
void fo_or_qkv_rows(const float *qkv, const float *rope, int64_t rows, int64_t heads, int64_t groups, float *q,
                    float *k, float *v);

/* Draft-head KV (src/draft_head.rs:177-220, 548-759): int8 rows with one
 * FP32 absmax scale per 64 values, group-major [8][capacity][64]; attention
 * of q [16][64] over the verified rows [max(0, bases - window), bases)
 * (window 0: all) and `chain` FP32 rows [chain][512]; out [16][64]. */
float fo_or_draft_quantize_row(const float *x, int8_t *codes);
void fo_or_draft_push(const float *keys, const float *values, int64_t rows, int64_t capacity, int64_t len,
                      int8_t *key_codes, float *key_scales, int8_t *value_codes, float *value_scales);
void fo_or_draft_attend(const int8_t *key_codes, const float *key_scales, const int8_t *value_codes,
                        const float *value_scales, int64_t capacity, const float *q, int64_t bases, int64_t window,
                        const float *chain_keys, const float *chain_values, int64_t chain, float *out);

/* OpenMP threads used by the parallel oracle loops (0 = library default). */
void fo_or_set_threads(int threads);
int fo_or_max_threads(void);

#ifdef __cplusplus
}
#endif
#endif
