/*
 * fo_attention.h -- C ABI of the B200 attention backend for falcon-ocr.
 *
 * This is the drop-in boundary of a `--backend cuda` for the reference's
 * attention operators.  Each entry point replaces one reference interface
 * (paths relative to the reference project root):
 *
 *   fo_attention                 kernels::attention_with
 *                                  src/kernels/attention/mod.rs:256-311
 *   fo_attention_prefill_bf16    kernels::attention_prefill_bf16
 *                                  src/kernels/attention/mod.rs:321-349
 *   fo_kv_seal                   SplitPrefix::from_compact  src/quant/kv.rs:225-236
 *   fo_kv_set_fast_exp           SplitPrefix::with_fast_exp src/quant/kv.rs:423-426
 *   fo_kv_seal_layer             model::cache::seal_layer   src/model/cache.rs:218-276
 *   fo_kv_append                 SplitPrefix::append        src/quant/kv.rs:430-449
 *   fo_kv_truncate_tail          SplitPrefix::truncate_tail src/quant/kv.rs:846-849
 *   fo_kv_tail_len               SplitPrefix::tail_len      src/quant/kv.rs:841-843
 *   fo_kv_bytes                  SplitPrefix::bytes         src/quant/kv.rs:523-525
 *   fo_kv_attention_decode       SplitPrefix::attention_decode      src/quant/kv.rs:568-576
 *   fo_kv_attention_decode_rows  SplitPrefix::attention_decode_rows src/quant/kv.rs:856-865
 *   fo_kv_attention_decode_batch one decode row per page, as Model::decode_batch_next
 *                                  calls LayerCache::attention per page (src/model/mod.rs:827-852)
 *   fo_kv_append_batch           one append per page, as Model::decode_batch_next calls
 *                                  SplitPrefix::append per page (src/model/mod.rs:760-852)
 *   fo_kv_plan_create/step/finish  the same append + one-row decode per page as a
 *                                  device-resident step (graph-capturable; no counterpart)
 *   fo_qkv_prefix_rows           model::fused::fused_prefix_rows (split, per-head RMS norm,
 *                                  RoPE, compact append, BF16 copies) src/model/fused.rs:17-116
 *   fo_kv_append_qkv             rope::split_norm_rope then SplitPrefix::append for decode
 *                                  rows, src/model/rope.rs:15-85, src/quant/kv.rs:430-449
 *   fo_draft_kv_create/destroy   DraftState::new with DraftKv::Q8   src/draft_head.rs:222-240
 *   fo_draft_kv_push             Kv::push / quantize_row             src/draft_head.rs:194-220
 *   fo_draft_attend              attend + group_q8                  src/draft_head.rs:548-759
 *
 * Entry points with no single reference counterpart (each says why below):
 *   fo_attention_prefill_bf16_rows[_split]  query-row bands of the BF16 prefill
 *                                  (the head-sharded multi-GPU prefill's unit)
 *   fo_sharded_prefill_bf16        one page's prefill with heads sharded over the ranks of
 *                                  an NCCL communicator, output all-gathered (BASELINE
 *                                  config 5b; the reference prefills on one host)
 *   fo_nccl_unique_id, fo_nccl_comm_init, fo_nccl_comm_destroy  its communicator
 *   fo_peer_block_register/destroy, fo_sharded_prefill_bf16_peers  the same prefill
 *                                  with the gather as NVLink peer stores from the kernels
 *   fo_convert_bf16                the Bf16Kv::Convert rounding on its own
 *   fo_decode_rows_static_scratch  verify decode with no device allocation,
 *   fo_decode_static_scratch_status  and its device error report
 *   fo_i8_*                        BASELINE config 4's INT8 KV format
 *   fo_selftest_bounded_wait       the kernels' bounded-wait failure path
 *
 * Conventions (mirroring the reference's, src/kernels/attention/mod.rs:159-195
 * and src/quant/kv.rs:248-295):
 *   - Every call returns an fo_status; FO_OK is 0.  Shape violations that the
 *     reference asserts on return FO_ERR_INVALID and write nothing; the seal
 *     errors the reference returns as anyhow::Result map to FO_ERR_PAIR,
 *     FO_ERR_NONFINITE, FO_ERR_OVERFLOW and FO_ERR_CAPACITY.
 *     fo_last_error() returns the calling thread's last message.
 *   - Buffers are caller-owned.  `mem` says whether the float pointers of a
 *     call are host (FO_MEM_HOST: copied to and from the device inside the
 *     call) or device (FO_MEM_DEVICE: read and written in place).  Outputs
 *     are overwritten, token-major [row][head][head_dim] FP32.
 *   - Work runs on the context's stream.  FO_MEM_HOST calls return after the
 *     output is on the host; FO_MEM_DEVICE calls return after launching.
 *   - Decode never allocates device memory: fo_kv_seal reserves every
 *     buffer a later append or decode on that cache needs.
 */
#ifndef FO_ATTENTION_H
#define FO_ATTENTION_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
    FO_OK = 0,
    FO_ERR_INVALID = 1,     /* null pointer or shape the reference asserts against */
    FO_ERR_PAIR = 2,        /* temporal keys differ inside a GQA pair (kv.rs:266-278) */
    FO_ERR_NONFINITE = 3,   /* non-finite value in a sealed prefix (kv.rs:288) */
    FO_ERR_OVERFLOW = 4,    /* Q8/Q16 code * scale overflowed (kv.rs:328, 355) */
    FO_ERR_CAPACITY = 5,    /* prefix_len == 0, capacity < prefix_len or above 3,000,000, or tail full */
    FO_ERR_CUDA = 6,        /* a CUDA runtime call failed; see fo_last_error() */
    FO_ERR_DECLINED = 7     /* shape outside a kernel's scope; nothing written */
} fo_status;

#define FO_MEM_DEVICE 0
#define FO_MEM_HOST 1

/* Split-cache record formats (src/quant/kv.rs:98-152; BF16 is new). */
#define FO_KV_F32 0
#define FO_KV_Q16 1
#define FO_KV_Q8 2
#define FO_KV_BF16 3
/* 4-bit codes -7..7, two per byte (element 2i in the low nibble), one BF16
 * scale per 32 elements (Records::Q4, kv.rs:109-114). */
#define FO_KV_Q4 4
/* Flag: every 32-element block of a record is stored rotated, H D x with H
 * the 32-point Sylvester Hadamard matrix and D a fixed sign pattern per
 * block kind (src/quant/rotation.rs); decode rotates each query head's
 * halves and un-rotates each output head's halves.  Valid with F32, Q8 and
 * Q4. */
#define FO_KV_ROTATED 16
#define FO_KV_Q8_ROT (FO_KV_Q8 | FO_KV_ROTATED) /* Kv::Q8Rot */
#define FO_KV_Q4_ROT (FO_KV_Q4 | FO_KV_ROTATED) /* Kv::Q4Rot */

/* ExpMode / PrefillSoftmax (src/kernels/attention/mod.rs:204-221). */
#define FO_EXP_EXACT 0
#define FO_EXP_FAST 1
#define FO_SOFTMAX_ONLINE 0
#define FO_SOFTMAX_STATIC 1

/* Geometry (src/kernels/attention/mod.rs:35-76). */
typedef struct {
    int64_t query_offset;
    int64_t image_start;
    int64_t image_end;
} fo_geometry;

/* CompactKv (src/kernels/attention/mod.rs:78-97): prefix_k
 * [prefix_len][n_heads][head_dim], generated_k [total_len - prefix_len]
 * [n_kv_heads][head_dim], v [total_len][n_kv_heads][head_dim]. */
typedef struct {
    const float *prefix_k;
    const float *generated_k;
    const float *v;
    int64_t prefix_len;
    int64_t total_len;
    int64_t n_heads;
    int64_t n_kv_heads;
    int64_t head_dim;
} fo_compact_kv;

/* PrefillOptions (src/kernels/attention/mod.rs:204-210). */
typedef struct {
    int32_t exp;          /* FO_EXP_EXACT | FO_EXP_FAST: the online softmax's exp */
    int32_t profile;      /* nonzero: record per-launch device times (fo_ctx_last_ms) */
    int32_t softmax;      /* BF16 kernel's softmax: FO_SOFTMAX_ONLINE | FO_SOFTMAX_STATIC */
    int32_t fp32_softmax; /* FP32 tiles' softmax */
} fo_prefill_options;

typedef struct fo_ctx fo_ctx;
typedef struct fo_kv_cache fo_kv_cache;
typedef struct fo_kv_plan fo_kv_plan;

/* Library version (major * 10000 + minor * 100 + patch). */
int fo_version(void);
/* The calling thread's last error message ("" when none). */
const char *fo_last_error(void);

/* A device context: device index and a CUDA stream (cudaStream_t passed as
 * void*; NULL is CUDA's default stream).  All work of calls made with this
 * context is ordered on that stream. */
int fo_ctx_create(int device, void *stream, fo_ctx **out);
int fo_ctx_destroy(fo_ctx *ctx);
int fo_ctx_synchronize(fo_ctx *ctx);
/* Device milliseconds of the last call's kernels when options.profile was set. */
int fo_ctx_last_ms(fo_ctx *ctx, float *ms);

/* Self-test of the kernels' bounded waits (no counterpart in the reference):
 * runs one CTA whose mbarrier wait never completes, so it gives up after
 * limit_ns nanoseconds, raises the context's error word and returns.  The
 * call synchronizes and returns FO_ERR_CUDA with the timeout message when
 * the wait gave up as designed (FO_OK would mean it did not); the context
 * stays usable. */
int fo_selftest_bounded_wait(fo_ctx *ctx, uint64_t limit_ns);

/* kernels::attention_with (mod.rs:256-311): any head_dim <= 256, prefix or
 * mixed caches, any query length.  query_len >= 4 with head_dim 64 runs the
 * FP32 tiles (options.fp32_softmax, options.exp); other shapes run the
 * online head.  q and output hold [query_len][n_heads][head_dim]. */
int fo_attention(fo_ctx *ctx, const float *q, const fo_compact_kv *kv, int64_t query_len, fo_geometry geometry,
                 const float *sinks, float *output, fo_prefill_options options, int mem);

/* kernels::attention_prefill_bf16 (mod.rs:321-349): the tcgen05 BF16 prefill
 * of a pure prefix (query_offset 0, query_len == prefix_len == total_len,
 * head_dim 64).  Returns FO_ERR_DECLINED, writing nothing, for other shapes
 * (the reference returns false).  keys_bf16 [total][n_heads][64] and
 * values_bf16 [total][n_kv_heads][64] are optional device BF16 copies
 * (Bf16Kv::Converted); when NULL the call converts kv's FP32 keys and
 * values into context scratch (Bf16Kv::Convert).  options.softmax selects
 * online or static shift; the static shift requires every score
 * |q.k| / 8 to stay below 80 (per-head RMS norms keep it below 8).  As in the
 * reference, which selects the static shift without checking scores, the
 * bound is not checked: outside it the static shift's results are undefined
 * (denominators overflow to inf or underflow to 0). */
int fo_attention_prefill_bf16(fo_ctx *ctx, const float *q, const fo_compact_kv *kv, int64_t query_len,
                              fo_geometry geometry, const float *sinks, float *output, const uint16_t *keys_bf16,
                              const uint16_t *values_bf16, fo_prefill_options options, int mem);

/* The BF16 prefill of query rows [query_begin, query_end) only (no
 * counterpart in the reference, which prefills a page whole): a pure prefix
 * of total_len positions with pre-converted BF16 keys [total][n_heads][64]
 * and values [total][n_kv_heads][64], device pointers only, q and output
 * FP32 [total][n_heads][64] (rows outside the range are not written).
 * query_begin is a multiple of 256 and query_end a multiple of 256 or
 * total_len.  It lets a caller pipeline the output: the head-sharded
 * multi-GPU prefill gathers each finished band of rows while the next one
 * computes. */
int fo_attention_prefill_bf16_rows(fo_ctx *ctx, const float *q, const uint16_t *keys_bf16,
                                   const uint16_t *values_bf16, int64_t total_len, int64_t n_heads, int64_t n_kv_heads,
                                   fo_geometry geometry, const float *sinks, float *output, int64_t query_begin,
                                   int64_t query_end, fo_prefill_options options);

/* fo_attention_prefill_bf16_rows with each query pair's key tiles cut into
 * kv_splits consecutive ranges (1..64), one CTA per range, combined in range
 * order with the sink by a second kernel.  For launches with fewer query
 * pairs x heads than the GPU has SMs (a band of a head-sharded page on many
 * GPUs), where the longest pairs would otherwise bound the launch.  Results
 * equal the unsplit call within rounding (the ranges' partial sums add in a
 * different order); the partials live in context scratch
 * (kv_splits x the launch's rows, rounded to 256, x n_heads x 65 floats).  With out_bf16 set, output is
 * BF16 [total][n_heads][64] instead (each value the FP32 result rounded to
 * nearest even as it is stored), the operand of the sharded prefill's
 * gather; 8-byte aligned then. */
int fo_attention_prefill_bf16_rows_split(fo_ctx *ctx, const float *q, const uint16_t *keys_bf16,
                                         const uint16_t *values_bf16, int64_t total_len, int64_t n_heads,
                                         int64_t n_kv_heads, fo_geometry geometry, const float *sinks, void *output,
                                         int32_t out_bf16, int64_t query_begin, int64_t query_end,
                                         fo_prefill_options options, int32_t kv_splits);

/* The head-sharded prefill of one page on this rank (one process per GPU;
 * `comm` an ncclComm_t of `world` ranks from the process's libnccl.so.2).
 * This rank holds n_heads query heads and their n_kv_heads KV groups: q
 * [total_len][n_heads][64] FP32, keys_bf16 [total_len][n_heads][64], values_bf16
 * [total_len][n_kv_heads][64], sinks [n_heads] (device pointers).  The rows
 * are computed in n_bands bands (256-row boundaries, latest first) with
 * kv_splits key ranges (0: enough for one CTA per SM); each band's BF16
 * output goes straight into this rank's slot of the band's block and the
 * block is all-gathered in place on the context's own comm stream while the
 * next band computes.  gathered (BF16, 16-byte aligned) holds the bands one
 * after another, each [world][rows][n_heads][64] rank-major: head j of rank
 * w is the page's head w * n_heads + j.  Every rank calls this with the same
 * shapes and bands.  On return the gathers are ordered before later work on
 * the context's stream. */
int fo_sharded_prefill_bf16(fo_ctx *ctx, void *comm, int32_t rank, int32_t world, const float *q,
                            const uint16_t *keys_bf16, const uint16_t *values_bf16, int64_t total_len,
                            int64_t n_heads, int64_t n_kv_heads, fo_geometry geometry, const float *sinks,
                            fo_prefill_options options, int32_t n_bands, int32_t kv_splits, uint16_t *gathered);
/* NCCL plumbing for it (a host with its own NCCL binding may pass its own
 * communicator instead): a 128-byte unique id from one rank, shared by the
 * caller; a communicator on the context's device. */
int fo_nccl_unique_id(uint8_t *id);
int fo_nccl_comm_init(fo_ctx *ctx, int32_t world, int32_t rank, const uint8_t *id, void **comm);
int fo_nccl_comm_destroy(void *comm);

/* The head-sharded prefill with the gather done by the kernels themselves:
 * fo_peer_block_register (collective: every rank of `comm` calls it with its
 * own device buffer of `bytes` bytes, an allocation that CUDA IPC can share,
 * on one node, at most 8 ranks) maps every rank's buffer into this process
 * over NVLink.  fo_sharded_prefill_bf16_peers then computes this rank's heads
 * (one launch over all rows) and its kernels store every finished BF16 row
 * into all ranks' buffers at [rank][total_len][n_heads][64] (plain peer
 * stores, overlapped with the computation; no multicast, no peer loads).  The
 * call starts with a barrier of the ranks (every rank's earlier work, such as
 * reads of the previous page, has completed before anyone overwrites its
 * buffer) and ends with one (every rank's stores have landed); both are
 * one-word NCCL all-reduces on the context's stream.  Results are bit for bit
 * those of fo_sharded_prefill_bf16 with one band and the same kv_splits. */
typedef struct fo_peer_block fo_peer_block;
int fo_peer_block_register(fo_ctx *ctx, void *comm, int32_t rank, int32_t world, uint16_t *gathered, int64_t bytes,
                           fo_peer_block **out);
int fo_peer_block_destroy(fo_peer_block *block);
int fo_sharded_prefill_bf16_peers(fo_ctx *ctx, fo_peer_block *block, const float *q, const uint16_t *keys_bf16,
                                  const uint16_t *values_bf16, int64_t total_len, int64_t n_heads, int64_t n_kv_heads,
                                  fo_geometry geometry, const float *sinks, fo_prefill_options options,
                                  int32_t kv_splits);

/* FP32 -> BF16 (round to nearest even) of n device values, the conversion
 * fo_attention_prefill_bf16 applies to Bf16Kv::Convert inputs. */
int fo_convert_bf16(fo_ctx *ctx, const float *src, uint16_t *dst, int64_t n);

/* SplitPrefix::from_compact (kv.rs:225-236): seal a compact prefix (k
 * [prefix_len][n_heads][64], v [prefix_len][n_kv_heads][64]) into
 * group-major records of `format`, with room for capacity - prefix_len
 * generated positions.  chunks is the reference's position-chunk request
 * (0 for its default); it only changes rounding, and the GPU partitions
 * positions by its own fixed split.  The cache keeps a reference to ctx. */
int fo_kv_seal(fo_ctx *ctx, const float *k, const float *v, int64_t prefix_len, int64_t capacity, int64_t n_heads,
               int64_t n_kv_heads, int64_t head_dim, int32_t format, int32_t chunks, int mem, fo_kv_cache **out);
int fo_kv_destroy(fo_kv_cache *cache);
/* seal_layer (src/model/cache.rs:218-276) for layer `layer` after its
 * prefill, on DEVICE pointers k, v (the compact prefix): filled must equal
 * prefix_len (a complete prefix); the records are Q8 when bit `layer` of
 * kv_q8_layers is set (Tuning::kv_q8_layers, cache.rs:247; layers past 63
 * never) and `mode` otherwise; the decode's fast exp is decode_fast_exp when
 * it is 0 or 1 (Tuning::decode_fast_exp) and otherwise fast_exps with a Q8
 * mode (default_fast_exp, kv.rs:182-184: the cache's mode, not the layer's
 * format, decides).  A compact-mode cache is never sealed: the caller keeps
 * its compact buffers. */
int fo_kv_seal_layer(fo_ctx *ctx, int32_t layer, uint64_t kv_q8_layers, int32_t mode, int32_t fast_exps,
                     int32_t decode_fast_exp, const float *k, const float *v, int64_t filled, int64_t prefix_len,
                     int64_t capacity, int64_t n_heads, int64_t n_kv_heads, int32_t chunks, fo_kv_cache **out);
/* SplitPrefix::with_fast_exp (kv.rs:423-426): the softmax's exp becomes
 * exp_poly (src/kernels/exp.rs:232-277) for single and verify rows alike. */
int fo_kv_set_fast_exp(fo_kv_cache *cache, int32_t fast);
/* SplitPrefix::append (kv.rs:430-449): rows of expanded k and v, each
 * [rows][n_heads][64], identical inside each GQA pair; the pair's first
 * head is stored.  Non-finite values give NaN blocks (kv.rs:451-455). */
int fo_kv_append(fo_kv_cache *cache, const float *k, const float *v, int64_t rows, int mem);
/* fo_kv_append on n caches in one launch, as the per-page appends of
 * Model::decode_batch_next (src/model/mod.rs:760-852): cache i takes `rows`
 * expanded rows from the DEVICE pointers k[i], v[i].  The caches share a
 * context, format and heads and are distinct; every capacity is checked
 * before anything is written (FO_ERR_CAPACITY leaves all caches as they
 * were).  The records equal those of n separate fo_kv_append calls. */
int fo_kv_append_batch(fo_kv_cache *const *caches, int64_t n, const float *const *k, const float *const *v,
                       int64_t rows);
/* A batch plan: the per-page append of one row and the one-row decode of
 * Model::decode_batch_next (src/model/mod.rs:760-852) for n caches, with its
 * launch descriptors resident on the device and moved on by one position per
 * step on the device, so a step needs no host work and can be captured in a
 * CUDA graph and replayed.  Cache i reads its new row from the DEVICE
 * pointers k[i], v[i] (expanded [1][n_heads][64]) and its query from q[i],
 * and writes its output to output[i], at every step: the caller refills
 * those buffers between steps.  The caches share context, format, heads and
 * exp, are distinct, and each has room for at least one more row.  While a
 * plan is open its caches take no other calls; fo_kv_plan_finish brings
 * their tail lengths back and frees the plan.  A step that finds a tail full
 * writes nothing more to it and repeats its last position; finish then
 * returns FO_ERR_CAPACITY. */
int fo_kv_plan_create(fo_kv_cache *const *caches, int64_t n, const float *const *k, const float *const *v,
                      const float *const *q, const float *const *sinks, float *const *output, fo_kv_plan **out);
int fo_kv_plan_step(fo_kv_plan *plan);
int fo_kv_plan_finish(fo_kv_plan *plan);

/* The fused QKV rows of a prefill (fused_prefix_rows, src/model/fused.rs:17-116;
 * the same arithmetic as split_norm_rope, src/model/rope.rs:15-85), on DEVICE
 * pointers: qkv [rows][n_heads*64 + 2*n_kv_heads*64] projection rows, rope
 * [rows][n_heads][32] {cos, sin} pairs.  Query head h and key head h (KV head
 * h / (n_heads / n_kv_heads)) are RMS-normalized (eps f32::EPSILON, the
 * reference's pairwise sum of squares) and rotated by rope[row][h]; q and k
 * get [rows][n_heads][64], v [rows][n_kv_heads][64] (a copy).  k_bf16 and
 * v_bf16 (nullable) get the BF16 copies (round to nearest even) in the same
 * layouts, the operands of fo_attention_prefill_bf16.  Bit for bit the
 * reference's row.  Buffers 8-byte aligned (BF16 copies 4-byte). */
int fo_qkv_prefix_rows(fo_ctx *ctx, const float *qkv, const float *rope, int64_t rows, int64_t n_heads,
                       int64_t n_kv_heads, float *q, float *k, float *v, uint16_t *k_bf16, uint16_t *v_bf16);
/* Decode rows of the same pass: q [rows][n_heads][64] as above, and each
 * row's keys and values appended to the cache's tail (the pair's first key
 * head, with its own rotation, and the group's value: what fo_kv_append
 * stores from split_norm_rope's expanded rows).  DEVICE pointers. */
int fo_kv_append_qkv(fo_kv_cache *cache, const float *qkv, const float *rope, int64_t rows, float *q);
/* SplitPrefix::truncate_tail (kv.rs:846-849). */
int fo_kv_truncate_tail(fo_kv_cache *cache, int64_t tail_len);
int64_t fo_kv_tail_len(const fo_kv_cache *cache);
int64_t fo_kv_prefix_len(const fo_kv_cache *cache);
/* Allocated record bytes, prefix and tail (kv.rs:523-525). */
int64_t fo_kv_bytes(const fo_kv_cache *cache);
/* Device pointers and strides of the records, for tests and tooling:
 * codes [groups][prefix_stride][160], scales [groups][prefix_stride][5],
 * tail_codes [groups][tail_stride][128], tail_scales [groups][tail_stride][4]. */
int fo_kv_records(const fo_kv_cache *cache, void **codes, void **scales, void **tail_codes, void **tail_scales,
                  int64_t *prefix_stride, int64_t *tail_stride);

/* SplitPrefix::attention_decode (kv.rs:568-576): q and output [n_heads][64];
 * total_len must equal prefix_len + tail_len. */
int fo_kv_attention_decode(fo_kv_cache *cache, const float *q, int64_t total_len, const float *sinks, float *output,
                           int mem);
/* SplitPrefix::attention_decode_rows (kv.rs:856-865): rows 1..8 (and at most
 * max(tail_len, 1)); row r sees prefix_len + tail_len - rows + 1 + r
 * positions and equals its single-row decode bit for bit. */
int fo_kv_attention_decode_rows(fo_kv_cache *cache, const float *q, int64_t rows, const float *sinks, float *output,
                                int mem);
/* One single-row decode per cache (independent pages), in one launch.  All
 * caches share one context and head shape; q[i], sinks[i], output[i] are
 * device pointers.  Each page's result equals its fo_kv_attention_decode. */
int fo_kv_attention_decode_batch(fo_kv_cache *const *caches, int64_t n, const float *const *q,
                                 const float *const *sinks, float *const *output);

/* Verify-row decode that allocates no device memory.  No counterpart in the
 * reference.  For callers that cannot allocate while they decode: a serving
 * runtime that owns all GPU memory through its own pool, or a decode loop
 * that must avoid cudaMalloc/cudaFree because they can synchronize the whole
 * device.  The caller passes the sealed records (as fo_kv_records describes
 * them), device q [rows][n_heads][64], sinks and output, and a stream (NULL
 * is the default stream); results equal fo_kv_attention_decode_rows'.  The
 * split partials live in one static device array of about 4.1 MiB that every
 * GPU loading the library holds until exit, which limits a call to 8 rows,
 * 16 heads and 16,384 positions (FO_ERR_CAPACITY beyond).  codes and
 * tail_codes must be 16-byte aligned and q 8-byte aligned (FO_ERR_INVALID
 * otherwise).  The first call on a device looks the array up and should come
 * before any stream capture (a failed lookup is retried by the next call);
 * calls that overlap on the GPU share the array and race.  If a bounded
 * device wait of a call gives up, that call's outputs are NaN and the next
 * fo_decode_static_scratch_status reports it. */
int fo_decode_rows_static_scratch(const void *codes, const uint16_t *scales, const void *tail_codes,
                                  const uint16_t *tail_scales, int32_t format, int64_t prefix_len,
                                  int64_t prefix_stride, int64_t tail_len, int64_t tail_stride, int64_t n_heads,
                                  int64_t n_kv_heads, const float *q, int64_t rows, const float *sinks,
                                  int32_t fast_exp, float *output, void *stream);
/* Device status of fo_decode_rows_static_scratch on the current device (no
 * counterpart in the reference): synchronizes `stream`, then returns
 * FO_ERR_CUDA if a bounded wait of any call since the last check gave up
 * (those calls wrote NaN outputs) and clears the report; FO_OK otherwise.
 * Allocates nothing. */
int fo_decode_static_scratch_status(void *stream);

/* BASELINE config 4's INT8 KV format (no counterpart in the reference,
 * whose INT8 KV is the Q8 record format above): keys and values of every head
 * stored apart as int8 codes [n_heads][len][64] with one FP32 scale per
 * (head, 64-position group) each; code = round-to-nearest-even(x / scale)
 * clamped to [-127, 127], scale = max |x| of the group / 127.  k and v are
 * [len][n_heads][64] FP32 (host or device per `mem`). */
typedef struct fo_i8_cache fo_i8_cache;
int fo_i8_seal(fo_ctx *ctx, const float *k, const float *v, int64_t len, int64_t n_heads, int mem,
               fo_i8_cache **out);
int fo_i8_destroy(fo_i8_cache *cache);
int64_t fo_i8_bytes(const fo_i8_cache *cache);
/* Device pointers to the cache's codes and scales (for tests and tools). */
int fo_i8_records(const fo_i8_cache *cache, const int8_t **k_codes, const float **k_scales, const int8_t **v_codes,
                  const float **v_scales);
/* One decode row per page, all pages in one launch: q[i] [n_heads][64],
 * sinks[i] [n_heads], output[i] [n_heads][64], device pointers; every head
 * attends over all len positions of its page. */
int fo_i8_decode_batch(fo_i8_cache *const *caches, int64_t n, const float *const *q, const float *const *sinks,
                       float *const *output, int32_t fast_exp);

/* The draft head's int8 key/value cache (DraftState's Kv::Q8,
 * src/draft_head.rs:177-220): each verified position's key and value,
 * [512] FP32 = 8 groups x 64, stored as int8 codes group-major
 * [8][capacity][64] with one FP32 scale per 64-value row, code =
 * round(v * 127 / max |row|) (half away from zero, clamped to +-127, NaN 0),
 * scale = max / 127. */
typedef struct fo_draft_kv fo_draft_kv;
int fo_draft_kv_create(fo_ctx *ctx, int64_t capacity, fo_draft_kv **out);
int fo_draft_kv_destroy(fo_draft_kv *kv);
/* Append `rows` positions: keys and values [rows][512] (host or device per
 * `mem`; device pointers 8-byte aligned). */
int fo_draft_kv_push(fo_draft_kv *kv, const float *keys, const float *values, int64_t rows, int mem);
int64_t fo_draft_kv_len(const fo_draft_kv *kv);
int64_t fo_draft_kv_bytes(const fo_draft_kv *kv);
/* Device pointers to the codes and scales (for tests and tools). */
int fo_draft_kv_records(const fo_draft_kv *kv, const int8_t **key_codes, const float **key_scales,
                        const int8_t **value_codes, const float **value_scales);
/* attend (src/draft_head.rs:548-627) with group_q8 (:706-759): the query
 * q [16][64] of heads 2g, 2g+1 over KV group g's verified rows
 * [max(0, bases - window), bases) (window 0: all of them) and then `chain`
 * FP32 rows chain_keys / chain_values [chain][512] (0..64 rows); scores
 * q.k / 8 (a row's dot times its key scale), softmax with the reference's
 * exp_poly, output = sum p * v (value scale folded into p) times 1 / sum,
 * [16][64].  bases <= fo_draft_kv_len; at least one row attended. */
int fo_draft_attend(fo_draft_kv *kv, const float *q, int64_t bases, int64_t window, const float *chain_keys,
                    const float *chain_values, int64_t chain, float *output, int mem);

#ifdef __cplusplus
}
#endif
#endif
