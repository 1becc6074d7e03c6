// fo_kernels.h -- launchers of the CUDA kernels (internal to libfo_cuda.so;
// the public boundary is include/fo_attention.h).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

cudaError_t fo_launch_online(const float *q, const float *prefix_k, const float *generated_k, const float *v,
                             const float *sinks, float *out, int64_t query_len, int64_t prefix_len, int64_t total_len,
                             int64_t n_heads, int64_t n_kv_heads, int64_t head_dim, int64_t query_offset,
                             int64_t image_start, int64_t image_end, int exp_fast, cudaStream_t stream);

cudaError_t fo_launch_prefill_f32(const float *q, const float *prefix_k, const float *generated_k, const float *v,
                                  const float *sinks, float *out, int64_t query_len, int64_t prefix_len,
                                  int64_t total_len, int64_t n_heads, int64_t n_kv_heads, int64_t query_offset,
                                  int64_t image_start, int64_t image_end, int softmax_static, int exp_fast,
                                  cudaStream_t stream);

cudaError_t fo_launch_convert_bf16(const float *src, uint16_t *dst, int64_t n, cudaStream_t stream);

// Seal: compact FP32 K [P][H][64], V [P][G][64] -> records [G][stride][160]
// and scales [G][stride][5]; raises FO_FLAG_* bits in *flags.
cudaError_t fo_launch_seal(const float *k, const float *v, int64_t prefix_len, int64_t heads, int64_t groups,
                           int format, void *codes, uint16_t *scales, int64_t stride, unsigned *flags,
                           cudaStream_t stream);
// The fused QKV rows (kv_cache.cu): split, per-head RMS norm and RoPE of
// projection rows qkv [rows][heads*64 + 2*groups*64] with rope
// [rows][heads][32][2]; q, k [rows][heads][64], v [rows][groups][64] and
// optional BF16 copies of k and v.
cudaError_t fo_launch_qkv_rows(const float *qkv, const float *rope, int64_t rows, int heads, int groups, float *q,
                               float *k, float *v, uint16_t *k_bf16, uint16_t *v_bf16, cudaStream_t stream);
// The same for decode rows: q, and the new keys and values appended as tail
// records first.. of a split cache.
cudaError_t fo_launch_qkv_append(const float *qkv, const float *rope, int64_t rows, int heads, int groups, float *q,
                                 int format, void *tail_codes, uint16_t *tail_scales, int64_t tail_stride,
                                 int64_t first, cudaStream_t stream);
// NCCL for the head-sharded prefill (sharded.cu), resolved at run time from
// libnccl.so.2; each returns 0, or -1 with a message in msg.
#define FO_NCCL_ID_BYTES 128
int fo_nccl_unique_id_impl(uint8_t *id, char *msg, size_t n);
int fo_nccl_comm_init_impl(int world, int rank, const uint8_t *id, void **comm, char *msg, size_t n);
int fo_nccl_comm_destroy_impl(void *comm, char *msg, size_t n);
int fo_nccl_gather_bf16(void *comm, uint16_t *block, size_t count, int rank, cudaStream_t stream, char *msg,
                        size_t n);
int fo_nccl_allgather_bytes(void *comm, const void *send, void *recv, size_t bytes, cudaStream_t stream, char *msg,
                            size_t n);
int fo_nccl_barrier(void *comm, int32_t *word, cudaStream_t stream, char *msg, size_t n);

struct fo_decode_page;

// Other ranks' destinations of a head-sharded prefill's BF16 rows: the same
// offset in each peer's gathered block, mapped into this process over NVLink
// (CUDA IPC).  The prefill kernels store every finished row there as well as
// locally (plain peer stores), so the gather overlaps the computation.
#define FO_MAX_PEERS 8
struct fo_peer_out {
    void *dst[FO_MAX_PEERS];
    int32_t n;
};

// One cache's share of a batched append: its expanded rows and tail.
struct fo_append_page {
    const float *k, *v;  // [rows][H][64]
    void *tail_codes;
    uint16_t *tail_scales;
    int64_t tail_stride, first;
};
// Device error bit: a batch plan step found a cache's tail full.
#define FO_DEVERR_CAPACITY 2u
// Append `rows` expanded rows to each of n pages in one launch.
// plan_pages (a batch plan's decode descriptors, or null): the append's first
// lane per page also sets that page's decode length (prefix + first + rows),
// or raises FO_DEVERR_CAPACITY in *err when the tail has no room.
cudaError_t fo_launch_append_batch(const fo_append_page *pages, int64_t n, int64_t rows, int64_t heads, int64_t groups,
                                   int format, fo_decode_page *plan_pages, unsigned *err, cudaStream_t stream);
// Append rows of expanded K, V [rows][H][64] as tail records at index first..
cudaError_t fo_launch_append(const float *k, const float *v, int64_t rows, int64_t heads, int64_t groups, int format,
                             void *tail_codes, uint16_t *tail_scales, int64_t tail_stride, int64_t first,
                             cudaStream_t stream);

// One decode page: a cache's records and the query rows against it.
struct alignas(64) fo_decode_page {
    CUtensorMap rec_map;   // prefix records as padded slots (fo_make_record_map); valid when has_map
    CUtensorMap tc_map;    // BF16 prefix records in 64-element swizzled boxes (fo_make_tc_maps)
    CUtensorMap tail_map;  // BF16 tail records likewise; valid when has_tail_map
    CUtensorMap s1_map;    // BF16 prefix records in 32-element boxes (64-byte swizzle): the second spatial half
    const void *codes;
    const uint16_t *scales;
    const void *tail_codes;
    const uint16_t *tail_scales;
    const float *q;      // [rows][H][64]
    const float *sinks;  // [H]
    float *out;          // [rows][H][64]
    float *part_o;       // [rows][H][splits][64] split partials
    float *part_ml;      // [rows][H][splits][2] (max, denominator)
    unsigned *err;       // error word for bounded waits that gave up (may be null)
    int64_t prefix_len, prefix_stride, tail_stride, last;  // last = prefix_len + tail_len
    int32_t rows, splits;                                   // splits = ceil(last / FO_SPLIT), or see prefix_splits
    int32_t has_map, has_tail_map;
    // 0: splits are FO_SPLIT positions from position 0 (decode.cu).  Otherwise
    // the prefix splits into this many FO_SPLIT-position splits and the tail
    // into its own, starting at prefix_len (decode_tc.cu): splits =
    // prefix_splits + ceil(tail_len / FO_SPLIT).
    int32_t prefix_splits;
    // With prefix_splits set: splits per partial ("unit"), and `splits` counts
    // units per row and head (fo_tc_layout).
    int32_t chunk;
    // Rotated records (FO_KV_ROTATED): the CUDA-core decode rotates each
    // query head's halves as it loads them, the merge un-rotates each output
    // head's halves before it stores them (kv.rs:83-96, 578-589).
    int32_t rotated;
};

// The tensor-core decode's maps of BF16 records (decode_tc.cu) for page p
// (codes, tail_codes, prefix_len and strides set); false if the encoder is
// unavailable or refuses (the caller then uses the CUDA-core decode).
bool fo_make_tc_maps(fo_decode_page *p, int64_t groups, int64_t tail_rows);
// Sets the tensor-core decode's split layout of page p (prefix_len set) with
// tail_len tail positions: prefix_splits, chunk and splits (units per row).
void fo_tc_layout(fo_decode_page *p, int64_t groups, int64_t tail_len);


// The tensor map the decode kernel loads prefix records through: records
// [groups][stride][160] of `format`, rows past prefix_len out of bounds, a
// box of one chunk of keys whose rows are padded to the kernel's slot size.
// Returns false if the driver's encoder is unavailable or refuses.
bool fo_make_record_map(CUtensorMap *map, const void *codes, int format, int64_t prefix_len, int64_t prefix_stride,
                        int64_t groups);

// Positions per decode split: the GPU's position partition.  Fixed, so a
// row's partition depends only on its own length (verify rows equal their
// single-row decodes bit for bit).
#define FO_SPLIT 128

// One page (descriptor read on the host, passed by value).
cudaError_t fo_launch_decode_one(const fo_decode_page *page, int format, int64_t groups, int fast_exp,
                                 cudaStream_t stream);
// One page of BF16 records on the tensor cores (decode_tc.cu) and its split
// merge; the page has prefix_splits and its tc maps set.
cudaError_t fo_launch_decode_tc(const fo_decode_page *page, int64_t groups, int fast_exp, cudaStream_t stream);
// The split merge of one page (a programmatic dependent of the decode just
// launched on `stream`).
cudaError_t fo_launch_decode_merge(const fo_decode_page *page, int64_t groups, cudaStream_t stream);
// n_pages pages whose descriptors are a device array.  advance (a batch
// plan's append descriptors, or null): the merge moves each page's next
// append index on by one once its append and decode are complete (a full tail
// keeps its capacity).
cudaError_t fo_launch_decode_batch(const fo_decode_page *dev_pages, int64_t n_pages, int format, int64_t groups,
                                   int fast_exp, int64_t max_splits, int max_rows, fo_append_page *advance,
                                   cudaStream_t stream);

// One page of BASELINE's INT8 KV format (decode_i8.cu): codes
// [heads][len][64], FP32 scales [heads][ceil(len / 64)], for keys and values.
struct fo_i8_page {
    const int8_t *k_codes, *v_codes;
    const float *k_scales, *v_scales;
    const float *q;      // [heads][64]
    const float *sinks;  // [heads]
    float *out;          // [heads][64]
    float *part_o;       // [heads][splits][64]
    float *part_ml;      // [heads][splits][2]
    unsigned *err;       // error word for bounded waits that gave up (may be null)
    int64_t len;
    int32_t splits;      // ceil(len / FO_I8_SPLIT)
};
#define FO_I8_SPLIT 1024

cudaError_t fo_launch_quantize_i8(const float *x, int64_t len, int64_t heads, int8_t *codes, float *scales,
                                  cudaStream_t stream);
cudaError_t fo_launch_decode_i8(const fo_i8_page *dev_pages, int64_t n_pages, int64_t heads, int32_t max_splits,
                                int fast_exp, cudaStream_t stream);

// The draft head's int8 KV (draft.cu; src/draft_head.rs:177-220, 548-759):
// codes [8][capacity][64] and one FP32 scale per row, for keys and values.
#define FO_DRAFT_KV_WIDTH 512  // KV_HEADS * HEAD_DIM (draft_head.rs:41)
#define FO_DRAFT_MAX_CHAIN 64  // FP32 chain rows one attention takes
cudaError_t fo_launch_draft_push(const float *keys, const float *values, int64_t rows, int64_t capacity, int64_t len,
                                 int8_t *key_codes, float *key_scales, int8_t *value_codes, float *value_scales,
                                 cudaStream_t stream);
#define FO_DRAFT_MAX_SPLITS 64  // CTAs per KV group of one attention
// part: [8][FO_DRAFT_MAX_SPLITS][2][64 + 2] partials; counters: [8], zeroed.
cudaError_t fo_launch_draft_attend(const int8_t *key_codes, const float *key_scales, const int8_t *value_codes,
                                   const float *value_scales, int64_t capacity, const float *q, int64_t start,
                                   int64_t n, const float *chain_keys, const float *chain_values, int64_t chain,
                                   float *part, unsigned *counters, float *out, cudaStream_t stream);

// The bounded-wait self-test kernel (selftest.cu).
cudaError_t fo_launch_bounded_wait(unsigned *err, unsigned long long limit_ns, cudaStream_t stream);

#ifdef __cplusplus
}
#endif
