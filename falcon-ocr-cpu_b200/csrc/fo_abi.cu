// fo_abi.cu -- host side of the C ABI (include/fo_attention.h): contexts,
// sealed caches, shape validation with the reference's rules, host/device
// staging and kernel dispatch.  Host code only; kernels live in the other
// .cu files of this directory.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdio>
#include <algorithm>
#include <cstring>
#include <string>
#include <vector>

#include "../../include/fo_attention.h"
#include "fo_common.cuh"
#include "fo_kernels.h"

#define FO_RECORD_ELEMS 160   // prefix record elements (src/quant/kv.rs:55)
#define FO_TAIL_ELEMS 128     // tail record elements (src/quant/kv.rs:60)
#define FO_MAX_ROWS_ABI 8     // verification rows (src/quant/kv.rs:68)

extern "C" cudaError_t fo_launch_prefill_bf16(const float *q, const uint16_t *keys_bf16, const uint16_t *values_bf16,
                                              const float *sinks, void *out, int out_bf16, int64_t total,
                                              int64_t n_heads, int64_t n_kv_heads, int64_t image_start,
                                              int64_t image_end,
                                              int64_t query_begin, int64_t query_end, int softmax_static, int exp_fast,
                                              unsigned *err, int n_split, float *part_o, float *part_ml,
                                              const fo_peer_out *peers, cudaStream_t stream);

#define FO_WAIT_LIMIT_MAX_NS 10000000000ull
#define FO_BATCH_PAGES 1024  // pages per batched launch

namespace {

thread_local std::string g_last_error;

int fail(int status, const char *fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return status;
}

int cuda_fail(cudaError_t e, const char *what) {
    return fail(FO_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

#define FO_CUDA(call, what)                         \
    do {                                            \
        cudaError_t e_ = (call);                    \
        if (e_ != cudaSuccess) return cuda_fail(e_, what); \
    } while (0)

// A device buffer that grows on demand (prefill staging and scratch only;
// decode paths use buffers reserved at seal time).
struct DevBuf {
    void *ptr = nullptr;
    size_t bytes = 0;
    cudaError_t ensure(size_t need) {
        if (need <= bytes) return cudaSuccess;
        if (ptr) cudaFree(ptr);
        ptr = nullptr;
        bytes = 0;
        cudaError_t e = cudaMalloc(&ptr, need);
        if (e == cudaSuccess) bytes = need;
        return e;
    }
    void release() {
        if (ptr) cudaFree(ptr);
        ptr = nullptr;
        bytes = 0;
    }
};

// Pinned host staging for the descriptors of batched launches, two slots:
// a slot is rewritten only after its previous upload has completed, so a call
// never waits for the kernels it launched before.
struct HostDesc {
    void *ptr[2] = {nullptr, nullptr};
    cudaEvent_t done[2] = {nullptr, nullptr};
    size_t bytes = 0;
    int next = 0;
    cudaError_t ensure(size_t need) {
        if (need <= bytes) return cudaSuccess;
        release();
        for (int i = 0; i < 2; i++) {
            cudaError_t e = cudaHostAlloc(&ptr[i], need, cudaHostAllocDefault);
            if (e == cudaSuccess) e = cudaEventCreateWithFlags(&done[i], cudaEventDisableTiming);
            if (e != cudaSuccess) return e;
        }
        bytes = need;
        return cudaSuccess;
    }
    // A free slot (its last upload finished) and its index.
    void *acquire(int &slot) {
        slot = next;
        next ^= 1;
        if (done[slot]) cudaEventSynchronize(done[slot]);
        return ptr[slot];
    }
    cudaError_t uploaded(int slot, cudaStream_t st) { return cudaEventRecord(done[slot], st); }
    void release() {
        for (int i = 0; i < 2; i++) {
            if (done[i]) cudaEventSynchronize(done[i]);
            if (ptr[i]) cudaFreeHost(ptr[i]);
            if (done[i]) cudaEventDestroy(done[i]);
            ptr[i] = nullptr;
            done[i] = nullptr;
        }
        bytes = 0;
    }
};

// Keeps the caller's current device and restores it on exit.
struct DeviceGuard {
    int prev = -1;
    explicit DeviceGuard(int dev) {
        cudaGetDevice(&prev);
        if (prev != dev) cudaSetDevice(dev);
    }
    ~DeviceGuard() {
        int cur = -1;
        cudaGetDevice(&cur);
        if (prev >= 0 && cur != prev) cudaSetDevice(prev);
    }
};

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }
bool aligned4(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 3) == 0; }

}  // namespace

struct fo_ctx {
    int device = 0;
    cudaStream_t stream = nullptr;
    bool own_stream = false;
    unsigned *flags = nullptr;                 // seal status bits
    unsigned *dev_err = nullptr;               // kernel error bits (bounded waits that gave up)
    DevBuf stage[6];                           // prefill host staging: q, prefix_k, generated_k, v, sinks, out
    DevBuf bf16_k, bf16_v;                     // Bf16Kv::Convert scratch
    DevBuf split_o, split_ml;                  // key-range split partials of the row-band prefill
    DevBuf pages;                              // decode batch descriptors (device)
    HostDesc host_pages;                       // and their pinned staging
    DevBuf append_pages;                       // batched-append descriptors (device)
    HostDesc host_append_pages;
    DevBuf i8_pages;                           // INT8-format decode descriptors (device)
    HostDesc host_i8_pages;
    cudaEvent_t ev0 = nullptr, ev1 = nullptr;
    float last_ms = 0.0f;
    // Host-buffer prefill pipeline: copy streams and per-band events.
    cudaStream_t h2d = nullptr, d2h = nullptr;
    std::vector<cudaEvent_t> band_ev;
    // Head-sharded prefill: the gathers' stream and its events.
    cudaStream_t comm = nullptr;
    std::vector<cudaEvent_t> comm_ev;
};

struct fo_kv_cache {
    fo_ctx *ctx = nullptr;
    int32_t format = 0;
    int32_t chunks = 0;
    int32_t fast_exp = 0;
    int64_t prefix_len = 0, capacity = 0, tail_capacity = 0, tail_len = 0;
    int64_t heads = 0, groups = 0;
    int64_t prefix_stride = 0, tail_stride = 0, max_splits = 0;
    void *codes = nullptr, *tail_codes = nullptr;
    uint16_t *scales = nullptr, *tail_scales = nullptr;
    float *part_o = nullptr, *part_ml = nullptr;     // decode split partials, rows <= 8

    float *q_stage = nullptr, *out_stage = nullptr;  // [8][H][64] host-mode staging
    float *sinks_stage = nullptr;                    // [H]
    float *rows_stage = nullptr;                     // [2][8][H][64] append staging
    size_t bytes = 0;                                // record bytes
    alignas(64) CUtensorMap rec_map;                 // prefix records for the decode kernel's TMA loads
    int has_map = 0;
    // BF16 records: the tensor-core decode's maps (decode_tc.cu), built at seal.
    alignas(64) CUtensorMap tc_map, tail_map, s1_map;
    int has_tc = 0, has_tail_map = 0;
};

// Every rank's gathered block of a head-sharded prefill, mapped into this
// process (CUDA IPC over NVLink): the destinations of the peer-store gather.
struct fo_peer_block {
    fo_ctx *ctx = nullptr;
    void *comm = nullptr;
    int32_t rank = 0, world = 0;
    uint16_t *local = nullptr;
    int64_t bytes = 0;
    uint16_t *block[FO_MAX_PEERS] = {};  // every rank's block (this rank's is `local`)
    void *opened[FO_MAX_PEERS] = {};     // IPC mappings to close
    int32_t *word = nullptr;             // the barriers' device word
};

// The draft head's int8 key/value cache (DraftState's Kv::Q8,
// src/draft_head.rs:177-220): codes [8][capacity][64], one scale per row.
struct fo_draft_kv {
    fo_ctx *ctx = nullptr;
    int64_t capacity = 0, len = 0;
    int8_t *key_codes = nullptr, *value_codes = nullptr;
    float *key_scales = nullptr, *value_scales = nullptr;
    float *part = nullptr;        // [8][FO_DRAFT_MAX_SPLITS][2][66] attention partials
    unsigned *counters = nullptr;  // [8] CTAs done per group (zero between calls)
    float *stage = nullptr;   // host-mode staging: q, out [16][64], chain keys and values
    size_t bytes = 0;
};

struct fo_i8_cache {
    fo_ctx *ctx = nullptr;
    int64_t len = 0, heads = 0, splits = 0;
    int8_t *k_codes = nullptr, *v_codes = nullptr;
    float *k_scales = nullptr, *v_scales = nullptr;
    float *part_o = nullptr, *part_ml = nullptr;  // decode partials [heads][splits][64], [..][2]
    size_t bytes = 0;                             // codes and scales
};

namespace {

// The record formats: an element format, optionally rotated (F32, Q8 and Q4
// only: Storage, kv.rs:128-152).
int element_format(int format) { return format & ~FO_KV_ROTATED; }

bool valid_format(int format) {
    const int e = element_format(format);
    if (format & ~(FO_KV_ROTATED | 7)) return false;
    if (e < FO_KV_F32 || e > FO_KV_Q4) return false;
    return !(format & FO_KV_ROTATED) || e == FO_KV_F32 || e == FO_KV_Q8 || e == FO_KV_Q4;
}

// Bytes of n record elements (Q4 packs two codes per byte; n even).
size_t code_bytes(int format, size_t n) {
    switch (element_format(format)) {
    case FO_KV_F32: return 4 * n;
    case FO_KV_Q16: return 2 * n;
    case FO_KV_Q8: return n;
    case FO_KV_BF16: return 2 * n;
    case FO_KV_Q4: return n / 2;
    }
    return 0;
}

bool coded(int format) {
    const int e = element_format(format);
    return e == FO_KV_Q16 || e == FO_KV_Q8 || e == FO_KV_Q4;
}

const char *format_name(int format) {
    switch (element_format(format)) {
    case FO_KV_Q16: return "Q16";
    case FO_KV_Q8: return "Q8";
    case FO_KV_Q4: return "Q4";
    }
    return "KV";
}

// CompactKv::validate (src/kernels/attention/mod.rs:159-195).
int validate_compact(const float *q, const fo_compact_kv *kv, int64_t query_len, const fo_geometry &g,
                     const float *sinks, const float *output) {
    if (!kv) return fail(FO_ERR_INVALID, "attention: null CompactKv");
    if (!(kv->head_dim > 0 && kv->n_heads > 0 && kv->n_kv_heads > 0))
        return fail(FO_ERR_INVALID, "attention head dimensions must be positive");
    if (kv->n_heads % kv->n_kv_heads != 0) return fail(FO_ERR_INVALID, "attention GQA grouping");
    if (kv->prefix_len < 0 || kv->prefix_len > kv->total_len) return fail(FO_ERR_INVALID, "attention prefix length");
    if (query_len < 0) return fail(FO_ERR_INVALID, "attention Q shape");
    if (!(g.image_start >= 0 && g.image_start <= g.image_end && g.image_end <= kv->prefix_len))
        return fail(FO_ERR_INVALID, "attention image must be inside the prefix");
    if (!(g.query_offset >= 0 && g.query_offset + query_len <= kv->total_len))
        return fail(FO_ERR_INVALID, "attention query interval");
    if (query_len > 0 && (!q || !output)) return fail(FO_ERR_INVALID, "attention Q/output pointer is null");
    if (!sinks) return fail(FO_ERR_INVALID, "attention sink pointer is null");
    if (kv->prefix_len > 0 && !kv->prefix_k) return fail(FO_ERR_INVALID, "attention prefix K pointer is null");
    if (kv->total_len > kv->prefix_len && !kv->generated_k)
        return fail(FO_ERR_INVALID, "attention generated K pointer is null");
    if (kv->total_len > 0 && !kv->v) return fail(FO_ERR_INVALID, "attention V pointer is null");
    return FO_OK;
}

struct Staged {
    const float *q, *pk, *gk, *v, *sinks;
    float *out;
};

// Host-mode inputs to device staging (FO_MEM_HOST), or the device pointers.
int stage_compact(fo_ctx *ctx, const float *q, const fo_compact_kv *kv, int64_t query_len, const float *sinks,
                  float *output, int mem, Staged *s) {
    const int64_t qn = query_len * kv->n_heads * kv->head_dim;
    const int64_t pkn = kv->prefix_len * kv->n_heads * kv->head_dim;
    const int64_t gkn = (kv->total_len - kv->prefix_len) * kv->n_kv_heads * kv->head_dim;
    const int64_t vn = kv->total_len * kv->n_kv_heads * kv->head_dim;
    if (mem == FO_MEM_DEVICE) {
        *s = {q, kv->prefix_k, kv->generated_k, kv->v, sinks, output};
        return FO_OK;
    }
    if (mem != FO_MEM_HOST) return fail(FO_ERR_INVALID, "mem must be FO_MEM_HOST or FO_MEM_DEVICE");
    const int64_t sizes[6] = {qn, pkn, gkn, vn, kv->n_heads, qn};
    const void *srcs[5] = {q, kv->prefix_k, kv->generated_k, kv->v, sinks};
    for (int i = 0; i < 6; i++) {
        FO_CUDA(ctx->stage[i].ensure((size_t)std::max<int64_t>(sizes[i], 1) * 4), "cudaMalloc(staging)");
        if (i < 5 && sizes[i] > 0)
            FO_CUDA(cudaMemcpyAsync(ctx->stage[i].ptr, srcs[i], (size_t)sizes[i] * 4, cudaMemcpyHostToDevice,
                                    ctx->stream),
                    "cudaMemcpyAsync(H2D)");
    }
    *s = {(const float *)ctx->stage[0].ptr, (const float *)ctx->stage[1].ptr, (const float *)ctx->stage[2].ptr,
          (const float *)ctx->stage[3].ptr, (const float *)ctx->stage[4].ptr, (float *)ctx->stage[5].ptr};
    return FO_OK;
}

// Reads and clears the context's device error word (after a synchronize).
int check_device_errors(fo_ctx *ctx) {
    unsigned bits = 0;
    FO_CUDA(cudaMemcpy(&bits, ctx->dev_err, sizeof bits, cudaMemcpyDeviceToHost), "cudaMemcpy(error word)");
    if (bits) {
        cudaMemset(ctx->dev_err, 0, sizeof bits);
        return fail(FO_ERR_CUDA, "a kernel wait exceeded its time limit and the kernel unwound (bits 0x%x)", bits);
    }
    return FO_OK;
}

int finish_host(fo_ctx *ctx, float *host_out, const float *dev_out, int64_t n, int mem) {
    if (mem == FO_MEM_HOST) {
        if (n > 0)
            FO_CUDA(cudaMemcpyAsync(host_out, dev_out, (size_t)n * 4, cudaMemcpyDeviceToHost, ctx->stream),
                    "cudaMemcpyAsync(D2H)");
        FO_CUDA(cudaStreamSynchronize(ctx->stream), "cudaStreamSynchronize");
        return check_device_errors(ctx);
    }
    return FO_OK;
}

int timed_begin(fo_ctx *ctx, bool on) {
    if (on) FO_CUDA(cudaEventRecord(ctx->ev0, ctx->stream), "cudaEventRecord");
    return FO_OK;
}
int timed_end(fo_ctx *ctx, bool on) {
    if (!on) return FO_OK;
    FO_CUDA(cudaEventRecord(ctx->ev1, ctx->stream), "cudaEventRecord");
    FO_CUDA(cudaEventSynchronize(ctx->ev1), "cudaEventSynchronize");
    FO_CUDA(cudaEventElapsedTime(&ctx->last_ms, ctx->ev0, ctx->ev1), "cudaEventElapsedTime");
    return FO_OK;
}

// Host-buffer BF16 prefill, pipelined over bands of query rows: the image rows
// (which need every image key) form the first band and the rest splits into at
// most four bands of at least 1,024 rows, all on 256-row boundaries.  Band b's
// keys, values and queries go up on the h2d stream; its BF16 conversion and
// prefill kernel run on the context's stream once they have landed; its output
// comes down on the d2h stream while later bands go up.  A band's kernel reads
// keys and values only below the end of its own rows (or of the image), which
// earlier bands have converted.  Returns after the last copy.
int prefill_bf16_host_pipelined(fo_ctx *ctx, const float *q, const fo_compact_kv *kv, const fo_geometry &geometry,
                                const float *sinks, float *output, const fo_prefill_options &options) {
    const int64_t T = kv->total_len, H = kv->n_heads, G = kv->n_kv_heads;
    std::vector<std::pair<int64_t, int64_t>> bands;
    int64_t first = std::min<int64_t>(T, (geometry.image_end + 255) / 256 * 256);
    if (first > 0) bands.push_back({0, first});
    const int64_t rest = T - first;
    if (rest > 0) {
        const int64_t nb = std::max<int64_t>(1, std::min<int64_t>(4, rest / 1024));
        const int64_t step = (rest + nb - 1) / nb;
        for (int64_t r = first; r < T;) {
            const int64_t e = std::min<int64_t>(T, (r + step + 255) / 256 * 256);
            bands.push_back({r, e});
            r = e;
        }
    }
    const size_t nb = bands.size();
    if (!ctx->h2d) FO_CUDA(cudaStreamCreateWithFlags(&ctx->h2d, cudaStreamNonBlocking), "cudaStreamCreate");
    if (!ctx->d2h) FO_CUDA(cudaStreamCreateWithFlags(&ctx->d2h, cudaStreamNonBlocking), "cudaStreamCreate");
    while (ctx->band_ev.size() < 2 * nb + 1) {
        cudaEvent_t e;
        FO_CUDA(cudaEventCreateWithFlags(&e, cudaEventDisableTiming), "cudaEventCreate");
        ctx->band_ev.push_back(e);
    }
    cudaEvent_t start = ctx->band_ev[0];
    const int64_t qn = T * H * 64, kn = T * H * 64, vn = T * G * 64;
    FO_CUDA(ctx->stage[0].ensure((size_t)qn * 4), "cudaMalloc(staging)");
    FO_CUDA(ctx->stage[1].ensure((size_t)kn * 4), "cudaMalloc(staging)");
    FO_CUDA(ctx->stage[3].ensure((size_t)vn * 4), "cudaMalloc(staging)");
    FO_CUDA(ctx->stage[4].ensure((size_t)H * 4), "cudaMalloc(staging)");
    FO_CUDA(ctx->stage[5].ensure((size_t)qn * 4), "cudaMalloc(staging)");
    FO_CUDA(ctx->bf16_k.ensure((size_t)kn * 2), "cudaMalloc(bf16 keys)");
    FO_CUDA(ctx->bf16_v.ensure((size_t)vn * 2), "cudaMalloc(bf16 values)");
    float *dq = (float *)ctx->stage[0].ptr, *dk = (float *)ctx->stage[1].ptr, *dv = (float *)ctx->stage[3].ptr;
    float *ds = (float *)ctx->stage[4].ptr, *dout = (float *)ctx->stage[5].ptr;
    uint16_t *kb = (uint16_t *)ctx->bf16_k.ptr, *vb = (uint16_t *)ctx->bf16_v.ptr;
    if (!aligned16(kb) || !aligned16(vb) || !aligned16(dq) || !aligned16(dout))
        return fail(FO_ERR_INVALID, "BF16 prefill buffers must be 16-byte aligned");
    // Earlier work on the context's stream (which may still read the staging
    // buffers) comes first.
    FO_CUDA(cudaEventRecord(start, ctx->stream), "cudaEventRecord");
    FO_CUDA(cudaStreamWaitEvent(ctx->h2d, start, 0), "cudaStreamWaitEvent");
    FO_CUDA(cudaMemcpyAsync(ds, sinks, (size_t)H * 4, cudaMemcpyHostToDevice, ctx->h2d), "cudaMemcpyAsync(H2D)");
    const bool prof = options.profile != 0;
    for (size_t b = 0; b < nb; b++) {
        const int64_t r0 = bands[b].first, r1 = bands[b].second;
        cudaEvent_t up = ctx->band_ev[1 + 2 * b], done = ctx->band_ev[2 + 2 * b];
        FO_CUDA(cudaMemcpyAsync(dk + r0 * H * 64, kv->prefix_k + r0 * H * 64, (size_t)(r1 - r0) * H * 64 * 4,
                                cudaMemcpyHostToDevice, ctx->h2d),
                "cudaMemcpyAsync(H2D)");
        FO_CUDA(cudaMemcpyAsync(dv + r0 * G * 64, kv->v + r0 * G * 64, (size_t)(r1 - r0) * G * 64 * 4,
                                cudaMemcpyHostToDevice, ctx->h2d),
                "cudaMemcpyAsync(H2D)");
        FO_CUDA(cudaMemcpyAsync(dq + r0 * H * 64, q + r0 * H * 64, (size_t)(r1 - r0) * H * 64 * 4,
                                cudaMemcpyHostToDevice, ctx->h2d),
                "cudaMemcpyAsync(H2D)");
        FO_CUDA(cudaEventRecord(up, ctx->h2d), "cudaEventRecord");
        FO_CUDA(cudaStreamWaitEvent(ctx->stream, up, 0), "cudaStreamWaitEvent");
        if (b == 0 && prof) FO_CUDA(cudaEventRecord(ctx->ev0, ctx->stream), "cudaEventRecord");
        cudaError_t e = fo_launch_convert_bf16(dk + r0 * H * 64, kb + r0 * H * 64, (r1 - r0) * H * 64, ctx->stream);
        if (e == cudaSuccess)
            e = fo_launch_convert_bf16(dv + r0 * G * 64, vb + r0 * G * 64, (r1 - r0) * G * 64, ctx->stream);
        if (e != cudaSuccess) return cuda_fail(e, "convert kernel launch");
        e = fo_launch_prefill_bf16(dq, kb, vb, ds, dout, 0, T, H, G, geometry.image_start, geometry.image_end, r0, r1,
                                   options.softmax == FO_SOFTMAX_STATIC, options.exp == FO_EXP_FAST, ctx->dev_err, 1,
                                   nullptr, nullptr, nullptr, ctx->stream);
        if (e != cudaSuccess) return cuda_fail(e, "BF16 prefill kernel launch");
        FO_CUDA(cudaEventRecord(done, ctx->stream), "cudaEventRecord");
    }
    if (prof) FO_CUDA(cudaEventRecord(ctx->ev1, ctx->stream), "cudaEventRecord");
    // The outputs come down band by band (issued after every upload, so a
    // pageable destination cannot hold up the uploads).
    for (size_t b = 0; b < nb; b++) {
        const int64_t r0 = bands[b].first, r1 = bands[b].second;
        FO_CUDA(cudaStreamWaitEvent(ctx->d2h, ctx->band_ev[2 + 2 * b], 0), "cudaStreamWaitEvent");
        FO_CUDA(cudaMemcpyAsync(output + r0 * H * 64, dout + r0 * H * 64, (size_t)(r1 - r0) * H * 64 * 4,
                                cudaMemcpyDeviceToHost, ctx->d2h),
                "cudaMemcpyAsync(D2H)");
    }
    FO_CUDA(cudaStreamSynchronize(ctx->d2h), "cudaStreamSynchronize");
    FO_CUDA(cudaStreamSynchronize(ctx->stream), "cudaStreamSynchronize");
    if (prof) FO_CUDA(cudaEventElapsedTime(&ctx->last_ms, ctx->ev0, ctx->ev1), "cudaEventElapsedTime");
    return check_device_errors(ctx);
}

}  // namespace

extern "C" {

// Lets other translation units of the library report through fo_last_error().
int fo_internal_fail(int status, const char *msg) { return fail(status, "%s", msg); }

int fo_version(void) { return 100; }

const char *fo_last_error(void) { return g_last_error.c_str(); }

int fo_ctx_create(int device, void *stream, fo_ctx **out) {
    if (!out) return fail(FO_ERR_INVALID, "fo_ctx_create: null output pointer");
    *out = nullptr;
    int count = 0;
    FO_CUDA(cudaGetDeviceCount(&count), "cudaGetDeviceCount");
    if (device < 0 || device >= count) return fail(FO_ERR_INVALID, "fo_ctx_create: no CUDA device %d", device);
    DeviceGuard guard(device);
    fo_ctx *ctx = new fo_ctx();
    ctx->device = device;
    // NULL is CUDA's default stream, as in the runtime API.
    ctx->stream = (cudaStream_t)stream;
    cudaError_t e = cudaMalloc(&ctx->flags, sizeof(unsigned));
    if (e == cudaSuccess) e = cudaMalloc(&ctx->dev_err, sizeof(unsigned));
    if (e == cudaSuccess) e = cudaMemset(ctx->dev_err, 0, sizeof(unsigned));
    if (e == cudaSuccess) e = cudaEventCreate(&ctx->ev0);
    if (e == cudaSuccess) e = cudaEventCreate(&ctx->ev1);
    if (e == cudaSuccess) e = ctx->pages.ensure(sizeof(fo_decode_page) * FO_BATCH_PAGES);
    if (e == cudaSuccess) e = ctx->host_pages.ensure(sizeof(fo_decode_page) * FO_BATCH_PAGES);
    if (e == cudaSuccess) e = ctx->append_pages.ensure(sizeof(fo_append_page) * FO_BATCH_PAGES);
    if (e == cudaSuccess) e = ctx->host_append_pages.ensure(sizeof(fo_append_page) * FO_BATCH_PAGES);
    if (e == cudaSuccess) e = ctx->i8_pages.ensure(sizeof(fo_i8_page) * FO_BATCH_PAGES);
    if (e == cudaSuccess) e = ctx->host_i8_pages.ensure(sizeof(fo_i8_page) * FO_BATCH_PAGES);
    if (e != cudaSuccess) {
        fo_ctx_destroy(ctx);
        return cuda_fail(e, "fo_ctx_create");
    }
    *out = ctx;
    return FO_OK;
}

int fo_ctx_destroy(fo_ctx *ctx) {
    if (!ctx) return FO_OK;
    DeviceGuard guard(ctx->device);
    if (ctx->stream) cudaStreamSynchronize(ctx->stream);
    for (auto &b : ctx->stage) b.release();
    ctx->bf16_k.release();
    ctx->bf16_v.release();
    ctx->split_o.release();
    ctx->split_ml.release();
    ctx->pages.release();
    ctx->host_pages.release();
    ctx->append_pages.release();
    ctx->host_append_pages.release();
    ctx->i8_pages.release();
    ctx->host_i8_pages.release();
    if (ctx->flags) cudaFree(ctx->flags);
    if (ctx->dev_err) cudaFree(ctx->dev_err);
    if (ctx->ev0) cudaEventDestroy(ctx->ev0);
    if (ctx->ev1) cudaEventDestroy(ctx->ev1);
    if (ctx->h2d) cudaStreamSynchronize(ctx->h2d);
    if (ctx->d2h) cudaStreamSynchronize(ctx->d2h);
    if (ctx->comm) cudaStreamSynchronize(ctx->comm);
    for (cudaEvent_t e : ctx->band_ev) cudaEventDestroy(e);
    for (cudaEvent_t e : ctx->comm_ev) cudaEventDestroy(e);
    if (ctx->comm) cudaStreamDestroy(ctx->comm);
    if (ctx->h2d) cudaStreamDestroy(ctx->h2d);
    if (ctx->d2h) cudaStreamDestroy(ctx->d2h);
    if (ctx->own_stream && ctx->stream) cudaStreamDestroy(ctx->stream);
    delete ctx;
    return FO_OK;
}

int fo_selftest_bounded_wait(fo_ctx *ctx, uint64_t limit_ns) {
    if (!ctx) return fail(FO_ERR_INVALID, "null context");
    if (limit_ns == 0 || limit_ns > FO_WAIT_LIMIT_MAX_NS) return fail(FO_ERR_INVALID, "limit_ns must be 1..10^10");
    DeviceGuard guard(ctx->device);
    cudaError_t e = fo_launch_bounded_wait(ctx->dev_err, (unsigned long long)limit_ns, ctx->stream);
    if (e != cudaSuccess) return cuda_fail(e, "bounded-wait self-test launch");
    FO_CUDA(cudaStreamSynchronize(ctx->stream), "cudaStreamSynchronize");
    return check_device_errors(ctx);
}

int fo_ctx_synchronize(fo_ctx *ctx) {
    if (!ctx) return fail(FO_ERR_INVALID, "null context");
    DeviceGuard guard(ctx->device);
    FO_CUDA(cudaStreamSynchronize(ctx->stream), "cudaStreamSynchronize");
    return check_device_errors(ctx);
}

int fo_ctx_last_ms(fo_ctx *ctx, float *ms) {
    if (!ctx || !ms) return fail(FO_ERR_INVALID, "null argument");
    *ms = ctx->last_ms;
    return FO_OK;
}

int fo_attention(fo_ctx *ctx, const float *q, const fo_compact_kv *kv, int64_t query_len, fo_geometry geometry,
                 const float *sinks, float *output, fo_prefill_options options, int mem) {
    int st = validate_compact(q, kv, query_len, geometry, sinks, output);
    if (st != FO_OK) return st;
    if (kv->head_dim > 256) return fail(FO_ERR_DECLINED, "attention: head_dim %lld above 256", (long long)kv->head_dim);
    if (!ctx) return fail(FO_ERR_INVALID, "null context");
    if (query_len == 0) return FO_OK;
    DeviceGuard guard(ctx->device);
    Staged s;
    if ((st = stage_compact(ctx, q, kv, query_len, sinks, output, mem, &s)) != FO_OK) return st;
    const bool tiles = query_len >= 4 && kv->head_dim == 64 && aligned16(s.q) && aligned16(s.pk) &&
                       aligned16(s.gk) && aligned16(s.v) && aligned16(s.out);
    if ((st = timed_begin(ctx, options.profile)) != FO_OK) return st;
    cudaError_t e;
    if (tiles) {
        // The FP32 tiles (prefill64.rs); static softmax only on pure prefixes.
        const int stat = options.fp32_softmax == FO_SOFTMAX_STATIC && kv->total_len == kv->prefix_len;
        e = fo_launch_prefill_f32(s.q, s.pk, s.gk, s.v, s.sinks, s.out, query_len, kv->prefix_len, kv->total_len,
                                  kv->n_heads, kv->n_kv_heads, geometry.query_offset, geometry.image_start,
                                  geometry.image_end, stat, options.exp == FO_EXP_FAST, ctx->stream);
    } else {
        // The online head (online.rs; decode64.rs for one query); decode
        // paths keep the platform exp (mod.rs:198-203).
        const int fast = query_len >= 4 && options.exp == FO_EXP_FAST;
        e = fo_launch_online(s.q, s.pk, s.gk, s.v, s.sinks, s.out, query_len, kv->prefix_len, kv->total_len,
                             kv->n_heads, kv->n_kv_heads, kv->head_dim, geometry.query_offset, geometry.image_start,
                             geometry.image_end, fast, ctx->stream);
    }
    if (e != cudaSuccess) return cuda_fail(e, "attention kernel launch");
    if ((st = timed_end(ctx, options.profile)) != FO_OK) return st;
    return finish_host(ctx, output, s.out, query_len * kv->n_heads * kv->head_dim, mem);
}

int fo_convert_bf16(fo_ctx *ctx, const float *src, uint16_t *dst, int64_t n) {
    if (!ctx || (n > 0 && (!src || !dst)) || n < 0) return fail(FO_ERR_INVALID, "fo_convert_bf16: bad argument");
    DeviceGuard guard(ctx->device);
    cudaError_t e = fo_launch_convert_bf16(src, dst, n, ctx->stream);
    if (e != cudaSuccess) return cuda_fail(e, "convert kernel launch");
    return FO_OK;
}

int fo_attention_prefill_bf16(fo_ctx *ctx, const float *q, const fo_compact_kv *kv, int64_t query_len,
                              fo_geometry geometry, const float *sinks, float *output, const uint16_t *keys_bf16,
                              const uint16_t *values_bf16, fo_prefill_options options, int mem) {
    int st = validate_compact(q, kv, query_len, geometry, sinks, output);
    if (st != FO_OK) return st;
    // mod.rs:333-339: a pure prefix prefilled whole, 64-wide heads.
    if (!(query_len >= 4 && kv->head_dim == 64 && geometry.query_offset == 0 && query_len == kv->total_len &&
          kv->total_len == kv->prefix_len))
        return fail(FO_ERR_DECLINED, "BF16 prefill declines this shape");
    if ((keys_bf16 == nullptr) != (values_bf16 == nullptr))
        return fail(FO_ERR_INVALID, "BF16 keys and values must both be given or both be null");
    if (keys_bf16 && mem != FO_MEM_DEVICE) return fail(FO_ERR_INVALID, "BF16 copies must be device pointers");
    if (!ctx) return fail(FO_ERR_INVALID, "null context");
    DeviceGuard guard(ctx->device);
    if (mem == FO_MEM_HOST) return prefill_bf16_host_pipelined(ctx, q, kv, geometry, sinks, output, options);
    const int64_t T = kv->total_len, H = kv->n_heads, G = kv->n_kv_heads;
    Staged s;
    // The FP32 keys and values are only read when converting.
    fo_compact_kv kv_stage = *kv;
    if (keys_bf16) {
        kv_stage.prefix_k = nullptr;
        kv_stage.v = nullptr;
        kv_stage.prefix_len = 0;
        kv_stage.total_len = 0;
    }
    if ((st = stage_compact(ctx, q, &kv_stage, query_len, sinks, output, mem, &s)) != FO_OK) return st;
    if ((st = timed_begin(ctx, options.profile)) != FO_OK) return st;
    const uint16_t *kb = keys_bf16, *vb = values_bf16;
    cudaError_t e;
    if (!kb) {
        FO_CUDA(ctx->bf16_k.ensure((size_t)T * H * 64 * 2), "cudaMalloc(bf16 keys)");
        FO_CUDA(ctx->bf16_v.ensure((size_t)T * G * 64 * 2), "cudaMalloc(bf16 values)");
        e = fo_launch_convert_bf16(s.pk, (uint16_t *)ctx->bf16_k.ptr, T * H * 64, ctx->stream);
        if (e == cudaSuccess) e = fo_launch_convert_bf16(s.v, (uint16_t *)ctx->bf16_v.ptr, T * G * 64, ctx->stream);
        if (e != cudaSuccess) return cuda_fail(e, "convert kernel launch");
        kb = (const uint16_t *)ctx->bf16_k.ptr;
        vb = (const uint16_t *)ctx->bf16_v.ptr;
    }
    if (!aligned16(kb) || !aligned16(vb) || !aligned16(s.q) || !aligned16(s.out))
        return fail(FO_ERR_INVALID, "BF16 prefill buffers must be 16-byte aligned");
    e = fo_launch_prefill_bf16(s.q, kb, vb, s.sinks, s.out, 0, T, H, G, geometry.image_start, geometry.image_end, 0, T,
                               options.softmax == FO_SOFTMAX_STATIC, options.exp == FO_EXP_FAST, ctx->dev_err, 1,
                               nullptr, nullptr, nullptr, ctx->stream);
    if (e != cudaSuccess) return cuda_fail(e, "BF16 prefill kernel launch");
    if ((st = timed_end(ctx, options.profile)) != FO_OK) return st;
    return finish_host(ctx, output, s.out, query_len * H * 64, mem);
}

int fo_attention_prefill_bf16_rows(fo_ctx *ctx, const float *q, const uint16_t *keys_bf16,
                                   const uint16_t *values_bf16, int64_t total_len, int64_t n_heads, int64_t n_kv_heads,
                                   fo_geometry geometry, const float *sinks, float *output, int64_t query_begin,
                                   int64_t query_end, fo_prefill_options options) {
    return fo_attention_prefill_bf16_rows_split(ctx, q, keys_bf16, values_bf16, total_len, n_heads, n_kv_heads,
                                                geometry, sinks, output, 0, query_begin, query_end, options, 1);
}

int fo_attention_prefill_bf16_rows_split(fo_ctx *ctx, const float *q, const uint16_t *keys_bf16,
                                         const uint16_t *values_bf16, int64_t total_len, int64_t n_heads,
                                         int64_t n_kv_heads, fo_geometry geometry, const float *sinks, void *output,
                                         int32_t out_bf16, int64_t query_begin, int64_t query_end,
                                         fo_prefill_options options, int32_t kv_splits) {
    if (!ctx) return fail(FO_ERR_INVALID, "null context");
    if (kv_splits < 1 || kv_splits > 64) return fail(FO_ERR_INVALID, "kv_splits must be 1..64");
    if (!q || !keys_bf16 || !values_bf16 || !sinks || !output) return fail(FO_ERR_INVALID, "null argument");
    if (!(total_len >= 4 && n_kv_heads >= 1 && n_heads >= n_kv_heads && n_heads % n_kv_heads == 0))
        return fail(FO_ERR_INVALID, "bad shape");
    if (geometry.query_offset != 0 || geometry.image_start < 0 || geometry.image_start > geometry.image_end ||
        geometry.image_end > total_len)
        return fail(FO_ERR_INVALID, "geometry must describe a pure prefix");
    if (!(query_begin >= 0 && query_begin <= query_end && query_end <= total_len && query_begin % 256 == 0 &&
          (query_end % 256 == 0 || query_end == total_len)))
        return fail(FO_ERR_INVALID, "query rows must be [begin, end) with begin and end multiples of 256 (or end = total)");
    if (!aligned16(keys_bf16) || !aligned16(values_bf16) || !aligned16(q) || !aligned16(output))
        return fail(FO_ERR_INVALID, "BF16 prefill buffers must be 16-byte aligned");
    DeviceGuard guard(ctx->device);
    float *po = nullptr, *pml = nullptr;
    if (kv_splits > 1) {
        // Partials of the launch's own query pairs only (rows from its first pair).
        const int64_t span = ((query_end + 255) / 256 - query_begin / 256) * 256;
        FO_CUDA(ctx->split_o.ensure((size_t)kv_splits * span * n_heads * 64 * 4), "cudaMalloc(split partials)");
        FO_CUDA(ctx->split_ml.ensure((size_t)kv_splits * span * n_heads * 2 * 4), "cudaMalloc(split partials)");
        po = (float *)ctx->split_o.ptr;
        pml = (float *)ctx->split_ml.ptr;
    }
    cudaError_t e = fo_launch_prefill_bf16(q, keys_bf16, values_bf16, sinks, output, out_bf16 != 0, total_len, n_heads,
                                           n_kv_heads,
                                           geometry.image_start, geometry.image_end, query_begin, query_end,
                                           options.softmax == FO_SOFTMAX_STATIC, options.exp == FO_EXP_FAST,
                                           ctx->dev_err, kv_splits, po, pml, nullptr, ctx->stream);
    if (e != cudaSuccess) return cuda_fail(e, "BF16 prefill kernel launch");
    return FO_OK;
}

// ------------------------------------------------- head-sharded prefill
int fo_nccl_unique_id(uint8_t *id) {
    if (!id) return fail(FO_ERR_INVALID, "fo_nccl_unique_id: null buffer");
    char msg[256];
    if (fo_nccl_unique_id_impl(id, msg, sizeof msg)) return fail(FO_ERR_CUDA, "%s", msg);
    return FO_OK;
}

int fo_nccl_comm_init(fo_ctx *ctx, int32_t world, int32_t rank, const uint8_t *id, void **comm) {
    if (!ctx || !id || !comm) return fail(FO_ERR_INVALID, "fo_nccl_comm_init: null argument");
    if (world < 1 || rank < 0 || rank >= world) return fail(FO_ERR_INVALID, "fo_nccl_comm_init: bad rank %d of %d", rank, world);
    *comm = nullptr;
    DeviceGuard guard(ctx->device);
    char msg[256];
    if (fo_nccl_comm_init_impl(world, rank, id, comm, msg, sizeof msg)) return fail(FO_ERR_CUDA, "%s", msg);
    return FO_OK;
}

int fo_nccl_comm_destroy(void *comm) {
    if (!comm) return FO_OK;
    char msg[256];
    if (fo_nccl_comm_destroy_impl(comm, msg, sizeof msg)) return fail(FO_ERR_CUDA, "%s", msg);
    return FO_OK;
}

int fo_sharded_prefill_bf16(fo_ctx *ctx, void *comm, int32_t rank, int32_t world, const float *q,
                            const uint16_t *keys_bf16, const uint16_t *values_bf16, int64_t total_len,
                            int64_t n_heads, int64_t n_kv_heads, fo_geometry geometry, const float *sinks,
                            fo_prefill_options options, int32_t n_bands, int32_t kv_splits, uint16_t *gathered) {
    if (!ctx || !comm || !gathered) return fail(FO_ERR_INVALID, "fo_sharded_prefill_bf16: null argument");
    if (world < 1 || rank < 0 || rank >= world) return fail(FO_ERR_INVALID, "fo_sharded_prefill_bf16: bad rank");
    if (n_bands < 1 || kv_splits < 0 || kv_splits > 64) return fail(FO_ERR_INVALID, "fo_sharded_prefill_bf16: bad bands or kv_splits");
    if (!aligned16(gathered)) return fail(FO_ERR_INVALID, "fo_sharded_prefill_bf16: gathered must be 16-byte aligned");
    if (total_len < 4 || n_heads < 1) return fail(FO_ERR_INVALID, "fo_sharded_prefill_bf16: bad shape");
    DeviceGuard guard(ctx->device);
    // Bands of about equal size on 256-row boundaries (the kernel's query pairs).
    const int64_t pairs = (total_len + 255) / 256;
    const int64_t nb = std::max<int64_t>(1, std::min<int64_t>(n_bands, pairs));
    std::vector<std::pair<int64_t, int64_t>> band;
    for (int64_t i = 0; i < nb; i++) {
        const int64_t b = (pairs * i / nb) * 256, e = std::min(total_len, (pairs * (i + 1) / nb) * 256);
        if (e > b) band.emplace_back(b, e);
    }
    if (kv_splits == 0) {
        // Enough key ranges that a band's launch has a CTA per SM (at most 8).
        int sms = 148;
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, ctx->device);
        int64_t least = pairs;
        for (auto &be : band) least = std::min<int64_t>(least, (be.second - be.first + 255) / 256);
        kv_splits = 1;
        while (kv_splits < 8 && least * n_heads * kv_splits < sms) kv_splits *= 2;
    }
    if (!ctx->comm) FO_CUDA(cudaStreamCreateWithFlags(&ctx->comm, cudaStreamNonBlocking), "cudaStreamCreate");
    while (ctx->comm_ev.size() < band.size() + 2) {
        cudaEvent_t e;
        FO_CUDA(cudaEventCreateWithFlags(&e, cudaEventDisableTiming), "cudaEventCreate");
        ctx->comm_ev.push_back(e);
    }
    // The gathers write peers' rows: after whatever the caller queued before.
    FO_CUDA(cudaEventRecord(ctx->comm_ev[0], ctx->stream), "cudaEventRecord");
    FO_CUDA(cudaStreamWaitEvent(ctx->comm, ctx->comm_ev[0], 0), "cudaStreamWaitEvent");
    const int64_t row_elems = n_heads * 64;
    char msg[256];
    for (int64_t i = (int64_t)band.size() - 1; i >= 0; i--) {
        const int64_t b = band[i].first, e = band[i].second, rows = e - b;
        uint16_t *block = gathered + world * b * row_elems;
        // Row r of this rank's slot lands at block + (rank * rows + r - b) * row_elems.
        uint16_t *out = block + (rank * rows - b) * row_elems;
        int st = fo_attention_prefill_bf16_rows_split(ctx, q, keys_bf16, values_bf16, total_len, n_heads, n_kv_heads,
                                                      geometry, sinks, out, 1, b, e, options, kv_splits);
        if (st != FO_OK) return st;
        cudaEvent_t done = ctx->comm_ev[1 + i];
        FO_CUDA(cudaEventRecord(done, ctx->stream), "cudaEventRecord");
        FO_CUDA(cudaStreamWaitEvent(ctx->comm, done, 0), "cudaStreamWaitEvent");
        if (fo_nccl_gather_bf16(comm, block, (size_t)(rows * row_elems), rank, ctx->comm, msg, sizeof msg))
            return fail(FO_ERR_CUDA, "%s", msg);
    }
    // The caller's stream sees the whole gathered page.
    cudaEvent_t all = ctx->comm_ev[band.size() + 1];
    FO_CUDA(cudaEventRecord(all, ctx->comm), "cudaEventRecord");
    FO_CUDA(cudaStreamWaitEvent(ctx->stream, all, 0), "cudaStreamWaitEvent");
    return FO_OK;
}

int fo_peer_block_destroy(fo_peer_block *pb) {
    if (!pb) return FO_OK;
    DeviceGuard guard(pb->ctx->device);
    cudaStreamSynchronize(pb->ctx->stream);
    for (int p = 0; p < FO_MAX_PEERS; p++)
        if (pb->opened[p]) cudaIpcCloseMemHandle(pb->opened[p]);
    if (pb->word) cudaFree(pb->word);
    delete pb;
    return FO_OK;
}

int fo_peer_block_register(fo_ctx *ctx, void *comm, int32_t rank, int32_t world, uint16_t *gathered, int64_t bytes,
                           fo_peer_block **out) {
    if (!out) return fail(FO_ERR_INVALID, "fo_peer_block_register: null output pointer");
    *out = nullptr;
    if (!ctx || !comm || !gathered) return fail(FO_ERR_INVALID, "fo_peer_block_register: null argument");
    if (world < 1 || world > FO_MAX_PEERS || rank < 0 || rank >= world)
        return fail(FO_ERR_INVALID, "fo_peer_block_register: rank %d of %d (at most %d ranks)", rank, world,
                    FO_MAX_PEERS);
    if (bytes <= 0 || !aligned16(gathered)) return fail(FO_ERR_INVALID, "fo_peer_block_register: bad buffer");
    DeviceGuard guard(ctx->device);
    // The allocation holding `gathered` (an IPC handle names a whole allocation).
    typedef CUresult (*AddressRange)(CUdeviceptr *, size_t *, CUdeviceptr);
    static AddressRange range = nullptr;
    if (!range) {
        void *fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &fn, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            return fail(FO_ERR_CUDA, "fo_peer_block_register: cuMemGetAddressRange is unavailable");
        range = reinterpret_cast<AddressRange>(fn);
    }
    CUdeviceptr base = 0;
    size_t size = 0;
    if (range(&base, &size, (CUdeviceptr)gathered) != CUDA_SUCCESS ||
        (uintptr_t)gathered + (size_t)bytes > (uintptr_t)base + size)
        return fail(FO_ERR_INVALID, "fo_peer_block_register: the buffer is not one device allocation");
    struct Entry {
        cudaIpcMemHandle_t handle;
        int64_t offset, bytes;
    } mine{};
    cudaError_t e = cudaIpcGetMemHandle(&mine.handle, reinterpret_cast<void *>(base));
    if (e != cudaSuccess) return cuda_fail(e, "fo_peer_block_register: cudaIpcGetMemHandle (an IPC-capable allocation is needed)");
    mine.offset = (int64_t)((uintptr_t)gathered - (uintptr_t)base);
    mine.bytes = bytes;
    // Every rank's entry, exchanged over the communicator.
    std::vector<Entry> all((size_t)world);
    void *d = nullptr;
    FO_CUDA(cudaMalloc(&d, sizeof(Entry) * (world + 1)), "cudaMalloc(handles)");
    char msg[256];
    e = cudaMemcpyAsync(d, &mine, sizeof mine, cudaMemcpyHostToDevice, ctx->stream);
    int st = 0;
    if (e == cudaSuccess)
        st = fo_nccl_allgather_bytes(comm, d, static_cast<char *>(d) + sizeof(Entry), sizeof(Entry), ctx->stream, msg,
                                     sizeof msg);
    if (e == cudaSuccess && !st)
        e = cudaMemcpyAsync(all.data(), static_cast<char *>(d) + sizeof(Entry), sizeof(Entry) * world,
                            cudaMemcpyDeviceToHost, ctx->stream);
    if (e == cudaSuccess && !st) e = cudaStreamSynchronize(ctx->stream);
    cudaFree(d);
    if (st) return fail(FO_ERR_CUDA, "%s", msg);
    if (e != cudaSuccess) return cuda_fail(e, "fo_peer_block_register: handle exchange");
    fo_peer_block *pb = new fo_peer_block();
    pb->ctx = ctx;
    pb->comm = comm;
    pb->rank = rank;
    pb->world = world;
    pb->local = gathered;
    pb->bytes = bytes;
    for (int p = 0; p < world; p++) {
        if (p == rank) {
            pb->block[p] = gathered;
            continue;
        }
        if (all[p].bytes != bytes) {
            fo_peer_block_destroy(pb);
            return fail(FO_ERR_INVALID, "fo_peer_block_register: rank %d registered %lld bytes, this rank %lld", p,
                        (long long)all[p].bytes, (long long)bytes);
        }
        void *ptr = nullptr;
        e = cudaIpcOpenMemHandle(&ptr, all[p].handle, cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess) {
            fo_peer_block_destroy(pb);
            return cuda_fail(e, "fo_peer_block_register: cudaIpcOpenMemHandle");
        }
        pb->opened[p] = ptr;
        pb->block[p] = reinterpret_cast<uint16_t *>(static_cast<char *>(ptr) + all[p].offset);
    }
    e = cudaMalloc(reinterpret_cast<void **>(&pb->word), sizeof(int32_t));
    if (e == cudaSuccess) e = cudaMemset(pb->word, 0, sizeof(int32_t));
    if (e != cudaSuccess) {
        fo_peer_block_destroy(pb);
        return cuda_fail(e, "fo_peer_block_register: cudaMalloc");
    }
    *out = pb;
    return FO_OK;
}

int fo_sharded_prefill_bf16_peers(fo_ctx *ctx, fo_peer_block *pb, const float *q, const uint16_t *keys_bf16,
                                  const uint16_t *values_bf16, int64_t total_len, int64_t n_heads, int64_t n_kv_heads,
                                  fo_geometry geometry, const float *sinks, fo_prefill_options options,
                                  int32_t kv_splits) {
    if (!ctx || !pb) return fail(FO_ERR_INVALID, "fo_sharded_prefill_bf16_peers: null argument");
    if (pb->ctx->device != ctx->device) return fail(FO_ERR_INVALID, "fo_sharded_prefill_bf16_peers: another device");
    if (kv_splits < 0 || kv_splits > 64) return fail(FO_ERR_INVALID, "fo_sharded_prefill_bf16_peers: bad kv_splits");
    if (total_len < 4 || n_heads < 1) return fail(FO_ERR_INVALID, "fo_sharded_prefill_bf16_peers: bad shape");
    const int64_t row_elems = n_heads * 64;
    if ((int64_t)pb->world * total_len * row_elems * 2 > pb->bytes)
        return fail(FO_ERR_INVALID, "fo_sharded_prefill_bf16_peers: the registered block holds fewer than %d x %lld rows",
                    pb->world, (long long)total_len);
    DeviceGuard guard(ctx->device);
    const int64_t pairs = (total_len + 255) / 256;
    if (kv_splits == 0) {
        // Enough key ranges that the launch has a CTA per SM (at most 8).
        int sms = 148;
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, ctx->device);
        kv_splits = 1;
        while (kv_splits < 8 && pairs * n_heads * kv_splits < sms) kv_splits *= 2;
    }
    char msg[256];
    // 1. Every rank is done with its blocks' previous contents (all work
    //    queued before this call on each rank's stream has completed).
    if (fo_nccl_barrier(pb->comm, pb->word, ctx->stream, msg, sizeof msg)) return fail(FO_ERR_CUDA, "%s", msg);
    // 2. This rank's rows, stored into its own block and, over NVLink, into
    //    every peer's at the same place [rank][rows][heads][64].
    const int64_t at = (int64_t)pb->rank * total_len * row_elems;
    fo_peer_out peers{};
    for (int p = 0; p < pb->world; p++)
        if (p != pb->rank) peers.dst[peers.n++] = pb->block[p] + at;
    float *po = nullptr, *pml = nullptr;
    if (kv_splits > 1) {
        FO_CUDA(ctx->split_o.ensure((size_t)kv_splits * pairs * 256 * n_heads * 64 * 4), "cudaMalloc(split partials)");
        FO_CUDA(ctx->split_ml.ensure((size_t)kv_splits * pairs * 256 * n_heads * 2 * 4), "cudaMalloc(split partials)");
        po = (float *)ctx->split_o.ptr;
        pml = (float *)ctx->split_ml.ptr;
    }
    cudaError_t e = fo_launch_prefill_bf16(q, keys_bf16, values_bf16, sinks, pb->local + at, 1, total_len, n_heads,
                                           n_kv_heads, geometry.image_start, geometry.image_end, 0, total_len,
                                           options.softmax == FO_SOFTMAX_STATIC, options.exp == FO_EXP_FAST,
                                           ctx->dev_err, kv_splits, po, pml, &peers, ctx->stream);
    if (e != cudaSuccess) return cuda_fail(e, "BF16 prefill kernel launch");
    // 3. Every rank's stores have landed: the whole page is in every block.
    if (fo_nccl_barrier(pb->comm, pb->word, ctx->stream, msg, sizeof msg)) return fail(FO_ERR_CUDA, "%s", msg);
    return FO_OK;
}

int fo_kv_seal_layer(fo_ctx *ctx, int32_t layer, uint64_t kv_q8_layers, int32_t mode, int32_t fast_exps,
                     int32_t decode_fast_exp, const float *k, const float *v, int64_t filled, int64_t prefix_len,
                     int64_t capacity, int64_t n_heads, int64_t n_kv_heads, int32_t chunks, fo_kv_cache **out) {
    if (!out) return fail(FO_ERR_INVALID, "fo_kv_seal_layer: null output pointer");
    *out = nullptr;
    if (layer < 0) return fail(FO_ERR_INVALID, "fo_kv_seal_layer: negative layer");
    if (!valid_format(mode)) return fail(FO_ERR_INVALID, "fo_kv_seal_layer: unknown mode %d", mode);
    // cache.rs:243-246
    if (filled != prefix_len) return fail(FO_ERR_INVALID, "seal only a complete prefix, before any text decode");
    // cache.rs:247-251: bit `layer` of the mask picks Q8 records (checked_shr: none past bit 63)
    const bool q8 = layer < 64 && ((kv_q8_layers >> layer) & 1u);
    const int32_t format = q8 ? FO_KV_Q8 : mode;
    fo_kv_cache *c = nullptr;
    int st = fo_kv_seal(ctx, k, v, prefix_len, capacity, n_heads, n_kv_heads, 64, format, chunks, FO_MEM_DEVICE, &c);
    if (st != FO_OK) return st;
    // kv.rs:182-184: the cache's mode, not this layer's format, picks the exp
    // (the 8-bit mode and the rotated research modes)
    const bool poly_mode = mode == FO_KV_Q8 || mode == FO_KV_Q8_ROT || mode == FO_KV_Q4_ROT;
    c->fast_exp = decode_fast_exp >= 0 ? decode_fast_exp != 0 : (fast_exps != 0 && poly_mode);
    *out = c;
    return FO_OK;
}

int fo_kv_destroy(fo_kv_cache *c) {
    if (!c) return FO_OK;
    DeviceGuard guard(c->ctx->device);
    cudaStreamSynchronize(c->ctx->stream);
    void *ptrs[] = {c->codes,   c->tail_codes, c->scales,    c->tail_scales, c->part_o,    c->part_ml,
                    c->q_stage, c->out_stage,  c->sinks_stage, c->rows_stage};
    for (void *p : ptrs)
        if (p) cudaFree(p);
    delete c;
    return FO_OK;
}

int fo_kv_seal(fo_ctx *ctx, const float *k, const float *v, int64_t prefix_len, int64_t capacity, int64_t n_heads,
               int64_t n_kv_heads, int64_t head_dim, int32_t format, int32_t chunks, int mem, fo_kv_cache **out) {
    if (!out) return fail(FO_ERR_INVALID, "fo_kv_seal: null output pointer");
    *out = nullptr;
    // kv.rs:248-263
    if (!(head_dim == 64 && n_heads == 2 * n_kv_heads && n_kv_heads >= 1 && n_kv_heads <= 8))
        return fail(FO_ERR_INVALID, "split cache requires Falcon 64-wide paired GQA heads");
    if (!(prefix_len > 0 && capacity >= prefix_len)) return fail(FO_ERR_CAPACITY, "invalid split-prefix capacity");
    // The split merge keeps two floats per split in shared memory.
    if (capacity > (int64_t)3000000) return fail(FO_ERR_CAPACITY, "split-prefix capacity above 3,000,000 positions");
    if (!valid_format(format)) return fail(FO_ERR_INVALID, "unknown split-cache format %d", format);
    if (!k || !v) return fail(FO_ERR_INVALID, "split prefix key/value pointer is null");
    if (mem != FO_MEM_HOST && mem != FO_MEM_DEVICE) return fail(FO_ERR_INVALID, "bad mem mode");
    if (!ctx) return fail(FO_ERR_INVALID, "null context");
    DeviceGuard guard(ctx->device);
    fo_kv_cache *c = new fo_kv_cache();
    c->ctx = ctx;
    c->format = format;
    c->chunks = chunks;
    c->prefix_len = prefix_len;
    c->capacity = capacity;
    c->tail_capacity = capacity - prefix_len;
    c->heads = n_heads;
    c->groups = n_kv_heads;
    c->prefix_stride = prefix_len;
    c->tail_stride = c->tail_capacity;
    c->max_splits = (capacity + FO_SPLIT - 1) / FO_SPLIT;
    const int64_t G = n_kv_heads, H = n_heads;
    const size_t prefix_bytes = code_bytes(format, (size_t)G * prefix_len * FO_RECORD_ELEMS);
    const size_t tail_bytes = code_bytes(format, (size_t)G * std::max<int64_t>(c->tail_capacity, 1) * FO_TAIL_ELEMS);
    const size_t scale_bytes = coded(format) ? (size_t)G * prefix_len * 5 * 2 : 16;
    const size_t tscale_bytes = coded(format) ? (size_t)G * std::max<int64_t>(c->tail_capacity, 1) * 4 * 2 : 16;
    cudaError_t e = cudaSuccess;
    auto alloc = [&](void **p, size_t n) {
        if (e == cudaSuccess) e = cudaMalloc(p, n);
    };
    alloc(&c->codes, prefix_bytes);
    alloc(&c->tail_codes, tail_bytes);
    alloc((void **)&c->scales, scale_bytes);
    alloc((void **)&c->tail_scales, tscale_bytes);
    // Partials for max_splits + 1 splits: the tensor-core decode splits the
    // prefix and the tail apart (at most one split more).
    alloc((void **)&c->part_o, (size_t)FO_MAX_ROWS_ABI * H * (c->max_splits + 1) * 64 * 4);
    alloc((void **)&c->part_ml, (size_t)FO_MAX_ROWS_ABI * H * (c->max_splits + 1) * 2 * 4);
    alloc((void **)&c->q_stage, (size_t)FO_MAX_ROWS_ABI * H * 64 * 4);
    alloc((void **)&c->out_stage, (size_t)FO_MAX_ROWS_ABI * H * 64 * 4);
    alloc((void **)&c->sinks_stage, (size_t)H * 4);
    alloc((void **)&c->rows_stage, (size_t)2 * FO_MAX_ROWS_ABI * H * 64 * 4);
    if (e != cudaSuccess) {
        fo_kv_destroy(c);
        return cuda_fail(e, "fo_kv_seal: cudaMalloc");
    }
    c->bytes = prefix_bytes + tail_bytes + (coded(format) ? scale_bytes + tscale_bytes : 0);
    // Without a tensor map the decode kernel copies record by record.
    c->has_map = fo_make_record_map(&c->rec_map, c->codes, format, prefix_len, c->prefix_stride, G) ? 1 : 0;
    if (format == FO_KV_BF16) {
        fo_decode_page tp{};
        tp.codes = c->codes;
        tp.tail_codes = c->tail_codes;
        tp.prefix_len = prefix_len;
        tp.prefix_stride = c->prefix_stride;
        tp.tail_stride = c->tail_stride;
        if (fo_make_tc_maps(&tp, G, c->tail_capacity)) {
            c->tc_map = tp.tc_map;
            c->s1_map = tp.s1_map;
            c->tail_map = tp.tail_map;
            c->has_tail_map = tp.has_tail_map;
            c->has_tc = 1;
        }
    }
    if (e == cudaSuccess) e = cudaMemsetAsync(c->tail_codes, 0, tail_bytes, ctx->stream);
    if (e == cudaSuccess) e = cudaMemsetAsync(c->tail_scales, 0, tscale_bytes, ctx->stream);
    const float *dk = k, *dv = v;
    if (e == cudaSuccess && mem == FO_MEM_HOST) {
        const size_t kn = (size_t)prefix_len * H * 64 * 4, vn = (size_t)prefix_len * G * 64 * 4;
        e = ctx->stage[1].ensure(kn);
        if (e == cudaSuccess) e = ctx->stage[3].ensure(vn);
        if (e == cudaSuccess) e = cudaMemcpyAsync(ctx->stage[1].ptr, k, kn, cudaMemcpyHostToDevice, ctx->stream);
        if (e == cudaSuccess) e = cudaMemcpyAsync(ctx->stage[3].ptr, v, vn, cudaMemcpyHostToDevice, ctx->stream);
        dk = (const float *)ctx->stage[1].ptr;
        dv = (const float *)ctx->stage[3].ptr;
    }
    if (e == cudaSuccess) e = cudaMemsetAsync(ctx->flags, 0, sizeof(unsigned), ctx->stream);
    if (e == cudaSuccess)
        e = fo_launch_seal(dk, dv, prefix_len, H, G, format, c->codes, c->scales, c->prefix_stride, ctx->flags,
                           ctx->stream);
    unsigned flags = 0;
    if (e == cudaSuccess) e = cudaMemcpyAsync(&flags, ctx->flags, sizeof flags, cudaMemcpyDeviceToHost, ctx->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
    if (e != cudaSuccess) {
        fo_kv_destroy(c);
        return cuda_fail(e, "fo_kv_seal");
    }
    // The reference validates every pair before anything else (kv.rs:265-278).
    if (flags & FO_FLAG_PAIR) {
        fo_kv_destroy(c);
        return fail(FO_ERR_PAIR, "temporal keys differ inside GQA pair; refusing illegal sharing");
    }
    if (flags & FO_FLAG_NONFINITE) {
        fo_kv_destroy(c);
        return fail(FO_ERR_NONFINITE, "nonfinite or incomplete KV group");
    }
    if (flags & FO_FLAG_ROTATED) {
        fo_kv_destroy(c);
        return fail(FO_ERR_OVERFLOW, "rotated KV group overflows");
    }
    if (flags & FO_FLAG_OVERFLOW) {
        fo_kv_destroy(c);
        return fail(FO_ERR_OVERFLOW, "%s KV conversion overflow", format_name(format));
    }
    *out = c;
    return FO_OK;
}

int fo_kv_set_fast_exp(fo_kv_cache *c, int32_t fast) {
    if (!c) return fail(FO_ERR_INVALID, "null cache");
    c->fast_exp = fast != 0;
    return FO_OK;
}

int fo_kv_append(fo_kv_cache *c, const float *k, const float *v, int64_t rows, int mem) {
    if (!c || (rows > 0 && (!k || !v)) || rows < 0) return fail(FO_ERR_INVALID, "fo_kv_append: bad argument");
    if (c->tail_len + rows > c->tail_capacity) return fail(FO_ERR_CAPACITY, "split tail capacity");
    if (mem != FO_MEM_HOST && mem != FO_MEM_DEVICE) return fail(FO_ERR_INVALID, "bad mem mode");
    DeviceGuard guard(c->ctx->device);
    const int64_t width = c->heads * 64;
    for (int64_t done = 0; done < rows;) {
        const int64_t n = mem == FO_MEM_HOST ? std::min<int64_t>(FO_MAX_ROWS_ABI, rows - done) : rows - done;
        const float *dk = k + done * width, *dv = v + done * width;
        if (mem == FO_MEM_HOST) {
            float *sk = c->rows_stage, *sv = c->rows_stage + FO_MAX_ROWS_ABI * width;
            FO_CUDA(cudaMemcpyAsync(sk, dk, (size_t)n * width * 4, cudaMemcpyHostToDevice, c->ctx->stream), "H2D");
            FO_CUDA(cudaMemcpyAsync(sv, dv, (size_t)n * width * 4, cudaMemcpyHostToDevice, c->ctx->stream), "H2D");
            dk = sk;
            dv = sv;
        }
        cudaError_t e = fo_launch_append(dk, dv, n, c->heads, c->groups, c->format, c->tail_codes, c->tail_scales,
                                         c->tail_stride, c->tail_len, c->ctx->stream);
        if (e != cudaSuccess) return cuda_fail(e, "append kernel launch");
        if (mem == FO_MEM_HOST) FO_CUDA(cudaStreamSynchronize(c->ctx->stream), "cudaStreamSynchronize");
        c->tail_len += n;
        done += n;
    }
    return FO_OK;
}

int fo_kv_append_batch(fo_kv_cache *const *caches, int64_t n, const float *const *k, const float *const *v,
                       int64_t rows) {
    if (!caches || !k || !v || n < 0 || rows < 0) return fail(FO_ERR_INVALID, "append batch: bad argument");
    if (n == 0 || rows == 0) return FO_OK;
    fo_ctx *ctx = caches[0] ? caches[0]->ctx : nullptr;
    if (!ctx) return fail(FO_ERR_INVALID, "append batch: null cache");
    const fo_kv_cache *c0 = caches[0];
    for (int64_t i = 0; i < n; i++) {
        const fo_kv_cache *c = caches[i];
        if (!c || !k[i] || !v[i]) return fail(FO_ERR_INVALID, "append batch: null entry %lld", (long long)i);
        if (c->ctx != ctx || c->format != c0->format || c->heads != c0->heads)
            return fail(FO_ERR_INVALID, "append batch: caches must share context, format and heads");
        if (c->tail_len + rows > c->tail_capacity)
            return fail(FO_ERR_CAPACITY, "append batch: cache %lld: split tail capacity", (long long)i);
    }
    {  // each cache's tail grows once per call
        std::vector<const fo_kv_cache *> seen(caches, caches + n);
        std::sort(seen.begin(), seen.end());
        if (std::adjacent_find(seen.begin(), seen.end()) != seen.end())
            return fail(FO_ERR_INVALID, "append batch: a cache appears twice");
    }
    DeviceGuard guard(ctx->device);
    for (int64_t base = 0; base < n; base += FO_BATCH_PAGES) {
        const int64_t m = std::min<int64_t>(FO_BATCH_PAGES, n - base);
        int slot = 0;
        fo_append_page *hp = static_cast<fo_append_page *>(ctx->host_append_pages.acquire(slot));
        for (int64_t i = 0; i < m; i++) {
            fo_kv_cache *c = caches[base + i];
            hp[i] = {k[base + i], v[base + i], c->tail_codes, c->tail_scales, c->tail_stride, c->tail_len};
        }
        FO_CUDA(cudaMemcpyAsync(ctx->append_pages.ptr, hp, (size_t)m * sizeof(fo_append_page),
                                cudaMemcpyHostToDevice, ctx->stream),
                "H2D(append pages)");
        FO_CUDA(ctx->host_append_pages.uploaded(slot, ctx->stream), "cudaEventRecord");
        cudaError_t e = fo_launch_append_batch((const fo_append_page *)ctx->append_pages.ptr, m, rows, c0->heads,
                                               c0->groups, c0->format, nullptr, nullptr, ctx->stream);
        if (e != cudaSuccess) return cuda_fail(e, "append batch launch");
        for (int64_t i = 0; i < m; i++) caches[base + i]->tail_len += rows;
    }
    return FO_OK;
}

static fo_decode_page make_page(const fo_kv_cache *c, const float *q, const float *sinks, float *out, int rows);

// A batch plan: device-resident descriptors of n caches' appends and
// single-row decodes, moved on by one position per step on the device.
struct fo_kv_plan {
    fo_ctx *ctx = nullptr;
    std::vector<fo_kv_cache *> caches;
    int32_t format = 0, fast_exp = 0;
    int64_t heads = 0, groups = 0, max_splits = 1;
    fo_append_page *ap = nullptr;  // [n] device
    fo_decode_page *dp = nullptr;  // [n] device
};

static void plan_free(fo_kv_plan *p) {
    if (p->ap) cudaFree(p->ap);
    if (p->dp) cudaFree(p->dp);
    delete p;
}

int fo_kv_plan_create(fo_kv_cache *const *caches, int64_t n, const float *const *k, const float *const *v,
                      const float *const *q, const float *const *sinks, float *const *output, fo_kv_plan **out) {
    if (!out) return fail(FO_ERR_INVALID, "fo_kv_plan_create: null output pointer");
    *out = nullptr;
    if (!caches || !k || !v || !q || !sinks || !output || n < 1)
        return fail(FO_ERR_INVALID, "fo_kv_plan_create: bad argument");
    fo_ctx *ctx = caches[0] ? caches[0]->ctx : nullptr;
    if (!ctx) return fail(FO_ERR_INVALID, "fo_kv_plan_create: null cache");
    const fo_kv_cache *c0 = caches[0];
    for (int64_t i = 0; i < n; i++) {
        const fo_kv_cache *c = caches[i];
        if (!c || !k[i] || !v[i] || !q[i] || !sinks[i] || !output[i])
            return fail(FO_ERR_INVALID, "fo_kv_plan_create: null entry %lld", (long long)i);
        if (c->ctx != ctx || c->format != c0->format || c->heads != c0->heads || c->fast_exp != c0->fast_exp)
            return fail(FO_ERR_INVALID, "fo_kv_plan_create: caches must share context, format, heads and exp");
        if (c->tail_len + 1 > c->tail_capacity)
            return fail(FO_ERR_CAPACITY, "fo_kv_plan_create: cache %lld has no tail room", (long long)i);
    }
    {
        std::vector<const fo_kv_cache *> seen(caches, caches + n);
        std::sort(seen.begin(), seen.end());
        if (std::adjacent_find(seen.begin(), seen.end()) != seen.end())
            return fail(FO_ERR_INVALID, "fo_kv_plan_create: a cache appears twice");
    }
    DeviceGuard guard(ctx->device);
    fo_kv_plan *p = new fo_kv_plan();
    p->ctx = ctx;
    p->caches.assign(caches, caches + n);
    p->format = c0->format;
    p->fast_exp = c0->fast_exp;
    p->heads = c0->heads;
    p->groups = c0->groups;
    std::vector<fo_append_page> ha((size_t)n);
    std::vector<fo_decode_page> hd((size_t)n);
    for (int64_t i = 0; i < n; i++) {
        fo_kv_cache *c = caches[i];
        ha[i] = {k[i], v[i], c->tail_codes, c->tail_scales, c->tail_stride, c->tail_len};
        // the decode of the step's row: it sees the position the append adds
        hd[i] = make_page(c, q[i], sinks[i], output[i], 1);
        hd[i].last = c->prefix_len + c->tail_len + 1;
        hd[i].splits = (int32_t)((hd[i].last + FO_SPLIT - 1) / FO_SPLIT);
        p->max_splits = std::max<int64_t>(p->max_splits, (c->prefix_len + c->tail_capacity + FO_SPLIT - 1) / FO_SPLIT);
    }
    cudaError_t e = cudaMalloc(&p->ap, sizeof(fo_append_page) * n);
    if (e == cudaSuccess) e = cudaMalloc(&p->dp, sizeof(fo_decode_page) * n);
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(p->ap, ha.data(), sizeof(fo_append_page) * n, cudaMemcpyHostToDevice, ctx->stream);
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(p->dp, hd.data(), sizeof(fo_decode_page) * n, cudaMemcpyHostToDevice, ctx->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
    if (e != cudaSuccess) {
        plan_free(p);
        return cuda_fail(e, "fo_kv_plan_create");
    }
    *out = p;
    return FO_OK;
}

int fo_kv_plan_step(fo_kv_plan *p) {
    if (!p) return fail(FO_ERR_INVALID, "fo_kv_plan_step: null plan");
    DeviceGuard guard(p->ctx->device);
    const int64_t n = (int64_t)p->caches.size();
    // The append also sets each page's decode length; the merge moves each
    // page's append index on for the next step.
    cudaError_t e = fo_launch_append_batch(p->ap, n, 1, p->heads, p->groups, p->format, p->dp, p->ctx->dev_err,
                                           p->ctx->stream);
    if (e == cudaSuccess)
        e = fo_launch_decode_batch(p->dp, n, p->format, p->groups, p->fast_exp, p->max_splits, 1, p->ap,
                                   p->ctx->stream);
    if (e != cudaSuccess) return cuda_fail(e, "batch plan step launch");
    return FO_OK;
}

int fo_kv_plan_finish(fo_kv_plan *p) {
    if (!p) return FO_OK;
    fo_ctx *ctx = p->ctx;
    DeviceGuard guard(ctx->device);
    const int64_t n = (int64_t)p->caches.size();
    std::vector<fo_append_page> ha((size_t)n);
    cudaError_t e = cudaMemcpyAsync(ha.data(), p->ap, sizeof(fo_append_page) * n, cudaMemcpyDeviceToHost,
                                    p->ctx->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(p->ctx->stream);
    unsigned bits = 0;
    if (e == cudaSuccess) e = cudaMemcpy(&bits, p->ctx->dev_err, sizeof bits, cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) {
        plan_free(p);
        return cuda_fail(e, "fo_kv_plan_finish");
    }
    // the next append index is the number of records written (a full tail
    // holds the capacity there)
    for (int64_t i = 0; i < n; i++)
        p->caches[i]->tail_len = std::min<int64_t>(ha[i].first, p->caches[i]->tail_capacity);
    plan_free(p);
    if (bits) {
        cudaMemset(ctx->dev_err, 0, sizeof bits);
        if (bits & FO_DEVERR_CAPACITY)
            return fail(FO_ERR_CAPACITY, "a batch plan step found a cache's tail full (later steps repeated its last position)");
        return fail(FO_ERR_CUDA, "a kernel wait exceeded its time limit and the kernel unwound (bits 0x%x)", bits);
    }
    return FO_OK;
}

static bool aligned8(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 7) == 0; }

int fo_qkv_prefix_rows(fo_ctx *ctx, const float *qkv, const float *rope, int64_t rows, int64_t n_heads,
                       int64_t n_kv_heads, float *q, float *k, float *v, uint16_t *k_bf16, uint16_t *v_bf16) {
    if (!ctx) return fail(FO_ERR_INVALID, "fo_qkv_prefix_rows: null context");
    if (rows < 0 || !(n_kv_heads >= 1 && n_heads >= n_kv_heads && n_heads % n_kv_heads == 0 && n_heads <= 64))
        return fail(FO_ERR_INVALID, "fo_qkv_prefix_rows: bad shape");
    if (rows == 0) return FO_OK;
    if (!qkv || !rope || !q || !k || !v) return fail(FO_ERR_INVALID, "fo_qkv_prefix_rows: null pointer");
    if (!aligned8(qkv) || !aligned8(rope) || !aligned8(q) || !aligned8(k) || !aligned8(v) ||
        (reinterpret_cast<uintptr_t>(k_bf16) & 3) || (reinterpret_cast<uintptr_t>(v_bf16) & 3))
        return fail(FO_ERR_INVALID, "fo_qkv_prefix_rows: buffers must be 8-byte aligned (BF16 copies 4-byte)");
    DeviceGuard guard(ctx->device);
    cudaError_t e = fo_launch_qkv_rows(qkv, rope, rows, (int)n_heads, (int)n_kv_heads, q, k, v, k_bf16, v_bf16,
                                       ctx->stream);
    if (e != cudaSuccess) return cuda_fail(e, "fused QKV rows launch");
    return FO_OK;
}

int fo_kv_append_qkv(fo_kv_cache *c, const float *qkv, const float *rope, int64_t rows, float *q) {
    if (!c || rows < 0) return fail(FO_ERR_INVALID, "fo_kv_append_qkv: bad argument");
    if (rows == 0) return FO_OK;
    if (!qkv || !rope || !q) return fail(FO_ERR_INVALID, "fo_kv_append_qkv: null pointer");
    if (!aligned8(qkv) || !aligned8(rope) || !aligned8(q))
        return fail(FO_ERR_INVALID, "fo_kv_append_qkv: buffers must be 8-byte aligned");
    if (c->tail_len + rows > c->tail_capacity) return fail(FO_ERR_CAPACITY, "split tail capacity");
    DeviceGuard guard(c->ctx->device);
    cudaError_t e = fo_launch_qkv_append(qkv, rope, rows, (int)c->heads, (int)c->groups, q, c->format, c->tail_codes,
                                         c->tail_scales, c->tail_stride, c->tail_len, c->ctx->stream);
    if (e != cudaSuccess) return cuda_fail(e, "fused QKV append launch");
    c->tail_len += rows;
    return FO_OK;
}

int fo_kv_truncate_tail(fo_kv_cache *c, int64_t tail_len) {
    if (!c) return fail(FO_ERR_INVALID, "null cache");
    if (tail_len < 0 || tail_len > c->tail_len) return fail(FO_ERR_INVALID, "cannot grow the tail by truncation");
    if (tail_len < c->tail_len) {
        // The dropped records go back to zero, as seal leaves the tail: the
        // tensor-core decode reads whole 128-position tiles of tail records,
        // and past the cache's end they must add nothing (zero keys, values).
        DeviceGuard guard(c->ctx->device);
        const size_t pitch = code_bytes(c->format, (size_t)c->tail_stride * FO_TAIL_ELEMS);
        FO_CUDA(cudaMemset2DAsync(static_cast<char *>(c->tail_codes) + code_bytes(c->format, (size_t)tail_len * FO_TAIL_ELEMS),
                                  pitch, 0, code_bytes(c->format, (size_t)(c->tail_len - tail_len) * FO_TAIL_ELEMS),
                                  (size_t)c->groups, c->ctx->stream),
                "cudaMemset2DAsync(tail records)");
        if (coded(c->format))
            FO_CUDA(cudaMemset2DAsync(c->tail_scales + (size_t)tail_len * 4, (size_t)c->tail_stride * 4 * 2, 0,
                                      (size_t)(c->tail_len - tail_len) * 4 * 2, (size_t)c->groups, c->ctx->stream),
                    "cudaMemset2DAsync(tail scales)");
    }
    c->tail_len = tail_len;
    return FO_OK;
}

int64_t fo_kv_tail_len(const fo_kv_cache *c) { return c ? c->tail_len : -1; }
int64_t fo_kv_prefix_len(const fo_kv_cache *c) { return c ? c->prefix_len : -1; }
int64_t fo_kv_bytes(const fo_kv_cache *c) { return c ? (int64_t)c->bytes : -1; }

int fo_kv_records(const fo_kv_cache *c, void **codes, void **scales, void **tail_codes, void **tail_scales,
                  int64_t *prefix_stride, int64_t *tail_stride) {
    if (!c) return fail(FO_ERR_INVALID, "null cache");
    if (codes) *codes = c->codes;
    if (scales) *scales = c->scales;
    if (tail_codes) *tail_codes = c->tail_codes;
    if (tail_scales) *tail_scales = c->tail_scales;
    if (prefix_stride) *prefix_stride = c->prefix_stride;
    if (tail_stride) *tail_stride = c->tail_stride;
    return FO_OK;
}

// A single-page decode of BF16 records runs on the tensor cores
// (decode_tc.cu) with its own split layout; others, and batches, on decode.cu.
static void use_tc_layout(const fo_kv_cache *c, fo_decode_page *p) {
    if (!c->has_tc || (c->tail_len > 0 && !c->has_tail_map)) return;
    p->tc_map = c->tc_map;
    p->s1_map = c->s1_map;
    p->tail_map = c->tail_map;
    p->has_tail_map = c->has_tail_map;
    fo_tc_layout(p, c->groups, c->tail_len);
}

static fo_decode_page make_page(const fo_kv_cache *c, const float *q, const float *sinks, float *out, int rows) {
    fo_decode_page p{};
    p.codes = c->codes;
    p.scales = c->scales;
    p.tail_codes = c->tail_codes;
    p.tail_scales = c->tail_scales;
    p.q = q;
    p.sinks = sinks;
    p.out = out;
    p.part_o = c->part_o;
    p.part_ml = c->part_ml;
    p.err = c->ctx->dev_err;
    p.rec_map = c->rec_map;
    p.has_map = c->has_map;
    p.prefix_len = c->prefix_len;
    p.prefix_stride = c->prefix_stride;
    p.tail_stride = c->tail_stride;
    p.last = c->prefix_len + c->tail_len;
    p.rows = rows;
    p.splits = (int32_t)((p.last + FO_SPLIT - 1) / FO_SPLIT);
    p.rotated = (c->format & FO_KV_ROTATED) ? 1 : 0;
    return p;
}

int fo_kv_attention_decode_rows(fo_kv_cache *c, const float *q, int64_t rows, const float *sinks, float *output,
                                int mem) {
    if (!c || !q || !sinks || !output) return fail(FO_ERR_INVALID, "decode: null argument");
    // kv.rs:858
    if (!(rows >= 1 && rows <= FO_MAX_ROWS_ABI && rows <= std::max<int64_t>(c->tail_len, 1)))
        return fail(FO_ERR_INVALID, "decode rows must be 1..8 and at most max(tail_len, 1)");
    if (mem != FO_MEM_HOST && mem != FO_MEM_DEVICE) return fail(FO_ERR_INVALID, "bad mem mode");
    DeviceGuard guard(c->ctx->device);
    cudaStream_t st = c->ctx->stream;
    const int64_t n = rows * c->heads * 64;
    const float *dq = q, *ds = sinks;
    float *dout = output;
    if (mem == FO_MEM_HOST) {
        FO_CUDA(cudaMemcpyAsync(c->q_stage, q, (size_t)n * 4, cudaMemcpyHostToDevice, st), "H2D");
        FO_CUDA(cudaMemcpyAsync(c->sinks_stage, sinks, (size_t)c->heads * 4, cudaMemcpyHostToDevice, st), "H2D");
        dq = c->q_stage;
        ds = c->sinks_stage;
        dout = c->out_stage;
    }
    fo_decode_page p = make_page(c, dq, ds, dout, (int)rows);
    use_tc_layout(c, &p);
    cudaError_t e = fo_launch_decode_one(&p, c->format, c->groups, c->fast_exp, st);
    if (e != cudaSuccess) return cuda_fail(e, "decode kernel launch");
    return finish_host(c->ctx, output, dout, n, mem);
}

int fo_kv_attention_decode(fo_kv_cache *c, const float *q, int64_t total_len, const float *sinks, float *output,
                           int mem) {
    if (!c) return fail(FO_ERR_INVALID, "null cache");
    if (total_len != c->prefix_len + c->tail_len)  // kv.rs:572
        return fail(FO_ERR_INVALID, "decode total_len must equal prefix_len + tail_len");
    if (!(c->tail_len >= 0)) return fail(FO_ERR_INVALID, "bad tail");
    // attention_decode over the whole cache is the one-row step.
    if (!c || !q || !sinks || !output) return fail(FO_ERR_INVALID, "decode: null argument");
    if (mem != FO_MEM_HOST && mem != FO_MEM_DEVICE) return fail(FO_ERR_INVALID, "bad mem mode");
    DeviceGuard guard(c->ctx->device);
    cudaStream_t st = c->ctx->stream;
    const int64_t n = c->heads * 64;
    const float *dq = q, *ds = sinks;
    float *dout = output;
    if (mem == FO_MEM_HOST) {
        FO_CUDA(cudaMemcpyAsync(c->q_stage, q, (size_t)n * 4, cudaMemcpyHostToDevice, st), "H2D");
        FO_CUDA(cudaMemcpyAsync(c->sinks_stage, sinks, (size_t)c->heads * 4, cudaMemcpyHostToDevice, st), "H2D");
        dq = c->q_stage;
        ds = c->sinks_stage;
        dout = c->out_stage;
    }
    fo_decode_page p = make_page(c, dq, ds, dout, 1);
    use_tc_layout(c, &p);
    cudaError_t e = fo_launch_decode_one(&p, c->format, c->groups, c->fast_exp, st);
    if (e != cudaSuccess) return cuda_fail(e, "decode kernel launch");
    return finish_host(c->ctx, output, dout, n, mem);
}

int fo_kv_attention_decode_batch(fo_kv_cache *const *caches, int64_t n, const float *const *q,
                                 const float *const *sinks, float *const *output) {
    if (!caches || !q || !sinks || !output || n < 0) return fail(FO_ERR_INVALID, "decode batch: null argument");
    if (n == 0) return FO_OK;
    fo_ctx *ctx = caches[0] ? caches[0]->ctx : nullptr;
    if (!ctx) return fail(FO_ERR_INVALID, "decode batch: null cache");
    const fo_kv_cache *c0 = caches[0];
    for (int64_t i = 0; i < n; i++) {
        const fo_kv_cache *c = caches[i];
        if (!c || !q[i] || !sinks[i] || !output[i]) return fail(FO_ERR_INVALID, "decode batch: null entry %lld", (long long)i);
        if (c->ctx != ctx || c->format != c0->format || c->groups != c0->groups || c->fast_exp != c0->fast_exp)
            return fail(FO_ERR_INVALID, "decode batch: caches must share context, format, heads and exp");
    }
    {  // each page's partials belong to its cache: pages must be distinct caches
        std::vector<const fo_kv_cache *> seen(caches, caches + n);
        std::sort(seen.begin(), seen.end());
        if (std::adjacent_find(seen.begin(), seen.end()) != seen.end())
            return fail(FO_ERR_INVALID, "decode batch: a cache appears twice");
    }
    DeviceGuard guard(ctx->device);
    for (int64_t base = 0; base < n; base += FO_BATCH_PAGES) {
        const int64_t m = std::min<int64_t>(FO_BATCH_PAGES, n - base);
        int slot = 0;
        fo_decode_page *hp = static_cast<fo_decode_page *>(ctx->host_pages.acquire(slot));
        int64_t max_splits = 1;
        for (int64_t i = 0; i < m; i++) {
            hp[i] = make_page(caches[base + i], q[base + i], sinks[base + i], output[base + i], 1);
            max_splits = std::max<int64_t>(max_splits, hp[i].splits);
        }
        FO_CUDA(cudaMemcpyAsync(ctx->pages.ptr, hp, (size_t)m * sizeof(fo_decode_page), cudaMemcpyHostToDevice,
                                ctx->stream),
                "H2D(pages)");
        FO_CUDA(ctx->host_pages.uploaded(slot, ctx->stream), "cudaEventRecord");
        cudaError_t e = fo_launch_decode_batch((const fo_decode_page *)ctx->pages.ptr, m, c0->format, c0->groups,
                                               c0->fast_exp, max_splits, 1, nullptr, ctx->stream);
        if (e != cudaSuccess) return cuda_fail(e, "decode batch launch");
    }
    return FO_OK;
}

int fo_i8_destroy(fo_i8_cache *c) {
    if (!c) return FO_OK;
    DeviceGuard guard(c->ctx->device);
    cudaStreamSynchronize(c->ctx->stream);
    void *ptrs[] = {c->k_codes, c->v_codes, c->k_scales, c->v_scales, c->part_o, c->part_ml};
    for (void *p : ptrs)
        if (p) cudaFree(p);
    delete c;
    return FO_OK;
}

int fo_i8_seal(fo_ctx *ctx, const float *k, const float *v, int64_t len, int64_t n_heads, int mem,
               fo_i8_cache **out) {
    if (!out) return fail(FO_ERR_INVALID, "fo_i8_seal: null output pointer");
    *out = nullptr;
    if (!ctx) return fail(FO_ERR_INVALID, "null context");
    if (!k || !v) return fail(FO_ERR_INVALID, "fo_i8_seal: null keys or values");
    if (!(len >= 1 && n_heads >= 1)) return fail(FO_ERR_INVALID, "fo_i8_seal: length and heads must be positive");
    if (mem != FO_MEM_HOST && mem != FO_MEM_DEVICE) return fail(FO_ERR_INVALID, "bad mem mode");
    DeviceGuard guard(ctx->device);
    fo_i8_cache *c = new fo_i8_cache();
    c->ctx = ctx;
    c->len = len;
    c->heads = n_heads;
    c->splits = (len + FO_I8_SPLIT - 1) / FO_I8_SPLIT;
    const int64_t groups = (len + 63) / 64;
    const size_t n = (size_t)len * n_heads * 64;
    cudaError_t e = cudaSuccess;
    auto alloc = [&](void **p, size_t bytes) {
        if (e == cudaSuccess) e = cudaMalloc(p, bytes);
    };
    alloc((void **)&c->k_codes, n);
    alloc((void **)&c->v_codes, n);
    alloc((void **)&c->k_scales, (size_t)n_heads * groups * 4);
    alloc((void **)&c->v_scales, (size_t)n_heads * groups * 4);
    alloc((void **)&c->part_o, (size_t)n_heads * c->splits * 64 * 4);
    alloc((void **)&c->part_ml, (size_t)n_heads * c->splits * 2 * 4);
    if (e != cudaSuccess) {
        fo_i8_destroy(c);
        return cuda_fail(e, "fo_i8_seal: cudaMalloc");
    }
    c->bytes = 2 * n + 2 * (size_t)n_heads * groups * 4;
    const float *dk = k, *dv = v;
    if (mem == FO_MEM_HOST) {
        e = ctx->stage[1].ensure(n * 4);
        if (e == cudaSuccess) e = ctx->stage[3].ensure(n * 4);
        if (e == cudaSuccess) e = cudaMemcpyAsync(ctx->stage[1].ptr, k, n * 4, cudaMemcpyHostToDevice, ctx->stream);
        if (e == cudaSuccess) e = cudaMemcpyAsync(ctx->stage[3].ptr, v, n * 4, cudaMemcpyHostToDevice, ctx->stream);
        dk = (const float *)ctx->stage[1].ptr;
        dv = (const float *)ctx->stage[3].ptr;
    }
    if (e == cudaSuccess) e = fo_launch_quantize_i8(dk, len, n_heads, c->k_codes, c->k_scales, ctx->stream);
    if (e == cudaSuccess) e = fo_launch_quantize_i8(dv, len, n_heads, c->v_codes, c->v_scales, ctx->stream);
    if (e == cudaSuccess && mem == FO_MEM_HOST) e = cudaStreamSynchronize(ctx->stream);
    if (e != cudaSuccess) {
        fo_i8_destroy(c);
        return cuda_fail(e, "fo_i8_seal");
    }
    *out = c;
    return FO_OK;
}

int64_t fo_i8_bytes(const fo_i8_cache *c) { return c ? (int64_t)c->bytes : -1; }

int fo_i8_records(const fo_i8_cache *c, const int8_t **k_codes, const float **k_scales, const int8_t **v_codes,
                  const float **v_scales) {
    if (!c) return fail(FO_ERR_INVALID, "null cache");
    if (k_codes) *k_codes = c->k_codes;
    if (k_scales) *k_scales = c->k_scales;
    if (v_codes) *v_codes = c->v_codes;
    if (v_scales) *v_scales = c->v_scales;
    return FO_OK;
}

int fo_i8_decode_batch(fo_i8_cache *const *caches, int64_t n, const float *const *q, const float *const *sinks,
                       float *const *output, int32_t fast_exp) {
    if (!caches || !q || !sinks || !output || n < 0) return fail(FO_ERR_INVALID, "i8 decode batch: null argument");
    if (n == 0) return FO_OK;
    fo_ctx *ctx = caches[0] ? caches[0]->ctx : nullptr;
    if (!ctx) return fail(FO_ERR_INVALID, "i8 decode batch: null cache");
    const int64_t heads = caches[0]->heads;
    for (int64_t i = 0; i < n; i++) {
        const fo_i8_cache *c = caches[i];
        if (!c || !q[i] || !sinks[i] || !output[i])
            return fail(FO_ERR_INVALID, "i8 decode batch: null entry %lld", (long long)i);
        if (c->ctx != ctx || c->heads != heads)
            return fail(FO_ERR_INVALID, "i8 decode batch: caches must share context and heads");
        if (!aligned16(q[i])) return fail(FO_ERR_INVALID, "i8 decode batch: queries must be 16-byte aligned");
    }
    {  // each page's partials belong to its cache: pages must be distinct caches
        std::vector<const fo_i8_cache *> seen(caches, caches + n);
        std::sort(seen.begin(), seen.end());
        if (std::adjacent_find(seen.begin(), seen.end()) != seen.end())
            return fail(FO_ERR_INVALID, "i8 decode batch: a cache appears twice");
    }
    DeviceGuard guard(ctx->device);
    for (int64_t base = 0; base < n; base += FO_BATCH_PAGES) {
        const int64_t m = std::min<int64_t>(FO_BATCH_PAGES, n - base);
        int slot = 0;
        fo_i8_page *hp = static_cast<fo_i8_page *>(ctx->host_i8_pages.acquire(slot));
        int32_t max_splits = 1;
        for (int64_t i = 0; i < m; i++) {
            const fo_i8_cache *c = caches[base + i];
            hp[i] = fo_i8_page{c->k_codes, c->v_codes, c->k_scales,  c->v_scales, q[base + i], sinks[base + i],
                               output[base + i], c->part_o, c->part_ml, ctx->dev_err, c->len, (int32_t)c->splits};
            max_splits = std::max<int32_t>(max_splits, (int32_t)c->splits);
        }
        FO_CUDA(cudaMemcpyAsync(ctx->i8_pages.ptr, hp, (size_t)m * sizeof(fo_i8_page), cudaMemcpyHostToDevice,
                                ctx->stream),
                "H2D(i8 pages)");
        FO_CUDA(ctx->host_i8_pages.uploaded(slot, ctx->stream), "cudaEventRecord");
        cudaError_t e = fo_launch_decode_i8((const fo_i8_page *)ctx->i8_pages.ptr, m, heads, max_splits, fast_exp,
                                            ctx->stream);
        if (e != cudaSuccess) return cuda_fail(e, "i8 decode launch");
    }
    return FO_OK;
}

// ------------------------------------------------------------ draft head KV
int fo_draft_kv_destroy(fo_draft_kv *kv) {
    if (!kv) return FO_OK;
    DeviceGuard guard(kv->ctx->device);
    cudaStreamSynchronize(kv->ctx->stream);
    void *ptrs[] = {kv->key_codes, kv->value_codes, kv->key_scales, kv->value_scales, kv->part, kv->counters,
                    kv->stage};
    for (void *p : ptrs)
        if (p) cudaFree(p);
    delete kv;
    return FO_OK;
}

// Host staging: q and out (16 x 64 each), chain keys and values (up to
// FO_DRAFT_MAX_CHAIN rows of 512 each); pushes from the host go through the
// chain part FO_DRAFT_MAX_CHAIN rows at a time.
static constexpr size_t DRAFT_STAGE_FLOATS = 2 * 1024 + 2 * (size_t)FO_DRAFT_MAX_CHAIN * FO_DRAFT_KV_WIDTH;

int fo_draft_kv_create(fo_ctx *ctx, int64_t capacity, fo_draft_kv **out) {
    if (!out) return fail(FO_ERR_INVALID, "fo_draft_kv_create: null output pointer");
    *out = nullptr;
    if (!ctx) return fail(FO_ERR_INVALID, "null context");
    if (capacity < 1 || capacity > (int64_t)1 << 24)
        return fail(FO_ERR_CAPACITY, "draft KV capacity must be 1..16,777,216 positions");
    DeviceGuard guard(ctx->device);
    fo_draft_kv *kv = new fo_draft_kv();
    kv->ctx = ctx;
    kv->capacity = capacity;
    const size_t rows = (size_t)8 * capacity;
    cudaError_t e = cudaSuccess;
    auto alloc = [&](void **p, size_t bytes) {
        if (e == cudaSuccess) e = cudaMalloc(p, bytes);
    };
    alloc((void **)&kv->key_codes, rows * 64);
    alloc((void **)&kv->value_codes, rows * 64);
    alloc((void **)&kv->key_scales, rows * 4);
    alloc((void **)&kv->value_scales, rows * 4);
    alloc((void **)&kv->part, (size_t)8 * FO_DRAFT_MAX_SPLITS * 2 * (64 + 2) * 4);
    alloc((void **)&kv->counters, 8 * sizeof(unsigned));
    alloc((void **)&kv->stage, DRAFT_STAGE_FLOATS * 4);
    if (e == cudaSuccess) e = cudaMemsetAsync(kv->counters, 0, 8 * sizeof(unsigned), ctx->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
    if (e != cudaSuccess) {
        fo_draft_kv_destroy(kv);
        return cuda_fail(e, "fo_draft_kv_create: cudaMalloc");
    }
    kv->bytes = 2 * rows * 64 + 2 * rows * 4;
    *out = kv;
    return FO_OK;
}

int64_t fo_draft_kv_len(const fo_draft_kv *kv) { return kv ? kv->len : -1; }
int64_t fo_draft_kv_bytes(const fo_draft_kv *kv) { return kv ? (int64_t)kv->bytes : -1; }

int fo_draft_kv_records(const fo_draft_kv *kv, const int8_t **key_codes, const float **key_scales,
                        const int8_t **value_codes, const float **value_scales) {
    if (!kv) return fail(FO_ERR_INVALID, "null draft KV");
    if (key_codes) *key_codes = kv->key_codes;
    if (key_scales) *key_scales = kv->key_scales;
    if (value_codes) *value_codes = kv->value_codes;
    if (value_scales) *value_scales = kv->value_scales;
    return FO_OK;
}

int fo_draft_kv_push(fo_draft_kv *kv, const float *keys, const float *values, int64_t rows, int mem) {
    if (!kv || rows < 0 || (rows > 0 && (!keys || !values))) return fail(FO_ERR_INVALID, "fo_draft_kv_push: bad argument");
    if (mem != FO_MEM_HOST && mem != FO_MEM_DEVICE) return fail(FO_ERR_INVALID, "bad mem mode");
    if (kv->len + rows > kv->capacity) return fail(FO_ERR_CAPACITY, "draft KV capacity");
    if (mem == FO_MEM_DEVICE && !(aligned8(keys) && aligned8(values)))
        return fail(FO_ERR_INVALID, "fo_draft_kv_push: keys and values must be 8-byte aligned");
    DeviceGuard guard(kv->ctx->device);
    cudaStream_t st = kv->ctx->stream;
    for (int64_t done = 0; done < rows;) {
        const int64_t n = mem == FO_MEM_HOST ? std::min<int64_t>(FO_DRAFT_MAX_CHAIN, rows - done) : rows - done;
        const float *dk = keys + done * FO_DRAFT_KV_WIDTH, *dv = values + done * FO_DRAFT_KV_WIDTH;
        if (mem == FO_MEM_HOST) {
            float *sk = kv->stage + 2048, *sv = sk + (size_t)FO_DRAFT_MAX_CHAIN * FO_DRAFT_KV_WIDTH;
            const size_t bytes = (size_t)n * FO_DRAFT_KV_WIDTH * 4;
            FO_CUDA(cudaMemcpyAsync(sk, dk, bytes, cudaMemcpyHostToDevice, st), "H2D(draft keys)");
            FO_CUDA(cudaMemcpyAsync(sv, dv, bytes, cudaMemcpyHostToDevice, st), "H2D(draft values)");
            dk = sk;
            dv = sv;
        }
        cudaError_t e = fo_launch_draft_push(dk, dv, n, kv->capacity, kv->len, kv->key_codes, kv->key_scales,
                                             kv->value_codes, kv->value_scales, st);
        if (e != cudaSuccess) return cuda_fail(e, "draft push launch");
        if (mem == FO_MEM_HOST) FO_CUDA(cudaStreamSynchronize(st), "cudaStreamSynchronize");
        kv->len += n;
        done += n;
    }
    return FO_OK;
}

int fo_draft_attend(fo_draft_kv *kv, const float *q, int64_t bases, int64_t window, const float *chain_keys,
                    const float *chain_values, int64_t chain, float *output, int mem) {
    if (!kv || !q || !output) return fail(FO_ERR_INVALID, "fo_draft_attend: null argument");
    if (mem != FO_MEM_HOST && mem != FO_MEM_DEVICE) return fail(FO_ERR_INVALID, "bad mem mode");
    if (bases < 0 || bases > kv->len) return fail(FO_ERR_INVALID, "fo_draft_attend: bases beyond the pushed rows");
    if (window < 0) return fail(FO_ERR_INVALID, "fo_draft_attend: negative window");
    if (chain < 0 || chain > FO_DRAFT_MAX_CHAIN)
        return fail(FO_ERR_INVALID, "fo_draft_attend: chain rows must be 0..%d", FO_DRAFT_MAX_CHAIN);
    if (chain > 0 && (!chain_keys || !chain_values)) return fail(FO_ERR_INVALID, "fo_draft_attend: null chain rows");
    // draft_head.rs:549-553: only the newest `window` verified rows (0: all)
    const int64_t start = window == 0 ? 0 : std::max<int64_t>(0, bases - window);
    const int64_t n = bases - start;
    if (n + chain == 0) return fail(FO_ERR_INVALID, "fo_draft_attend: nothing to attend to");
    if (mem == FO_MEM_DEVICE &&
        !(aligned16(q) && aligned4(output) && (chain == 0 || (aligned16(chain_keys) && aligned8(chain_values)))))
        return fail(FO_ERR_INVALID, "fo_draft_attend: q and chain keys must be 16-byte aligned, chain values 8");
    DeviceGuard guard(kv->ctx->device);
    cudaStream_t st = kv->ctx->stream;
    const float *dq = q, *dk = chain_keys, *dv = chain_values;
    float *dout = output;
    if (mem == FO_MEM_HOST) {
        float *sq = kv->stage, *so = kv->stage + 1024, *sk = kv->stage + 2048;
        float *sv = sk + (size_t)FO_DRAFT_MAX_CHAIN * FO_DRAFT_KV_WIDTH;
        FO_CUDA(cudaMemcpyAsync(sq, q, 1024 * 4, cudaMemcpyHostToDevice, st), "H2D(draft q)");
        if (chain > 0) {
            const size_t bytes = (size_t)chain * FO_DRAFT_KV_WIDTH * 4;
            FO_CUDA(cudaMemcpyAsync(sk, chain_keys, bytes, cudaMemcpyHostToDevice, st), "H2D(chain keys)");
            FO_CUDA(cudaMemcpyAsync(sv, chain_values, bytes, cudaMemcpyHostToDevice, st), "H2D(chain values)");
        }
        dq = sq;
        dk = sk;
        dv = sv;
        dout = so;
    }
    cudaError_t e = fo_launch_draft_attend(kv->key_codes, kv->key_scales, kv->value_codes, kv->value_scales,
                                           kv->capacity, dq, start, n, dk, dv, chain, kv->part, kv->counters, dout,
                                           st);
    if (e != cudaSuccess) return cuda_fail(e, "draft attention launch");
    if (mem == FO_MEM_HOST) {
        FO_CUDA(cudaMemcpyAsync(output, dout, 1024 * 4, cudaMemcpyDeviceToHost, st), "D2H(draft out)");
        FO_CUDA(cudaStreamSynchronize(st), "cudaStreamSynchronize");
    }
    return FO_OK;
}

}  // extern "C"
