// decode_static.cu -- verify-row decode that allocates nothing.
//
// Some callers cannot allocate device memory when they decode: a serving
// runtime that owns every byte of the GPU through its own pool, or a decode
// loop that must not call cudaMalloc/cudaFree, which can synchronize the
// whole device and stall the other streams that share it.  This entry point
// takes the sealed records, the queries, the sinks and the output from the
// caller, and keeps the split-KV partials (the only scratch the decode
// kernels need) in one fixed array compiled into this library.
//
// Limits: at most FO_STATIC_ROWS rows, FO_STATIC_HEADS query heads and
// FO_STATIC_POSITIONS cached positions (prefix + tail), the shapes of the
// reference model (8 verification rows, 16 heads, a 16,384-token context);
// larger calls are refused.  Every GPU that loads this library holds the
// array (about 4.1 MiB) until the process exits.
//
// The first call on each device looks the array's device address up
// (cudaGetSymbolAddress, with that device current); make that first call
// before any stream capture.  A lookup that fails is not remembered: the next
// call tries again.  All calls share the one array: calls whose kernels
// overlap on the GPU (other streams, other threads) race on it and must be
// serialized by the caller.  The decode kernel writes every partial that the
// merge kernel after it reads, so nothing in the array needs initializing or
// clearing between calls.
//
// Errors the kernels find on the device (a bounded wait that gave up) land in
// a second static word: the merge kernel then writes NaN outputs instead of
// stale partials, and fo_decode_static_scratch_status reports the word (and
// clears it) once the caller's stream has drained.
#include <cstdio>
#include <mutex>

#include "../../include/fo_attention.h"
#include "fo_common.cuh"
#include "fo_kernels.h"

#define FO_STATIC_ROWS 8
#define FO_STATIC_HEADS 16
#define FO_STATIC_POSITIONS 16384
// One split more than the positions need: BF16 records split the prefix and
// the tail apart (decode_tc.cu).
#define FO_STATIC_SPLITS (FO_STATIC_POSITIONS / FO_SPLIT + 1)
#define FO_STATIC_O_FLOATS (FO_STATIC_ROWS * FO_STATIC_HEADS * FO_STATIC_SPLITS * FO_HD)
#define FO_STATIC_ML_FLOATS (FO_STATIC_ROWS * FO_STATIC_HEADS * FO_STATIC_SPLITS * 2)
#define FO_STATIC_FLOATS (FO_STATIC_O_FLOATS + FO_STATIC_ML_FLOATS)

// The decode partials: split outputs [rows][heads][splits][64], then their
// (max, denominator) [rows][heads][splits][2].
static __device__ __align__(256) float g_decode_scratch[FO_STATIC_FLOATS];
// Error bits of the kernels these calls launch (FO_DEVERR_*; 0 when none).
static __device__ unsigned g_decode_static_err;

namespace {

constexpr int kMaxDevices = 64;
std::mutex g_setup_mutex;
float *g_scratch_ptr[kMaxDevices];
unsigned *g_err_ptr[kMaxDevices];

thread_local char g_msg[256];

// The device addresses of the static array and error word on the current
// device `dev`, looked up once; a failed lookup is retried on the next call.
cudaError_t device_symbols(int dev, float **scratch, unsigned **err) {
    std::lock_guard<std::mutex> lock(g_setup_mutex);
    if (!g_scratch_ptr[dev] || !g_err_ptr[dev]) {
        void *p = nullptr, *w = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_decode_scratch);
        if (e == cudaSuccess) e = cudaGetSymbolAddress(&w, g_decode_static_err);
        if (e != cudaSuccess || !p || !w) {
            cudaGetLastError();  // the failed lookup is not left pending for the caller
            return e != cudaSuccess ? e : cudaErrorInvalidSymbol;
        }
        g_scratch_ptr[dev] = static_cast<float *>(p);
        g_err_ptr[dev] = static_cast<unsigned *>(w);
    }
    *scratch = g_scratch_ptr[dev];
    *err = g_err_ptr[dev];
    return cudaSuccess;
}

bool aligned(const void *p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }

}  // namespace

// Defined in fo_abi.cu: records a message for fo_last_error().
extern "C" int fo_internal_fail(int status, const char *msg);

extern "C" int fo_decode_rows_static_scratch(const void *codes, const uint16_t *scales, const void *tail_codes,
                                             const uint16_t *tail_scales, int32_t format, int64_t prefix_len,
                                             int64_t prefix_stride, int64_t tail_len, int64_t tail_stride,
                                             int64_t n_heads, int64_t n_kv_heads, const float *q, int64_t rows,
                                             const float *sinks, int32_t fast_exp, float *output, void *stream) {
    if (!codes || !q || !sinks || !output || (tail_len > 0 && !tail_codes))
        return fo_internal_fail(FO_ERR_INVALID, "static-scratch decode: null pointer");
    // An element format, optionally rotated (F32, Q8 and Q4 only).
    const int element = format & ~FO_KV_ROTATED;
    const bool rotated = (format & FO_KV_ROTATED) != 0;
    if ((format & ~(FO_KV_ROTATED | 7)) || element < FO_KV_F32 || element > FO_KV_Q4 ||
        (rotated && element != FO_KV_F32 && element != FO_KV_Q8 && element != FO_KV_Q4))
        return fo_internal_fail(FO_ERR_INVALID, "static-scratch decode: unknown record format");
    if ((element == FO_KV_Q8 || element == FO_KV_Q16 || element == FO_KV_Q4) &&
        (!scales || (tail_len > 0 && !tail_scales)))
        return fo_internal_fail(FO_ERR_INVALID, "static-scratch decode: coded records need their scales");
    // The records are staged with bulk copies (16-byte aligned sources); the
    // queries are read two floats at a time, the scales as 16-bit words.
    if (!aligned(codes, 16) || (tail_len > 0 && !aligned(tail_codes, 16)) || !aligned(q, 8) ||
        !aligned(output, 4) || !aligned(sinks, 4) || (scales && !aligned(scales, 2)) ||
        (tail_scales && !aligned(tail_scales, 2)))
        return fo_internal_fail(FO_ERR_INVALID,
                                "static-scratch decode: codes and tail_codes must be 16-byte aligned, q 8-byte aligned");
    if (!(n_kv_heads >= 1 && n_heads == 2 * n_kv_heads))
        return fo_internal_fail(FO_ERR_INVALID, "static-scratch decode: heads must be paired GQA heads");
    if (!(prefix_len >= 1 && tail_len >= 0 && prefix_stride >= prefix_len && tail_stride >= tail_len))
        return fo_internal_fail(FO_ERR_INVALID, "static-scratch decode: bad prefix/tail lengths or strides");
    if (!(rows >= 1 && rows <= FO_STATIC_ROWS && rows <= (tail_len > 1 ? tail_len : 1)))
        return fo_internal_fail(FO_ERR_INVALID, "static-scratch decode: rows must be 1..8 and at most max(tail_len, 1)");
    const int64_t last = prefix_len + tail_len;
    if (n_heads > FO_STATIC_HEADS || last > FO_STATIC_POSITIONS) {
        snprintf(g_msg, sizeof g_msg,
                 "static-scratch decode: %lld heads and %lld positions exceed the static scratch limit "
                 "(%d heads, %d positions)",
                 (long long)n_heads, (long long)last, FO_STATIC_HEADS, FO_STATIC_POSITIONS);
        return fo_internal_fail(FO_ERR_CAPACITY, g_msg);
    }
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess || dev < 0 || dev >= kMaxDevices)
        return fo_internal_fail(FO_ERR_CUDA, "static-scratch decode: no usable current device");
    // Once per device, with that device current: the array's device address.
    float *base = nullptr;
    unsigned *err_word = nullptr;
    e = device_symbols(dev, &base, &err_word);
    if (e != cudaSuccess) {
        snprintf(g_msg, sizeof g_msg, "static-scratch decode: cudaGetSymbolAddress failed: %s", cudaGetErrorString(e));
        return fo_internal_fail(FO_ERR_CUDA, g_msg);
    }
    fo_decode_page p{};
    p.codes = codes;
    p.scales = scales;
    p.tail_codes = tail_codes;
    p.tail_scales = tail_scales;
    p.q = q;
    p.sinks = sinks;
    p.out = output;
    p.err = err_word;
    p.part_o = base;
    p.part_ml = base + FO_STATIC_O_FLOATS;
    p.has_map = fo_make_record_map(&p.rec_map, codes, format, prefix_len, prefix_stride, n_kv_heads) ? 1 : 0;
    p.prefix_len = prefix_len;
    p.prefix_stride = prefix_stride;
    p.tail_stride = tail_stride;
    p.last = last;
    p.rows = (int32_t)rows;
    p.splits = (int32_t)((last + FO_SPLIT - 1) / FO_SPLIT);
    p.rotated = rotated ? 1 : 0;
    if (format == FO_KV_BF16 && fo_make_tc_maps(&p, n_kv_heads, tail_len)) {
        // The tensor-core decode's split layout (prefix and tail apart), as
        // fo_kv_attention_decode_rows uses for BF16 records; the tail map ends
        // at tail_len, so records past it are never read.
        fo_tc_layout(&p, n_kv_heads, tail_len);
    }
    e = fo_launch_decode_one(&p, format, n_kv_heads, fast_exp != 0, (cudaStream_t)stream);
    if (e != cudaSuccess) {
        snprintf(g_msg, sizeof g_msg, "static-scratch decode launch: %s", cudaGetErrorString(e));
        return fo_internal_fail(FO_ERR_CUDA, g_msg);
    }
    return FO_OK;
}

extern "C" int fo_decode_static_scratch_status(void *stream) {
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess || dev < 0 || dev >= kMaxDevices)
        return fo_internal_fail(FO_ERR_CUDA, "static-scratch status: no usable current device");
    float *base = nullptr;
    unsigned *err_word = nullptr;
    if ((e = device_symbols(dev, &base, &err_word)) != cudaSuccess) {
        snprintf(g_msg, sizeof g_msg, "static-scratch status: cudaGetSymbolAddress failed: %s", cudaGetErrorString(e));
        return fo_internal_fail(FO_ERR_CUDA, g_msg);
    }
    const cudaStream_t st = (cudaStream_t)stream;
    unsigned bits = 0;
    e = cudaMemcpyAsync(&bits, err_word, sizeof bits, cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e == cudaSuccess && bits) e = cudaMemsetAsync(err_word, 0, sizeof bits, st);
    if (e == cudaSuccess && bits) e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) {
        snprintf(g_msg, sizeof g_msg, "static-scratch status: %s", cudaGetErrorString(e));
        return fo_internal_fail(FO_ERR_CUDA, g_msg);
    }
    if (bits) {
        snprintf(g_msg, sizeof g_msg,
                 "static-scratch decode: a kernel wait exceeded its time limit (bits 0x%x); the outputs of the "
                 "calls since the last status check are NaN",
                 bits);
        return fo_internal_fail(FO_ERR_CUDA, g_msg);
    }
    return FO_OK;
}
