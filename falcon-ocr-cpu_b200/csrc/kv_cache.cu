// kv_cache.cu -- sealing a compact prefix into split records and appending
// generated positions (reference: SplitPrefix::seal, src/quant/kv.rs:239-418;
// push_unique, :456-513; codec, src/quant/kv/codec.rs:9-83), plus the FP32 to
// BF16 conversion of prefill operands (prefill64/bf16.rs:190-223).
//
// Records are group-major: for group g and prefix position t the record
// `[T 32 | S(2g) 32 | S(2g+1) 32 | V 64]` lives at codes[(g * stride + t) * 160]
// with its five BF16 block scales at scales[(g * stride + t) * 5]; tail
// records `[K 64 | V 64]` at tail_codes[(g * tail_stride + i) * 128] with four
// scales.  Codes are integers computed exactly as the reference does: the
// f64 quotient value / scale rounded to nearest even and clamped, so they
// match it bit for bit.
#include "fo_common.cuh"
#include "fo_kernels.h"

namespace fo {

enum { KV_F32 = 0, KV_Q16 = 1, KV_Q8 = 2, KV_BF16 = 3 };

// codec.rs:60-63 (clamp, then round half to even; |x| < 2^51).
__device__ __forceinline__ double round_clamped(double x, double limit) {
    if (isnan(x)) return x;
    x = x < -limit ? -limit : (x > limit ? limit : x);
    return rint(x);
}

// codec.rs:11-32: absmax over `limit`, at least the smallest subnormal.
__device__ __forceinline__ float block_scale(float max, double limit) {
    if (max == 0.0f) return 0.0f;
    float s = (float)((double)max / limit);
    const float tiny = __uint_as_float(1u);
    return s > tiny ? s : tiny;
}

// Encode one 32-element block held one value per lane.  `nan_on_nonfinite`
// is the tail rule (a non-finite block gets a NaN scale, kv.rs:474-478);
// the prefix instead rejects non-finite input before encoding.
__device__ __forceinline__ void encode_block(float x, int format, void *codes, uint16_t *scales, int64_t at,
                                             bool nan_on_nonfinite, unsigned *flags) {
    const int lane = threadIdx.x & 31;
    if (format == KV_F32) {
        reinterpret_cast<float *>(codes)[at + lane] = x;
        return;
    }
    if (format == KV_BF16) {
        reinterpret_cast<uint16_t *>(codes)[at + lane] = bf16_rne(x);
        return;
    }
    const bool q8 = format == KV_Q8;
    const double limit = q8 ? 127.0 : 32767.0;
    const float mx = warp_max(fabsf(x));  // NaN-ignoring, as Rust f32::max
    const bool finite = __all_sync(0xffffffffu, isfinite(x));
    const float raw = (nan_on_nonfinite && !finite) ? __uint_as_float(0x7FC00000u) : block_scale(mx, limit);
    const uint16_t stored = bf16_up(raw);
    const float scale = bf16_f32(stored);
    if (lane == 0) scales[at / 32] = stored;
    int code = 0;
    if (scale != 0.0f) {
        const double r = round_clamped((double)x / (double)scale, limit);
        code = isnan(r) ? 0 : (int)r;  // Rust `as` casts NaN to 0
    }
    if (q8)
        reinterpret_cast<int8_t *>(codes)[at + lane] = (int8_t)code;
    else
        reinterpret_cast<int16_t *>(codes)[at + lane] = (int16_t)code;
    if (!nan_on_nonfinite && !isfinite((float)code * scale)) atomicOr(flags, FO_FLAG_OVERFLOW);
}

// One warp per (group, position) record.
__global__ void seal_kernel(const float *__restrict__ k, const float *__restrict__ v, int64_t prefix_len,
                            int64_t heads, int64_t groups, int format, void *codes, uint16_t *scales, int64_t stride,
                            unsigned *flags) {
    const int64_t rec = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (rec >= groups * prefix_len) return;
    const int64_t g = rec / prefix_len, t = rec % prefix_len;
    const float *ka = k + (t * heads + 2 * g) * FO_HD;  // head 2g
    const float *kb = ka + FO_HD;                        // head 2g + 1
    const float *vv = v + (t * groups + g) * FO_HD;
    // kv.rs:266-278: the temporal halves must be bit-identical.
    if (__any_sync(0xffffffffu, __float_as_uint(ka[lane]) != __float_as_uint(kb[lane]))) {
        if (lane == 0) atomicOr(flags, FO_FLAG_PAIR);
        return;
    }
    float x[5];
    x[0] = ka[lane];           // T
    x[1] = ka[32 + lane];      // S(2g)
    x[2] = kb[32 + lane];      // S(2g+1)
    x[3] = vv[lane];           // V 0..32
    x[4] = vv[32 + lane];      // V 32..64
    bool ok = true;
#pragma unroll
    for (int b = 0; b < 5; b++) ok = ok && isfinite(x[b]);
    if (!__all_sync(0xffffffffu, ok)) {  // kv.rs:288
        if (lane == 0) atomicOr(flags, FO_FLAG_NONFINITE);
        return;
    }
    const int64_t base = (g * stride + t) * FO_RECORD;
#pragma unroll
    for (int b = 0; b < 5; b++) encode_block(x[b], format, codes, scales, base + 32 * b, false, flags);
}

// Tail record `first + r` of group g from expanded row r: the group's first
// head (kv.rs:437-447); one warp, a lane per dimension pair.
__device__ __forceinline__ void append_record(const float *__restrict__ k, const float *__restrict__ v, int64_t r,
                                              int64_t g, int64_t heads, int format, void *tail_codes,
                                              uint16_t *tail_scales, int64_t tail_stride, int64_t first, int lane) {
    const float *kr = k + (r * heads + 2 * g) * FO_HD;
    const float *vr = v + (r * heads + 2 * g) * FO_HD;
    const int64_t base = (g * tail_stride + first + r) * FO_TAIL_RECORD;
    encode_block(kr[lane], format, tail_codes, tail_scales, base, true, nullptr);
    encode_block(kr[32 + lane], format, tail_codes, tail_scales, base + 32, true, nullptr);
    encode_block(vr[lane], format, tail_codes, tail_scales, base + 64, true, nullptr);
    encode_block(vr[32 + lane], format, tail_codes, tail_scales, base + 96, true, nullptr);
}

// One warp per (row, group) tail record.
__global__ void append_kernel(const float *__restrict__ k, const float *__restrict__ v, int64_t rows, int64_t heads,
                              int64_t groups, int format, void *tail_codes, uint16_t *tail_scales,
                              int64_t tail_stride, int64_t first) {
    const int64_t w = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    if (w >= rows * groups) return;
    append_record(k, v, w / groups, w % groups, heads, format, tail_codes, tail_scales, tail_stride, first,
                  threadIdx.x & 31);
}

// The same over many caches at once: one warp per (page, row, group).
__global__ void append_batch_kernel(const fo_append_page *__restrict__ pages, int64_t n, int64_t rows,
                                    int64_t heads, int64_t groups, int format) {
    const int64_t w = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int64_t per_page = rows * groups;
    if (w >= n * per_page) return;
    const int64_t i = w / per_page, rg = w - i * per_page;
    const fo_append_page &pg = pages[i];
    append_record(pg.k, pg.v, rg / groups, rg % groups, heads, format, pg.tail_codes, pg.tail_scales,
                  pg.tail_stride, pg.first, threadIdx.x & 31);
}

// FP32 -> BF16, eight values per thread (16-byte stores).
__global__ void convert_bf16_kernel(const float *__restrict__ src, uint16_t *__restrict__ dst, int64_t n) {
    const int64_t i8 = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) * 8;
    if (i8 + 8 <= n && ((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst)) & 15) == 0) {
        const float4 a = *reinterpret_cast<const float4 *>(src + i8);
        const float4 b = *reinterpret_cast<const float4 *>(src + i8 + 4);
        uint4 o;
        o.x = bf16_rne(a.x) | ((uint32_t)bf16_rne(a.y) << 16);
        o.y = bf16_rne(a.z) | ((uint32_t)bf16_rne(a.w) << 16);
        o.z = bf16_rne(b.x) | ((uint32_t)bf16_rne(b.y) << 16);
        o.w = bf16_rne(b.z) | ((uint32_t)bf16_rne(b.w) << 16);
        *reinterpret_cast<uint4 *>(dst + i8) = o;
    } else {
        for (int64_t i = i8; i < n && i < i8 + 8; i++) dst[i] = bf16_rne(src[i]);
    }
}

}  // namespace fo

extern "C" cudaError_t fo_launch_seal(const float *k, const float *v, int64_t prefix_len, int64_t heads,
                                      int64_t groups, int format, void *codes, uint16_t *scales, int64_t stride,
                                      unsigned *flags, cudaStream_t stream) {
    const int64_t warps = groups * prefix_len;
    if (warps == 0) return cudaSuccess;
    const int threads = 256;
    const int64_t blocks = (warps * 32 + threads - 1) / threads;
    fo::seal_kernel<<<(unsigned)blocks, threads, 0, stream>>>(k, v, prefix_len, heads, groups, format, codes, scales,
                                                              stride, flags);
    return cudaGetLastError();
}

extern "C" cudaError_t fo_launch_append(const float *k, const float *v, int64_t rows, int64_t heads, int64_t groups,
                                        int format, void *tail_codes, uint16_t *tail_scales, int64_t tail_stride,
                                        int64_t first, cudaStream_t stream) {
    const int64_t warps = rows * groups;
    if (warps == 0) return cudaSuccess;
    const int threads = 256;
    const int64_t blocks = (warps * 32 + threads - 1) / threads;
    fo::append_kernel<<<(unsigned)blocks, threads, 0, stream>>>(k, v, rows, heads, groups, format, tail_codes,
                                                                tail_scales, tail_stride, first);
    return cudaGetLastError();
}

extern "C" cudaError_t fo_launch_append_batch(const fo_append_page *pages, int64_t n, int64_t rows, int64_t heads,
                                              int64_t groups, int format, cudaStream_t stream) {
    const int64_t warps = n * rows * groups;
    if (warps == 0) return cudaSuccess;
    const int threads = 256;
    const int64_t blocks = (warps * 32 + threads - 1) / threads;
    fo::append_batch_kernel<<<(unsigned)blocks, threads, 0, stream>>>(pages, n, rows, heads, groups, format);
    return cudaGetLastError();
}

extern "C" cudaError_t fo_launch_convert_bf16(const float *src, uint16_t *dst, int64_t n, cudaStream_t stream) {
    if (n == 0) return cudaSuccess;
    const int threads = 256;
    const int64_t blocks = ((n + 7) / 8 + threads - 1) / threads;
    fo::convert_bf16_kernel<<<(unsigned)blocks, threads, 0, stream>>>(src, dst, n);
    return cudaGetLastError();
}
