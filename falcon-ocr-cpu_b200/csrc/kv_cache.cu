// kv_cache.cu -- sealing a compact prefix into split records and appending
// generated positions (reference: SplitPrefix::seal, src/quant/kv.rs:239-418;
// push_unique, :456-513; codec, src/quant/kv/codec.rs:9-83), plus the FP32 to
// BF16 conversion of prefill operands (prefill64/bf16.rs:190-223).
//
// Records are group-major: for group g and prefix position t the record
// `[T 32 | S(2g) 32 | S(2g+1) 32 | V 64]` lives at codes[(g * stride + t) * 160]
// with its five BF16 block scales at scales[(g * stride + t) * 5]; tail
// records `[K 64 | V 64]` at tail_codes[(g * tail_stride + i) * 128] with four
// scales (element offsets: Q4 packs two codes per byte, element 2i in the
// low nibble).  Codes are integers computed exactly as the reference does:
// the f64 quotient value / scale rounded to nearest even and clamped, so they
// match it bit for bit.  Rotated formats (FO_KV_ROTATED: Kv::Q8Rot, Kv::Q4Rot
// and the rotated FP32 test storage) first rotate every 32-element block,
// H D x (src/quant/rotation.rs:100-104), with the warp's lanes as the block's
// elements: the sign flips, then the five butterfly stages across lanes.
#include "fo_common.cuh"
#include "fo_kernels.h"

namespace fo {

enum { KV_F32 = 0, KV_Q16 = 1, KV_Q8 = 2, KV_BF16 = 3, KV_Q4 = 4, KV_ROTATED = 16 };

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
    if (format == KV_Q4) {
        // codec.rs:87-122: absmax / 7, codes -7..7 packed two per byte
        // (element 2i in the low nibble); a non-finite block gets a NaN scale.
        const float mx = warp_max(fabsf(x));
        const bool finite = __all_sync(0xffffffffu, isfinite(x));
        const uint16_t stored = bf16_up(finite ? block_scale(mx, 7.0) : __uint_as_float(0x7FC00000u));
        const float scale = bf16_f32(stored);
        if (lane == 0) scales[at / 32] = stored;
        int code = 0;
        if (scale != 0.0f) {
            const double r = round_clamped((double)x / (double)scale, 7.0);
            code = isnan(r) ? 0 : (int)r;
        }
        const int high = __shfl_down_sync(0xffffffffu, code, 1);
        if ((lane & 1) == 0)
            reinterpret_cast<uint8_t *>(codes)[(at + lane) / 2] = (uint8_t)((code & 0xF) | ((high & 0xF) << 4));
        // kv.rs:381-383: codes are at most 7 in magnitude
        if (!nan_on_nonfinite && lane == 0 && !isfinite(7.0f * scale)) atomicOr(flags, FO_FLAG_OVERFLOW);
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
    if (format & KV_ROTATED) {
        // kv.rs:289-293: every block rotated after the pair check (which saw
        // the unrotated keys); kinds [T, S, S, V0, V1].
        const int kinds[5] = {0, 1, 1, 2, 3};
        ok = true;
#pragma unroll
        for (int b = 0; b < 5; b++) {
            x[b] = rotate_lane(x[b], kinds[b], lane);
            ok = ok && isfinite(x[b]);
        }
        if (!__all_sync(0xffffffffu, ok)) {
            if (lane == 0) atomicOr(flags, FO_FLAG_ROTATED);
            return;
        }
    }
    const int64_t base = (g * stride + t) * FO_RECORD;
#pragma unroll
    for (int b = 0; b < 5; b++) encode_block(x[b], format & ~KV_ROTATED, codes, scales, base + 32 * b, false, flags);
}

// Tail record blocks [K 0..32 | K 32..64 | V 0..32 | V 32..64] (one value per
// lane each): rotated when the format is (kv.rs:466-468, kinds T, S, V0, V1),
// then encoded with the tail's rule for non-finite blocks.
__device__ __forceinline__ void encode_tail_record(float k0, float k1, float v0, float v1, int format,
                                                   void *tail_codes, uint16_t *tail_scales, int64_t base, int lane) {
    float x[4] = {k0, k1, v0, v1};
    if (format & KV_ROTATED) {
#pragma unroll
        for (int b = 0; b < 4; b++) x[b] = rotate_lane(x[b], b, lane);
    }
#pragma unroll
    for (int b = 0; b < 4; b++)
        encode_block(x[b], format & ~KV_ROTATED, tail_codes, tail_scales, base + 32 * b, true, nullptr);
}

// Tail record `first + r` of group g from expanded row r: the group's first
// head (kv.rs:437-447); one warp, a lane per dimension pair.
__device__ __forceinline__ void append_record(const float *__restrict__ k, const float *__restrict__ v, int64_t r,
                                              int64_t g, int64_t heads, int format, void *tail_codes,
                                              uint16_t *tail_scales, int64_t tail_stride, int64_t first, int lane) {
    const float *kr = k + (r * heads + 2 * g) * FO_HD;
    const float *vr = v + (r * heads + 2 * g) * FO_HD;
    const int64_t base = (g * tail_stride + first + r) * FO_TAIL_RECORD;
    encode_tail_record(kr[lane], kr[32 + lane], vr[lane], vr[32 + lane], format, tail_codes, tail_scales, base, lane);
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
                                    int64_t heads, int64_t groups, int format, fo_decode_page *dp, unsigned *err) {
    const int64_t w = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int64_t per_page = rows * groups;
    if (w >= n * per_page) return;
    const int64_t i = w / per_page, rg = w - i * per_page;
    const fo_append_page &pg = pages[i];
    if (dp && rg == 0 && (threadIdx.x & 31) == 0) {
        // A batch plan's step (one lane per page): the page's decode covers
        // the rows appended now; a tail without room for them writes nothing,
        // keeps its decode length and raises the capacity bit.
        if (pg.first + rows > pg.tail_stride) {
            if (err) atomicOr(err, FO_DEVERR_CAPACITY);
        } else {
            dp[i].last = dp[i].prefix_len + pg.first + rows;
            dp[i].splits = (int32_t)((dp[i].last + FO_SPLIT - 1) / FO_SPLIT);
        }
    }
    if (pg.first + rg / groups >= pg.tail_stride) return;  // a full batch-plan tail
    append_record(pg.k, pg.v, rg / groups, rg % groups, heads, format, pg.tail_codes, pg.tail_scales,
                  pg.tail_stride, pg.first, threadIdx.x & 31);
}

// ------------------------------------------------------- fused QKV rows
// One head of the fused QKV rows (src/model/fused.rs:96-116 and :184-223):
// lane l holds dimensions 2l and 2l + 1 (the rotation's pair l).  The sum of
// squares follows sum_squares_pairwise's tree (src/kernels/mod.rs:535-555):
// two 32-value leaves (lanes 0-15 and 16-31), in each partial[i] +=
// partial[i + w] for w = 16, 8, 4, 2, 1 (lanes l and l + w/2 here), then
// leaf 0 + leaf 1; rms_scale's 1 / sqrt(sum / 64 + f32::EPSILON) with IEEE
// square root and reciprocal (mod.rs:531-533); then x * scale and the
// unfused rotation a*cos - b*sin, a*sin + b*cos.
__device__ __forceinline__ float2 norm_rope_pair(float2 x, float2 cs) {
    float px = __fmul_rn(x.x, x.x), py = __fmul_rn(x.y, x.y);
#pragma unroll
    for (int off = 8; off >= 1; off >>= 1) {
        const float ox = __shfl_down_sync(0xffffffffu, px, off), oy = __shfl_down_sync(0xffffffffu, py, off);
        px = __fadd_rn(px, ox);
        py = __fadd_rn(py, oy);
    }
    const float leaf = __fadd_rn(px, py);  // in lanes 0 and 16
    const float sum = __fadd_rn(__shfl_sync(0xffffffffu, leaf, 0), __shfl_sync(0xffffffffu, leaf, 16));
    const float scale = __frcp_rn(__fsqrt_rn(__fadd_rn(__fdiv_rn(sum, 64.0f), 1.1920928955078125e-7f)));
    const float a = __fmul_rn(x.x, scale), b = __fmul_rn(x.y, scale);
    return make_float2(__fsub_rn(__fmul_rn(a, cs.x), __fmul_rn(b, cs.y)),
                       __fadd_rn(__fmul_rn(a, cs.y), __fmul_rn(b, cs.x)));
}

// Prefill rows (fused_prefix_rows, fused.rs:17-93): one warp per (row, head)
// writes query head h and key head h (from KV head h / (heads / groups)),
// rotated by rope[row][h]; warps of heads h < groups also copy value head h.
// BF16 copies (round to nearest even) when kb / vb are given.
__global__ void qkv_rows_kernel(const float *__restrict__ qkv, const float *__restrict__ rope, int64_t rows,
                                int heads, int groups, float *__restrict__ q, float *__restrict__ k,
                                float *__restrict__ v, uint32_t *__restrict__ kb, uint32_t *__restrict__ vb) {
    const int64_t w = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (w >= rows * heads) return;
    const int64_t r = w / heads;
    const int h = (int)(w - r * heads);
    const int64_t qdim = (int64_t)heads * FO_HD, kdim = (int64_t)groups * FO_HD;
    const float *src = qkv + r * (qdim + 2 * kdim);
    const float2 cs = reinterpret_cast<const float2 *>(rope + (r * heads + h) * FO_HD)[lane];
    const float2 yq = norm_rope_pair(reinterpret_cast<const float2 *>(src + h * FO_HD)[lane], cs);
    const float2 yk =
        norm_rope_pair(reinterpret_cast<const float2 *>(src + qdim + (h / (heads / groups)) * FO_HD)[lane], cs);
    const int64_t o = (r * heads + h) * FO_HD;
    reinterpret_cast<float2 *>(q + o)[lane] = yq;
    reinterpret_cast<float2 *>(k + o)[lane] = yk;
    if (kb) kb[o / 2 + lane] = (uint32_t)bf16_rne(yk.x) | ((uint32_t)bf16_rne(yk.y) << 16);
    if (h < groups) {
        const float2 xv = reinterpret_cast<const float2 *>(src + qdim + kdim + h * FO_HD)[lane];
        const int64_t ov = (r * groups + h) * FO_HD;
        reinterpret_cast<float2 *>(v + ov)[lane] = xv;
        if (vb) vb[ov / 2 + lane] = (uint32_t)bf16_rne(xv.x) | ((uint32_t)bf16_rne(xv.y) << 16);
    }
}

// Decode rows (split_norm_rope, rope.rs:15-85, then SplitPrefix::append,
// kv.rs:430-449): warps of the first rows * heads write the rotated queries;
// then one warp per (row, group) builds the pair's first key head (its own
// rotation) and the group's value and encodes tail record first + row, as
// append_record does with expanded rows.
__global__ void qkv_append_kernel(const float *__restrict__ qkv, const float *__restrict__ rope, int64_t rows,
                                  int heads, int groups, float *__restrict__ q, int format, void *tail_codes,
                                  uint16_t *tail_scales, int64_t tail_stride, int64_t first) {
    const int64_t w = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    const int64_t qdim = (int64_t)heads * FO_HD, kdim = (int64_t)groups * FO_HD;
    if (w < rows * heads) {
        const int64_t r = w / heads;
        const int h = (int)(w - r * heads);
        const float *src = qkv + r * (qdim + 2 * kdim);
        const float2 cs = reinterpret_cast<const float2 *>(rope + (r * heads + h) * FO_HD)[lane];
        reinterpret_cast<float2 *>(q + (r * heads + h) * FO_HD)[lane] =
            norm_rope_pair(reinterpret_cast<const float2 *>(src + h * FO_HD)[lane], cs);
        return;
    }
    const int64_t w2 = w - rows * heads;
    if (w2 >= rows * groups) return;
    const int64_t r = w2 / groups;
    const int g = (int)(w2 - r * groups), h = g * (heads / groups);
    const float *src = qkv + r * (qdim + 2 * kdim);
    const float2 cs = reinterpret_cast<const float2 *>(rope + (r * heads + h) * FO_HD)[lane];
    const float2 yk = norm_rope_pair(reinterpret_cast<const float2 *>(src + qdim + g * FO_HD)[lane], cs);
    // to the record's layout: lane l encodes dimensions l and 32 + l
    const int sl = lane >> 1;
    const float a0 = __shfl_sync(0xffffffffu, yk.x, sl), a1 = __shfl_sync(0xffffffffu, yk.y, sl);
    const float b0 = __shfl_sync(0xffffffffu, yk.x, 16 + sl), b1 = __shfl_sync(0xffffffffu, yk.y, 16 + sl);
    const float *vr = src + qdim + kdim + g * FO_HD;
    const int64_t base = ((int64_t)g * tail_stride + first + r) * FO_TAIL_RECORD;
    encode_tail_record((lane & 1) ? a1 : a0, (lane & 1) ? b1 : b0, vr[lane], vr[32 + lane], format, tail_codes,
                       tail_scales, base, lane);
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
                                              int64_t groups, int format, fo_decode_page *plan_pages, unsigned *err,
                                              cudaStream_t stream) {
    const int64_t warps = n * rows * groups;
    if (warps == 0) return cudaSuccess;
    const int threads = 256;
    const int64_t blocks = (warps * 32 + threads - 1) / threads;
    fo::append_batch_kernel<<<(unsigned)blocks, threads, 0, stream>>>(pages, n, rows, heads, groups, format,
                                                                      plan_pages, err);
    return cudaGetLastError();
}

extern "C" cudaError_t fo_launch_qkv_rows(const float *qkv, const float *rope, int64_t rows, int heads, int groups,
                                          float *q, float *k, float *v, uint16_t *k_bf16, uint16_t *v_bf16,
                                          cudaStream_t stream) {
    const int64_t warps = rows * heads;
    if (warps == 0) return cudaSuccess;
    const int threads = 256;
    const int64_t blocks = (warps * 32 + threads - 1) / threads;
    fo::qkv_rows_kernel<<<(unsigned)blocks, threads, 0, stream>>>(qkv, rope, rows, heads, groups, q, k, v,
                                                                  reinterpret_cast<uint32_t *>(k_bf16),
                                                                  reinterpret_cast<uint32_t *>(v_bf16));
    return cudaGetLastError();
}

extern "C" cudaError_t fo_launch_qkv_append(const float *qkv, const float *rope, int64_t rows, int heads, int groups,
                                            float *q, int format, void *tail_codes, uint16_t *tail_scales,
                                            int64_t tail_stride, int64_t first, cudaStream_t stream) {
    const int64_t warps = rows * (heads + groups);
    if (warps == 0) return cudaSuccess;
    const int threads = 256;
    const int64_t blocks = (warps * 32 + threads - 1) / threads;
    fo::qkv_append_kernel<<<(unsigned)blocks, threads, 0, stream>>>(qkv, rope, rows, heads, groups, q, format,
                                                                    tail_codes, tail_scales, tail_stride, first);
    return cudaGetLastError();
}

extern "C" cudaError_t fo_launch_convert_bf16(const float *src, uint16_t *dst, int64_t n, cudaStream_t stream) {
    if (n == 0) return cudaSuccess;
    const int threads = 256;
    const int64_t blocks = ((n + 7) / 8 + threads - 1) / threads;
    fo::convert_bf16_kernel<<<(unsigned)blocks, threads, 0, stream>>>(src, dst, n);
    return cudaGetLastError();
}
