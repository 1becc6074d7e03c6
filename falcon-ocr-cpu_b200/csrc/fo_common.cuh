// fo_common.cuh -- shared device helpers of the B200 attention backend.
//
// Arithmetic restated from the reference (paths relative to its project
// root); CUDA's own math functions are called, never re-implemented.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#define FO_HD 64            // head_dim of every fixed-width kernel
#define FO_RECORD 160       // prefix record elements (src/quant/kv.rs:55)
#define FO_TAIL_RECORD 128  // tail record elements (src/quant/kv.rs:60)
#define FO_MAX_ROWS 8       // verification rows (src/quant/kv.rs:68)

// Device status bits the seal kernel raises (checked on the host).
#define FO_FLAG_PAIR 1u
#define FO_FLAG_NONFINITE 2u
#define FO_FLAG_OVERFLOW 4u
#define FO_FLAG_ROTATED 8u  // a rotated block is no longer finite (kv.rs:289-293)

// The record format's rotation flag (FO_KV_ROTATED of the C ABI).
#define FO_KV_ROTATED_BIT 16

namespace fo {

__host__ __device__ __forceinline__ int64_t min64(int64_t a, int64_t b) { return a < b ? a : b; }
__host__ __device__ __forceinline__ int64_t max64(int64_t a, int64_t b) { return a > b ? a : b; }

// ---- rotation of 32-value blocks (src/quant/rotation.rs) ----
// The sign pattern D of block kind k (0 temporal key half, 1 spatial key
// half, 2 value 0..32, 3 value 32..64): the low 32 bits of SplitMix64's
// output for the state SEED + (k + 1) * GAMMA, SEED = "KVROTATE" read
// big-endian (rotation.rs:36-61).
constexpr uint64_t splitmix64_out(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
    return z ^ (z >> 31);
}
constexpr uint32_t rotation_signs(int kind) {
    return (uint32_t)splitmix64_out(0x4b56524f54415445ull + (uint64_t)(kind + 1) * 0x9e3779b97f4a7c15ull);
}
// The reference's own known answers (rotation.rs:163-166).
static_assert(rotation_signs(0) == 0x04dcf6b7u && rotation_signs(1) == 0x871f5f8bu &&
                  rotation_signs(2) == 0x489ce13cu && rotation_signs(3) == 0x4a81cbcbu,
              "rotation sign words");

// One stage of the Sylvester butterflies over elements held one per lane
// group: element i pairs with i ^ half; the low one becomes a + b, the high
// one a - b (a the low element, rotation.rs:71-84).  `partner` is the other
// element, `high` whether this one is the high element.
__device__ __forceinline__ float butterfly(float x, float partner, bool high) {
    return high ? __fsub_rn(partner, x) : __fadd_rn(x, partner);
}

// x <- H D x for a block held one element per lane (lane = element index):
// the stored form of a key or value block (rotation.rs:100-104).
__device__ __forceinline__ float rotate_lane(float x, int kind, int lane) {
    x = __uint_as_float(__float_as_uint(x) ^ (((rotation_signs(kind) >> lane) & 1u) << 31));
#pragma unroll
    for (int half = 1; half < 32; half <<= 1) x = butterfly(x, __shfl_xor_sync(0xffffffffu, x, half), lane & half);
    return x;
}

__device__ __forceinline__ float bits_f32(uint32_t u) { return __uint_as_float(u); }
__device__ __forceinline__ uint32_t f32_bits(float f) { return __float_as_uint(f); }

// BF16 bits widened exactly (src/quant/kv/codec.rs:48-50).
__device__ __forceinline__ float bf16_f32(uint16_t b) { return __uint_as_float((uint32_t)b << 16); }

// Round to nearest even; NaN stays a quiet NaN with its sign and payload top
// bits (half::bf16::from_f32, which the reference's BF16 paths use).
__device__ __forceinline__ uint16_t bf16_rne(float x) {
    uint32_t u = __float_as_uint(x);
    if ((u & 0x7FFFFFFFu) > 0x7F800000u) return (uint16_t)((u >> 16) | 0x40u);
    u += 0x7FFFu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

// Smallest BF16 at or above a positive finite scale, 0 or NaN
// (src/quant/kv/codec.rs:37-44).
__device__ __forceinline__ uint16_t bf16_up(float scale) {
    if (isnan(scale)) return 0x7FC0;
    uint32_t bits = __float_as_uint(scale);
    uint16_t high = (uint16_t)(bits >> 16);
    return (bits & 0xFFFFu) ? (uint16_t)(high + 1) : high;
}

// The reference's portable polynomial exp (src/kernels/exp.rs:232-277,
// Cephes-style constants published there).  Written with explicit FMAs in
// the reference's order; used where the reference selects its fast exp.
__device__ __forceinline__ float exp_poly_unchecked(float x) {
    const float LOG2E = 1.44269504088896340736f;
    const float LN2_HI = 0.6933594f, LN2_LO = -2.1219444e-4f;
    float n = rintf(__fmul_rn(x, LOG2E));
    float r = __fmaf_rn(n, -LN2_HI, x);
    r = __fmaf_rn(n, -LN2_LO, r);
    float p = 1.9875691e-4f;
    p = __fmaf_rn(p, r, 1.3981999e-3f);
    p = __fmaf_rn(p, r, 8.333452e-3f);
    p = __fmaf_rn(p, r, 4.1665796e-2f);
    p = __fmaf_rn(p, r, 0.16666665f);
    p = __fmaf_rn(p, r, 0.5f);
    float y = __fadd_rn(__fmaf_rn(p, __fmul_rn(r, r), r), 1.0f);
    return __fmul_rn(y, __uint_as_float((uint32_t)((int)n + 127) << 23));
}

__device__ __forceinline__ float exp_poly(float x) {
    if (isnan(x)) return x;
    if (x < -87.0f) return 0.0f;
    if (x > 88.376f) return INFINITY;
    return exp_poly_unchecked(x);
}

// The softmax exp: CUDA's accurate expf, or the reference's exp_poly.
template <bool FAST>
__device__ __forceinline__ float softmax_exp(float x) {
    if constexpr (FAST) return exp_poly(x); else return expf(x);
}

// Exact integer codes as floats without the conversion unit (which runs at
// a fraction of the FMA rate): a code c, offset to be non-negative, is
// placed in the mantissa of 2^23 (byte permute) and 2^23 plus the offset is
// subtracted; every step is exact.
// The four signed bytes of w.
__device__ __forceinline__ void s8x4_f32(uint32_t w, float *out) {
    const uint32_t u = w ^ 0x80808080u;
    // (2^23 + 128 + c) - (2^23 + 128) is exact; two codes per packed subtract.
    const float2 lo = __fadd2_rn(make_float2(__uint_as_float(__byte_perm(u, 0x4B000000u, 0x7540u)),
                                             __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7541u))),
                                 make_float2(-8388736.0f, -8388736.0f));
    const float2 hi = __fadd2_rn(make_float2(__uint_as_float(__byte_perm(u, 0x4B000000u, 0x7542u)),
                                             __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7543u))),
                                 make_float2(-8388736.0f, -8388736.0f));
    out[0] = lo.x;
    out[1] = lo.y;
    out[2] = hi.x;
    out[3] = hi.y;
}
// The two signed bytes in the low half of w (as a 16-bit load returns them).
__device__ __forceinline__ void s8x2_f32(uint32_t w, float &lo, float &hi) {
    const uint32_t u = w ^ 0x8080u;
    const float2 x = __fadd2_rn(make_float2(__uint_as_float(__byte_perm(u, 0x4B000000u, 0x7540u)),
                                            __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7541u))),
                                make_float2(-8388736.0f, -8388736.0f));
    lo = x.x;
    hi = x.y;
}
// The signed 4-bit codes of a byte (codec.rs:127-129: element 2i in the
// low nibble), exactly: each nibble with its sign bit flipped is the code + 8,
// placed in the mantissa of 2^23 and shifted back.
__device__ __forceinline__ void s4x2_f32(uint32_t byte, float &lo, float &hi) {
    const uint32_t u = byte ^ 0x88u;
    const float2 x = __fadd2_rn(make_float2(__uint_as_float(0x4B000000u | (u & 0xFu)),
                                            __uint_as_float(0x4B000000u | ((u >> 4) & 0xFu))),
                                make_float2(-8388616.0f, -8388616.0f));
    lo = x.x;
    hi = x.y;
}
// The eight codes of w's four bytes in element order (byte k: 2k, 2k + 1).
__device__ __forceinline__ void s4x8_f32(uint32_t w, float *f) {
    const uint32_t u = w ^ 0x88888888u;
    const uint32_t lo = u & 0x0F0F0F0Fu, hi = (u >> 4) & 0x0F0F0F0Fu;
#pragma unroll
    for (int k = 0; k < 4; k++) {
        const float2 x = __fadd2_rn(make_float2(__uint_as_float(__byte_perm(lo, 0x4B000000u, 0x7540u + k)),
                                                __uint_as_float(__byte_perm(hi, 0x4B000000u, 0x7540u + k))),
                                    make_float2(-8388616.0f, -8388616.0f));
        f[2 * k] = x.x;
        f[2 * k + 1] = x.y;
    }
}
// The two signed 16-bit halves of w.
__device__ __forceinline__ void s16x2_f32(uint32_t w, float &lo, float &hi) {
    const uint32_t u = w ^ 0x80008000u;
    const float2 x = __fadd2_rn(make_float2(__uint_as_float(__byte_perm(u, 0x4B000000u, 0x7510u)),
                                            __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7532u))),
                                make_float2(-8421376.0f, -8421376.0f));
    lo = x.x;
    hi = x.y;
}

// Rust f32::max: the non-NaN operand when one is NaN (fmaxf semantics).
__device__ __forceinline__ float rmax(float a, float b) { return fmaxf(a, b); }

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Geometry (src/kernels/attention/mod.rs:35-76): the keys [0, end) that the
// query at absolute position `a` sees.
__device__ __forceinline__ int64_t visible_end(int64_t a, int64_t image_start, int64_t image_end) {
    return (a >= image_start && a < image_end) ? image_end : a + 1;
}

// The sink epilogue (src/kernels/attention/online.rs:145-149).
__device__ __forceinline__ float sink_scale(float sink, float lse) { return 1.0f / (1.0f + expf(sink - lse)); }

}  // namespace fo
