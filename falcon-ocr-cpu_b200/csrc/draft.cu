// draft.cu -- the draft head's int8 key/value cache and its attention on the
// device (reference: DraftState's Kv::Q8 and quantize_row,
// src/draft_head.rs:177-220; attend and group_q8, :548-759).
//
// Layout as the reference's: codes [8 groups][capacity][64] int8 and one
// FP32 scale per 64-value row, for keys and for values, so a group's rows
// are contiguous.  A push quantizes one (row, group, key|value) per warp, two
// values per lane.  The attention is one CTA per KV group (two query heads):
// a thread per position computes both heads' scores (int8 codes widened
// exactly, FMA with the query, times key_scale / 8; the FP32 chain rows'
// dots / 8) into a scratch row, the block takes the maxima, exp_poly (the
// reference's vector exp) and the sums, then a warp per position stride
// accumulates p * value_scale * v with a lane per two dimensions, and the
// warps' partial outputs add in warp order before the scale by 1 / sum.
#include "fo_common.cuh"
#include "fo_kernels.h"

namespace fo {

// quantize_row (draft_head.rs:213-220) of a 64-value row held two per lane:
// absmax (NaN-ignoring fold from 0), codes round(v * 127 / max) clamped to
// +-127 (half away from zero; NaN codes 0), scale max / 127.
__device__ __forceinline__ void draft_quantize(float2 x, int8_t *codes, float *scale, int lane) {
    const float m = fmaxf(warp_max(fmaxf(fabsf(x.x), fabsf(x.y))), 0.0f);
    const float inverse = m > 0.0f ? 127.0f / m : 0.0f;
    auto code = [&](float v) -> int8_t {
        const float r = roundf(v * inverse);
        if (isnan(r)) return 0;
        return (int8_t)fminf(fmaxf(r, -127.0f), 127.0f);
    };
    reinterpret_cast<char2 *>(codes)[lane] = make_char2(code(x.x), code(x.y));
    if (lane == 0) *scale = m / 127.0f;
}

// Kv::push (draft_head.rs:194-210) of `rows` positions at index `len`: one
// warp per (row, group, key | value).
__global__ void draft_push_kernel(const float *__restrict__ keys, const float *__restrict__ values, int64_t rows,
                                  int64_t capacity, int64_t len, int8_t *key_codes, float *key_scales,
                                  int8_t *value_codes, float *value_scales) {
    const int64_t w = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (w >= rows * 16) return;
    const int64_t r = w / 16;
    const int g = (int)((w % 16) >> 1);
    const bool value = w & 1;
    const float2 x = reinterpret_cast<const float2 *>((value ? values : keys) + r * FO_DRAFT_KV_WIDTH + g * FO_HD)[lane];
    const int64_t row = g * capacity + len + r;
    draft_quantize(x, (value ? value_codes : key_codes) + row * FO_HD, (value ? value_scales : key_scales) + row,
                   lane);
}

constexpr int DRAFT_THREADS = 256;

// attend + group_q8 for group blockIdx.x over verified rows [start, start + n)
// and `chain` FP32 rows; scores is [8][2][n + chain] scratch.
__global__ void __launch_bounds__(DRAFT_THREADS) draft_attend_kernel(
    const int8_t *__restrict__ key_codes, const float *__restrict__ key_scales, const int8_t *__restrict__ value_codes,
    const float *__restrict__ value_scales, int64_t capacity, const float *__restrict__ q, int64_t start, int64_t n,
    const float *__restrict__ chain_keys, const float *__restrict__ chain_values, int64_t chain, float *scores,
    float *__restrict__ out) {
    constexpr int NW = DRAFT_THREADS / 32;
    const int g = blockIdx.x, t = threadIdx.x, lane = t & 31, warp = t >> 5;
    __shared__ float qs[2][FO_HD];
    __shared__ float red[2][2][NW];
    __shared__ float2 osum[NW][2][FO_HD / 2];
    if (t < 2 * FO_HD) qs[t / FO_HD][t % FO_HD] = q[2 * g * FO_HD + t];  // heads 2g, 2g + 1
    __syncthreads();
    const int64_t total = n + chain;
    float *s0 = scores + (int64_t)g * 2 * total, *s1 = s0 + total;
    // Scores, a thread per position: both heads' dots with one key row.
    float m0 = -INFINITY, m1 = -INFINITY;
    for (int64_t i = t; i < total; i += DRAFT_THREADS) {
        float d0 = 0.0f, d1 = 0.0f;
        if (i < n) {
            const int64_t row = g * capacity + start + i;
            const int4 *kr = reinterpret_cast<const int4 *>(key_codes + row * FO_HD);
#pragma unroll
            for (int c = 0; c < 4; c++) {
                const int4 w = kr[c];
                const uint32_t ws[4] = {(uint32_t)w.x, (uint32_t)w.y, (uint32_t)w.z, (uint32_t)w.w};
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    float f[4];
                    s8x4_f32(ws[j], f);
#pragma unroll
                    for (int b = 0; b < 4; b++) {
                        const int d = 16 * c + 4 * j + b;
                        d0 = fmaf(qs[0][d], f[b], d0);
                        d1 = fmaf(qs[1][d], f[b], d1);
                    }
                }
            }
            const float f = key_scales[row] * 0.125f;  // key_scale * (1 / sqrt(64))
            d0 *= f;
            d1 *= f;
        } else {
            const float4 *k = reinterpret_cast<const float4 *>(chain_keys + (i - n) * FO_DRAFT_KV_WIDTH + g * FO_HD);
#pragma unroll
            for (int c = 0; c < FO_HD / 4; c++) {
                const float4 kv = k[c];
                d0 = fmaf(qs[0][4 * c], kv.x, d0);
                d1 = fmaf(qs[1][4 * c], kv.x, d1);
                d0 = fmaf(qs[0][4 * c + 1], kv.y, d0);
                d1 = fmaf(qs[1][4 * c + 1], kv.y, d1);
                d0 = fmaf(qs[0][4 * c + 2], kv.z, d0);
                d1 = fmaf(qs[1][4 * c + 2], kv.z, d1);
                d0 = fmaf(qs[0][4 * c + 3], kv.w, d0);
                d1 = fmaf(qs[1][4 * c + 3], kv.w, d1);
            }
            d0 *= 0.125f;
            d1 *= 0.125f;
        }
        s0[i] = d0;
        s1[i] = d1;
        m0 = fmaxf(m0, d0);
        m1 = fmaxf(m1, d1);
    }
    m0 = warp_max(m0);
    m1 = warp_max(m1);
    if (lane == 0) {
        red[0][0][warp] = m0;
        red[0][1][warp] = m1;
    }
    __syncthreads();
#pragma unroll
    for (int w = 0; w < NW; w++) {
        m0 = fmaxf(m0, red[0][0][w]);
        m1 = fmaxf(m1, red[0][1][w]);
    }
    // p = exp(s - max) with the reference's vector exp (exp_poly), and sums.
    float l0 = 0.0f, l1 = 0.0f;
    for (int64_t i = t; i < total; i += DRAFT_THREADS) {
        const float e0 = exp_poly(s0[i] - m0), e1 = exp_poly(s1[i] - m1);
        s0[i] = e0;
        s1[i] = e1;
        l0 += e0;
        l1 += e1;
    }
    l0 = warp_sum(l0);
    l1 = warp_sum(l1);
    if (lane == 0) {
        red[1][0][warp] = l0;
        red[1][1][warp] = l1;
    }
    __syncthreads();  // also publishes every thread's probabilities
    float sum0 = 0.0f, sum1 = 0.0f;
#pragma unroll
    for (int w = 0; w < NW; w++) {
        sum0 += red[1][0][w];
        sum1 += red[1][1][w];
    }
    // O = sum_t p_t * value_scale_t * v_t (+ the chain rows' p * v), a lane
    // per two dimensions, a warp per position stride.
    float2 o0 = make_float2(0.0f, 0.0f), o1 = make_float2(0.0f, 0.0f);
    for (int64_t i = warp; i < total; i += NW) {
        float p0 = s0[i], p1 = s1[i];
        float2 v;
        if (i < n) {
            const int64_t row = g * capacity + start + i;
            const float f = value_scales[row];
            p0 *= f;
            p1 *= f;
            const char2 c = reinterpret_cast<const char2 *>(value_codes + row * FO_HD)[lane];
            v = make_float2((float)c.x, (float)c.y);
        } else {
            v = reinterpret_cast<const float2 *>(chain_values + (i - n) * FO_DRAFT_KV_WIDTH + g * FO_HD)[lane];
        }
        o0 = make_float2(fmaf(p0, v.x, o0.x), fmaf(p0, v.y, o0.y));
        o1 = make_float2(fmaf(p1, v.x, o1.x), fmaf(p1, v.y, o1.y));
    }
    osum[warp][0][lane] = o0;
    osum[warp][1][lane] = o1;
    __syncthreads();
    if (t < 2 * FO_HD) {
        const int h = t / FO_HD, d = t % FO_HD;
        const float *po = reinterpret_cast<const float *>(&osum[0][h][0]);
        float o = 0.0f;
#pragma unroll
        for (int w = 0; w < NW; w++) o += po[w * 2 * FO_HD + d];
        out[(2 * g + h) * FO_HD + d] = o * (1.0f / (h ? sum1 : sum0));
    }
}

}  // namespace fo

extern "C" cudaError_t fo_launch_draft_push(const float *keys, const float *values, int64_t rows, int64_t capacity,
                                            int64_t len, int8_t *key_codes, float *key_scales, int8_t *value_codes,
                                            float *value_scales, cudaStream_t stream) {
    if (rows <= 0) return cudaSuccess;
    const int64_t warps = rows * 16;
    const unsigned blocks = (unsigned)((warps * 32 + 255) / 256);
    fo::draft_push_kernel<<<blocks, 256, 0, stream>>>(keys, values, rows, capacity, len, key_codes, key_scales,
                                                      value_codes, value_scales);
    return cudaGetLastError();
}

extern "C" cudaError_t fo_launch_draft_attend(const int8_t *key_codes, const float *key_scales,
                                              const int8_t *value_codes, const float *value_scales, int64_t capacity,
                                              const float *q, int64_t start, int64_t n, const float *chain_keys,
                                              const float *chain_values, int64_t chain, float *scores, float *out,
                                              cudaStream_t stream) {
    fo::draft_attend_kernel<<<8, fo::DRAFT_THREADS, 0, stream>>>(key_codes, key_scales, value_codes, value_scales,
                                                                capacity, q, start, n, chain_keys, chain_values,
                                                                chain, scores, out);
    return cudaGetLastError();
}
