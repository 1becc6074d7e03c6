// draft.cu -- the draft head's int8 key/value cache and its attention on the
// device (reference: DraftState's Kv::Q8 and quantize_row,
// src/draft_head.rs:177-220; attend and group_q8, :548-759).
//
// Layout as the reference's: codes [8 groups][capacity][64] int8 and one
// FP32 scale per 64-value row, for keys and for values, so a group's rows
// are contiguous.  A push quantizes one (row, group, key|value) per warp, two
// values per lane.  The attention is one CTA per KV group (two query heads):
// split over the positions: each CTA of a group streams its range in
// sub-chunks of 128 positions (a thread per position for both heads' scores:
// int8 codes widened exactly, FMA with the query, times key_scale / 8; the
// FP32 chain rows' dots / 8), keeps a running maximum (the reference takes
// one maximum over all scores; the rescaling differs from it by rounding
// only), p = exp_poly (the reference's vector exp), and accumulates
// p * value_scale * v with a warp per position and a lane per two dimensions;
// the last CTA of the group merges the partials in order and scales by 1 / sum.
#include "fo_common.cuh"
#include "fo_kernels.h"

#include <algorithm>

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

constexpr int DRAFT_THREADS = 128;  // four warps; a thread per position of a sub-chunk
constexpr int DRAFT_SUB = 128;      // positions per sub-chunk

// Both heads' dots with one int8 key row (64 codes, widened exactly).
__device__ __forceinline__ void draft_dot_i8(const int4 *kr, const float (*qs)[FO_HD], float &d0, float &d1) {
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
}

// Both heads' dots with one FP32 chain key (64 values).
__device__ __forceinline__ void draft_dot_f32(const float *row, const float (*qs)[FO_HD], float &d0, float &d1) {
    const float4 *k = reinterpret_cast<const float4 *>(row);
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
}

// Block reductions over the four warps (max or sum), both heads at once.
__device__ __forceinline__ float2 draft_block_max(float2 v, float2 *red, int lane, int warp) {
    v = make_float2(warp_max(v.x), warp_max(v.y));
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float2 r = red[0];
#pragma unroll
    for (int w = 1; w < DRAFT_THREADS / 32; w++) r = make_float2(fmaxf(r.x, red[w].x), fmaxf(r.y, red[w].y));
    __syncthreads();
    return r;
}
__device__ __forceinline__ float2 draft_block_sum(float2 v, float2 *red, int lane, int warp) {
    v = make_float2(warp_sum(v.x), warp_sum(v.y));
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float2 r = red[0];
#pragma unroll
    for (int w = 1; w < DRAFT_THREADS / 32; w++) r = make_float2(r.x + red[w].x, r.y + red[w].y);
    __syncthreads();
    return r;
}

// attend + group_q8 for group blockIdx.y: CTA blockIdx.x of gridDim.x takes
// positions [x * per, (x + 1) * per) of the group's n verified rows
// [start, start + n) followed by its `chain` FP32 rows, in sub-chunks of
// DRAFT_SUB (scores, running maximum with the rescale of the running sum and
// output, p = exp_poly(s - max), O += p * value_scale * v), and writes its
// partial (max, sum, output) of both heads.  The last CTA of the group to
// finish (a counter per group, reset by that CTA) combines the partials in
// CTA order: M = max of the maxima, each partial scaled by exp(m - M), and
// out = O * (1 / sum).
__global__ void __launch_bounds__(DRAFT_THREADS) draft_attend_kernel(
    const int8_t *__restrict__ key_codes, const float *__restrict__ key_scales, const int8_t *__restrict__ value_codes,
    const float *__restrict__ value_scales, int64_t capacity, const float *__restrict__ q, int64_t start, int64_t n,
    const float *__restrict__ chain_keys, const float *__restrict__ chain_values, int64_t chain, int64_t per,
    float *__restrict__ part, unsigned *__restrict__ counters, float *__restrict__ out) {
    constexpr int NW = DRAFT_THREADS / 32;
    const int g = blockIdx.y, x = blockIdx.x, t = threadIdx.x, lane = t & 31, warp = t >> 5;
    __shared__ float qs[2][FO_HD];
    __shared__ float2 sc[DRAFT_SUB];  // this sub-chunk's (head 0, head 1) scores, then probabilities
    __shared__ __align__(16) int8_t vsm[DRAFT_SUB][FO_HD];  // its verified value rows
    __shared__ float vsc[DRAFT_SUB];                        // and their scales
    __shared__ float2 red[NW];
    __shared__ float2 osum[NW][2][FO_HD / 2];
    __shared__ bool last;
    __shared__ float2 mf[FO_DRAFT_MAX_SPLITS][2];  // merge: per partial (max, sum), then (factor, sum)
    // The query goes to shared memory while the first sub-chunk's rows load.
    if (t < 2 * FO_HD) qs[t / FO_HD][t % FO_HD] = q[2 * g * FO_HD + t];  // heads 2g, 2g + 1
    const int64_t total = n + chain, rowbase = g * capacity + start;
    const int64_t a = (int64_t)x * per, b = min64(a + per, total);
    float2 m = make_float2(-INFINITY, -INFINITY), l = make_float2(0.0f, 0.0f);
    float2 o0 = make_float2(0.0f, 0.0f), o1 = make_float2(0.0f, 0.0f);  // this warp's, dims 2 lane, 2 lane + 1
    for (int64_t c0 = a; c0 < b; c0 += DRAFT_SUB) {
        const int cn = (int)min64(DRAFT_SUB, b - c0);
        const int64_t i = c0 + t;
        const bool verified = t < cn && i < n, chained = t < cn && i >= n;
        // The position's key and value rows and scales are read together, so
        // they arrive within one memory latency (and, for the first
        // sub-chunk, while the query is still on its way to shared memory).
        int4 krow[4], vrow[4];
        float kscale = 0.0f, vscale = 0.0f;
        if (verified) {
            const int4 *kr = reinterpret_cast<const int4 *>(key_codes + (rowbase + i) * FO_HD);
            const int4 *vr = reinterpret_cast<const int4 *>(value_codes + (rowbase + i) * FO_HD);
#pragma unroll
            for (int c = 0; c < 4; c++) {
                krow[c] = kr[c];
                vrow[c] = vr[c];
            }
            kscale = key_scales[rowbase + i];
            vscale = value_scales[rowbase + i];
        }
        if (c0 == a) __syncthreads();  // every thread: the query is in shared memory
        float2 s = make_float2(-INFINITY, -INFINITY);
        if (verified) {
            float d0 = 0.0f, d1 = 0.0f;
            draft_dot_i8(krow, qs, d0, d1);
            const float f = kscale * 0.125f;  // key_scale * (1 / sqrt(64))
            s = make_float2(d0 * f, d1 * f);
#pragma unroll
            for (int c = 0; c < 4; c++) reinterpret_cast<int4 *>(vsm[t])[c] = vrow[c];
            vsc[t] = vscale;
        } else if (chained) {
            float d0 = 0.0f, d1 = 0.0f;
            draft_dot_f32(chain_keys + (i - n) * FO_DRAFT_KV_WIDTH + g * FO_HD, qs, d0, d1);
            s = make_float2(d0 * 0.125f, d1 * 0.125f);
        }
        const float2 cm = draft_block_max(s, red, lane, warp);
        const float2 mn = make_float2(fmaxf(m.x, cm.x), fmaxf(m.y, cm.y));
        const float2 alpha = make_float2(m.x == -INFINITY ? 0.0f : exp_poly(m.x - mn.x),
                                         m.y == -INFINITY ? 0.0f : exp_poly(m.y - mn.y));
        m = mn;
        float2 p = make_float2(0.0f, 0.0f);
        if (t < cn) p = make_float2(exp_poly(s.x - m.x), exp_poly(s.y - m.y));
        sc[t] = p;
        const float2 ls = draft_block_sum(p, red, lane, warp);  // its barrier publishes sc
        l = make_float2(__fmaf_rn(l.x, alpha.x, ls.x), __fmaf_rn(l.y, alpha.y, ls.y));
        o0 = make_float2(o0.x * alpha.x, o0.y * alpha.x);
        o1 = make_float2(o1.x * alpha.y, o1.y * alpha.y);
        // O += p * v: warp w takes positions w, w + 4, ... of the sub-chunk.
#pragma unroll 8
        for (int j = warp; j < cn; j += NW) {
            const int64_t i = c0 + j;
            float2 pj = sc[j];
            float2 v;
            if (i < n) {
                const float f = vsc[j];
                pj = make_float2(pj.x * f, pj.y * f);
                const char2 c = reinterpret_cast<const char2 *>(vsm[j])[lane];
                v = make_float2((float)c.x, (float)c.y);
            } else {
                v = reinterpret_cast<const float2 *>(chain_values + (i - n) * FO_DRAFT_KV_WIDTH + g * FO_HD)[lane];
            }
            o0 = make_float2(fmaf(pj.x, v.x, o0.x), fmaf(pj.x, v.y, o0.y));
            o1 = make_float2(fmaf(pj.y, v.x, o1.x), fmaf(pj.y, v.y, o1.y));
        }
        __syncthreads();  // sc, vsm and vsc are rewritten by the next sub-chunk
    }
    osum[warp][0][lane] = o0;
    osum[warp][1][lane] = o1;
    __syncthreads();
    // This CTA's partial: [2 heads][64 + 2] = output, max, sum.
    float *mine = part + ((int64_t)g * gridDim.x + x) * 2 * (FO_HD + 2);
    if (t < 2 * FO_HD) {
        const int h = t / FO_HD, d = t % FO_HD;
        const float *po = reinterpret_cast<const float *>(&osum[0][h][0]);
        float acc = 0.0f;
#pragma unroll
        for (int w = 0; w < NW; w++) acc += po[w * 2 * FO_HD + d];
        mine[h * (FO_HD + 2) + d] = acc;
        if (d == 0) {
            mine[h * (FO_HD + 2) + FO_HD] = h ? m.y : m.x;
            mine[h * (FO_HD + 2) + FO_HD + 1] = h ? l.y : l.x;
        }
    }
    __threadfence();
    __syncthreads();
    if (t == 0) {
        const unsigned done = atomicAdd(&counters[g], 1u);
        last = done == gridDim.x - 1;
        if (last) counters[g] = 0;  // ready for the next call
    }
    __syncthreads();
    if (!last) return;
    __threadfence();
    // The merge, in CTA order.  Every partial's (max, sum) of both heads is
    // loaded at once; then thread (h, d) takes the maximum and sums the
    // scaled partial outputs, their loads in flight together.
    const int nc = (int)gridDim.x;
    const float *gp = part + (int64_t)g * nc * 2 * (FO_HD + 2);
    if (t < 2 * nc) {
        const float *pc = gp + (t >> 1) * 2 * (FO_HD + 2) + (t & 1) * (FO_HD + 2);
        mf[t >> 1][t & 1] = make_float2(__ldcg(pc + FO_HD), __ldcg(pc + FO_HD + 1));
    }
    __syncthreads();
    if (t < 2 * FO_HD) {
        const int h = t / FO_HD, d = t % FO_HD;
        float M = -INFINITY;
        for (int c = 0; c < nc; c++) M = fmaxf(M, mf[c][h].x);
        float acc = 0.0f, sum = 0.0f;
#pragma unroll 8
        for (int c = 0; c < nc; c++) {
            const float2 ml = mf[c][h];
            const float o = __ldcg(gp + c * 2 * (FO_HD + 2) + h * (FO_HD + 2) + d);
            if (ml.x == -INFINITY) continue;  // a CTA with no position
            const float f = exp_poly(ml.x - M);
            sum = __fmaf_rn(ml.y, f, sum);
            acc = __fmaf_rn(o, f, acc);
        }
        out[(2 * g + h) * FO_HD + d] = acc * (1.0f / sum);
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
                                              const float *chain_values, int64_t chain, float *part,
                                              unsigned *counters, float *out, cudaStream_t stream) {
    // Positions per CTA: a multiple of the sub-chunk, at most FO_DRAFT_MAX_SPLITS CTAs per group.
    const int64_t total = n + chain;
    const int64_t subs = (total + fo::DRAFT_SUB - 1) / fo::DRAFT_SUB;
    const int64_t splits = std::min<int64_t>(subs, FO_DRAFT_MAX_SPLITS);
    const int64_t per = ((subs + splits - 1) / splits) * fo::DRAFT_SUB;
    const int64_t grid = (total + per - 1) / per;
    fo::draft_attend_kernel<<<dim3((unsigned)grid, 8), fo::DRAFT_THREADS, 0, stream>>>(
        key_codes, key_scales, value_codes, value_scales, capacity, q, start, n, chain_keys, chain_values, chain, per,
        part, counters, out);
    return cudaGetLastError();
}
