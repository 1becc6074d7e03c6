// decode.cu -- split-KV decode and speculative-verify attention over the
// split cache (reference: SplitPrefix::attention_decode / attention_decode_rows,
// src/quant/kv.rs:565-972; per-group kernels pair / pair_rows,
// src/quant/kv/decode.rs:305-677; merge, src/quant/kv.rs:775-813).
//
// Grid (split, group, page).  A CTA streams the records of one KV group over
// a fixed range of FO_SPLIT positions and serves both heads of the group and
// every verification row, as the reference's pair_rows does: each 128-key
// tile's keys and values are loaded and dequantized once (fl(code * scale),
// decode.rs:151-187) and every row runs over them.  Per row and head it keeps
// the reference's online state (tile max, rescale before PV, exp(s - max)),
// then writes an unnormalized partial; merge_kernel combines the partials of
// each row in position order and applies the sink.  Rows only ever see their
// own positions (row r: prefix + tail - rows + 1 + r, kv.rs:851-855) and the
// split boundaries are absolute, so every verification row equals its
// single-row decode bit for bit.
#include "fo_common.cuh"
#include "fo_kernels.h"

namespace fo {

constexpr int DEC_THREADS = 256;
constexpr int DEC_TILE = 128;  // keys per tile (src/quant/kv.rs:64)
constexpr int L_STRIDE = 132;  // padded logits row (floats) per (row, head)

enum { DF32 = 0, DQ16 = 1, DQ8 = 2, DBF16 = 3 };

// 32 consecutive decoded values of a record block starting at element `e`
// (a multiple of 32): fl(code * bf16 scale) for coded formats.
template <int F>
__device__ __forceinline__ void load_block(const void *codes, const uint16_t *scales, int64_t e, float *out) {
    if constexpr (F == DF32) {
        const float4 *p = reinterpret_cast<const float4 *>(reinterpret_cast<const float *>(codes) + e);
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const float4 x = __ldg(p + i);
            out[4 * i] = x.x;
            out[4 * i + 1] = x.y;
            out[4 * i + 2] = x.z;
            out[4 * i + 3] = x.w;
        }
    } else if constexpr (F == DBF16) {
        const uint4 *p = reinterpret_cast<const uint4 *>(reinterpret_cast<const uint16_t *>(codes) + e);
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const uint4 x = __ldg(p + i);
            const uint32_t w[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
            for (int c = 0; c < 4; c++) {
                out[8 * i + 2 * c] = __uint_as_float(w[c] << 16);
                out[8 * i + 2 * c + 1] = __uint_as_float(w[c] & 0xFFFF0000u);
            }
        }
    } else if constexpr (F == DQ16) {
        const float s = bf16_f32(__ldg(scales + e / 32));
        const uint4 *p = reinterpret_cast<const uint4 *>(reinterpret_cast<const int16_t *>(codes) + e);
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const uint4 x = __ldg(p + i);
            const uint32_t w[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
            for (int c = 0; c < 4; c++) {
                out[8 * i + 2 * c] = __fmul_rn((float)(int16_t)(w[c] & 0xFFFFu), s);
                out[8 * i + 2 * c + 1] = __fmul_rn((float)(int16_t)(w[c] >> 16), s);
            }
        }
    } else {  // DQ8
        const float s = bf16_f32(__ldg(scales + e / 32));
        const uint4 *p = reinterpret_cast<const uint4 *>(reinterpret_cast<const int8_t *>(codes) + e);
#pragma unroll
        for (int i = 0; i < 2; i++) {
            const uint4 x = __ldg(p + i);
            const uint32_t w[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
            for (int c = 0; c < 4; c++)
#pragma unroll
                for (int b = 0; b < 4; b++)
                    out[16 * i + 4 * c + b] = __fmul_rn((float)(int8_t)((w[c] >> (8 * b)) & 0xFFu), s);
        }
    }
}

template <int F, bool FAST>
__global__ void __launch_bounds__(DEC_THREADS) decode_kernel(fo_decode_page page0, const fo_decode_page *pages,
                                                             int64_t groups) {
    __shared__ __align__(16) float q_s[FO_MAX_ROWS][2][FO_HD];
    __shared__ __align__(16) float l_s[FO_MAX_ROWS * 2][L_STRIDE];
    __shared__ __align__(16) float v_s[DEC_TILE][FO_HD];
    __shared__ float m_st[FO_MAX_ROWS * 2], d_st[FO_MAX_ROWS * 2], a_st[FO_MAX_ROWS * 2];

    const fo_decode_page pg = pages ? pages[blockIdx.z] : page0;
    const int s = blockIdx.x;
    if (s >= pg.splits) return;
    const int64_t g = blockIdx.y;
    const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
    const int R = pg.rows;
    const int64_t H = 2 * groups;
    const int64_t p0 = (int64_t)s * FO_SPLIT;
    const int64_t p_end = min64(p0 + FO_SPLIT, pg.last);

    for (int i = t; i < R * 2 * FO_HD; i += DEC_THREADS) {
        const int r = i / (2 * FO_HD), h = (i / FO_HD) & 1, d = i % FO_HD;
        q_s[r][h][d] = pg.q[(r * H + 2 * g + h) * FO_HD + d];
    }
    if (t < 2 * R) {
        m_st[t] = -INFINITY;
        d_st[t] = 0.0f;
    }
    // PV ownership: warp = row, lane -> (head, 4 dimensions).
    const int pv_h = lane >> 4, pv_d = (lane & 15) * 4;
    float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};

    for (int64_t k0 = p0; k0 < p_end; k0 += DEC_TILE) {
        const int tile_len = (int)min64(DEC_TILE, p_end - k0);
        __syncthreads();
        // Values of the tile, dequantized once: thread -> (key, half).
        {
            const int j = t >> 1, half = t & 1;
            if (j < tile_len) {
                const int64_t pos = k0 + j;
                float vals[32];
                if (pos < pg.prefix_len)
                    load_block<F>(pg.codes, pg.scales, (g * pg.prefix_stride + pos) * FO_RECORD + 96 + 32 * half, vals);
                else
                    load_block<F>(pg.tail_codes, pg.tail_scales,
                                  (g * pg.tail_stride + (pos - pg.prefix_len)) * FO_TAIL_RECORD + 64 + 32 * half, vals);
#pragma unroll
                for (int c0 = 0; c0 < 8; c0++) {
                    const int c = (c0 + lane) & 7;  // rotate 16-byte slots: conflict-free stores
                    float4 x;
                    x.x = vals[4 * c];
                    x.y = vals[4 * c + 1];
                    x.z = vals[4 * c + 2];
                    x.w = vals[4 * c + 3];
                    *reinterpret_cast<float4 *>(&v_s[j][32 * half + 4 * c]) = x;
                }
            }
        }
        // Logits: thread -> (key, head); both halves of the head's key.
        {
            const int j = t & (DEC_TILE - 1), h = t >> 7;
            if (j < tile_len) {
                const int64_t pos = k0 + j;
                float key[FO_HD];
                if (pos < pg.prefix_len) {
                    const int64_t e = (g * pg.prefix_stride + pos) * FO_RECORD;
                    load_block<F>(pg.codes, pg.scales, e, key);                   // T
                    load_block<F>(pg.codes, pg.scales, e + 32 + 32 * h, key + 32);  // S(2g+h)
                } else {
                    const int64_t e = (g * pg.tail_stride + (pos - pg.prefix_len)) * FO_TAIL_RECORD;
                    load_block<F>(pg.tail_codes, pg.tail_scales, e, key);
                    load_block<F>(pg.tail_codes, pg.tail_scales, e + 32, key + 32);
                }
                for (int r = 0; r < R; r++) {
                    float d0 = 0.f, d1 = 0.f, d2 = 0.f, d3 = 0.f;
#pragma unroll
                    for (int d = 0; d < FO_HD; d += 4) {
                        const float4 qv = *reinterpret_cast<const float4 *>(&q_s[r][h][d]);
                        d0 = fmaf(qv.x, key[d], d0);
                        d1 = fmaf(qv.y, key[d + 1], d1);
                        d2 = fmaf(qv.z, key[d + 2], d2);
                        d3 = fmaf(qv.w, key[d + 3], d3);
                    }
                    l_s[r * 2 + h][j] = ((d0 + d1) + (d2 + d3)) * 0.125f;
                }
            }
        }
        __syncthreads();
        // Online softmax per (row, head): warp per pair.
        for (int pi = warp; pi < 2 * R; pi += DEC_THREADS / 32) {
            const int r = pi >> 1;
            const int64_t row_len = pg.last - R + 1 + r;
            const int len = (int)max64(0, min64(tile_len, row_len - k0));
            if (len == 0) {
                if (lane == 0) a_st[pi] = 1.0f;
                continue;
            }
            float x[DEC_TILE / 32];
            float bm = -INFINITY;
#pragma unroll
            for (int i = 0; i < DEC_TILE / 32; i++) {
                const int j = lane + 32 * i;
                x[i] = j < len ? l_s[pi][j] : -INFINITY;
                bm = rmax(bm, x[i]);
            }
            bm = warp_max(bm);
            const float m_old = m_st[pi];
            const float m_new = rmax(m_old, bm);
            const float alpha = m_old == -INFINITY ? 0.0f : expf(m_old - m_new);
            float psum = 0.0f;
#pragma unroll
            for (int i = 0; i < DEC_TILE / 32; i++) {
                const int j = lane + 32 * i;
                const float p = j < len ? softmax_exp<FAST>(x[i] - m_new) : 0.0f;
                l_s[pi][j] = p;
                psum += p;
            }
            psum = warp_sum(psum);
            if (lane == 0) {
                a_st[pi] = alpha;
                m_st[pi] = m_new;
                d_st[pi] = d_st[pi] * alpha + psum;
            }
        }
        __syncthreads();
        // O += P V for this warp's row.
        if (warp < R) {
            const int r = warp, pi = 2 * r + pv_h;
            const int64_t row_len = pg.last - R + 1 + r;
            const int len = (int)max64(0, min64(tile_len, row_len - k0));
            if (len > 0) {
                const float alpha = a_st[pi];
#pragma unroll
                for (int c = 0; c < 4; c++) acc[c] *= alpha;
                for (int j = 0; j < len; j++) {
                    const float p = l_s[pi][j];
                    const float4 v = *reinterpret_cast<const float4 *>(&v_s[j][pv_d]);
                    acc[0] = fmaf(p, v.x, acc[0]);
                    acc[1] = fmaf(p, v.y, acc[1]);
                    acc[2] = fmaf(p, v.z, acc[2]);
                    acc[3] = fmaf(p, v.w, acc[3]);
                }
            }
        }
    }
    __syncthreads();
    if (warp < R) {
        const int64_t row_head = (int64_t)warp * H + 2 * g + pv_h;
        *reinterpret_cast<float4 *>(pg.part_o + (row_head * pg.splits + s) * FO_HD + pv_d) =
            make_float4(acc[0], acc[1], acc[2], acc[3]);
    }
    if (t < 2 * R) {
        const int64_t row_head = (int64_t)(t >> 1) * H + 2 * g + (t & 1);
        pg.part_ml[(row_head * pg.splits + s) * 2] = m_st[t];
        pg.part_ml[(row_head * pg.splits + s) * 2 + 1] = d_st[t];
    }
}

// Merge the position splits of every (row, head) in order, then the sink
// (src/quant/kv.rs:775-813).  One warp per (row, head), two dims per lane.
__global__ void merge_kernel(fo_decode_page page0, const fo_decode_page *pages, int64_t heads) {
    const fo_decode_page pg = pages ? pages[blockIdx.y] : page0;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t rh = (int64_t)blockIdx.x * (blockDim.x >> 5) + warp;
    if (rh >= (int64_t)pg.rows * heads) return;
    const int64_t r = rh / heads, h = rh % heads;
    const int64_t row_len = pg.last - pg.rows + 1 + r;
    const int n = (int)((row_len + FO_SPLIT - 1) / FO_SPLIT);
    const float *po = pg.part_o + rh * pg.splits * FO_HD;
    const float *pml = pg.part_ml + rh * pg.splits * 2;
    float m, den, o0, o1;
    if (n == 1) {  // a single scan: its state as is
        m = pml[0];
        den = pml[1];
        o0 = po[lane];
        o1 = po[32 + lane];
    } else {
        m = -INFINITY;
        for (int s = 0; s < n; s++) m = rmax(m, pml[2 * s]);
        den = 0.0f;
        o0 = 0.0f;
        o1 = 0.0f;
        for (int s = 0; s < n; s++) {
            const float pm = pml[2 * s];
            if (pm == -INFINITY) continue;
            const float f = expf(pm - m);
            den = fmaf(pml[2 * s + 1], f, den);
            o0 = fmaf(po[s * FO_HD + lane], f, o0);
            o1 = fmaf(po[s * FO_HD + 32 + lane], f, o1);
        }
    }
    const float lse = m + logf(den);
    const float ss = sink_scale(pg.sinks[h], lse);
    float *out = pg.out + rh * FO_HD;
    out[lane] = (o0 / den) * ss;
    out[32 + lane] = (o1 / den) * ss;
}

}  // namespace fo

static cudaError_t launch_decode(const fo_decode_page &page0, const fo_decode_page *dev_pages, int64_t n_pages,
                                 int format, int64_t groups, int fast_exp, int64_t max_splits, int max_rows,
                                 cudaStream_t stream) {
    if (n_pages <= 0 || max_splits <= 0) return cudaSuccess;
    dim3 grid((unsigned)max_splits, (unsigned)groups, (unsigned)n_pages);
#define FO_DECODE_CASE(F)                                                                              \
    case F:                                                                                            \
        if (fast_exp)                                                                                  \
            fo::decode_kernel<F, true><<<grid, fo::DEC_THREADS, 0, stream>>>(page0, dev_pages, groups); \
        else                                                                                           \
            fo::decode_kernel<F, false><<<grid, fo::DEC_THREADS, 0, stream>>>(page0, dev_pages, groups); \
        break;
    switch (format) {
        FO_DECODE_CASE(fo::DF32)
        FO_DECODE_CASE(fo::DQ16)
        FO_DECODE_CASE(fo::DQ8)
        FO_DECODE_CASE(fo::DBF16)
    default:
        return cudaErrorInvalidValue;
    }
#undef FO_DECODE_CASE
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    const int64_t heads = 2 * groups;
    const int warps_per_block = 4;
    dim3 mgrid((unsigned)((max_rows * heads + warps_per_block - 1) / warps_per_block), (unsigned)n_pages);
    fo::merge_kernel<<<mgrid, warps_per_block * 32, 0, stream>>>(page0, dev_pages, heads);
    return cudaGetLastError();
}

extern "C" cudaError_t fo_launch_decode_one(const fo_decode_page *page, int format, int64_t groups, int fast_exp,
                                            cudaStream_t stream) {
    return launch_decode(*page, nullptr, 1, format, groups, fast_exp, page->splits, page->rows, stream);
}

extern "C" cudaError_t fo_launch_decode_batch(const fo_decode_page *dev_pages, int64_t n_pages, int format,
                                              int64_t groups, int fast_exp, int64_t max_splits, int max_rows,
                                              cudaStream_t stream) {
    fo_decode_page none{};
    return launch_decode(none, dev_pages, n_pages, format, groups, fast_exp, max_splits, max_rows, stream);
}
