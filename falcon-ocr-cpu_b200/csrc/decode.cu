// decode.cu -- split-KV decode and speculative-verify attention over the
// split cache (reference: SplitPrefix::attention_decode / attention_decode_rows,
// src/quant/kv.rs:565-972; per-group kernels pair / pair_rows,
// src/quant/kv/decode.rs:305-677; merge, src/quant/kv.rs:775-813).
//
// Grid (split, group, page).  A CTA covers FO_SPLIT positions of one KV
// group and serves both heads of the group and every verification row, as the
// reference's pair_rows does: each record is loaded and dequantized once
// (fl(code * scale), decode.rs:151-187) and every row runs over it.  Each of
// its eight warps streams its own 32-key chunks with no block-wide barrier
// (lane = key for the loads and logits, lane = two output dimensions for PV)
// and keeps the reference's online state per row and head (chunk max,
// rescale before PV, exp(s - max)).  The warps then combine, in warp order,
// into the split's unnormalized partial.  The last CTA of a group to finish
// (an atomic counter per group, no waiting) merges the splits of every row in
// position order with the reference's merge arithmetic and applies the sink;
// it resets the counter for the next call.  Rows only see their own positions
// (row r: prefix + tail - rows + 1 + r, kv.rs:851-855) and split boundaries
// are absolute, so every verification row equals its single-row decode bit
// for bit.
#include "fo_common.cuh"
#include "fo_kernels.h"

namespace fo {

constexpr int DEC_WARPS = 8;
constexpr int DEC_THREADS = 32 * DEC_WARPS;
constexpr int CHUNK = 32;                                        // keys per warp step (one per lane)
constexpr int CHUNKS_PER_WARP = FO_SPLIT / (CHUNK * DEC_WARPS);  // a split is DEC_WARPS x this many chunks
constexpr int V_LD = FO_HD + 4;                                  // padded value row (floats)
// Dynamic shared memory: q [8][2][64], per-warp values [32][V_LD] (reused for
// the warps' outputs [2 * 8][64]), per-warp probabilities [16][32], per-warp
// max and sum [16] each.
constexpr int SM_Q = FO_MAX_ROWS * 2 * FO_HD;
constexpr int SM_V = DEC_WARPS * CHUNK * V_LD;
constexpr int SM_P = DEC_WARPS * 2 * FO_MAX_ROWS * CHUNK;
constexpr int SM_ML = DEC_WARPS * 2 * FO_MAX_ROWS;
constexpr size_t DEC_SMEM = sizeof(float) * (SM_Q + SM_V + SM_P + 2 * SM_ML) + 16;
static_assert(DEC_WARPS * 2 * FO_MAX_ROWS * FO_HD <= SM_V, "warp outputs fit the value buffers");

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

template <int F, bool FAST, int R>
__global__ void __launch_bounds__(DEC_THREADS, 2) decode_kernel(fo_decode_page page0, const fo_decode_page *pages,
                                                                int64_t groups) {
    extern __shared__ __align__(16) float dsm[];
    float(*q_s)[2][FO_HD] = reinterpret_cast<float(*)[2][FO_HD]>(dsm);
    float *v_base = dsm + SM_Q;
    float *p_base = v_base + SM_V;
    float *m_base = p_base + SM_P;
    float *l_base = m_base + SM_ML;
    int *last_flag = reinterpret_cast<int *>(l_base + SM_ML);

    const fo_decode_page pg = pages ? pages[blockIdx.z] : page0;
    const int s = blockIdx.x;
    if (s >= pg.splits) return;
    const int64_t g = blockIdx.y;
    const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
    const int64_t H = 2 * groups;
    const int64_t p0 = (int64_t)s * FO_SPLIT;
    const int64_t p_end = min64(p0 + FO_SPLIT, pg.last);

    for (int i = t; i < R * 2 * FO_HD; i += DEC_THREADS) {
        const int r = i / (2 * FO_HD), h = (i / FO_HD) & 1, d = i % FO_HD;
        q_s[r][h][d] = pg.q[(r * H + 2 * g + h) * FO_HD + d];
    }
    // Per (row, head): the online state (warp-uniform, in shared memory) and
    // this lane's two output dimensions 2*lane, 2*lane + 1 (registers).
    float *mr = m_base + warp * 2 * FO_MAX_ROWS, *lr = l_base + warp * 2 * FO_MAX_ROWS;
    if (lane < 2 * R) {
        mr[lane] = -INFINITY;
        lr[lane] = 0.0f;
    }
    __syncthreads();
    float o0[2 * R], o1[2 * R];
#pragma unroll
    for (int rh = 0; rh < 2 * R; rh++) {
        o0[rh] = 0.0f;
        o1[rh] = 0.0f;
    }
    float(*vw)[V_LD] = reinterpret_cast<float(*)[V_LD]>(v_base + warp * CHUNK * V_LD);
    float(*pw)[CHUNK] = reinterpret_cast<float(*)[CHUNK]>(p_base + warp * 2 * FO_MAX_ROWS * CHUNK);
    for (int c = 0; c < CHUNKS_PER_WARP; c++) {
        const int64_t k0 = p0 + (int64_t)(warp * CHUNKS_PER_WARP + c) * CHUNK;
        if (k0 >= p_end) break;  // warp-uniform
        const int64_t pos = k0 + lane;
        const bool live = pos < p_end;
        const bool prefix = pos < pg.prefix_len;
        const int64_t rec = prefix ? (g * pg.prefix_stride + pos) * FO_RECORD
                                   : (g * pg.tail_stride + (pos - pg.prefix_len)) * FO_TAIL_RECORD;
        const void *codes = prefix ? pg.codes : pg.tail_codes;
        const uint16_t *scales = prefix ? pg.scales : pg.tail_scales;
        // This lane's value row, dequantized once for every row and head.
        {
            float vals[32];
#pragma unroll
            for (int half = 0; half < 2; half++) {
                if (live)
                    load_block<F>(codes, scales, rec + (prefix ? 96 : 64) + 32 * half, vals);
                else
#pragma unroll
                    for (int i = 0; i < 32; i++) vals[i] = 0.0f;
#pragma unroll
                for (int i = 0; i < 8; i++)
                    *reinterpret_cast<float4 *>(&vw[lane][32 * half + 4 * i]) =
                        make_float4(vals[4 * i], vals[4 * i + 1], vals[4 * i + 2], vals[4 * i + 3]);
            }
        }
        // Logits of every (row, head): the shared temporal half once for both
        // heads, then each head's spatial half (a tail record has one key for
        // both heads).
        float lg[2 * R];
        {
            float key[32];
            if (live)
                load_block<F>(codes, scales, rec, key);
            else
#pragma unroll
                for (int i = 0; i < 32; i++) key[i] = 0.0f;
#pragma unroll
            for (int rh = 0; rh < 2 * R; rh++) {
                const float *qv = q_s[rh >> 1][rh & 1];
                float d0 = 0.f, d1 = 0.f, d2 = 0.f, d3 = 0.f;
#pragma unroll
                for (int d = 0; d < 32; d += 4) {
                    const float4 x = *reinterpret_cast<const float4 *>(qv + d);
                    d0 = fmaf(x.x, key[d], d0);
                    d1 = fmaf(x.y, key[d + 1], d1);
                    d2 = fmaf(x.z, key[d + 2], d2);
                    d3 = fmaf(x.w, key[d + 3], d3);
                }
                lg[rh] = (d0 + d1) + (d2 + d3);
            }
#pragma unroll
            for (int h = 0; h < 2; h++) {
                if (live) load_block<F>(codes, scales, rec + (prefix ? 32 + 32 * h : 32), key);
#pragma unroll
                for (int r = 0; r < R; r++) {
                    const float *qv = q_s[r][h] + 32;
                    float d0 = 0.f, d1 = 0.f, d2 = 0.f, d3 = 0.f;
#pragma unroll
                    for (int d = 0; d < 32; d += 4) {
                        const float4 x = *reinterpret_cast<const float4 *>(qv + d);
                        d0 = fmaf(x.x, key[d], d0);
                        d1 = fmaf(x.y, key[d + 1], d1);
                        d2 = fmaf(x.z, key[d + 2], d2);
                        d3 = fmaf(x.w, key[d + 3], d3);
                    }
                    lg[2 * r + h] = (lg[2 * r + h] + ((d0 + d1) + (d2 + d3))) * 0.125f;
                }
            }
        }
        // Online softmax of the chunk per (row, head).
#pragma unroll
        for (int rh = 0; rh < 2 * R; rh++) {
            const int64_t row_len = pg.last - R + 1 + (rh >> 1);
            const bool valid = pos < row_len;
            const float x = valid ? lg[rh] : -INFINITY;
            const float bm = warp_max(x);
            if (bm == -INFINITY) {  // no position of this row in the chunk (warp-uniform)
                pw[rh][lane] = 0.0f;
                continue;
            }
            const float m_old = mr[rh];
            const float m_new = rmax(m_old, bm);
            const float alpha = m_old == -INFINITY ? 0.0f : expf(m_old - m_new);
            const float p = valid ? softmax_exp<FAST>(x - m_new) : 0.0f;
            pw[rh][lane] = p;
            const float l_new = lr[rh] * alpha + warp_sum(p);
            __syncwarp();
            if (lane == 0) {
                lr[rh] = l_new;
                mr[rh] = m_new;
            }
            o0[rh] *= alpha;
            o1[rh] *= alpha;
        }
        __syncwarp();
        // O += P V in key order; this lane's two dimensions.
#pragma unroll
        for (int j4 = 0; j4 < CHUNK / 4; j4++) {
            float2 v[4];
#pragma unroll
            for (int jj = 0; jj < 4; jj++) v[jj] = *reinterpret_cast<const float2 *>(&vw[4 * j4 + jj][2 * lane]);
#pragma unroll
            for (int rh = 0; rh < 2 * R; rh++) {
                const float4 p = *reinterpret_cast<const float4 *>(&pw[rh][4 * j4]);
                o0[rh] = fmaf(p.x, v[0].x, o0[rh]);
                o1[rh] = fmaf(p.x, v[0].y, o1[rh]);
                o0[rh] = fmaf(p.y, v[1].x, o0[rh]);
                o1[rh] = fmaf(p.y, v[1].y, o1[rh]);
                o0[rh] = fmaf(p.z, v[2].x, o0[rh]);
                o1[rh] = fmaf(p.z, v[2].y, o1[rh]);
                o0[rh] = fmaf(p.w, v[3].x, o0[rh]);
                o1[rh] = fmaf(p.w, v[3].y, o1[rh]);
            }
        }
        __syncwarp();
    }
    // Combine the warps in warp order (kv.rs:775-813 arithmetic) into this
    // split's partial.
    float *ow = v_base;  // [DEC_WARPS][2 * FO_MAX_ROWS][FO_HD]
    __syncthreads();
#pragma unroll
    for (int rh = 0; rh < 2 * R; rh++)
        *reinterpret_cast<float2 *>(&ow[(warp * 2 * FO_MAX_ROWS + rh) * FO_HD + 2 * lane]) = make_float2(o0[rh], o1[rh]);
    __syncthreads();
    for (int e = t; e < 2 * R * FO_HD; e += DEC_THREADS) {
        const int rh = e / FO_HD, d = e % FO_HD;
        float m = -INFINITY;
#pragma unroll
        for (int w = 0; w < DEC_WARPS; w++) m = rmax(m, m_base[w * 2 * FO_MAX_ROWS + rh]);
        float den = 0.0f, acc = 0.0f;
        if (m != -INFINITY) {
#pragma unroll
            for (int w = 0; w < DEC_WARPS; w++) {
                const float mw = m_base[w * 2 * FO_MAX_ROWS + rh];
                if (mw == -INFINITY) continue;
                const float f = expf(mw - m);
                den = fmaf(l_base[w * 2 * FO_MAX_ROWS + rh], f, den);
                acc = fmaf(ow[(w * 2 * FO_MAX_ROWS + rh) * FO_HD + d], f, acc);
            }
        }
        const int64_t row_head = (int64_t)(rh >> 1) * H + 2 * g + (rh & 1);
        pg.part_o[(row_head * pg.splits + s) * FO_HD + d] = acc;
        if (d == 0) {
            pg.part_ml[(row_head * pg.splits + s) * 2] = m;
            pg.part_ml[(row_head * pg.splits + s) * 2 + 1] = den;
        }
    }
    // The group's last split to finish merges (threadfence reduction: no
    // CTA ever waits for another).
    __threadfence();
    __syncthreads();
    if (t == 0) *last_flag = atomicAdd(pg.counters + g, 1u) == (unsigned)(pg.splits - 1);
    __syncthreads();
    if (!*last_flag) return;
    __threadfence();
    for (int e = t; e < 2 * R * FO_HD; e += DEC_THREADS) {
        const int rh = e / FO_HD, d = e % FO_HD;
        const int64_t r = rh >> 1, h = 2 * g + (rh & 1);
        const int64_t row_head = r * H + h;
        const int64_t row_len = pg.last - R + 1 + r;
        const int n = (int)((row_len + FO_SPLIT - 1) / FO_SPLIT);
        const float *po = pg.part_o + row_head * pg.splits * FO_HD;
        const float *pml = pg.part_ml + row_head * pg.splits * 2;
        float m = -INFINITY;
        for (int k = 0; k < n; k++) m = rmax(m, __ldcg(pml + 2 * k));
        float den = 0.0f, acc = 0.0f;
        for (int k = 0; k < n; k++) {
            const float pm = __ldcg(pml + 2 * k);
            if (pm == -INFINITY) continue;
            const float f = expf(pm - m);
            den = fmaf(__ldcg(pml + 2 * k + 1), f, den);
            acc = fmaf(__ldcg(po + k * FO_HD + d), f, acc);
        }
        const float lse = m + logf(den);
        pg.out[row_head * FO_HD + d] = (acc / den) * sink_scale(pg.sinks[h], lse);
    }
    if (t == 0) pg.counters[g] = 0u;  // ready for the next call on this cache
}

}  // namespace fo

// Launches one instantiation, raising its dynamic shared-memory limit once.
template <int F, bool FAST, int R>
static cudaError_t launch_one(dim3 grid, const fo_decode_page &page0, const fo_decode_page *dev_pages,
                              int64_t groups, cudaStream_t stream) {
    static bool configured = false;
    if (!configured) {
        cudaError_t e = cudaFuncSetAttribute(fo::decode_kernel<F, FAST, R>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, (int)fo::DEC_SMEM);
        if (e != cudaSuccess) return e;
        configured = true;
    }
    fo::decode_kernel<F, FAST, R><<<grid, fo::DEC_THREADS, fo::DEC_SMEM, stream>>>(page0, dev_pages, groups);
    return cudaGetLastError();
}

template <int F, bool FAST>
static cudaError_t launch_rows(dim3 grid, int rows, const fo_decode_page &page0, const fo_decode_page *dev_pages,
                               int64_t groups, cudaStream_t stream) {
    switch (rows) {
    case 1: return launch_one<F, FAST, 1>(grid, page0, dev_pages, groups, stream);
    case 2: return launch_one<F, FAST, 2>(grid, page0, dev_pages, groups, stream);
    case 3: return launch_one<F, FAST, 3>(grid, page0, dev_pages, groups, stream);
    case 4: return launch_one<F, FAST, 4>(grid, page0, dev_pages, groups, stream);
    case 5: return launch_one<F, FAST, 5>(grid, page0, dev_pages, groups, stream);
    case 6: return launch_one<F, FAST, 6>(grid, page0, dev_pages, groups, stream);
    case 7: return launch_one<F, FAST, 7>(grid, page0, dev_pages, groups, stream);
    case 8: return launch_one<F, FAST, 8>(grid, page0, dev_pages, groups, stream);
    }
    return cudaErrorInvalidValue;
}

static cudaError_t launch_decode(const fo_decode_page &page0, const fo_decode_page *dev_pages, int64_t n_pages,
                                 int format, int64_t groups, int fast_exp, int64_t max_splits, int rows,
                                 cudaStream_t stream) {
    if (n_pages <= 0 || max_splits <= 0) return cudaSuccess;
    dim3 grid((unsigned)max_splits, (unsigned)groups, (unsigned)n_pages);
    switch (format) {
    case fo::DF32: return fast_exp ? launch_rows<fo::DF32, true>(grid, rows, page0, dev_pages, groups, stream)
                                   : launch_rows<fo::DF32, false>(grid, rows, page0, dev_pages, groups, stream);
    case fo::DQ16: return fast_exp ? launch_rows<fo::DQ16, true>(grid, rows, page0, dev_pages, groups, stream)
                                   : launch_rows<fo::DQ16, false>(grid, rows, page0, dev_pages, groups, stream);
    case fo::DQ8: return fast_exp ? launch_rows<fo::DQ8, true>(grid, rows, page0, dev_pages, groups, stream)
                                  : launch_rows<fo::DQ8, false>(grid, rows, page0, dev_pages, groups, stream);
    case fo::DBF16: return fast_exp ? launch_rows<fo::DBF16, true>(grid, rows, page0, dev_pages, groups, stream)
                                    : launch_rows<fo::DBF16, false>(grid, rows, page0, dev_pages, groups, stream);
    }
    return cudaErrorInvalidValue;
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
