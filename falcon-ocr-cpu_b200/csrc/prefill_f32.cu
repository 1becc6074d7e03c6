// prefill_f32.cu -- exact-mode prefill attention on FP32 CUDA cores
// (reference: the FP32 prefill tiles, src/kernels/attention/prefill64.rs:179-715,
// and their static-shift softmax, prefill64/static_shift.rs:129-161).
//
// One CTA computes 64 queries of one head against every key tile they see:
// Q (transposed), K (transposed) and V tiles staged in shared memory,
// S = scale * Q K^T with an 8x4 register tile per thread, the prefix-LM mask
// as a per-row visible end, then the online softmax (block max, rescale of
// output and denominator, exp(s - max)) or the static shift (exp_poly of the
// score, no maximum), then O += P V with an 8x4 register tile.  Keys of a
// mixed cache are read from the prefix (per query head) or generated rows
// (per KV head), as CompactKv::key does (src/kernels/attention/mod.rs:143-151).
#include "fo_common.cuh"
#include "fo_kernels.h"

namespace fo {

constexpr int F32_QT = 64;  // queries per CTA
constexpr int F32_KT = 64;  // keys per tile
constexpr int F32_LD = 68;  // padded row stride (floats) of the transposed tiles
constexpr int F32_THREADS = 128;

struct F32Args {
    const float *q, *prefix_k, *generated_k, *v, *sinks;
    float *out;
    int64_t query_len, prefix_len, total_len, n_heads, n_kv_heads;
    int64_t query_offset, image_start, image_end;
};

template <bool STATIC, bool FAST>
__global__ void __launch_bounds__(F32_THREADS) prefill_f32_kernel(F32Args a) {
    extern __shared__ __align__(16) float smem[];
    float *Qt = smem;                    // [64 d][F32_LD]  Qt[d][row]
    float *Kt = Qt + FO_HD * F32_LD;     // [64 d][F32_LD]  Kt[d][key]
    float *Vs = Kt + FO_HD * F32_LD;     // [64 key][64 d]
    float *Ps = Vs + F32_KT * FO_HD;     // [64 row][F32_LD]

    const int t = threadIdx.x, ty = t >> 4, tx = t & 15;
    const int64_t tiles = (a.query_len + F32_QT - 1) / F32_QT;
    const int64_t tile = tiles - 1 - blockIdx.x;  // heaviest (latest) tiles first
    const int64_t head = blockIdx.y;
    const int64_t kv_head = head / (a.n_heads / a.n_kv_heads);
    const int64_t q0 = tile * F32_QT;
    const int queries = (int)min64(F32_QT, a.query_len - q0);
    const int64_t qw = a.n_heads * FO_HD, kvw = a.n_kv_heads * FO_HD;

    // Tile span (src/kernels/attention/prefill64/span.rs:9-20).
    const int64_t first_abs = a.query_offset + q0, last_abs = first_abs + queries - 1;
    int64_t tile_end = last_abs + 1;
    if (first_abs < a.image_end && last_abs >= a.image_start) tile_end = max(tile_end, a.image_end);

    // Q tile, transposed.
    for (int i = t; i < F32_QT * 16; i += F32_THREADS) {
        const int r = i >> 4, c = i & 15;
        float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
        if (r < queries) x = *reinterpret_cast<const float4 *>(a.q + (q0 + r) * qw + head * FO_HD + 4 * c);
        Qt[(4 * c + 0) * F32_LD + r] = x.x;
        Qt[(4 * c + 1) * F32_LD + r] = x.y;
        Qt[(4 * c + 2) * F32_LD + r] = x.z;
        Qt[(4 * c + 3) * F32_LD + r] = x.w;
    }
    // Per-row state: rows ty*8 + i.
    // Outputs as (dims 4 tx, 4 tx + 1) and (4 tx + 2, 4 tx + 3) pairs of the
    // packed FMA (each half an ordinary fmaf).
    int64_t vend[8];
    float m[8], l[8];
    float2 acc[8][2];
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const int64_t abs_row = first_abs + ty * 8 + i;
        vend[i] = visible_end(abs_row, a.image_start, a.image_end);
        m[i] = -INFINITY;
        l[i] = 0.0f;
        acc[i][0] = acc[i][1] = make_float2(0.0f, 0.0f);
    }
    const float scale = 0.125f;  // (64 as f32).sqrt().recip()

    for (int64_t k0 = 0; k0 < tile_end; k0 += F32_KT) {
        __syncthreads();  // previous tile's readers are done
        for (int i = t; i < F32_KT * 16; i += F32_THREADS) {
            const int j = i >> 4, c = i & 15;
            const int64_t pos = k0 + j;
            float4 kx = make_float4(0.f, 0.f, 0.f, 0.f), vx = kx;
            if (pos < tile_end) {
                const float *kr = pos < a.prefix_len ? a.prefix_k + pos * qw + head * FO_HD
                                                     : a.generated_k + (pos - a.prefix_len) * kvw + kv_head * FO_HD;
                kx = *reinterpret_cast<const float4 *>(kr + 4 * c);
                vx = *reinterpret_cast<const float4 *>(a.v + pos * kvw + kv_head * FO_HD + 4 * c);
            }
            Kt[(4 * c + 0) * F32_LD + j] = kx.x;
            Kt[(4 * c + 1) * F32_LD + j] = kx.y;
            Kt[(4 * c + 2) * F32_LD + j] = kx.z;
            Kt[(4 * c + 3) * F32_LD + j] = kx.w;
            *reinterpret_cast<float4 *>(Vs + j * FO_HD + 4 * c) = vx;
        }
        __syncthreads();

        // S = Q K^T: rows ty*8..+8, keys tx*4..+4 (key pairs in packed FMA).
        float2 s2[8][2];
#pragma unroll
        for (int i = 0; i < 8; i++) s2[i][0] = s2[i][1] = make_float2(0.0f, 0.0f);
#pragma unroll 8
        for (int d = 0; d < FO_HD; d++) {
            const float4 qa = *reinterpret_cast<const float4 *>(Qt + d * F32_LD + ty * 8);
            const float4 qb = *reinterpret_cast<const float4 *>(Qt + d * F32_LD + ty * 8 + 4);
            const float4 kb = *reinterpret_cast<const float4 *>(Kt + d * F32_LD + tx * 4);
            const float qv[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
#pragma unroll
            for (int i = 0; i < 8; i++) {
                s2[i][0] = __ffma2_rn(make_float2(qv[i], qv[i]), make_float2(kb.x, kb.y), s2[i][0]);
                s2[i][1] = __ffma2_rn(make_float2(qv[i], qv[i]), make_float2(kb.z, kb.w), s2[i][1]);
            }
        }
        float s[8][4];
#pragma unroll
        for (int i = 0; i < 8; i++) {
            s[i][0] = s2[i][0].x;
            s[i][1] = s2[i][0].y;
            s[i][2] = s2[i][1].x;
            s[i][3] = s2[i][1].y;
        }
        // Mask, softmax, P to shared memory.
#pragma unroll
        for (int i = 0; i < 8; i++) {
            float p[4];
            if constexpr (STATIC) {
                float rsum = 0.0f;
#pragma unroll
                for (int c = 0; c < 4; c++) {
                    const int64_t key = k0 + tx * 4 + c;
                    p[c] = key < vend[i] ? exp_poly_unchecked(s[i][c] * scale) : 0.0f;
                    rsum += p[c];
                }
#pragma unroll
                for (int o = 8; o > 0; o >>= 1) rsum += __shfl_xor_sync(0xffffffffu, rsum, o);
                l[i] += rsum;
            } else {
                float bm = -INFINITY;
#pragma unroll
                for (int c = 0; c < 4; c++) {
                    const int64_t key = k0 + tx * 4 + c;
                    s[i][c] = key < vend[i] ? s[i][c] * scale : -INFINITY;
                    bm = rmax(bm, s[i][c]);
                }
#pragma unroll
                for (int o = 8; o > 0; o >>= 1) bm = fmaxf(bm, __shfl_xor_sync(0xffffffffu, bm, o));
                const float new_max = rmax(m[i], bm);
                float rescale = 1.0f, rsum = 0.0f;
                if (new_max != -INFINITY) {
                    rescale = m[i] == -INFINITY ? 0.0f : softmax_exp<FAST>(m[i] - new_max);
#pragma unroll
                    for (int c = 0; c < 4; c++) {
                        p[c] = softmax_exp<FAST>(s[i][c] - new_max);
                        rsum += p[c];
                    }
                    m[i] = new_max;
                } else {
#pragma unroll
                    for (int c = 0; c < 4; c++) p[c] = 0.0f;
                }
#pragma unroll
                for (int o = 8; o > 0; o >>= 1) rsum += __shfl_xor_sync(0xffffffffu, rsum, o);
                l[i] = l[i] * rescale + rsum;
                acc[i][0] = __fmul2_rn(acc[i][0], make_float2(rescale, rescale));
                acc[i][1] = __fmul2_rn(acc[i][1], make_float2(rescale, rescale));
            }
            *reinterpret_cast<float4 *>(Ps + (ty * 8 + i) * F32_LD + tx * 4) = make_float4(p[0], p[1], p[2], p[3]);
        }
        __syncthreads();

        // O += P V: rows ty*8..+8, dims tx*4..+4.
        const int kmax = (int)min64(F32_KT, tile_end - k0);
        for (int j4 = 0; j4 < kmax; j4 += 4) {
            float4 pv[8];
#pragma unroll
            for (int i = 0; i < 8; i++) pv[i] = *reinterpret_cast<const float4 *>(Ps + (ty * 8 + i) * F32_LD + j4);
#pragma unroll
            for (int jj = 0; jj < 4; jj++) {
                const float4 vb = *reinterpret_cast<const float4 *>(Vs + (j4 + jj) * FO_HD + tx * 4);
#pragma unroll
                for (int i = 0; i < 8; i++) {
                    const float p = jj == 0 ? pv[i].x : jj == 1 ? pv[i].y : jj == 2 ? pv[i].z : pv[i].w;
                    acc[i][0] = __ffma2_rn(make_float2(p, p), make_float2(vb.x, vb.y), acc[i][0]);
                    acc[i][1] = __ffma2_rn(make_float2(p, p), make_float2(vb.z, vb.w), acc[i][1]);
                }
            }
        }
    }
    // Epilogue: normalize and apply the sink (prefill64.rs:468-479).
    const float sink = a.sinks[head];
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const int r = ty * 8 + i;
        if (r >= queries) continue;
        const float lse = STATIC ? logf(l[i]) : m[i] + logf(l[i]);
        const float ss = sink_scale(sink, lse);
        float4 o;
        o.x = (acc[i][0].x / l[i]) * ss;
        o.y = (acc[i][0].y / l[i]) * ss;
        o.z = (acc[i][1].x / l[i]) * ss;
        o.w = (acc[i][1].y / l[i]) * ss;
        *reinterpret_cast<float4 *>(a.out + (q0 + r) * qw + head * FO_HD + tx * 4) = o;
    }
}

}  // namespace fo

extern "C" cudaError_t fo_launch_prefill_f32(const float *q, const float *prefix_k, const float *generated_k,
                                             const float *v, const float *sinks, float *out, int64_t query_len,
                                             int64_t prefix_len, int64_t total_len, int64_t n_heads,
                                             int64_t n_kv_heads, int64_t query_offset, int64_t image_start,
                                             int64_t image_end, int softmax_static, int exp_fast,
                                             cudaStream_t stream) {
    fo::F32Args a{q,         prefix_k,   generated_k,  v,           sinks,      out,      query_len,
                  prefix_len, total_len, n_heads,      n_kv_heads,  query_offset, image_start, image_end};
    if (query_len == 0) return cudaSuccess;
    const size_t smem = sizeof(float) * (3 * FO_HD * fo::F32_LD + fo::F32_KT * FO_HD);
    dim3 grid((unsigned)((query_len + fo::F32_QT - 1) / fo::F32_QT), (unsigned)n_heads);
    auto launch = [&](auto kernel) -> cudaError_t {
        cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        kernel<<<grid, fo::F32_THREADS, smem, stream>>>(a);
        return cudaGetLastError();
    };
    if (softmax_static) return launch(fo::prefill_f32_kernel<true, false>);
    if (exp_fast) return launch(fo::prefill_f32_kernel<false, true>);
    return launch(fo::prefill_f32_kernel<false, false>);
}
