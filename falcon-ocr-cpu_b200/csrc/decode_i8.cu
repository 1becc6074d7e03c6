// decode_i8.cu -- the INT8 KV format of BASELINE's config 4 and single-row
// decode attention over many pages of it.  The reference has no such format
// (its INT8 KV is the Q8 record format of src/quant/kv.rs, decoded by
// decode.cu); this one stores keys and values of every head separately,
// [head][position][64] int8, with one FP32 scale per (head, 64-position group)
// for keys and values apart.  Codes are round-to-nearest-even of x / scale,
// clamped to [-127, 127], as the reference's codec rounds
// (src/quant/kv/codec.rs:60-83); scale = max |x| over the group / 127.
//
// Decode: grid (split, head, page), a CTA per FO_I8_SPLIT positions of one
// head of one page.  Each warp streams its keys in 32-key chunks through two
// shared-memory buffers: one lane bulk-copies a chunk's key rows and value
// rows (2 KB each, contiguous) two chunks ahead, so every warp keeps about
// 8 KB in flight without a load on its dependency chain.  From shared
// memory: logits with lane = key (the 64 codes of a key), the online softmax
// per chunk, and O += P V with lane = two output dimensions.  Codes become floats exactly without the conversion
// unit, and each group's scale multiplies once (a logit, or p) instead of
// every code.  The warps combine into the split's partial; a merge
// kernel (a programmatic dependent) folds the splits and applies the sink.
#include "fo_common.cuh"
#include "fo_kernels.h"
#include "sm100.cuh"

#include <algorithm>
#include <atomic>

namespace fo {

constexpr int I8_WARPS = 8;
constexpr int I8_THREADS = 32 * I8_WARPS;
constexpr int I8_KEYS_PER_WARP = FO_I8_SPLIT / I8_WARPS;
constexpr int I8_GROUP = 64;
constexpr int I8_DSMEM = 2 * I8_WARPS * 2 * 32 * 64;  // key and value row buffers

// ---------------------------------------------------------------- quantize
// A CTA per (head, 64-position group): max |x| over the group, scale, codes.
__global__ void __launch_bounds__(256) quantize_i8_kernel(const float *x, int64_t len, int64_t heads, int8_t *codes,
                                                          float *scales) {
    __shared__ float red[8];
    const int64_t h = blockIdx.y, grp = blockIdx.x;
    const int t = threadIdx.x;
    const int64_t p0 = grp * I8_GROUP;
    const int n = (int)min64(I8_GROUP, len - p0) * 64;
    float v[16];
    float m = 0.0f;
#pragma unroll
    for (int i = 0; i < 16; i++) {
        const int e = t + i * 256;  // element of the group: position e / 64, dim e % 64
        v[i] = e < n ? x[((p0 + e / 64) * heads + h) * 64 + e % 64] : 0.0f;
        m = fmaxf(m, fabsf(v[i]));
    }
    m = warp_max(m);
    if ((t & 31) == 0) red[t >> 5] = m;
    __syncthreads();
    m = red[0];
#pragma unroll
    for (int w = 1; w < 8; w++) m = fmaxf(m, red[w]);
    const float scale = __fdiv_rn(m, 127.0f);
    if (t == 0) scales[h * ((len + I8_GROUP - 1) / I8_GROUP) + grp] = scale;
#pragma unroll
    for (int i = 0; i < 16; i++) {
        const int e = t + i * 256;
        if (e >= n) continue;
        int c = 0;
        if (scale > 0.0f) c = (int)fminf(fmaxf(rintf(__fdiv_rn(v[i], scale)), -127.0f), 127.0f);
        codes[(h * len + p0 + e / 64) * 64 + e % 64] = (int8_t)c;
    }
}

// ------------------------------------------------------------------ decode
template <bool FAST>
__global__ void __launch_bounds__(I8_THREADS, 3) decode_i8_kernel(const fo_i8_page *pages, int64_t heads) {
    __shared__ float ow[I8_WARPS][64];
    __shared__ __align__(16) float qs[64];  // the head's query row
    __shared__ float mw[I8_WARPS], lw[I8_WARPS];
    // Per warp, two buffers of 32 key rows and 32 value rows (dynamic: 64 KB).
    extern __shared__ __align__(128) int8_t i8_rows[];
    int8_t(*kbuf)[2][32 * 64] = reinterpret_cast<int8_t(*)[2][32 * 64]>(i8_rows);
    int8_t(*vbuf)[2][32 * 64] = reinterpret_cast<int8_t(*)[2][32 * 64]>(i8_rows + I8_WARPS * 2 * 32 * 64);
    __shared__ __align__(8) uint64_t bars[I8_WARPS][2];
    __shared__ int abort_flag;
    // The merge kernel may launch now; it waits for this grid to finish.
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const fo_i8_page &pg = pages[blockIdx.z];
    const int s = blockIdx.x;
    if (s >= pg.splits) return;
    const int64_t h = blockIdx.y, len = pg.len;
    const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
    const int64_t groups = (len + I8_GROUP - 1) / I8_GROUP;
    const int8_t *kc = pg.k_codes + h * len * 64;
    const int8_t *vc = pg.v_codes + h * len * 64;
    const float *ks = pg.k_scales + h * groups, *vs = pg.v_scales + h * groups;
    if (t < 2 * I8_WARPS) sm100::mbar_init(&bars[t / 2][t % 2], 1);
    if (t == 0) abort_flag = 0;
    if (t < 16) reinterpret_cast<float4 *>(qs)[t] = __ldg(reinterpret_cast<const float4 *>(pg.q + h * 64) + t);
    __syncthreads();
    const int64_t w0 = (int64_t)s * FO_I8_SPLIT + (int64_t)warp * I8_KEYS_PER_WARP;
    const int64_t w1 = min64(w0 + I8_KEYS_PER_WARP, min64((int64_t)(s + 1) * FO_I8_SPLIT, len));
    const int n_chunks = (int)max64(0, (w1 - w0 + 31) / 32);
    // Chunk c's key and value rows into buffer c & 1.
    auto stage = [&](int c) {
        const int64_t k0 = w0 + 32 * c;
        const uint32_t bytes = (uint32_t)min64(32, w1 - k0) * 64;
        uint64_t *bar = &bars[warp][c & 1];
        sm100::mbar_expect_tx(bar, 2 * bytes);
        sm100::bulk_g2s(kbuf[warp][c & 1], kc + k0 * 64, bytes, bar);
        sm100::bulk_g2s(vbuf[warp][c & 1], vc + k0 * 64, bytes, bar);
    };
    if (lane == 0)
        for (int c = 0; c < min(2, n_chunks); c++) stage(c);
    // P V runs in half warps: lanes 16 h + i take the keys of parity h and
    // output dimensions 4 i .. 4 i + 3, as (d, d + 1), (d + 2, d + 3) pairs.
    const int half = lane >> 4, dq = 4 * (lane & 15);
    float m_st = -INFINITY, l_st = 0.0f;
    float2 oa = make_float2(0.0f, 0.0f), ob = make_float2(0.0f, 0.0f);
    bool ok = true;
    int c = 0;
    for (; c < n_chunks; c++) {
        const int64_t k0 = w0 + 32 * c;
        const int nk = (int)min64(32, w1 - k0);
        ok = sm100::mbar_wait(&bars[warp][c & 1], (c >> 1) & 1, &abort_flag, pg.err);
        if (!ok) break;
        const int8_t *kb = kbuf[warp][c & 1], *vb = vbuf[warp][c & 1];
        // Logit of this lane's key: (q . codes) * scale / 8 (the group's
        // scale factored out of the dot product).
        float x;
        {
            const uint4 *kp = reinterpret_cast<const uint4 *>(kb + min(lane, nk - 1) * 64);
            const float sc = __ldg(ks + (k0 + min(lane, nk - 1)) / I8_GROUP);
            // Dimensions d % 4 = 0, 1 (a01) and 2, 3 (a23) in packed FMA,
            // each half an ordinary fmaf.
            float2 a01 = make_float2(0.f, 0.f), a23 = make_float2(0.f, 0.f);
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const uint4 wv = kp[i];
                const uint32_t ww[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    float cf[4];
                    s8x4_f32(ww[j], cf);
                    const float4 qv = reinterpret_cast<const float4 *>(qs)[4 * i + j];
                    a01 = __ffma2_rn(make_float2(qv.x, qv.y), make_float2(cf[0], cf[1]), a01);
                    a23 = __ffma2_rn(make_float2(qv.z, qv.w), make_float2(cf[2], cf[3]), a23);
                }
            }
            x = lane < nk ? __fmul_rn(__fmul_rn(__fadd_rn(__fadd_rn(a01.x, a01.y), __fadd_rn(a23.x, a23.y)), sc),
                                      0.125f)
                          : -INFINITY;
        }
        // Online softmax of the chunk (chunk max, rescale, exp(s - max)).
        const float cm = warp_max(x);
        const float m_new = rmax(m_st, cm);
        const float alpha = m_st == -INFINITY ? 0.0f : expf(__fsub_rn(m_st, m_new));
        const float p = lane < nk ? softmax_exp<FAST>(__fsub_rn(x, m_new)) : 0.0f;
        l_st = __fadd_rn(__fmul_rn(l_st, alpha), warp_sum(p));
        m_st = m_new;
        oa = __fmul2_rn(oa, make_float2(alpha, alpha));
        ob = __fmul2_rn(ob, make_float2(alpha, alpha));
        // O += P V over the keys of this half's parity, the value scale
        // folded into p (a chunk never straddles a group).
        const float ps = __fmul_rn(p, __ldg(vs + k0 / I8_GROUP));
        auto pv = [&](int j) {
            const float pj = __shfl_sync(0xffffffffu, ps, min(j, 31));
            if (j < nk) {
                float v[4];
                s8x4_f32(*reinterpret_cast<const uint32_t *>(vb + j * 64 + dq), v);
                oa = __ffma2_rn(make_float2(pj, pj), make_float2(v[0], v[1]), oa);
                ob = __ffma2_rn(make_float2(pj, pj), make_float2(v[2], v[3]), ob);
            }
        };
        if (nk == 32) {
#pragma unroll
            for (int j2 = 0; j2 < 16; j2++) pv(2 * j2 + half);
        } else {
            for (int j2 = 0; j2 < (nk + 1) / 2; j2++) pv(2 * j2 + half);
        }
        __syncwarp();
        if (lane == 0 && c + 2 < n_chunks) {
            sm100::fence_proxy_async_smem();  // this chunk's reads before the copies' writes
            stage(c + 2);
        }
    }
    if (!ok) {
        // A wait that gave up (error word raised): let this warp's copies in
        // flight (chunks c and c + 1) land before the CTA can exit.
        if (lane == 0) {
            sm100::mbar_wait_drain(&bars[warp][c & 1], (c >> 1) & 1);
            if (c + 1 < n_chunks) sm100::mbar_wait_drain(&bars[warp][(c + 1) & 1], ((c + 1) >> 1) & 1);
        }
        m_st = -INFINITY;
        l_st = 0.0f;
        oa = ob = make_float2(0.0f, 0.0f);
    }
    // The even-key and odd-key halves of this lane's dimensions.
    oa.x = __fadd_rn(oa.x, __shfl_xor_sync(0xffffffffu, oa.x, 16));
    oa.y = __fadd_rn(oa.y, __shfl_xor_sync(0xffffffffu, oa.y, 16));
    ob.x = __fadd_rn(ob.x, __shfl_xor_sync(0xffffffffu, ob.x, 16));
    ob.y = __fadd_rn(ob.y, __shfl_xor_sync(0xffffffffu, ob.y, 16));
    // Combine the warps in order into the split's partial.
    if (lane == 0) {
        mw[warp] = m_st;
        lw[warp] = l_st;
    }
    if (half == 0) *reinterpret_cast<float4 *>(&ow[warp][dq]) = make_float4(oa.x, oa.y, ob.x, ob.y);
    __syncthreads();
    if (t < 64) {
        float m = -INFINITY;
#pragma unroll
        for (int w = 0; w < I8_WARPS; w++) m = rmax(m, mw[w]);
        float den = 0.0f, acc = 0.0f;
#pragma unroll
        for (int w = 0; w < I8_WARPS; w++) {
            if (mw[w] == -INFINITY) continue;
            const float f = expf(__fsub_rn(mw[w], m));
            den = fmaf(lw[w], f, den);
            acc = fmaf(ow[w][t], f, acc);
        }
        const int64_t idx = h * pg.splits + s;
        pg.part_o[idx * 64 + t] = acc;
        if (t == 0) {
            pg.part_ml[idx * 2] = m;
            pg.part_ml[idx * 2 + 1] = den;
        }
    }
}

// The splits of every head of a page in order, and the sink; a CTA per
// (head, page), a thread per dimension.
__global__ void __launch_bounds__(64) merge_i8_kernel(const fo_i8_page *pages, int64_t heads) {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const fo_i8_page &pg = pages[blockIdx.y];
    const int64_t h = blockIdx.x;
    const int d = threadIdx.x;
    const float *ml = pg.part_ml + h * pg.splits * 2;
    const float *po = pg.part_o + h * pg.splits * 64 + d;
    float m = -INFINITY;
    for (int k = 0; k < pg.splits; k++) m = rmax(m, __ldcg(ml + 2 * k));
    float den = 0.0f, acc = 0.0f;
    for (int k = 0; k < pg.splits; k++) {
        const float mk = __ldcg(ml + 2 * k);
        if (mk == -INFINITY) continue;
        const float f = expf(__fsub_rn(mk, m));
        den = fmaf(__ldcg(ml + 2 * k + 1), f, den);
        acc = fmaf(__ldcg(po + (int64_t)k * 64), f, acc);
    }
    const float lse = m + logf(den);
    pg.out[h * 64 + d] = (acc / den) * sink_scale(pg.sinks[h], lse);
}

}  // namespace fo

extern "C" cudaError_t fo_launch_quantize_i8(const float *x, int64_t len, int64_t heads, int8_t *codes, float *scales,
                                             cudaStream_t stream) {
    if (len <= 0) return cudaSuccess;
    dim3 grid((unsigned)((len + fo::I8_GROUP - 1) / fo::I8_GROUP), (unsigned)heads);
    fo::quantize_i8_kernel<<<grid, 256, 0, stream>>>(x, len, heads, codes, scales);
    return cudaGetLastError();
}

extern "C" cudaError_t fo_launch_decode_i8(const fo_i8_page *dev_pages, int64_t n_pages, int64_t heads,
                                           int32_t max_splits, int fast_exp, cudaStream_t stream) {
    if (n_pages <= 0 || max_splits <= 0) return cudaSuccess;
    dim3 grid((unsigned)max_splits, (unsigned)heads, (unsigned)n_pages);
    // The attribute belongs to each device's context: set once per device.
    static std::atomic<unsigned long long> configured{0};
    int dev = 0;
    cudaGetDevice(&dev);
    const unsigned long long bit = 1ull << (dev & 63);
    if (!(configured.load() & bit)) {
        cudaError_t e = cudaFuncSetAttribute(fo::decode_i8_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             fo::I8_DSMEM);
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(fo::decode_i8_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     fo::I8_DSMEM);
        if (e != cudaSuccess) return e;
        configured.fetch_or(bit);
    }
    if (fast_exp)
        fo::decode_i8_kernel<true><<<grid, fo::I8_THREADS, fo::I8_DSMEM, stream>>>(dev_pages, heads);
    else
        fo::decode_i8_kernel<false><<<grid, fo::I8_THREADS, fo::I8_DSMEM, stream>>>(dev_pages, heads);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)heads, (unsigned)n_pages);
    cfg.blockDim = dim3(64);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, fo::merge_i8_kernel, dev_pages, heads);
}
