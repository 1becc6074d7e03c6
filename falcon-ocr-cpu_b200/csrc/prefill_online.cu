// prefill_online.cu -- the online-softmax head for every cache layout and
// head width (reference: src/kernels/attention/online.rs:89-169, and the
// decode64 fixed-width form src/kernels/attention/decode64.rs:22-44).
//
// One warp per (query, head): 128-key tiles, block maximum, rescale of the
// output and denominator before PV, exp(score - max), the sink applied once
// at the end.  Lanes own keys during QK and dimensions during PV.  It serves
// the shapes the FP32 tiles do not (head_dim != 64, fewer than 4 queries)
// and is the generic path of the C ABI.
#include "fo_common.cuh"
#include "fo_kernels.h"

namespace fo {

constexpr int ONLINE_TILE = 128;
constexpr int ONLINE_WARPS = 8;
constexpr int ONLINE_MAX_HD = 256;

struct OnlineArgs {
    const float *q, *prefix_k, *generated_k, *v, *sinks;
    float *out;
    int64_t query_len, prefix_len, total_len, n_heads, n_kv_heads, head_dim;
    int64_t query_offset, image_start, image_end;
};

__device__ __forceinline__ const float *key_row(const OnlineArgs &a, int64_t pos, int64_t head) {
    if (pos < a.prefix_len) return a.prefix_k + (pos * a.n_heads + head) * a.head_dim;
    int64_t repeat = a.n_heads / a.n_kv_heads;
    return a.generated_k + ((pos - a.prefix_len) * a.n_kv_heads + head / repeat) * a.head_dim;
}

template <bool FAST>
__global__ void __launch_bounds__(ONLINE_WARPS * 32) online_head_kernel(OnlineArgs a) {
    __shared__ float s_q[ONLINE_WARPS][ONLINE_MAX_HD];
    __shared__ float s_p[ONLINE_WARPS][ONLINE_TILE];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t qh = (int64_t)blockIdx.x * ONLINE_WARPS + warp;
    if (qh >= a.query_len * a.n_heads) return;
    const int64_t query = qh / a.n_heads, head = qh % a.n_heads;
    const int64_t kv_head = head / (a.n_heads / a.n_kv_heads);
    const int hd = (int)a.head_dim;
    const float scale = 1.0f / sqrtf((float)hd);  // (head_dim as f32).sqrt().recip()
    const int64_t vend = visible_end(a.query_offset + query, a.image_start, a.image_end);
    const float *qv = a.q + qh * hd;
    for (int d = lane; d < hd; d += 32) s_q[warp][d] = qv[d];
    __syncwarp();

    float acc[ONLINE_MAX_HD / 32];
#pragma unroll
    for (int i = 0; i < ONLINE_MAX_HD / 32; i++) acc[i] = 0.0f;
    float running_max = -INFINITY, denominator = 0.0f;

    for (int64_t start = 0; start < vend; start += ONLINE_TILE) {
        const int len = (int)min64(ONLINE_TILE, vend - start);
        float logit[ONLINE_TILE / 32];
        float block_max = -INFINITY;
#pragma unroll
        for (int i = 0; i < ONLINE_TILE / 32; i++) {
            const int j = lane + 32 * i;
            logit[i] = -INFINITY;
            if (j < len) {
                const float *kr = key_row(a, start + j, head);
                float dot = 0.0f;
                for (int d = 0; d < hd; d++) dot = fmaf(s_q[warp][d], kr[d], dot);
                logit[i] = dot * scale;
                block_max = rmax(block_max, logit[i]);
            }
        }
        block_max = warp_max(block_max);
        const float new_max = rmax(running_max, block_max);
        const float rescale = running_max == -INFINITY ? 0.0f : expf(running_max - new_max);
#pragma unroll
        for (int i = 0; i < ONLINE_MAX_HD / 32; i++) acc[i] *= rescale;
        denominator *= rescale;
        float psum = 0.0f;
#pragma unroll
        for (int i = 0; i < ONLINE_TILE / 32; i++) {
            const int j = lane + 32 * i;
            float p = 0.0f;
            if (j < len) p = softmax_exp<FAST>(logit[i] - new_max);
            s_p[warp][j] = p;
            psum += p;
        }
        denominator += warp_sum(psum);
        __syncwarp();
        for (int j = 0; j < len; j++) {
            const float p = s_p[warp][j];
            const float *vr = a.v + ((start + j) * a.n_kv_heads + kv_head) * hd;
#pragma unroll
            for (int i = 0; i < ONLINE_MAX_HD / 32; i++) {
                const int d = lane + 32 * i;
                if (d < hd) acc[i] = fmaf(p, vr[d], acc[i]);
            }
        }
        __syncwarp();
        running_max = new_max;
    }
    const float lse = running_max + logf(denominator);
    const float ss = sink_scale(a.sinks[head], lse);
    float *out = a.out + qh * hd;
#pragma unroll
    for (int i = 0; i < ONLINE_MAX_HD / 32; i++) {
        const int d = lane + 32 * i;
        if (d < hd) out[d] = (acc[i] / denominator) * ss;
    }
}

}  // namespace fo

extern "C" cudaError_t fo_launch_online(const float *q, const float *prefix_k, const float *generated_k,
                                        const float *v, const float *sinks, float *out, int64_t query_len,
                                        int64_t prefix_len, int64_t total_len, int64_t n_heads, int64_t n_kv_heads,
                                        int64_t head_dim, int64_t query_offset, int64_t image_start,
                                        int64_t image_end, int exp_fast, cudaStream_t stream) {
    fo::OnlineArgs a{q,       prefix_k, generated_k, v,          sinks,        out,         query_len,
                     prefix_len, total_len, n_heads,  n_kv_heads, head_dim, query_offset, image_start, image_end};
    const int64_t warps = query_len * n_heads;
    if (warps == 0) return cudaSuccess;
    dim3 grid((unsigned)((warps + fo::ONLINE_WARPS - 1) / fo::ONLINE_WARPS));
    if (exp_fast)
        fo::online_head_kernel<true><<<grid, fo::ONLINE_WARPS * 32, 0, stream>>>(a);
    else
        fo::online_head_kernel<false><<<grid, fo::ONLINE_WARPS * 32, 0, stream>>>(a);
    return cudaGetLastError();
}
