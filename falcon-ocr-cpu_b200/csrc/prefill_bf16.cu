// prefill_bf16.cu -- BF16 prefill attention on the sm_100a tensor cores
// (reference: prefill64/bf16.rs:78-481 with the online softmax, and its
// static-shift softmax, prefill64/bf16/static_shift.rs:1-340).
//
// Semantics kept from the reference: Q, K, V and the probabilities are
// rounded to BF16 (round to nearest even); scores, softmax state, the PV
// accumulator and the output stay FP32; the prefix-LM mask hides key > query
// unless both are image tokens (src/kernels/attention/mod.rs:70-75); the
// sink enters once at the end through sigmoid(lse - sink).  The static shift
// computes p = 2^(scale * log2(e) * q.k) without a running maximum and sums
// the BF16-rounded p (bf16/static_shift.rs:8-23); the online softmax sums the
// unrounded p (bf16.rs:327-356) and, as the reference does, rescales the
// output and denominator whenever a tile raises the row maximum, so the
// largest probability is exactly 1 and loses nothing to BF16 rounding.
//
// Structure (one CTA = two 128-query tiles of one head, sharing K/V tiles):
//   warp 8     TMA producer: K and V tiles [128 keys][64] BF16, 128-byte
//              swizzle, NS-stage ring with full/empty mbarriers;
//   warp 9     MMA issuer (one thread): S_t = Q_t K^T (M128 N128 K64) into
//              TMEM, then O_t += P_t V (M128 N64 K128); tcgen05.commit
//              signals every consumer; it also owns the TMEM allocation;
//   warps 0-7  two softmax warpgroups, one per Q tile, one thread per query
//              row: Q row to BF16 in shared memory, S row from TMEM
//              (tcgen05.ld), mask, exp2, BF16 P row back to TMEM (tcgen05.st),
//              and the epilogue O / l * sink from TMEM.
// TMEM columns: S0 [0,128) S1 [128,256) O0 [256,320) O1 [320,384) P0 [384,448)
// P1 [448,512).  P_t holds the BF16 probabilities (two per 32-bit column) and
// is the PV MMA's A operand straight from TMEM, so PV reads only V from
// shared memory.
// Every wait is bounded (sm100.cuh); on a timeout the CTA unwinds, waits for
// its own copies and MMAs, frees TMEM and reports through the error word.
#include <cudaTypedefs.h>

#include "fo_common.cuh"
#include "fo_kernels.h"
#include "sm100.cuh"

namespace fo {
using namespace sm100;

constexpr int BT_STAGES = 4;
constexpr int BT_THREADS = 320;
constexpr uint32_t BT_TILE = 128 * 128;  // one [128][64] BF16 tile, bytes
constexpr uint32_t OFF_Q = 0;
constexpr uint32_t OFF_K = 2 * BT_TILE;
constexpr uint32_t OFF_V = OFF_K + BT_STAGES * BT_TILE;
constexpr uint32_t OFF_BAR = OFF_V + BT_STAGES * BT_TILE;
// barriers: q_full, k_full[NS], k_empty[NS], v_full[NS], v_empty[NS],
// s_full[2], s_empty[2], p_full[2], p_empty[2], mma_done
constexpr int NBAR = 1 + 4 * BT_STAGES + 8 + 1;
constexpr uint32_t SMEM_BYTES = OFF_BAR + NBAR * 8 + 16 + 1024;
constexpr uint32_t TMEM_COLS = 512;

struct Bf16Args {
    const float *q, *sinks;
    void *out;      // [T][H][64] FP32, or BF16 when out_bf16
    int out_bf16;   // round the output to BF16 (nearest even) as it is stored
    unsigned *err;
    int64_t total, n_heads, n_kv_heads, image_start, image_end;
    int64_t pair_begin, pair_end;  // the 256-query pairs [begin, end) this launch computes
    // Key-range split (SPLIT kernels): each pair's key tiles in n_split
    // consecutive ranges, one CTA per range, writing unnormalized partials
    // [n_split][rows][H][64] and (max in log2 units, denominator)
    // [n_split][rows][H], rows counted from the launch's first pair (rows =
    // 256 x its pairs).
    int n_split;
    float *part_o, *part_ml;
    fo_peer_out peers;  // other ranks' BF16 destinations (n = 0: none)
};

// Bounded wait that ignores the abort flag (for copies/MMAs that complete on
// their own), used while unwinding.
__device__ __forceinline__ void drain_wait(uint64_t *bar, uint32_t phase) {
    const uint64_t t0 = globaltimer();
    while (!mbar_try_wait(bar, phase))
        if (globaltimer() - t0 > FO_WAIT_NS) break;
}

template <bool STATIC, bool SPLIT>
__global__ void __launch_bounds__(BT_THREADS, 1)
    prefill_bf16_kernel(const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmv, Bf16Args a) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + OFF_BAR);
    uint64_t *q_full = bars;
    uint64_t *k_full = bars + 1, *k_empty = k_full + BT_STAGES;
    uint64_t *v_full = k_empty + BT_STAGES, *v_empty = v_full + BT_STAGES;
    uint64_t *s_full = v_empty + BT_STAGES, *s_empty = s_full + 2;
    uint64_t *p_full = s_empty + 2, *p_empty = p_full + 2;
    uint64_t *mma_done = p_empty + 2;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + NBAR);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t T = a.total, H = a.n_heads;
    // Blocks start in index order, x fastest: every head of the heaviest
    // (latest) query pair first, so the longest CTAs start earliest.
    const int64_t pair = a.pair_end - 1 - (SPLIT ? blockIdx.y / a.n_split : blockIdx.y);
    const int64_t head = blockIdx.x;
    const int64_t kv_head = head / (H / a.n_kv_heads);
    const int64_t q0 = pair * 256;
    // Tile span over both Q tiles (src/kernels/attention/prefill64/span.rs:9-20).
    const int64_t last_abs = min64(q0 + 255, T - 1);
    int64_t tile_end = last_abs + 1;
    if (q0 < a.image_end && last_abs >= a.image_start) tile_end = max64(tile_end, a.image_end);
    // This CTA's key tiles: [jbase, jbase + nkv) (all of them unless split).
    int jbase = 0, nkv = (int)((tile_end + 127) / 128);
    const int part = SPLIT ? (int)(blockIdx.y % a.n_split) : 0;
    if constexpr (SPLIT) {
        const int all = nkv;
        jbase = (int)((int64_t)part * all / a.n_split);
        nkv = (int)((int64_t)(part + 1) * all / a.n_split) - jbase;
        if (nkv == 0) {
            // An empty range (a pair with fewer tiles than ranges): an empty
            // partial, before any barrier or tensor memory is set up.
            if (threadIdx.x < 256) {
                const int64_t row = q0 + threadIdx.x;
                if (row < T) {
                    const int64_t idx = ((int64_t)part * ((a.pair_end - a.pair_begin) * 256) + (row - a.pair_begin * 256)) * H + head;
                    float4 *dst = reinterpret_cast<float4 *>(a.part_o + idx * FO_HD);
#pragma unroll
                    for (int i = 0; i < 16; i++) dst[i] = make_float4(0.f, 0.f, 0.f, 0.f);
                    *reinterpret_cast<float2 *>(a.part_ml + idx * 2) = make_float2(-INFINITY, 0.0f);
                }
            }
            return;
        }
    }

    if (threadIdx.x == 0) {
        mbar_init(q_full, 256);
        for (int s = 0; s < BT_STAGES; s++) {
            mbar_init(k_full + s, 1);
            mbar_init(k_empty + s, 1);
            mbar_init(v_full + s, 1);
            mbar_init(v_empty + s, 1);
        }
        for (int t = 0; t < 2; t++) {
            mbar_init(s_full + t, 1);
            mbar_init(s_empty + t, 128);
            mbar_init(p_full + t, 128);
            mbar_init(p_empty + t, 1);
        }
        mbar_init(mma_done, 1);
        *abort_flag = 0;
        mbar_fence_init();
    }
    if (warp == 9) tmem_alloc(tmem_slot, TMEM_COLS);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const uint32_t sQ = smem_u32(smem + OFF_Q), sK = smem_u32(smem + OFF_K), sV = smem_u32(smem + OFF_V);

    if (warp < 8) {
        // ------------------------------------------------ softmax warpgroups
        const int t = warp >> 2, wq = warp & 3, r = threadIdx.x & 127;
        const int64_t row = q0 + 128 * t + r;
        {
            // Q row to BF16 (round to nearest even), 128-byte swizzled rows.
            uint32_t w[32];
            if (row < T) {
                const float4 *src = reinterpret_cast<const float4 *>(a.q + (row * H + head) * FO_HD);
#pragma unroll
                for (int i = 0; i < 16; i++) {
                    const float4 x = __ldg(src + i);
                    w[2 * i] = pack_bf16(x.x, x.y);
                    w[2 * i + 1] = pack_bf16(x.z, x.w);
                }
            } else {
#pragma unroll
                for (int i = 0; i < 32; i++) w[i] = 0;
            }
            const uint32_t base = sQ + t * BT_TILE + r * 128;
#pragma unroll
            for (int c = 0; c < 8; c++)
                st_shared_v4(base + ((c ^ (r & 7)) << 4), w[4 * c], w[4 * c + 1], w[4 * c + 2], w[4 * c + 3]);
            fence_proxy_async_smem();
            mbar_arrive(q_full);
        }
        const int64_t vend = row < T ? visible_end(row, a.image_start, a.image_end) : 0;
        const uint32_t lane_base = (uint32_t)(32 * wq) << 16;
        const uint32_t s_tm = tmem + lane_base + 128 * t;
        const uint32_t o_tm = tmem + lane_base + 256 + 64 * t;
        const uint32_t p_tm = tmem + lane_base + 384 + 64 * t;
        const float C = 0.125f * 1.44269504088896340736f;  // scale * log2(e)
        float l = 0.0f, m2 = -INFINITY;
        bool ok = true;
        for (int j = 0; j < nkv; j++) {
            ok = __all_sync(0xffffffffu, mbar_wait(s_full + t, j & 1, abort_flag, a.err));
            if (!ok) break;
            tc_fence_after();
            uint32_t s[128];
            FO_TMEM_LD32(s_tm + 0, (s + 0));
            FO_TMEM_LD32(s_tm + 32, (s + 32));
            FO_TMEM_LD32(s_tm + 64, (s + 64));
            FO_TMEM_LD32(s_tm + 96, (s + 96));
            tmem_wait_ld();
            tc_fence_before();
            mbar_arrive(s_empty + t);
            const int nvis = (int)max64(0, min64(128, vend - 128 * (int64_t)(jbase + j)));
            // Whole tile visible for every row of the warp: the common case
            // runs without any per-key mask (a separate copy of the loop).
            const bool full = __all_sync(0xffffffffu, nvis >= 128);
            // Scaled scores, two at a time: t = s * (scale * log2 e).
            float2 tt[64];
#pragma unroll
            for (int i = 0; i < 64; i++)
                tt[i] = __fmul2_rn(make_float2(__uint_as_float(s[2 * i]), __uint_as_float(s[2 * i + 1])),
                                   make_float2(C, C));
            float factor = 1.0f;
            if constexpr (!STATIC) {
                float bm = -INFINITY;
                if (full) {
#pragma unroll
                    for (int i = 0; i < 64; i++) bm = fmaxf(bm, fmaxf(tt[i].x, tt[i].y));
                } else {
#pragma unroll
                    for (int i = 0; i < 64; i++) {
                        if (2 * i < nvis) bm = fmaxf(bm, tt[i].x);
                        if (2 * i + 1 < nvis) bm = fmaxf(bm, tt[i].y);
                    }
                }
                if (bm > m2) {  // also true on the first visible tile
                    if (m2 != -INFINITY) factor = ex2(m2 - bm);
                    m2 = bm;
                }
                const float shift = m2 == -INFINITY ? 0.0f : m2;
#pragma unroll
                for (int i = 0; i < 64; i++) tt[i] = __fadd2_rn(tt[i], make_float2(-shift, -shift));
                l *= factor;
            }
            // The probabilities, packed to BF16 pairs in registers, so this
            // overlaps PV_t(j-1), which still reads the P tile.  The static
            // shift sums the rounded probabilities PV multiplies (four
            // running sums, even key first within a pair); the online softmax
            // sums the unrounded ones.
            float2 ls[2] = {make_float2(0.0f, 0.0f), make_float2(0.0f, 0.0f)};
            float la[4] = {0.0f, 0.0f, 0.0f, 0.0f};
            uint32_t pk[64];
            auto pair = [&](int i, float x0, float x1) {
                pk[i] = pack_bf16(x0, x1);
                if constexpr (STATIC)
                    la[i & 3] = add_bf16x2_f32(la[i & 3], pk[i]);
                else
                    ls[i & 1] = __fadd2_rn(ls[i & 1], make_float2(x0, x1));
            };
            if constexpr (STATIC) {
                // The reference's own 2^t (degree-3 polynomial in f = t - n,
                // times 2^n) for every probability: its 7.5e-5 relative error
                // decides some BF16 roundings of P, so the SFU's (nearly exact)
                // exp2 would move them away from the reference's.
                if (full) {
#pragma unroll
                    for (int i = 0; i < 64; i++) {
                        const float2 e = ex2_poly2_inrange(tt[i]);
                        pair(i, e.x, e.y);
                    }
                } else {
#pragma unroll
                    for (int i = 0; i < 64; i++) {
                        const float2 e = ex2_poly2(tt[i]);
                        pair(i, 2 * i < nvis ? e.x : 0.0f, 2 * i + 1 < nvis ? e.y : 0.0f);
                    }
                }
            } else if (full) {
                // 4 of every 16 exponentials run on the FMA pipes (ex2_fit5, as
                // accurate as the SFU's), the rest on the SFU, which would
                // otherwise bound the loop.
#pragma unroll
                for (int i = 0; i < 64; i++) {
                    if ((i & 3) == 3) {
                        const float2 e = ex2_fit5(tt[i]);
                        pair(i, e.x, e.y);
                    } else {
                        pair(i, ex2(tt[i].x), ex2(tt[i].y));
                    }
                }
            } else {
#pragma unroll
                for (int i = 0; i < 64; i++)
                    pair(i, 2 * i < nvis ? ex2(tt[i].x) : 0.0f, 2 * i + 1 < nvis ? ex2(tt[i].y) : 0.0f);
            }
            if constexpr (STATIC)
                l += (la[0] + la[1]) + (la[2] + la[3]);
            else
                l += (ls[0].x + ls[0].y) + (ls[1].x + ls[1].y);
            // P_t is free once PV_t(j-1) has completed.
            if (j > 0) {
                ok = __all_sync(0xffffffffu, mbar_wait(p_empty + t, (j - 1) & 1, abort_flag, a.err));
                if (!ok) break;
            }
            if constexpr (!STATIC) {
                if (__any_sync(0xffffffffu, factor != 1.0f)) {
                    // Rescale this row of O_t (PV_t(j-1) is complete).
                    tc_fence_after();
                    uint32_t o[32];
#pragma unroll
                    for (int h = 0; h < 2; h++) {
                        FO_TMEM_LD32(o_tm + 32 * h, o);
                        tmem_wait_ld();
#pragma unroll
                        for (int i = 0; i < 32; i++) o[i] = __float_as_uint(__uint_as_float(o[i]) * factor);
                        FO_TMEM_ST32(o_tm + 32 * h, o);
                    }
                    tmem_wait_st();
                }
            }
            // P_t row r (keys 2i, 2i+1 in the low, high half of column i).
            FO_TMEM_ST32(p_tm, (pk + 0));
            FO_TMEM_ST32(p_tm + 32, (pk + 32));
            tmem_wait_st();
            tc_fence_before();
            mbar_arrive(p_full + t);
        }
        if (ok) ok = __all_sync(0xffffffffu, mbar_wait(p_empty + t, (nkv - 1) & 1, abort_flag, a.err));
        if (ok) {
            tc_fence_after();
            uint32_t o[64];
            FO_TMEM_LD32(o_tm, (o + 0));
            FO_TMEM_LD32(o_tm + 32, (o + 32));
            tmem_wait_ld();
            if (SPLIT && row < T) {
                // The range's unnormalized output, its max and denominator.
                const int64_t idx = ((int64_t)part * ((a.pair_end - a.pair_begin) * 256) + (row - a.pair_begin * 256)) * H + head;
                float4 *dst = reinterpret_cast<float4 *>(a.part_o + idx * FO_HD);
#pragma unroll
                for (int i = 0; i < 16; i++)
                    dst[i] = make_float4(__uint_as_float(o[4 * i]), __uint_as_float(o[4 * i + 1]),
                                         __uint_as_float(o[4 * i + 2]), __uint_as_float(o[4 * i + 3]));
                *reinterpret_cast<float2 *>(a.part_ml + idx * 2) = make_float2(STATIC ? 0.0f : m2, l);
            } else if (row < T) {
                const float lse = STATIC ? logf(l) : m2 * 0.69314718055994530942f + logf(l);
                const float ss = sink_scale(a.sinks[head], lse);
                if (a.out_bf16) {
                    // BF16 row to this tile's Q buffer (free once the tile's MMAs
                    // are done): 128-byte rows, 16-byte chunks XOR-swizzled by row.
                    uint8_t *stage = smem + OFF_Q + t * BT_TILE + r * 128;
#pragma unroll
                    for (int c = 0; c < 8; c++) {
                        uint32_t w[4];
#pragma unroll
                        for (int k = 0; k < 4; k++) {
                            const float x0 = (__uint_as_float(o[8 * c + 2 * k]) / l) * ss;
                            const float x1 = (__uint_as_float(o[8 * c + 2 * k + 1]) / l) * ss;
                            w[k] = (uint32_t)bf16_rne(x0) | ((uint32_t)bf16_rne(x1) << 16);
                        }
                        *reinterpret_cast<uint4 *>(stage + ((c ^ (r & 7)) << 4)) = make_uint4(w[0], w[1], w[2], w[3]);
                    }
                } else {
                    const int64_t at = (row * H + head) * FO_HD;
#pragma unroll
                    for (int i = 0; i < 16; i++) {
                        float4 v;
                        v.x = (__uint_as_float(o[4 * i]) / l) * ss;
                        v.y = (__uint_as_float(o[4 * i + 1]) / l) * ss;
                        v.z = (__uint_as_float(o[4 * i + 2]) / l) * ss;
                        v.w = (__uint_as_float(o[4 * i + 3]) / l) * ss;
                        reinterpret_cast<float4 *>(static_cast<float *>(a.out) + at)[i] = v;
                    }
                }
            }
        }
        if constexpr (!SPLIT) {
            if (a.out_bf16) {
                // The tile's four warps store whole 128-byte rows of one head,
                // coalesced, into this rank's block and every peer's (the
                // head-sharded prefill's gather as NVLink stores).  The barrier
                // is reached once by all four warps; rows of a warp whose waits
                // gave up are not stored.
                __shared__ int ok_w[2][4];
                if (lane == 0) ok_w[t][wq] = ok;
                asm volatile("bar.sync %0, 128;" ::"r"(1 + t) : "memory");
                const uint8_t *stage = smem + OFF_Q + t * BT_TILE;
#pragma unroll 2
                for (int it = 0; it < 8; it++) {
                    const int rr = wq * 32 + it * 4 + (lane >> 3), c = lane & 7;
                    const int64_t grow = q0 + 128 * t + rr;
                    if (grow < T && ok_w[t][rr >> 5]) {
                        const uint4 v = *reinterpret_cast<const uint4 *>(stage + rr * 128 + ((c ^ (rr & 7)) << 4));
                        const int64_t at = (grow * H + head) * FO_HD + 8 * c;
                        *reinterpret_cast<uint4 *>(static_cast<uint16_t *>(a.out) + at) = v;
                        for (int p = 0; p < a.peers.n; p++)
                            *reinterpret_cast<uint4 *>(static_cast<uint16_t *>(a.peers.dst[p]) + at) = v;
                    }
                }
                if (a.peers.n) __threadfence_system();
            }
        }
    } else if (warp == 8) {
        // ------------------------------------------------------ TMA producer
        if (lane == 0) {
            tma_prefetch(&tmk);
            tma_prefetch(&tmv);
            int issued = 0;
            bool ok = true;
            for (int j = 0; j < nkv && ok; j++) {
                const int st = j % BT_STAGES, u = j / BT_STAGES;
                if (u > 0 && !(ok = mbar_wait(k_empty + st, (u - 1) & 1, abort_flag, a.err))) break;
                mbar_expect_tx(k_full + st, BT_TILE);
                tma_load_3d(smem + OFF_K + st * BT_TILE, &tmk, k_full + st, 0, (int)head, 128 * (jbase + j));
                if (u > 0 && !(ok = mbar_wait(v_empty + st, (u - 1) & 1, abort_flag, a.err))) {
                    issued = 2 * j + 1;
                    break;
                }
                mbar_expect_tx(v_full + st, BT_TILE);
                tma_load_3d(smem + OFF_V + st * BT_TILE, &tmv, v_full + st, 0, (int)kv_head, 128 * (jbase + j));
                issued = 2 * j + 2;
            }
            if (!ok) {
                // Unwinding: let the copies still in flight land before exit.
                for (int i = max(0, issued - 2 * BT_STAGES); i < issued; i++) {
                    const int j = i >> 1, st = j % BT_STAGES;
                    drain_wait((i & 1) ? v_full + st : k_full + st, (j / BT_STAGES) & 1);
                }
            }
        }
    } else {
        // ------------------------------------------------------- MMA issuer
        // The whole warp runs the loop and its waits, so descriptors and
        // addresses stay warp-uniform (uniform registers); one elected lane
        // issues each group of MMAs and its commits.
        {
            const uint32_t idS = idesc_bf16(128, 128, 0), idPV = idesc_bf16(128, 64, 1);
            // Descriptors are built once; a K step or stage only moves the
            // start-address field (16-byte units, no carry below 256 KB).
            const uint64_t dQ = sdesc_sw128(sQ, 16, 1024), dK = sdesc_sw128(sK, 16, 1024);
            const uint64_t dV = sdesc_sw128(sV, BT_TILE, 1024);
            constexpr uint32_t TILE16 = BT_TILE >> 4;
            auto issue_s = [&](int t, int st) {
                const uint64_t a = dQ + t * TILE16, b = dK + st * TILE16;
                const uint32_t d = tmem + 128 * t;
                if (elect_one()) {
                    mma_bf16(d, a, b, idS, 0);
#pragma unroll
                    for (int kk = 1; kk < 4; kk++) mma_bf16(d, a + 2 * kk, b + 2 * kk, idS, 1);
                    mma_commit(s_full + t);
                }
                __syncwarp();
            };
            auto issue_pv = [&](int t, int st, int j) {
                const uint32_t a = tmem + 384 + 64 * t;  // P_t: 8 columns per 16 keys
                const uint64_t b = dV + st * TILE16;
                const uint32_t d = tmem + 256 + 64 * t;
                if (elect_one()) {
                    mma_bf16_ts(d, a, b, idPV, j > 0);
#pragma unroll
                    for (int kk = 1; kk < 8; kk++) mma_bf16_ts(d, a + 8 * kk, b + kk * (2048 >> 4), idPV, 1);
                    mma_commit(p_empty + t);
                }
                __syncwarp();
            };
            auto commit = [&](uint64_t *bar) {
                if (elect_one()) mma_commit(bar);
                __syncwarp();
            };
            bool ok = mbar_wait(q_full, 0, abort_flag, a.err) && mbar_wait(k_full, 0, abort_flag, a.err);
            ok = __all_sync(0xffffffffu, ok);
            if (ok) {
                tc_fence_after();
                issue_s(0, 0);
                issue_s(1, 0);
                commit(k_empty + 0);
            }
            // Issue order: S_t(j) and PV_t(j) in increasing j for each tile t,
            // but the two tiles do not wait for each other: the warp polls
            // every pending operation's barriers and issues whichever is
            // ready (S_t(j + 1) needs K(j + 1) and the softmax's load of
            // S_t(j); PV_t(j) needs V(j) and P_t(j)).  A K (V) stage is
            // released once both tiles' S (PV) have been issued from it.
            int ns[2] = {1, 1}, np[2] = {0, 0};  // next S and PV index per tile
            uint64_t t_last = globaltimer();
            while (ok && (np[0] < nkv || np[1] < nkv)) {
                bool progress = false;
#pragma unroll
                for (int t = 0; t < 2; t++) {
                    const int js = ns[t];
                    if (js < nkv) {
                        const int st = js % BT_STAGES;
                        bool ready = mbar_try_wait(k_full + st, (js / BT_STAGES) & 1) &&
                                     mbar_try_wait(s_empty + t, (js - 1) & 1);
                        ready = __shfl_sync(0xffffffffu, ready, 0);
                        if (ready) {
                            tc_fence_after();
                            issue_s(t, st);
                            ns[t] = js + 1;
                            if (ns[t ^ 1] > js) commit(k_empty + st);  // both tiles are done with K(js)
                            progress = true;
                        }
                    }
                    const int jp = np[t];
                    if (jp < nkv && jp < ns[t]) {
                        const int st = jp % BT_STAGES;
                        bool ready = mbar_try_wait(v_full + st, (jp / BT_STAGES) & 1) &&
                                     mbar_try_wait(p_full + t, jp & 1);
                        ready = __shfl_sync(0xffffffffu, ready, 0);
                        if (ready) {
                            tc_fence_after();
                            issue_pv(t, st, jp);
                            np[t] = jp + 1;
                            if (np[t ^ 1] > jp) commit(v_empty + st);  // both tiles are done with V(jp)
                            progress = true;
                        }
                    }
                }
                if (progress) {
                    t_last = globaltimer();
                } else if (globaltimer() - t_last > FO_WAIT_NS || *abort_flag) {
                    // Nothing became ready within the bound: unwind.
                    if (lane == 0 && !*abort_flag) {
                        *abort_flag = 1;
                        if (a.err) atomicOr(a.err, FO_DEVERR_WAIT_TIMEOUT);
                    }
                    ok = false;
                }
                ok = __shfl_sync(0xffffffffu, ok, 0);
            }
            // Every issued MMA completes before TMEM is released.
            commit(mma_done);
            if (lane == 0) drain_wait(mma_done, 0);
            __syncwarp();
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 9) {
        tc_fence_after();
        tmem_dealloc(tmem, TMEM_COLS);
    }
}

// Combines the key ranges of a split launch in range order and applies the
// sink: a warp per (row, head), two output dimensions per lane.  Static shift:
// the ranges' outputs and denominators add (one fixed shift); online: each is
// scaled by 2^(m_r - M) first.
template <bool STATIC>
__global__ void __launch_bounds__(256) prefill_split_merge_kernel(const float *part_o, const float *part_ml,
                                                                  const float *sinks, void *out, int out_bf16,
                                                                  int64_t span, int64_t base, int64_t H, int64_t row0,
                                                                  int64_t rows, int n_split,
                                                                  const __grid_constant__ fo_peer_out peers) {
    const int64_t w = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
    if (w >= rows * H) return;
    const int lane = threadIdx.x & 31;
    const int64_t row = row0 + w / H, head = w % H;
    float M = 0.0f;
    if constexpr (!STATIC) {
        M = -INFINITY;
        for (int r = 0; r < n_split; r++) M = rmax(M, part_ml[(((int64_t)r * span + row - base) * H + head) * 2]);
    }
    float l = 0.0f, o0 = 0.0f, o1 = 0.0f;
    for (int r = 0; r < n_split; r++) {
        const int64_t idx = ((int64_t)r * span + row - base) * H + head;
        const float2 ml = *reinterpret_cast<const float2 *>(part_ml + idx * 2);
        float f = 1.0f;
        if constexpr (!STATIC) {
            if (ml.x == -INFINITY) continue;
            f = exp2f(__fsub_rn(ml.x, M));
        }
        const float2 o = *reinterpret_cast<const float2 *>(part_o + idx * FO_HD + 2 * lane);
        o0 = fmaf(o.x, f, o0);
        o1 = fmaf(o.y, f, o1);
        l = fmaf(ml.y, f, l);
    }
    const float lse = STATIC ? logf(l) : M * 0.69314718055994530942f + logf(l);
    const float ss = sink_scale(sinks[head], lse);
    const float y0 = (o0 / l) * ss, y1 = (o1 / l) * ss;
    const int64_t at = (row * H + head) * FO_HD + 2 * lane;
    if (out_bf16) {
        const uint32_t w = (uint32_t)bf16_rne(y0) | ((uint32_t)bf16_rne(y1) << 16);
        *reinterpret_cast<uint32_t *>(static_cast<uint16_t *>(out) + at) = w;
        for (int p = 0; p < peers.n; p++) *reinterpret_cast<uint32_t *>(static_cast<uint16_t *>(peers.dst[p]) + at) = w;
        if (peers.n) __threadfence_system();
    } else {
        *reinterpret_cast<float2 *>(static_cast<float *>(out) + at) = make_float2(y0, y1);
    }
}

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn) {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }
    return fn;
}

// [rows][heads][64] BF16, box of 128 rows of one head, 128-byte swizzle.
static bool make_map(CUtensorMap *m, const uint16_t *base, int64_t rows, int64_t heads) {
    auto fn = encode_fn();
    if (!fn) return false;
    cuuint64_t dims[3] = {64, (cuuint64_t)heads, (cuuint64_t)rows};
    cuuint64_t strides[2] = {64 * 2, (cuuint64_t)heads * 64 * 2};
    cuuint32_t box[3] = {64, 1, 128};
    cuuint32_t estr[3] = {1, 1, 1};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<uint16_t *>(base), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace fo

extern "C" cudaError_t fo_launch_prefill_bf16(const float *q, const uint16_t *keys_bf16, const uint16_t *values_bf16,
                                              const float *sinks, void *out, int out_bf16, int64_t total,
                                              int64_t n_heads,
                                              int64_t n_kv_heads, int64_t image_start, int64_t image_end,
                                              int64_t query_begin, int64_t query_end, int softmax_static, int exp_fast,
                                              unsigned *err, int n_split, float *part_o, float *part_ml,
                                              const fo_peer_out *peers, cudaStream_t stream) {
    (void)exp_fast;  // the tensor-core softmax always takes the hardware exp2
    fo_peer_out none{};
    const fo_peer_out po = peers ? *peers : none;
    if (po.n < 0 || po.n > FO_MAX_PEERS || (po.n > 0 && !out_bf16)) return cudaErrorInvalidValue;
    if (total == 0 || query_end <= query_begin) return cudaSuccess;
    if (n_split < 1 || (n_split > 1 && (!part_o || !part_ml))) return cudaErrorInvalidValue;
    CUtensorMap mk, mv;
    if (!fo::make_map(&mk, keys_bf16, total, n_heads) || !fo::make_map(&mv, values_bf16, total, n_kv_heads))
        return cudaErrorInvalidValue;
    const int64_t pb = query_begin / 256, pe = (query_end + 255) / 256;
    fo::Bf16Args args{q, sinks, out, out_bf16 != 0, err, total, n_heads, n_kv_heads, image_start, image_end, pb, pe,
                      n_split, part_o, part_ml, po};
    if ((pe - pb) * n_split > 65535) return cudaErrorInvalidValue;  // grid y limit
    dim3 grid((unsigned)n_heads, (unsigned)((pe - pb) * n_split));
    auto launch = [&](auto kernel) -> cudaError_t {
        cudaError_t e =
            cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)fo::SMEM_BYTES);
        if (e != cudaSuccess) return e;
        kernel<<<grid, fo::BT_THREADS, fo::SMEM_BYTES, stream>>>(mk, mv, args);
        return cudaGetLastError();
    };
    if (n_split == 1)
        return softmax_static ? launch(fo::prefill_bf16_kernel<true, false>)
                              : launch(fo::prefill_bf16_kernel<false, false>);
    cudaError_t e = softmax_static ? launch(fo::prefill_bf16_kernel<true, true>)
                                   : launch(fo::prefill_bf16_kernel<false, true>);
    if (e != cudaSuccess) return e;
    const int64_t rows = query_end - query_begin;
    const unsigned blocks = (unsigned)((rows * n_heads + 7) / 8);
    if (softmax_static)
        fo::prefill_split_merge_kernel<true><<<blocks, 256, 0, stream>>>(part_o, part_ml, sinks, out, out_bf16,
                                                                         (pe - pb) * 256, pb * 256, n_heads,
                                                                         query_begin, rows, n_split, po);
    else
        fo::prefill_split_merge_kernel<false><<<blocks, 256, 0, stream>>>(part_o, part_ml, sinks, out, out_bf16,
                                                                          (pe - pb) * 256, pb * 256, n_heads,
                                                                          query_begin, rows, n_split, po);
    return cudaGetLastError();
}
