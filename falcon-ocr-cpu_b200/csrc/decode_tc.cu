// decode_tc.cu -- split-cache verify decode over BF16 records on the sm_100a
// tensor cores (reference: SplitPrefix::attention_decode_rows and its per-group
// kernel pair_rows, src/quant/kv.rs:856-972, src/quant/kv/decode.rs:551-677;
// merge and sink, src/quant/kv.rs:775-813).
//
// The CUDA-core decode (decode.cu) spends ~20 FP32 instructions per (key,
// group) on five verify rows and runs at a quarter of HBM speed.  Here the
// dot products go to tcgen05 and the CUDA cores only run the softmax:
//
//   split     128 keys of one KV group: of the prefix records, or of the tail
//             records (splits never straddle the two, so a split is one TMA
//             tile; the partition depends only on prefix_len, so every verify
//             row still equals its single-row decode bit for bit);
//   unit      `chunk` consecutive splits of one group (chunk chosen from the
//             prefix length so that the units about fill the GPU); a CTA
//             walks whole units and leaves one partial per unit and row;
//   TMA warps (warps 8 and 11) boxes of 128 records in two 4-stage rings:
//             the keys ([T|S0] in 64-element boxes with the 128-byte
//             swizzle and [S1] in 32-element boxes with the 64-byte swizzle
//             of prefix records, [K] of tail records), freed when their QK
//             is done, and the values ([V]), freed when their PV is done;
//   QK warp   (warp 9) S = keys x Q' (M128 K64, keys in TMEM lanes: the temporal
//             half for both heads at N64, each spatial half at N32), S and P'
//             double-buffered;
//   PV warp   (warp 10) O += P' x V (M64 N64 K128), summed in TMEM over the
//             whole unit;
//   8 warps   (warps 0-7) one thread per (head, key): logits, p = exp(s -
//             m_ref) against the row's reference maximum, P' to shared memory,
//             and the thread's share of the row sums l.  m_ref is the unit's
//             first maximum and moves only when a split's maximum passes it by
//             more than TAU (a vote of the head's four warps); the head's two
//             warps whose TMEM lane quadrants hold its O rows then rescale O in
//             place, and write the unit's partial at its end.  The split merge
//             (decode.cu) follows as a programmatic dependent launch.
//
// Exactness: Q' holds each FP32 query as three BF16 terms (hi + mid + lo ==
// q exactly), so every product with a BF16 key is exact and S is the FP32
// dot product up to accumulation order.  P' holds each probability as two
// BF16 terms (hi + lo == p to 2^-18) in two groups of M rows, which the
// unit's end adds; the row sums add the FP32 p.  The output agrees
// with the reference's FP32 decode over the same records within
// 1e-5 * (1 + |b|).
//
// Verify rows: every row's logits, maxima, O and l columns come from its own
// query and keys only, with the same instructions whatever the number of
// rows (a row's reference maximum moves on its own keys only; a rescale
// multiplies the other rows by exactly 1), and a split that holds none of a
// row's keys leaves that row's unit partial untouched.  Keys a row does not see get p = 0; with finite values
// that adds an exact zero to its O column.  A non-finite value in one of the
// last rows - 1 positions (a NaN draft) is taken out of the MMA and added by
// the CUDA cores to exactly the rows that see it.  Positions past the cache's
// end are zero in memory (seal clears the tail, truncation clears what it
// drops) or lie outside the tensor map, so they add nothing either.
#include <cudaTypedefs.h>

#include <algorithm>
#include <atomic>

#include "fo_common.cuh"
#include "fo_kernels.h"
#include "sm100.cuh"

namespace fo {
namespace tc {
using namespace sm100;

constexpr int KEY_WARPS = 8;
constexpr int THREADS = 384;  // warps 0-7 (head, key), 8 key TMA, 9 QK issue, 10 PV issue, 11 value TMA
constexpr int W_TMA = 8, W_QK = 9, W_PV = 10, W_VTMA = 11;
// Separate rings for the keys and the values of a split: a key stage is
// free once its QK is done, a value stage once its PV is.
constexpr int KST = 4, VST = 4;
// A row's reference maximum moves only when a split's maximum passes it by
// more than TAU, so probabilities stay below e^8 and O is rescaled in TMEM
// only then (never, for ordinary data, after a unit's first split).
constexpr float TAU = 8.0f;
constexpr uint32_t BOX = 128 * 128;        // 128 records x 128 bytes (64 BF16, 128-byte swizzle)
constexpr uint32_t HBOX = 128 * 64;        // 128 records x 64 bytes (32 BF16, 64-byte swizzle)
constexpr uint32_t KSTAGE = BOX + HBOX;    // [T|S0] and [S1] of a prefix split, [K] of a tail split
constexpr uint32_t OFF_V = KST * KSTAGE;   // value ring: [V] boxes
constexpr uint32_t QTILE = 32 * 128;       // Q' of one head: 32 rows x 64 BF16
constexpr uint32_t OFF_Q = OFF_V + VST * BOX;
constexpr uint32_t OFF_P = OFF_Q + 2 * 2 * QTILE;  // two Q' buffers x two heads
// P' double buffer: [key][64 M rows] BF16, M row = 32 * head + 16 * term + row
// (term 0 = hi, 1 = lo), i.e. 16-byte chunk 4 * head + 2 * term of the key's
// row; the odd chunks stay zero.  An M64 MMA puts M rows 16q .. 16q + 15 in
// TMEM lanes 32q .. 32q + 15, so head h's hi rows of O lie in lane quadrant
// 2h and its lo rows in quadrant 2h + 1: the head's own key warps of those
// quadrants can rescale and read them.
constexpr uint32_t OFF_RED = OFF_P + 2 * BOX;
// per-warp row maxima of a split, [split parity][2 heads][4 warps][8 rows],
// then per-warp row sums of a unit, [2 heads][4 warps][8 rows]
constexpr uint32_t RED_FLOATS = 2 * 2 * 4 * 8 + 2 * 4 * 8;
constexpr uint32_t OFF_WIN = OFF_RED + RED_FLOATS * 4;
// draft-window list of each head's current unit, 32-bit words: { count,
// tail row[8], p[8 keys][8 rows], reference max[8 keys][8 rows] }
constexpr uint32_t WIN_WORDS = 1 + 8 + 64 + 64;
constexpr uint32_t ACC_STRIDE = 68;
// O's lo rows handed from a head's lo warp to its hi warp at a unit's end:
// [2 heads][8 rows][68] floats.
constexpr uint32_t OFF_LO = (OFF_WIN + 2 * WIN_WORDS * 4 + 15) / 16 * 16;
constexpr uint32_t OFF_BAR = OFF_LO + 2 * 8 * ACC_STRIDE * 4;
// k_full[4] k_empty[4] v_full[4] v_empty[4] s_full[2] s_empty[2] q_full[2] p_full pv_done[2] qk_drain pv_drain
constexpr int NBAR = 2 * KST + 2 * VST + 2 + 2 + 2 + 1 + 2 + 2;
// after the barriers: TMEM address and abort flag
constexpr uint32_t SMEM = OFF_BAR + NBAR * 8 + 16 + 1024;
// S double-buffered [0, 128); O [128, 192), summed over a unit.
constexpr uint32_t TMEM_COLS = 256;
constexpr uint32_t TM_O = 128;
static_assert(SMEM <= 227 * 1024, "shared memory per CTA");

// Instruction descriptor, kind::f16, BF16 inputs, FP32 accumulator.
__host__ __device__ constexpr uint32_t idesc(uint32_t m, uint32_t n, uint32_t a_mn, uint32_t b_mn) {
    return (1u << 4) | (1u << 7) | (1u << 10) | (a_mn << 15) | (b_mn << 16) | ((n >> 3) << 17) | ((m >> 4) << 24);
}

struct Args {
    int64_t H, prefix_len, last, len0;  // len0 = last - rows + 1: keys every row sees
    int32_t prefix_splits, tail_splits, chunk, prefix_units, units;  // units per group and row
    uint32_t n_units;                                                 // groups x units (< 2^24)
};

__device__ __forceinline__ void drain_wait(uint64_t *bar, uint32_t phase) {
    const uint64_t t0 = globaltimer();
    while (!mbar_try_wait(bar, phase))
        if (globaltimer() - t0 > FO_WAIT_NS) break;
}

// Named barriers of head h's four key warps: 1 + h, the per-split vote on
// whether any row's reference maximum moves; 3 + h, the meeting at a unit's
// end; 5 + h (64 threads), its hi and lo warps there.  Every warp passes each of
// them the same number of times, also after a bounded wait gave up (it then
// skips the work), so no warp waits for one that left.
__device__ __forceinline__ bool vote_head(int h, bool v) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 q, %1, 0;\n\tbar.red.or.pred p, %2, 128, q;\n\tselp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(r)
        : "r"((uint32_t)v), "r"(1 + h)
        : "memory");
    return r != 0;
}
__device__ __forceinline__ void bar_named(int id, int n) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
}

__device__ __forceinline__ float warp_max_redux(float v) {
    float r;
    asm volatile("redux.sync.max.f32 %0, %1, 0xffffffff;" : "=f"(r) : "f"(v));
    return r;
}

// The decode's exp: CUDA's SFU exp2 of x * log2(e) (within 2e-7 relative of
// expf for the softmax's x <= 0 down to -20, and underflowing like it), or the
// reference's exp_poly when the cache asks for its fast exp.
template <bool FAST>
__device__ __forceinline__ float key_exp(float x) {
    if constexpr (FAST) {
        return exp_poly(x);
    } else {
        return ex2(__fmul_rn(x, 1.44269504088896340736f));
    }
}

// Walks a CTA's units and their splits in order: group, split index, and
// whether the split opens or closes its unit.
struct Walk {
    uint32_t U, U_end;
    int g;                     // unit, end, the unit's group
    int u, s, s_first, s_end;  // the unit's index within its group, split, first and end split
    __device__ __forceinline__ void unit_bounds(const Args &a) {
        if (u < a.prefix_units) {
            s = u * a.chunk;
            s_end = min(s + a.chunk, a.prefix_splits);
        } else {
            s = a.prefix_splits + (u - a.prefix_units) * a.chunk;
            s_end = min(s + a.chunk, a.prefix_splits + a.tail_splits);
        }
        s_first = s;
    }
    __device__ __forceinline__ void start(const Args &a, uint32_t u0, uint32_t u1) {
        U = u0;
        U_end = u1;
        g = (int)(U / (uint32_t)a.units);  // the walk's one division
        u = (int)U - g * a.units;
        s = s_first = s_end = 0;
        if (U < U_end) unit_bounds(a);
    }
    __device__ __forceinline__ bool valid() const { return U < U_end; }
    __device__ __forceinline__ int group(const Args &) const { return g; }
    __device__ __forceinline__ int unit(const Args &) const { return u; }
    __device__ __forceinline__ bool first_of_unit() const { return s == s_first; }
    __device__ __forceinline__ bool last_of_unit() const { return s + 1 == s_end; }
    __device__ __forceinline__ void next(const Args &a) {
        if (++s >= s_end && ++U < U_end) {
            if (++u == a.units) {
                u = 0;
                g++;
            }
            unit_bounds(a);
        }
    }
};

// A split's positions [k0, k1) and its first record row in its map.
struct Split {
    int64_t k0, k1;
    bool tail;
    int row0;
};
__device__ __forceinline__ Split split_of(const Args &a, int s) {
    Split x;
    if (s < a.prefix_splits) {
        x.k0 = (int64_t)s * 128;
        x.k1 = min64(x.k0 + 128, a.prefix_len);
        x.tail = false;
        x.row0 = s * 128;
    } else {
        const int t = s - a.prefix_splits;
        x.k0 = a.prefix_len + (int64_t)t * 128;
        x.k1 = min64(x.k0 + 128, a.last);
        x.tail = true;
        x.row0 = t * 128;
    }
    return x;
}

// The key boxes of local split i (the walk's current split) into key stage
// i mod KST: [T|S0] and [S1] of a prefix split, [K] of a tail split.
__device__ __forceinline__ void issue_k(const fo_decode_page &pg, const Args &a, uint8_t *smem, uint64_t *k_full,
                                        const Walk &wk, int i) {
    const int st = i % KST;
    const int g = wk.group(a);
    const Split x = split_of(a, wk.s);
    uint8_t *dst = smem + st * KSTAGE;
    // Records are read once per call: first out of L2.
    const uint64_t pol = l2_evict_first();
    if (!x.tail) {
        mbar_expect_tx(k_full + st, BOX + HBOX);
        tma_load_3d_hint(dst, &pg.tc_map, k_full + st, 0, x.row0, g, pol);
        tma_load_3d_hint(dst + BOX, &pg.s1_map, k_full + st, 64, x.row0, g, pol);
    } else {
        mbar_expect_tx(k_full + st, BOX);
        tma_load_3d_hint(dst, &pg.tail_map, k_full + st, 0, x.row0, g, pol);
    }
}

// The value box of local split i into value stage i mod VST.
__device__ __forceinline__ void issue_v(const fo_decode_page &pg, const Args &a, uint8_t *smem, uint64_t *v_full,
                                        const Walk &wk, int i) {
    const int st = i % VST;
    const int g = wk.group(a);
    const Split x = split_of(a, wk.s);
    const uint64_t pol = l2_evict_first();
    mbar_expect_tx(v_full + st, BOX);
    tma_load_3d_hint(smem + OFF_V + st * BOX, x.tail ? &pg.tail_map : &pg.tc_map, v_full + st, x.tail ? 64 : 96,
                     x.row0, g, pol);
}

// Q' of group g's head h into buffer qb (kept out of the per-split loop):
// thread key < 64 takes (row r, 8-dimension chunk c) and writes the three
// BF16 terms of q[r][2g + h] (hi, mid, lo; their sum is the FP32 value).
__device__ __noinline__ void build_qprime(const float *q, uint8_t *smem, int64_t H, int g, int h, int key, int qb,
                                          int R) {
    const int r = key >> 3, c = key & 7;
    if (key >= 64 || r >= R) return;
    const float4 *src = reinterpret_cast<const float4 *>(q + ((int64_t)r * H + 2 * g + h) * FO_HD + 8 * c);
    const float4 x0 = __ldg(src), x1 = __ldg(src + 1);
    const float v[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
    uint32_t wv[3][4];
#pragma unroll
    for (int e = 0; e < 4; e++) {
        float hi[2], mi[2], lo[2];
#pragma unroll
        for (int k2 = 0; k2 < 2; k2++) {
            const float xv = v[2 * e + k2];
            hi[k2] = bf16_f32(bf16_rne(xv));
            const float r1 = __fsub_rn(xv, hi[k2]);
            mi[k2] = bf16_f32(bf16_rne(r1));
            lo[k2] = __fsub_rn(r1, mi[k2]);
        }
        wv[0][e] = pack_bf16(hi[0], hi[1]);
        wv[1][e] = pack_bf16(mi[0], mi[1]);
        wv[2][e] = pack_bf16(lo[0], lo[1]);
    }
#pragma unroll
    for (int term = 0; term < 3; term++) {
        const int row = term * 8 + r;
        const uint32_t addr = smem_u32(smem + OFF_Q + (qb * 2 + h) * QTILE + row * 128) + ((c ^ r) << 4);
        st_shared_v4(addr, wv[term][0], wv[term][1], wv[term][2], wv[term][3]);
    }
}

// A unit's end for the head's hi and lo warps (lo_warp: the lo one), kept
// out of the per-split loop (it runs once per unit): once the unit's last PV
// is in, the lo warp hands O's lo rows over through shared memory and the hi
// warp adds them to its hi rows, adds the draft window's non-finite values
// (the list the key warps recorded, factors rebased to the final reference
// maximum) and writes the unit's partial (lane r: row r) with the row sums
// the four warps left in shared memory.  Both warps pass the pair's named
// barrier whatever happened; a failed wait (ok false) skips the work.
__device__ __noinline__ void unit_partial(const fo_decode_page &pg, uint8_t *smem, uint32_t tq, int h, bool lo_warp,
                                          int lane, int R, bool ok, float m_fin, uint64_t *pv_done,
                                          uint32_t phase, volatile int *abort_flag, int64_t H, int g, int unit,
                                          int64_t prefix_len, int64_t len0) {
    const float NEG_INF = -INFINITY;
    const float *lsum = reinterpret_cast<const float *>(smem + OFF_RED) + 2 * 2 * 4 * 8 + h * 32;
    int *win = reinterpret_cast<int *>(smem + OFF_WIN) + h * WIN_WORDS;
    const bool o_ok = ok && __all_sync(0xffffffffu, mbar_wait(pv_done, phase, abort_flag, pg.err));
    if (o_ok) tc_fence_after();
    float *lo = reinterpret_cast<float *>(smem + OFF_LO) + (h * 8 + (lane & 7)) * ACC_STRIDE;
    if (lo_warp && o_ok) {
        for (int half = 0; half < 2; half++) {
            uint32_t o[32];
            FO_TMEM_LD32(tq + TM_O + 32 * half, o);
            tmem_wait_ld();
            if (lane < R) {
                float4 *dst = reinterpret_cast<float4 *>(lo + 32 * half);
#pragma unroll
                for (int d = 0; d < 8; d++)
                    dst[d] = make_float4(__uint_as_float(o[4 * d]), __uint_as_float(o[4 * d + 1]),
                                         __uint_as_float(o[4 * d + 2]), __uint_as_float(o[4 * d + 3]));
            }
        }
    }
    bar_named(5 + h, 64);
    if (!lo_warp && o_ok) {
        const int64_t row_head = (int64_t)lane * H + 2 * g + h;
        const int64_t idx = row_head * pg.splits + unit;
        float4 *dst = reinterpret_cast<float4 *>(pg.part_o + idx * FO_HD);
        const bool live = lane < R && m_fin != NEG_INF;
        const int nw = live ? win[0] : 0;
        const float *wp = reinterpret_cast<const float *>(win + 9);
        const float *wm = reinterpret_cast<const float *>(win + 9 + 64);
        for (int half = 0; half < 2; half++) {
            uint32_t o[32];
            FO_TMEM_LD32(tq + TM_O + 32 * half, o);
            tmem_wait_ld();
            if (live) {
                float ov[32];
                const float4 *lv = reinterpret_cast<const float4 *>(lo + 32 * half);
#pragma unroll
                for (int d = 0; d < 8; d++) {
                    const float4 l4 = lv[d];
                    ov[4 * d] = __fadd_rn(__uint_as_float(o[4 * d]), l4.x);
                    ov[4 * d + 1] = __fadd_rn(__uint_as_float(o[4 * d + 1]), l4.y);
                    ov[4 * d + 2] = __fadd_rn(__uint_as_float(o[4 * d + 2]), l4.z);
                    ov[4 * d + 3] = __fadd_rn(__uint_as_float(o[4 * d + 3]), l4.w);
                }
                for (int e = 0; e < nw; e++) {
                    const int tr = win[1 + e];
                    if (prefix_len + tr >= len0 + lane) continue;  // this row does not see it
                    const float pk = __fmul_rn(wp[e * 8 + lane], expf(__fsub_rn(wm[e * 8 + lane], m_fin)));
                    const uint16_t *vr = reinterpret_cast<const uint16_t *>(pg.tail_codes) +
                                         ((int64_t)g * pg.tail_stride + tr) * FO_TAIL_RECORD + 64 + 32 * half;
#pragma unroll
                    for (int d = 0; d < 32; d++) ov[d] = fmaf(pk, bf16_f32(vr[d]), ov[d]);
                }
#pragma unroll
                for (int d = 0; d < 8; d++)
                    dst[half * 8 + d] = make_float4(ov[4 * d], ov[4 * d + 1], ov[4 * d + 2], ov[4 * d + 3]);
            } else if (lane < R) {
                // No key of the unit is this row's: an empty partial.
#pragma unroll
                for (int d = 0; d < 8; d++) dst[half * 8 + d] = make_float4(0.f, 0.f, 0.f, 0.f);
            }
        }
        if (lane < R) {
            float l_run = 0.0f;
            if (live)
                l_run = __fadd_rn(__fadd_rn(__fadd_rn(lsum[lane], lsum[8 + lane]), lsum[16 + lane]), lsum[24 + lane]);
            *reinterpret_cast<float2 *>(pg.part_ml + idx * 2) = make_float2(m_fin, l_run);
        }
    }
    if (o_ok) tc_fence_before();
    if (!lo_warp) {
        __syncwarp();
        if (lane == 0) win[0] = 0;  // this warp is the list's last reader
    }
}

template <bool FAST, int R>
__global__ void __launch_bounds__(THREADS, 1)
    decode_tc_kernel(const __grid_constant__ fo_decode_page pg, const Args a) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + OFF_BAR);
    uint64_t *k_full = bars, *k_empty = k_full + KST, *v_full = k_empty + KST, *v_empty = v_full + VST;
    uint64_t *s_full = v_empty + VST, *s_empty = s_full + 2, *q_full = s_empty + 2;
    uint64_t *p_full = q_full + 2, *pv_done = p_full + 1, *qk_drain = pv_done + 2, *pv_drain = qk_drain + 1;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + NBAR);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t u0 = blockIdx.x * a.n_units / gridDim.x;
    const uint32_t u1 = (blockIdx.x + 1) * a.n_units / gridDim.x;

    // The key TMA thread starts the first loads of both rings before anything
    // else and sets the other barriers up before the CTA-wide barrier (the
    // ring buffers are not touched by the rest of the setup).
    Walk twk;
    int t_issued = 0;
    if (threadIdx.x == W_TMA * 32) {
        for (int s = 0; s < KST; s++) {
            mbar_init(k_full + s, 1);
            mbar_init(k_empty + s, 1);
        }
        for (int s = 0; s < VST; s++) {
            mbar_init(v_full + s, 1);
            mbar_init(v_empty + s, 1);
        }
        mbar_fence_init();
        tma_prefetch(&pg.tc_map);
        tma_prefetch(&pg.s1_map);
        Walk vwk;
        vwk.start(a, u0, u1);
        twk.start(a, u0, u1);
        for (int i = 0; i < KST || i < VST; i++) {
            if (i < KST && twk.valid()) {
                issue_k(pg, a, smem, k_full, twk, i);
                t_issued = i + 1;
                twk.next(a);
            }
            if (i < VST && vwk.valid()) {
                issue_v(pg, a, smem, v_full, vwk, i);
                vwk.next(a);
            }
        }
        for (int b = 0; b < 2; b++) {
            mbar_init(s_full + b, 1);
            mbar_init(s_empty + b, KEY_WARPS);
            mbar_init(q_full + b, KEY_WARPS);
            mbar_init(pv_done + b, 1);
        }
        mbar_init(p_full, KEY_WARPS);
        mbar_init(qk_drain, 1);
        mbar_init(pv_drain, 1);
        *abort_flag = 0;
        mbar_fence_init();
        if (pg.has_tail_map) tma_prefetch(&pg.tail_map);
    }
    if (warp < KEY_WARPS) {
        // Zero what the loop never writes: Q' rows of absent verify rows and
        // its padding rows (R..7 of each term, 24..31), and P' chunks 1, 3, 5
        // and 7 of every key's row (both buffers); empty window lists.
        const int t = threadIdx.x;
        for (int idx = t; idx < 2 * 2 * 32 * 8; idx += 32 * KEY_WARPS) {
            const int chunk = idx & 7, row = (idx >> 3) & 31;
            if (row >= 24 || (row & 7) >= R)
                *reinterpret_cast<uint4 *>(smem + OFF_Q + (idx >> 8) * QTILE + row * 128 + ((chunk ^ (row & 7)) << 4)) =
                    make_uint4(0, 0, 0, 0);
        }
        for (int idx = t; idx < 2 * 128 * 4; idx += 32 * KEY_WARPS) {
            const int tile = idx >> 9, key = (idx >> 2) & 127, chunk = 2 * (idx & 3) + 1;
            *reinterpret_cast<uint4 *>(smem + OFF_P + tile * BOX + key * 128 + ((chunk ^ (key & 7)) << 4)) =
                make_uint4(0, 0, 0, 0);
        }
        if (t < 2) reinterpret_cast<int *>(smem + OFF_WIN)[t * WIN_WORDS] = 0;
        fence_proxy_async_smem();
    }
    if (warp == W_PV) tmem_alloc(tmem_slot, TMEM_COLS);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    // The merge kernel may launch now; it waits for this grid to finish.
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

    if (warp == W_TMA) {
        // ------------------------------------------------------ key TMA
        if (lane == 0) {
            bool ok = true;
            for (int i = t_issued; twk.valid() && ok; i++, twk.next(a)) {
                const int st = i % KST, u = i / KST;
                if (!(ok = mbar_wait(k_empty + st, (u - 1) & 1, abort_flag, pg.err))) break;
                issue_k(pg, a, smem, k_full, twk, i);
                t_issued = i + 1;
            }
            if (!ok)
                for (int i = max(0, t_issued - KST); i < t_issued; i++) drain_wait(k_full + i % KST, (i / KST) & 1);
        }
    } else if (warp == W_VTMA) {
        // ---------------------------------------------------- value TMA
        // The key TMA thread issued the first VST value stages.
        if (lane == 0) {
            Walk wk;
            wk.start(a, u0, u1);
            int i = 0, issued = 0;
            for (; i < VST && wk.valid(); i++) wk.next(a);
            issued = i;
            bool ok = true;
            for (; wk.valid() && ok; i++, wk.next(a)) {
                const int st = i % VST, u = i / VST;
                if (!(ok = mbar_wait(v_empty + st, (u - 1) & 1, abort_flag, pg.err))) break;
                issue_v(pg, a, smem, v_full, wk, i);
                issued = i + 1;
            }
            if (!ok)
                for (int j = max(0, issued - VST); j < issued; j++) drain_wait(v_full + j % VST, (j / VST) & 1);
        }
    } else if (warp == W_QK) {
        // ------------------------------------------------------- QK issue
        // S(i) = keys x Q' once the split's records, Q' (on a group change)
        // and S buffer i & 1 are in.
        const uint32_t iT = idesc(128, 64, 0, 0), iS = idesc(128, 32, 0, 0);
        const uint32_t sQ = smem_u32(smem + OFF_Q);
        bool ok = true;
        int q_uses[2] = {0, 0};
        int qb = 1, prev_g = -1;
        Walk wk;
        wk.start(a, u0, u1);
        for (int i = 0; wk.valid() && ok; i++, wk.next(a)) {
            const int st = i % KST, sb = i & 1;
            const int g = wk.group(a);
            if (g != prev_g) {
                qb ^= 1;
                ok = __all_sync(0xffffffffu, mbar_wait(q_full + qb, q_uses[qb] & 1, abort_flag, pg.err));
                q_uses[qb]++;
                prev_g = g;
                if (!ok) break;
            }
            ok = __all_sync(0xffffffffu, mbar_wait(k_full + st, (i / KST) & 1, abort_flag, pg.err));
            if (ok && i >= 2)
                ok = __all_sync(0xffffffffu, mbar_wait(s_empty + sb, ((i - 2) >> 1) & 1, abort_flag, pg.err));
            if (!ok) break;
            tc_fence_after();
            const bool tail = wk.s >= a.prefix_splits;
            const uint32_t b0 = smem_u32(smem + st * KSTAGE), b1 = b0 + BOX;
            const uint64_t dK0 = sdesc_sw128(b0, 16, 1024);
            // Head 1's spatial half: the [S1] box of a prefix record (64-byte
            // rows), the key's own second half in a tail record.
            const uint64_t dK1s = tail ? dK0 + (64 >> 4) : sdesc_sw64(b1, 16, 512);
            const uint64_t dQ0 = sdesc_sw128(sQ + (qb * 2) * QTILE, 16, 1024);
            const uint64_t dQ1 = sdesc_sw128(sQ + (qb * 2 + 1) * QTILE, 16, 1024);
            const uint32_t d = tmem + sb * 64;
            if (elect_one()) {
                // The temporal half against both heads' queries at once (N64:
                // head 1's Q' rows follow head 0's), then each spatial half.
                mma_bf16(d, dK0, dQ0, iT, 0);
                mma_bf16(d, dK0 + 2, dQ0 + 2, iT, 1);
                mma_bf16(d, dK0 + 4, dQ0 + 4, iS, 1);
                mma_bf16(d, dK0 + 6, dQ0 + 6, iS, 1);
                mma_bf16(d + 32, dK1s, dQ1 + 4, iS, 1);
                mma_bf16(d + 32, dK1s + 2, dQ1 + 6, iS, 1);
                mma_commit(s_full + sb);
                mma_commit(k_empty + st);
            }
            __syncwarp();
        }
        if (elect_one()) mma_commit(qk_drain);
        __syncwarp();
        if (lane == 0) drain_wait(qk_drain, 0);
        __syncwarp();
    } else if (warp == W_PV) {
        // ------------------------------------------------------- PV issue
        // O += P'(j) V(j) over the split's 128 keys (8 K16 steps) once P'(j)
        // is in (and O rescaled where the split moved a reference maximum);
        // a unit's first split starts O afresh.  PV(j)'s completion frees P'
        // buffer j & 1 and the split's value stage.
        const uint32_t iPV = idesc(64, 64, 1, 1);
        const uint32_t sP = smem_u32(smem + OFF_P);
        bool ok = true;
        Walk wk;
        wk.start(a, u0, u1);
        for (int j = 0; wk.valid() && ok; j++, wk.next(a)) {
            const int st = j % VST;
            ok = __all_sync(0xffffffffu, mbar_wait(p_full, j & 1, abort_flag, pg.err));
            if (ok) ok = __all_sync(0xffffffffu, mbar_wait(v_full + st, (j / VST) & 1, abort_flag, pg.err));
            if (!ok) break;
            tc_fence_after();
            const bool first = wk.first_of_unit();
            const uint64_t dV = sdesc_sw128(smem_u32(smem + OFF_V + st * BOX), BOX, 1024);
            const uint64_t dP = sdesc_sw128(sP + (j & 1) * BOX, BOX, 1024);
            if (elect_one()) {
#pragma unroll
                for (int kk = 0; kk < 8; kk++)
                    mma_bf16(tmem + TM_O, dP + kk * (2048 >> 4), dV + kk * (2048 >> 4), iPV, kk != 0 || !first);
                mma_commit(pv_done + (j & 1));
                mma_commit(v_empty + st);
            }
            __syncwarp();
        }
        if (elect_one()) mma_commit(pv_drain);
        __syncwarp();
        if (lane == 0) drain_wait(pv_drain, 0);
        __syncwarp();
    } else {
        // ---------------------------------------------- (head, key) warps
        const int h = warp >> 2;         // this warp's head of the group
        const int qd = warp & 3;         // TMEM lane quadrant of this warp (and its index in the head)
        const int key = qd * 32 + lane;  // the key this thread owns in a split
        const bool hi_warp = qd == 2 * h, lo_warp = qd == 2 * h + 1;  // holders of the head's O rows
        const uint32_t tq = tmem + ((uint32_t)(qd * 32) << 16);
        const int64_t H = a.H;
        const float NEG_INF = -INFINITY;
        float *red = reinterpret_cast<float *>(smem + OFF_RED);
        float *lsum = red + 2 * 2 * 4 * 8 + h * 32;  // the head's per-warp row sums [warp][row]
        int *win = reinterpret_cast<int *>(smem + OFF_WIN) + h * WIN_WORDS;
        bool ok = true;
        int qb = 1, prev_g = -1;
        // The unit's reference maxima per row (the same in all the head's
        // threads): every p of the unit is exp(s - m_ref) with the m_ref of
        // its split, O and the row sums follow each move of m_ref.  l_acc:
        // this thread's key slot's share of the row sums.
        float m_ref[R], l_acc[R];
#pragma unroll
        for (int r = 0; r < R; r++) {
            m_ref[r] = NEG_INF;
            l_acc[r] = 0.0f;
        }
        Walk wk;
        wk.start(a, u0, u1);
        for (int i = 0; wk.valid(); i++, wk.next(a)) {
            const int sb = i & 1;
            const int g = wk.group(a);
            const Split x = split_of(a, wk.s);
            float *sm = red + (sb * 2 + h) * 32;  // this split's maxima [warp][row]
            float lg[R];
            bool need = false;
            if (ok && g != prev_g) {
                // Q' of this group's head h: row (term * 8 + r) holds term (hi,
                // mid, lo) of q[r][2g + h], three BF16 values summing to the
                // FP32 query exactly; thread key < 64 takes (row r, 8-dimension
                // chunk c).  The buffer's previous readers (the QK of the group
                // before last) finished before the last split's S was read.
                qb ^= 1;
                build_qprime(pg.q, smem, H, g, h, key, qb, R);
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) mbar_arrive(q_full + qb);
                prev_g = g;
            }
            if (ok) ok = __all_sync(0xffffffffu, mbar_wait(s_full + sb, (i >> 1) & 1, abort_flag, pg.err));
            if (ok) {
                tc_fence_after();
                uint32_t sv[32];
                FO_TMEM_LD32(tq + sb * 64 + h * 32, sv);
                tmem_wait_ld();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(s_empty + sb);
                // Logits of this key for every row: the three query terms'
                // dot products added in a fixed order, scaled by 1/8 (qk_row:
                // s * scale).  Row r sees positions [0, len0 + r).
                const int64_t pos = x.k0 + key;
#pragma unroll
                for (int r = 0; r < R; r++) {
                    const float dot = __fadd_rn(__fadd_rn(__uint_as_float(sv[r]), __uint_as_float(sv[8 + r])),
                                                __uint_as_float(sv[16 + r]));
                    lg[r] = (pos < x.k1 && pos < a.len0 + r) ? __fmul_rn(dot, 0.125f) : NEG_INF;
                }
                // This warp's row maxima; a row whose maximum passes its
                // reference by more than TAU (or gets its first key) asks the
                // head to move the reference.
#pragma unroll
                for (int r = 0; r < R; r++) {
                    const float m = warp_max_redux(lg[r]);
                    if (lane == 0) sm[qd * 8 + r] = m;
                    need |= m_ref[r] == NEG_INF ? m != NEG_INF : m > __fadd_rn(m_ref[r], TAU);
                }
            }
            need = vote_head(h, need);
            if (ok && *abort_flag) ok = false;
            float p[R];
            if (ok) {
                bool rescale = false;
                float alpha[R];
#pragma unroll
                for (int r = 0; r < R; r++) alpha[r] = 1.0f;
                if (need) {
#pragma unroll
                    for (int r = 0; r < R; r++) {
                        float m = NEG_INF;
#pragma unroll
                        for (int ww = 0; ww < 4; ww++) m = rmax(m, sm[ww * 8 + r]);
                        if (m_ref[r] == NEG_INF) {
                            m_ref[r] = m;  // O and the row sums are still zero
                        } else if (m > __fadd_rn(m_ref[r], TAU)) {
                            alpha[r] = expf(__fsub_rn(m_ref[r], m));
                            m_ref[r] = m;
                            l_acc[r] = __fmul_rn(l_acc[r], alpha[r]);
                            rescale = true;
                        }
                    }
                }
#pragma unroll
                for (int r = 0; r < R; r++) {
                    p[r] = lg[r] == NEG_INF ? 0.0f : key_exp<FAST>(__fsub_rn(lg[r], m_ref[r]));
                    l_acc[r] = __fadd_rn(l_acc[r], p[r]);
                }
                if (rescale && (hi_warp || lo_warp)) {
                    // O rows of this head hold the unit so far against the old
                    // references: scale them once PV of the split before (an
                    // earlier split of this unit) is in, before PV of this one.
                    ok = __all_sync(0xffffffffu,
                                    mbar_wait(pv_done + ((i - 1) & 1), ((i - 1) >> 1) & 1, abort_flag, pg.err));
                    if (ok) {
                        tc_fence_after();
                        float al = 1.0f;
#pragma unroll
                        for (int r = 0; r < R; r++)
                            if (lane == r) al = alpha[r];
#pragma unroll
                        for (int half = 0; half < 2; half++) {
                            uint32_t o[32];
                            FO_TMEM_LD32(tq + TM_O + 32 * half, o);
                            tmem_wait_ld();
#pragma unroll
                            for (int d = 0; d < 32; d++) o[d] = __float_as_uint(__fmul_rn(__uint_as_float(o[d]), al));
                            FO_TMEM_ST32(tq + TM_O + 32 * half, o);
                        }
                        tmem_wait_st();
                        tc_fence_before();
                    }
                }
            }
            if (ok) {
                // The draft window [len0, last) of a tail split: a key whose value
                // row holds a non-finite number leaves the MMA (head 0's thread of
                // the key zeroes its staged row) and the unit's end adds it to the
                // rows that see it.  Both heads test the row in global memory, so
                // neither test depends on the other's zeroing.
                const int64_t pos = x.k0 + key;
                bool nonfinite = false;
                if (x.tail && pos >= a.len0 && pos < x.k1) {
                    const uint4 *vg = reinterpret_cast<const uint4 *>(
                        reinterpret_cast<const uint16_t *>(pg.tail_codes) +
                        ((int64_t)g * pg.tail_stride + (pos - a.prefix_len)) * FO_TAIL_RECORD + 64);
#pragma unroll
                    for (int c = 0; c < 8; c++) {
                        const uint4 q4 = vg[c];
                        const uint32_t ws[4] = {q4.x, q4.y, q4.z, q4.w};
#pragma unroll
                        for (int e = 0; e < 4; e++)
                            nonfinite |= ((ws[e] & 0x7F80u) == 0x7F80u) || ((ws[e] & 0x7F800000u) == 0x7F800000u);
                    }
                }
                if (nonfinite) {
                    const int e = atomicAdd(win, 1);  // at most rows - 1 keys a unit
                    win[1 + e] = (int)(pos - a.prefix_len);
                    float *wp = reinterpret_cast<float *>(win + 9) + e * 8;
                    float *wm = reinterpret_cast<float *>(win + 9 + 64) + e * 8;
#pragma unroll
                    for (int r = 0; r < 8; r++) {
                        wp[r] = r < R ? p[r < R ? r : 0] : 0.0f;
                        wm[r] = r < R ? m_ref[r < R ? r : 0] : 0.0f;
                    }
                    if (h == 0) {
                        drain_wait(v_full + i % VST, (i / VST) & 1);  // the row's arrival, observed here
                        const uint32_t vrow = smem_u32(smem + OFF_V + (i % VST) * BOX + key * 128);
#pragma unroll
                        for (int c = 0; c < 8; c++) st_shared_v4(vrow + (c << 4), 0u, 0u, 0u, 0u);
                    }
                }
                // P' of this key into buffer i & 1 once PV of split i - 2 (that
                // buffer's last reader) is done.
                if (i >= 2)
                    ok = __all_sync(0xffffffffu,
                                    mbar_wait(pv_done + (i & 1), ((i - 2) >> 1) & 1, abort_flag, pg.err));
            }
            if (ok) {
                uint32_t hi[4], lo[4];
#pragma unroll
                for (int r2 = 0; r2 < 4; r2++) {
                    const float a0 = 2 * r2 < R ? p[2 * r2 < R ? 2 * r2 : 0] : 0.0f;
                    const float a1 = 2 * r2 + 1 < R ? p[2 * r2 + 1 < R ? 2 * r2 + 1 : 0] : 0.0f;
                    const uint32_t ph = pack_bf16(a0, a1);
                    hi[r2] = ph;
                    lo[r2] = pack_bf16(__fsub_rn(a0, __uint_as_float(ph << 16)),
                                       __fsub_rn(a1, __uint_as_float(ph & 0xFFFF0000u)));
                }
                const uint32_t prow = smem_u32(smem + OFF_P + (i & 1) * BOX + key * 128);
                st_shared_v4(prow + (uint32_t)(((4 * h) ^ (key & 7)) << 4), hi[0], hi[1], hi[2], hi[3]);
                st_shared_v4(prow + (uint32_t)(((4 * h + 2) ^ (key & 7)) << 4), lo[0], lo[1], lo[2], lo[3]);
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) mbar_arrive(p_full);
            }
            if (wk.last_of_unit()) {
                // The unit's end: the row sums over the head's 128 key slots
                // (a butterfly per warp, then the four warps in order); once
                // the unit's last PV is in, the head's hi warp adds O's lo rows
                // to its hi rows, adds the draft window's non-finite values and
                // writes the unit's partial (lane r: row r).  The meeting
                // orders the window list and the row sums.
#pragma unroll
                for (int r = 0; r < R; r++) {
                    float v = l_acc[r];
#pragma unroll
                    for (int o = 16; o > 0; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
                    if (lane == 0) lsum[qd * 8 + r] = v;
                    l_acc[r] = 0.0f;
                }
                bar_named(3 + h, 128);
                if (hi_warp || lo_warp) {
                    float m_fin = NEG_INF;
#pragma unroll
                    for (int r = 0; r < R; r++)
                        if (lane == r) m_fin = m_ref[r];
                    unit_partial(pg, smem, tq, h, lo_warp, lane, R, ok, m_fin, pv_done + (i & 1), (i >> 1) & 1,
                                 abort_flag, H, g, wk.unit(a), a.prefix_len, a.len0);
                }
#pragma unroll
                for (int r = 0; r < R; r++) m_ref[r] = NEG_INF;
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == W_PV) {
        tc_fence_after();
        tmem_dealloc(tmem, TMEM_COLS);
    }
}

}  // namespace tc
}  // namespace fo

// Tensor maps of the BF16 records for this kernel: prefix records
// [groups][stride][160] and tail records [groups][tail_stride][128], boxes of
// 64 elements x 128 records with the 128-byte swizzle.
static PFN_cuTensorMapEncodeTiled_v12000 tc_encoder() {
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

static bool tc_map(CUtensorMap *map, const void *base, int64_t elems, int64_t rows, int64_t stride_rows,
                   int64_t groups, uint32_t box_elems = 64) {
    auto fn = tc_encoder();
    if (!fn || rows <= 0 || rows >= (int64_t(1) << 31) || (reinterpret_cast<uintptr_t>(base) & 15)) return false;
    cuuint64_t dims[3] = {(cuuint64_t)elems, (cuuint64_t)rows, (cuuint64_t)groups};
    cuuint64_t strides[2] = {(cuuint64_t)elems * 2, (cuuint64_t)stride_rows * elems * 2};
    cuuint32_t box[3] = {box_elems, 128, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void *>(base), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, box_elems == 64 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool fo_make_tc_maps(fo_decode_page *p, int64_t groups, int64_t tail_rows) {
    if (!tc_map(&p->tc_map, p->codes, FO_RECORD, p->prefix_len, p->prefix_stride, groups)) return false;
    if (!tc_map(&p->s1_map, p->codes, FO_RECORD, p->prefix_len, p->prefix_stride, groups, 32)) return false;
    p->has_tail_map = 0;
    if (tail_rows > 0) {
        if (!tc_map(&p->tail_map, p->tail_codes, FO_TAIL_RECORD, tail_rows, p->tail_stride, groups)) return false;
        p->has_tail_map = 1;
    }
    return true;
}

// SMs of the current device (looked up once per device).
static int device_sms() {
    static std::atomic<int> sms_of[64];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 148;
    int s = sms_of[dev & 63].load();
    if (!s) {
        if (cudaDeviceGetAttribute(&s, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || s <= 0) s = 148;
        sms_of[dev & 63].store(s);
    }
    return s;
}

void fo_tc_layout(fo_decode_page *p, int64_t groups, int64_t tail_len) {
    const int sp = (int)((p->prefix_len + FO_SPLIT - 1) / FO_SPLIT);
    const int st = (int)((tail_len + FO_SPLIT - 1) / FO_SPLIT);
    // Units of `chunk` splits: about one per SM for the prefix, leaving room
    // for the tail's units (the chunk depends on the prefix alone).
    const int64_t room = std::max<int64_t>(device_sms() - 2 * groups, groups);
    const int chunk = (int)std::max<int64_t>(1, ((int64_t)sp * groups + room - 1) / room);
    p->prefix_splits = sp;
    p->chunk = chunk;
    p->splits = (sp + chunk - 1) / chunk + (st + chunk - 1) / chunk;  // units per row and head
}

template <bool FAST, int R>
static cudaError_t launch_tc(const fo_decode_page &pg, int64_t groups, cudaStream_t stream) {
    static std::atomic<unsigned long long> configured{0};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    const unsigned long long bit = 1ull << (dev & 63);
    if (!(configured.load() & bit)) {
        e = cudaFuncSetAttribute(fo::tc::decode_tc_kernel<FAST, R>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)fo::tc::SMEM);
        if (e != cudaSuccess) return e;
        configured.fetch_or(bit);
    }
    fo::tc::Args a;
    a.H = 2 * groups;
    a.prefix_len = pg.prefix_len;
    a.last = pg.last;
    a.len0 = pg.last - pg.rows + 1;
    a.prefix_splits = pg.prefix_splits;
    a.tail_splits = (int32_t)((pg.last - pg.prefix_len + FO_SPLIT - 1) / FO_SPLIT);
    a.chunk = pg.chunk;
    a.prefix_units = (pg.prefix_splits + pg.chunk - 1) / pg.chunk;
    a.units = pg.splits;
    if ((int64_t)pg.splits * groups >= (int64_t(1) << 24)) return cudaErrorInvalidValue;
    a.n_units = (uint32_t)(pg.splits * groups);
    const unsigned grid = (unsigned)std::min<int64_t>(a.n_units, device_sms());
    fo::tc::decode_tc_kernel<FAST, R><<<grid, fo::tc::THREADS, fo::tc::SMEM, stream>>>(pg, a);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    return fo_launch_decode_merge(&pg, groups, stream);
}

extern "C" cudaError_t fo_launch_decode_tc(const fo_decode_page *page, int64_t groups, int fast_exp,
                                           cudaStream_t stream) {
    const fo_decode_page &p = *page;
    if (p.rows < 1 || p.rows > FO_MAX_ROWS || !p.prefix_splits || p.chunk < 1) return cudaErrorInvalidValue;
#define FO_TC_ROWS(R)                                                                                   \
    case R:                                                                                             \
        e = fast_exp ? launch_tc<true, R>(p, groups, stream) : launch_tc<false, R>(p, groups, stream); \
        break;
    cudaError_t e = cudaErrorInvalidValue;
    switch (p.rows) {
        FO_TC_ROWS(1)
        FO_TC_ROWS(2)
        FO_TC_ROWS(3)
        FO_TC_ROWS(4)
        FO_TC_ROWS(5)
        FO_TC_ROWS(6)
        FO_TC_ROWS(7)
        FO_TC_ROWS(8)
    }
#undef FO_TC_ROWS
    return e;
}
