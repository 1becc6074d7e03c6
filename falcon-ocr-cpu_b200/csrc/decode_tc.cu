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
//   TMA warp  (warp 10) boxes of 128 records x 64 BF16 (128-byte swizzle) through a
//             3-stage ring: [T|S0], [S1|V0..31] and [V] of prefix records,
//             [K] and [V] of tail records;
//   MMA warp  (warp 11) S = keys x Q' (M128 K64, keys in TMEM lanes: the temporal
//             half for both heads at N64, each spatial half at N32); then
//             O = P' x V (M64 N64 K128) and the row sums l = P' x 1 (N8),
//             S, P', O and l double-buffered;
//   8 warps   (warps 2-9) one thread per (head, key): logits, the row maxima
//             over the split (redux, then the head's four warps through a
//             named barrier and shared memory), p = exp(s - max), P' to shared
//             memory;
//   2 warps   (warps 0, 1: TMEM lane quadrants 0 and 1) read O's hi and lo
//             rows and fold each split into its unit's running partial,
//             written at the unit's end, off the key warps' path.
//
// Exactness: Q' holds each FP32 query as three BF16 terms (hi + mid + lo ==
// q exactly), so every product with a BF16 key is exact and S is the FP32
// dot product up to accumulation order.  P' holds each probability as two
// BF16 terms (hi + lo == p to 2^-18) in two groups of M rows, which the
// epilogue adds, for O and l alike.  The output agrees
// with the reference's FP32 decode over the same records within
// 1e-5 * (1 + |b|).
//
// Verify rows: every row's logits, maxima, O and l columns come from its own
// query and keys only, with the same instructions whatever the number of
// rows, and a split that holds none of a row's keys leaves that row's unit
// partial untouched.  Keys a row does not see get p = 0; with finite values
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
constexpr int THREADS = 384;  // warps 0-1 epilogue, 2-9 (head, key), 10 TMA, 11 MMA
constexpr int W_TMA = 10, W_MMA = 11;
constexpr int RING = 8;       // per-split statistics and window records, by split index mod 8
constexpr int STAGES = 3;
constexpr uint32_t BOX = 128 * 128;   // 128 records x 128 bytes
constexpr uint32_t STAGE = 3 * BOX;   // three boxes per split
constexpr uint32_t QTILE = 32 * 128;  // Q' of one head: 32 rows x 64 BF16
constexpr uint32_t OFF_Q = STAGES * STAGE;
constexpr uint32_t OFF_P = OFF_Q + 2 * 2 * QTILE;  // two Q' buffers x two heads
// P' double buffer: [key][64 M rows] BF16, M row = term * 16 + head * 8 + row
// (term 0 = hi, 1 = lo; rows 32..63 zero).
constexpr uint32_t OFF_ONES = OFF_P + 2 * BOX;  // 256 bytes of BF16 ones: the row-sum MMA's operand
constexpr uint32_t OFF_RED = OFF_ONES + 256;
// row maxima: [RING][2 heads][4 warps][8 rows] floats
constexpr uint32_t RED_FLOATS = RING * 2 * 4 * 8;
constexpr uint32_t OFF_WIN = OFF_RED + RED_FLOATS * 4;
// draft-window fallback per [RING][2 heads]: { count, keys[8], p[8 keys][8
// rows] } in 32-bit words.  The key warps run at most RING - 1 splits ahead
// of the epilogue (P' of split i waits for PV of split i - 2, which waits for
// the epilogue of split i - 4), so a slot is free when they come back to it.
constexpr uint32_t WIN_WORDS = 1 + 8 + 8 * 8;
// [2 heads][8 rows][68] floats: the epilogue lanes' running unit partials
// (64 dimensions, padded against bank conflicts); and the lo rows of O handed
// from one epilogue warp to the other, [2 parities][2 heads][8 rows][68].
constexpr uint32_t ACC_STRIDE = 68;
constexpr uint32_t OFF_ACC = (OFF_WIN + RING * 2 * WIN_WORDS * 4 + 15) / 16 * 16;
constexpr uint32_t OFF_LO = OFF_ACC + 2 * 8 * ACC_STRIDE * 4;
constexpr uint32_t OFF_BAR = OFF_LO + 2 * 2 * 8 * ACC_STRIDE * 4;
// full[3] empty[3] s_full[2] s_empty[2] q_full[2] p_full pv_done[2]
// o_empty[2] lo_ready[2] mma_done
constexpr int NBAR = 2 * STAGES + 2 + 2 + 2 + 1 + 2 + 2 + 2 + 1;
constexpr uint32_t SMEM = OFF_BAR + NBAR * 8 + 16 + 1024;
// S, O and the row sums l double-buffered: S [0, 128), O [128, 256), l [256, 272).
constexpr uint32_t TMEM_COLS = 512;
constexpr uint32_t TM_O = 128, TM_L = 256;
static_assert(SMEM <= 227 * 1024, "shared memory per CTA");

// Instruction descriptor, kind::f16, BF16 inputs, FP32 accumulator.
__host__ __device__ constexpr uint32_t idesc(uint32_t m, uint32_t n, uint32_t a_mn, uint32_t b_mn) {
    return (1u << 4) | (1u << 7) | (1u << 10) | (a_mn << 15) | (b_mn << 16) | ((n >> 3) << 17) | ((m >> 4) << 24);
}

struct Args {
    int64_t H, prefix_len, last, len0;  // len0 = last - rows + 1: keys every row sees
    int32_t prefix_splits, tail_splits, chunk, prefix_units, units;  // units per group and row
    int64_t n_units;                                                  // groups x units
};

__device__ __forceinline__ void drain_wait(uint64_t *bar, uint32_t phase) {
    const uint64_t t0 = globaltimer();
    while (!mbar_try_wait(bar, phase))
        if (globaltimer() - t0 > FO_WAIT_NS) break;
}

// The exchange among a head's four key warps (named barrier 1 + head, 128
// threads).  Every key warp passes it once per split, also after a bounded
// wait gave up (it then skips the split's work), so no warp waits here for
// one that left.
__device__ __forceinline__ void sync_head(int h) {
    asm volatile("bar.sync %0, 128;" ::"r"(1 + h) : "memory");
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
// whether the split closes its unit.
struct Walk {
    int64_t U, U_end, g;  // unit, end, the unit's group
    int u, s, s_end;      // the unit's index within its group, split, end
    __device__ __forceinline__ void unit_bounds(const Args &a) {
        if (u < a.prefix_units) {
            s = u * a.chunk;
            s_end = min(s + a.chunk, a.prefix_splits);
        } else {
            s = a.prefix_splits + (u - a.prefix_units) * a.chunk;
            s_end = min(s + a.chunk, a.prefix_splits + a.tail_splits);
        }
    }
    __device__ __forceinline__ void start(const Args &a, int64_t u0, int64_t u1) {
        U = u0;
        U_end = u1;
        g = U / a.units;  // the walk's one division
        u = (int)(U - g * a.units);
        s = s_end = 0;
        if (U < U_end) unit_bounds(a);
    }
    __device__ __forceinline__ bool valid() const { return U < U_end; }
    __device__ __forceinline__ int64_t group(const Args &) const { return g; }
    __device__ __forceinline__ int unit(const Args &) const { return u; }
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

// The TMA loads of local split i (the walk's current split) into stage
// i mod STAGES: three boxes of a prefix split, two of a tail split.
__device__ __forceinline__ void issue_tma(const fo_decode_page &pg, const Args &a, uint8_t *smem, uint64_t *full,
                                          const Walk &wk, int i) {
    const int st = i % STAGES;
    const int g = (int)wk.group(a);
    const Split x = split_of(a, wk.s);
    uint8_t *dst = smem + st * STAGE;
    if (!x.tail) {
        mbar_expect_tx(full + st, 3 * BOX);
        tma_load_3d(dst, &pg.tc_map, full + st, 0, x.row0, g);
        tma_load_3d(dst + BOX, &pg.tc_map, full + st, 64, x.row0, g);
        tma_load_3d(dst + 2 * BOX, &pg.tc_map, full + st, 96, x.row0, g);
    } else {
        mbar_expect_tx(full + st, 2 * BOX);
        tma_load_3d(dst, &pg.tail_map, full + st, 0, x.row0, g);
        tma_load_3d(dst + 2 * BOX, &pg.tail_map, full + st, 64, x.row0, g);
    }
}

template <bool FAST, int R>
__global__ void __launch_bounds__(THREADS, 1)
    decode_tc_kernel(const __grid_constant__ fo_decode_page pg, const Args a) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + OFF_BAR);
    uint64_t *full = bars, *empty = bars + STAGES;
    uint64_t *s_full = bars + 2 * STAGES, *s_empty = s_full + 2, *q_full = s_empty + 2;
    uint64_t *p_full = q_full + 2, *pv_done = p_full + 1, *o_empty = pv_done + 2, *lo_ready = o_empty + 2;
    uint64_t *mma_done = lo_ready + 2;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + NBAR);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t u0 = (int64_t)blockIdx.x * a.n_units / gridDim.x;
    const int64_t u1 = (int64_t)(blockIdx.x + 1) * a.n_units / gridDim.x;

    // The TMA thread sets the barriers up and starts the first loads before
    // the CTA-wide barrier (the stage buffers are not touched by the rest of
    // the setup).
    Walk twk;
    int t_issued = 0;
    if (threadIdx.x == W_TMA * 32) {
        for (int s = 0; s < STAGES; s++) {
            mbar_init(full + s, 1);
            mbar_init(empty + s, 1);
        }
        for (int b = 0; b < 2; b++) {
            mbar_init(s_full + b, 1);
            mbar_init(s_empty + b, KEY_WARPS);
            mbar_init(q_full + b, KEY_WARPS);
            mbar_init(pv_done + b, 1);
            mbar_init(o_empty + b, 2);  // both epilogue warps
            mbar_init(lo_ready + b, 1);
        }
        mbar_init(p_full, KEY_WARPS);
        mbar_init(mma_done, 1);
        *abort_flag = 0;
        mbar_fence_init();
        tma_prefetch(&pg.tc_map);
        if (pg.has_tail_map) tma_prefetch(&pg.tail_map);
        twk.start(a, u0, u1);
        for (; twk.valid() && t_issued < STAGES; t_issued++, twk.next(a)) issue_tma(pg, a, smem, full, twk, t_issued);
    }
    if (warp >= 2 && warp < 2 + KEY_WARPS) {
        // Zero what the loop never writes: Q' rows of absent verify rows and
        // its padding rows (R..7 of each term, 24..31), and P' rows 32..63
        // (logical chunks 4..7 of every key's row, both buffers).
        const int t = threadIdx.x - 64;
        for (int idx = t; idx < 2 * 2 * 32 * 8; idx += 32 * KEY_WARPS) {
            const int chunk = idx & 7, row = (idx >> 3) & 31;
            if (row >= 24 || (row & 7) >= R)
                *reinterpret_cast<uint4 *>(smem + OFF_Q + (idx >> 8) * QTILE + row * 128 + ((chunk ^ (row & 7)) << 4)) =
                    make_uint4(0, 0, 0, 0);
        }
        for (int idx = t; idx < 2 * 128 * 4; idx += 32 * KEY_WARPS) {
            const int tile = idx >> 9, key = (idx >> 2) & 127, chunk = 4 + (idx & 3);
            *reinterpret_cast<uint4 *>(smem + OFF_P + tile * BOX + key * 128 + ((chunk ^ (key & 7)) << 4)) =
                make_uint4(0, 0, 0, 0);
        }
        if (t < 16)
            *reinterpret_cast<uint4 *>(smem + OFF_ONES + 16 * t) =
                make_uint4(0x3F803F80u, 0x3F803F80u, 0x3F803F80u, 0x3F803F80u);
        fence_proxy_async_smem();
    }
    if (warp == W_MMA) tmem_alloc(tmem_slot, TMEM_COLS);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    // The merge kernel may launch now; it waits for this grid to finish.
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

    if (warp == W_TMA) {
        // ---------------------------------------------------------- TMA
        if (lane == 0) {
            bool ok = true;
            for (int i = t_issued; twk.valid() && ok; i++, twk.next(a)) {
                const int st = i % STAGES, u = i / STAGES;
                if (!(ok = mbar_wait(empty + st, (u - 1) & 1, abort_flag, pg.err))) break;
                issue_tma(pg, a, smem, full, twk, i);
                t_issued = i + 1;
            }
            if (!ok)
                for (int i = max(0, t_issued - STAGES); i < t_issued; i++)
                    drain_wait(full + i % STAGES, (i / STAGES) & 1);
        }
    } else if (warp == W_MMA) {
        // ---------------------------------------------------------- MMA
        const uint32_t iT = idesc(128, 64, 0, 0), iS = idesc(128, 32, 0, 0), iPV = idesc(64, 64, 1, 1);
        const uint32_t iL = idesc(64, 8, 1, 0);
        const uint32_t sQ = smem_u32(smem + OFF_Q), sP = smem_u32(smem + OFF_P);
        // The ones operand (N8 x K16, no swizzle): every K step reads the same
        // 256 bytes of BF16 ones.
        const uint64_t dOnes = sdesc_none(smem_u32(smem + OFF_ONES), 128, 256);
        bool ok = true;
        int q_uses[2] = {0, 0};
        int qb = 1;
        int64_t prev_g = -1;
        auto issue_pv = [&](int j) {
            // O = P' V and l = P' 1 over the split's 128 keys (8 K16 steps) into
            // buffer j & 1.
            const int st = j % STAGES;
            const uint64_t dV = sdesc_sw128(smem_u32(smem + st * STAGE + 2 * BOX), BOX, 1024);
            const uint64_t dP = sdesc_sw128(sP + (j & 1) * BOX, BOX, 1024);
            if (elect_one()) {
#pragma unroll
                for (int kk = 0; kk < 8; kk++) {
                    mma_bf16(tmem + TM_O + (j & 1) * 64, dP + kk * (2048 >> 4), dV + kk * (2048 >> 4), iPV, kk != 0);
                    mma_bf16(tmem + TM_L + (j & 1) * 8, dP + kk * (2048 >> 4), dOnes, iL, kk != 0);
                }
                mma_commit(pv_done + (j & 1));
                mma_commit(empty + st);
            }
            __syncwarp();
        };
        Walk wk;
        wk.start(a, u0, u1);
        int i = 0;
        for (; wk.valid() && ok; i++, wk.next(a)) {
            const int st = i % STAGES, u = i / STAGES, sb = i & 1;
            const int64_t g = wk.group(a);
            if (g != prev_g) {
                qb ^= 1;
                ok = __all_sync(0xffffffffu, mbar_wait(q_full + qb, q_uses[qb] & 1, abort_flag, pg.err));
                q_uses[qb]++;
                prev_g = g;
                if (!ok) break;
            }
            ok = __all_sync(0xffffffffu, mbar_wait(full + st, u & 1, abort_flag, pg.err));
            if (ok && i >= 2)
                ok = __all_sync(0xffffffffu, mbar_wait(s_empty + sb, ((i - 2) >> 1) & 1, abort_flag, pg.err));
            if (!ok) break;
            tc_fence_after();
            const bool tail = wk.s >= a.prefix_splits;
            const uint32_t b0 = smem_u32(smem + st * STAGE), b1 = b0 + BOX;
            const uint64_t dK0 = sdesc_sw128(b0, 16, 1024);
            // Head 1's spatial half: the [S1|V] box of a prefix record, the
            // key's own second half in a tail record.
            const uint64_t dK1s = tail ? dK0 + (64 >> 4) : sdesc_sw128(b1, 16, 1024);
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
            }
            __syncwarp();
            if (i >= 1) {
                // PV of the previous split once its probabilities are in and
                // the epilogue has read the O two splits back (same buffer).
                ok = __all_sync(0xffffffffu, mbar_wait(p_full, (i - 1) & 1, abort_flag, pg.err));
                if (ok && i >= 3)
                    ok = __all_sync(0xffffffffu,
                                    mbar_wait(o_empty + ((i - 1) & 1), ((i - 3) >> 1) & 1, abort_flag, pg.err));
                if (!ok) break;
                tc_fence_after();
                issue_pv(i - 1);
            }
        }
        if (ok && i > 0) {
            const int j = i - 1;
            ok = __all_sync(0xffffffffu, mbar_wait(p_full, j & 1, abort_flag, pg.err));
            if (ok && j >= 2)
                ok = __all_sync(0xffffffffu, mbar_wait(o_empty + (j & 1), ((j - 2) >> 1) & 1, abort_flag, pg.err));
            if (ok) {
                tc_fence_after();
                issue_pv(j);
            }
        }
        if (elect_one()) mma_commit(mma_done);
        __syncwarp();
        if (lane == 0) drain_wait(mma_done, 0);
        __syncwarp();
    } else if (warp >= 2) {
        // ---------------------------------------------- (head, key) warps
        const int hw = warp - 2;         // 0..7
        const int h = hw >> 2;           // this warp's head of the group
        const int w4 = hw & 3;           // warp index within the head
        const int qd = warp & 3;         // TMEM lane quadrant of this warp
        const int key = qd * 32 + lane;  // the key this thread owns in a split
        const int64_t H = a.H;
        const float NEG_INF = -INFINITY;
        float *red = reinterpret_cast<float *>(smem + OFF_RED);
        bool ok = true;
        int qb = 1;
        int64_t prev_g = -1;
        Walk wk;
        wk.start(a, u0, u1);
        for (int i = 0; wk.valid(); i++, wk.next(a)) {
            const int sb = i & 1, slot = i % RING;
            const int64_t g = wk.group(a);
            const Split x = split_of(a, wk.s);
            float *sm = red + ((slot * 2 + h) * 4) * 8;  // maxima [warp][row]
            int *wi = reinterpret_cast<int *>(smem + OFF_WIN) + (slot * 2 + h) * WIN_WORDS;
            float lg[R];
            if (ok && g != prev_g) {
                // Q' of this group's head h: row (term * 8 + r) holds term (hi,
                // mid, lo) of q[r][2g + h], three BF16 values summing to the
                // FP32 query exactly; thread key < 64 takes (row r, 8-dimension
                // chunk c).  The buffer's previous readers (the QK of the group
                // before last) finished before the last split's S was read.
                qb ^= 1;
                const int r = key >> 3, c = key & 7;
                if (key < 64 && r < R) {
                    const float4 *src =
                        reinterpret_cast<const float4 *>(pg.q + ((int64_t)r * H + 2 * g + h) * FO_HD + 8 * c);
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
                        const uint32_t addr =
                            smem_u32(smem + OFF_Q + (qb * 2 + h) * QTILE + row * 128) + ((c ^ r) << 4);
                        st_shared_v4(addr, wv[term][0], wv[term][1], wv[term][2], wv[term][3]);
                    }
                }
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) mbar_arrive(q_full + qb);
                prev_g = g;
            }
            if (ok) ok = __all_sync(0xffffffffu, mbar_wait(s_full + sb, (i >> 1) & 1, abort_flag, pg.err));
            if (ok) {
                tc_fence_after();
                uint32_t sv[32];
                FO_TMEM_LD32(tmem + ((uint32_t)(qd * 32) << 16) + sb * 64 + h * 32, sv);
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
                // Row maxima over the split's keys: per warp here, over the
                // head's four warps after the exchange.
#pragma unroll
                for (int r = 0; r < R; r++) {
                    const float m = warp_max_redux(lg[r]);
                    if (lane == 0) sm[w4 * 8 + r] = m;
                }
                if (w4 == 0 && lane == 0) wi[0] = 0;  // this split's window record
            }
            sync_head(h);
            if (!ok || *abort_flag) {
                ok = false;
                continue;  // the remaining splits only pass the exchange
            }
            float p[R];
#pragma unroll
            for (int r = 0; r < R; r++) {
                float m = NEG_INF;
#pragma unroll
                for (int ww = 0; ww < 4; ww++) m = rmax(m, sm[ww * 8 + r]);
                p[r] = lg[r] == NEG_INF ? 0.0f : key_exp<FAST>(__fsub_rn(lg[r], m));
            }
            // The draft window [len0, last) of a tail split: a key whose value
            // row holds a non-finite number leaves the MMA (head 0's thread of
            // the key zeroes its staged row) and the epilogue adds it to the
            // rows that see it.  Both heads test the row in global memory, so
            // neither test depends on the other's zeroing.
            const int64_t pos = x.k0 + key;
            bool nonfinite = false;
            if (x.tail && pos >= a.len0 && pos < x.k1) {
                const uint4 *vg = reinterpret_cast<const uint4 *>(
                    reinterpret_cast<const uint16_t *>(pg.tail_codes) +
                    (g * pg.tail_stride + (pos - a.prefix_len)) * FO_TAIL_RECORD + 64);
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
                const int e = atomicAdd(wi, 1);  // at most rows - 1 keys
                wi[1 + e] = key;
                float *wp = reinterpret_cast<float *>(wi + 9) + e * 8;
#pragma unroll
                for (int r = 0; r < 8; r++) wp[r] = r < R ? p[r < R ? r : 0] : 0.0f;
                if (h == 0) {
                    drain_wait(full + i % STAGES, (i / STAGES) & 1);  // the row's arrival, observed here
                    const uint32_t vrow = smem_u32(smem + (i % STAGES) * STAGE + 2 * BOX + key * 128);
#pragma unroll
                    for (int c = 0; c < 8; c++) st_shared_v4(vrow + (c << 4), 0u, 0u, 0u, 0u);
                }
            }
            // P' of this key into buffer i & 1 once PV of split i - 2 (that
            // buffer's last reader) is done: hi terms in M rows 8h .. 8h + 7,
            // lo terms in rows 16 + 8h .. 16 + 8h + 7.
            if (i >= 2 && !(ok = __all_sync(0xffffffffu, mbar_wait(pv_done + (i & 1), ((i - 2) >> 1) & 1,
                                                                   abort_flag, pg.err))))
                continue;
            {
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
                st_shared_v4(prow + (uint32_t)((h ^ (key & 7)) << 4), hi[0], hi[1], hi[2], hi[3]);
                st_shared_v4(prow + (uint32_t)(((2 + h) ^ (key & 7)) << 4), lo[0], lo[1], lo[2], lo[3]);
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) mbar_arrive(p_full);
        }
    } else {
        // ------------------------------------------------ epilogue (warps 0, 1)
        // Warp 0 reads O's hi rows (TMEM lanes 8h + r of quadrant 0), warp 1
        // its lo rows (quadrant 1) and hands them over through shared memory;
        // warp 0 folds hi + lo of each split into the unit's partial (lane
        // 8h + r: head h, row r) and writes it at the unit's end.
        const bool hi_warp = warp == 0;
        const int h = lane >> 3, er = lane & 7;
        const bool erow = lane < 16 && er < R;
        const int64_t H = a.H;
        const float NEG_INF = -INFINITY;
        const float *red = reinterpret_cast<const float *>(smem + OFF_RED);
        float *o_acc = reinterpret_cast<float *>(smem + OFF_ACC) + (lane & 15) * ACC_STRIDE;
        float m_run = NEG_INF, l_run = 0.0f;
        bool ok = true;
        Walk wk;
        wk.start(a, u0, u1);
        for (int j = 0; wk.valid() && ok; j++, wk.next(a)) {
            const int slot = j % RING;
            // Split j's PV: pv_done[j & 1] moves on only after this split's
            // o_empty, so its phase cannot be overtaken.
            if (!(ok = __all_sync(0xffffffffu, mbar_wait(pv_done + (j & 1), (j >> 1) & 1, abort_flag, pg.err))))
                break;
            tc_fence_after();
            const uint32_t tO = tmem + ((uint32_t)(warp * 32) << 16) + TM_O + (j & 1) * 64;
            float *lo = reinterpret_cast<float *>(smem + OFF_LO) + ((j & 1) * 16 + (lane & 15)) * ACC_STRIDE;
            const float l_part = __uint_as_float(tmem_ld1(tmem + ((uint32_t)(warp * 32) << 16) + TM_L + (j & 1) * 8));
            if (!hi_warp) {
                tmem_wait_ld();
                if (erow) lo[64] = l_part;
#pragma unroll
                for (int half = 0; half < 2; half++) {
                    uint32_t o[32];
                    FO_TMEM_LD32(tO + 32 * half, o);
                    tmem_wait_ld();
                    if (erow) {
                        float4 *dst = reinterpret_cast<float4 *>(lo + 32 * half);
#pragma unroll
                        for (int d = 0; d < 8; d++)
                            dst[d] = make_float4(__uint_as_float(o[4 * d]), __uint_as_float(o[4 * d + 1]),
                                                 __uint_as_float(o[4 * d + 2]), __uint_as_float(o[4 * d + 3]));
                    }
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(lo_ready + (j & 1));
                    mbar_arrive(o_empty + (j & 1));
                }
                continue;
            }
            // This split's max of row (h, er): the head's four warps (the key
            // warps wrote them before this split's P').
            float m_split = NEG_INF;
            if (erow) {
                const float *sm = red + ((slot * 2 + h) * 4) * 8;
#pragma unroll
                for (int ww = 0; ww < 4; ww++) m_split = rmax(m_split, sm[ww * 8 + er]);
            }
            const bool live = erow && m_split != NEG_INF;
            const bool first = m_run == NEG_INF;
            float fa = 1.0f, fb = 1.0f, m_new = m_split;
            if (live && !first) {
                m_new = rmax(m_run, m_split);
                fa = expf(__fsub_rn(m_run, m_new));
                fb = expf(__fsub_rn(m_split, m_new));
            }
            // Non-finite values of the draft window, added for the rows that
            // see them (the MMA saw their value rows as zero).
            const int *wr = reinterpret_cast<const int *>(smem + OFF_WIN) + (slot * 2 + h) * WIN_WORDS;
            const int nw = live ? wr[0] : 0;
            const Split x = split_of(a, wk.s);
            const int64_t g = wk.group(a);
            uint32_t o[2][32];
            FO_TMEM_LD32(tO, o[0]);
            FO_TMEM_LD32(tO + 32, o[1]);
            tmem_wait_ld();
            tc_fence_before();
            if (!(ok = __all_sync(0xffffffffu, mbar_wait(lo_ready + (j & 1), (j >> 1) & 1, abort_flag, pg.err))))
                break;
            // The split's row sum: the hi and lo terms' l columns.
            const float l_split = erow ? __fadd_rn(l_part, lo[64]) : 0.0f;
#pragma unroll
            for (int half = 0; half < 2; half++) {
                if (live) {
                    float ov[32];
                    const float4 *lv = reinterpret_cast<const float4 *>(lo + 32 * half);
#pragma unroll
                    for (int d = 0; d < 8; d++) {
                        const float4 l4 = lv[d];
                        ov[4 * d] = __fadd_rn(__uint_as_float(o[half][4 * d]), l4.x);
                        ov[4 * d + 1] = __fadd_rn(__uint_as_float(o[half][4 * d + 1]), l4.y);
                        ov[4 * d + 2] = __fadd_rn(__uint_as_float(o[half][4 * d + 2]), l4.z);
                        ov[4 * d + 3] = __fadd_rn(__uint_as_float(o[half][4 * d + 3]), l4.w);
                    }
                    for (int e = 0; e < nw; e++) {
                        const int kl = wr[1 + e];
                        if (x.k0 + kl >= a.len0 + er) continue;  // this row does not see it
                        const float pk = reinterpret_cast<const float *>(wr + 9)[e * 8 + er];
                        const uint16_t *vr = reinterpret_cast<const uint16_t *>(pg.tail_codes) +
                                             (g * pg.tail_stride + (x.k0 + kl - a.prefix_len)) * FO_TAIL_RECORD + 64 +
                                             32 * half;
                        for (int d = 0; d < 32; d++) ov[d] = fmaf(pk, bf16_f32(vr[d]), ov[d]);
                    }
                    float4 *acc = reinterpret_cast<float4 *>(o_acc + 32 * half);
#pragma unroll
                    for (int d = 0; d < 8; d++) {
                        float4 y = first ? make_float4(0.f, 0.f, 0.f, 0.f) : acc[d];
                        y.x = first ? ov[4 * d] : fmaf(ov[4 * d], fb, __fmul_rn(y.x, fa));
                        y.y = first ? ov[4 * d + 1] : fmaf(ov[4 * d + 1], fb, __fmul_rn(y.y, fa));
                        y.z = first ? ov[4 * d + 2] : fmaf(ov[4 * d + 2], fb, __fmul_rn(y.z, fa));
                        y.w = first ? ov[4 * d + 3] : fmaf(ov[4 * d + 3], fb, __fmul_rn(y.w, fa));
                        acc[d] = y;
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(o_empty + (j & 1));
            if (live) {
                l_run = first ? l_split : fmaf(l_split, fb, __fmul_rn(l_run, fa));
                m_run = m_new;
            }
            if (wk.last_of_unit()) {
                if (erow) {
                    const int64_t row_head = (int64_t)er * H + 2 * g + h;
                    const int64_t idx = row_head * pg.splits + wk.unit(a);
                    float4 *dst = reinterpret_cast<float4 *>(pg.part_o + idx * FO_HD);
                    const float4 *acc = reinterpret_cast<const float4 *>(o_acc);
                    if (m_run == NEG_INF) {
                        // No key of the unit is this row's: an empty partial.
#pragma unroll
                        for (int d = 0; d < 16; d++) dst[d] = make_float4(0.f, 0.f, 0.f, 0.f);
                    } else {
#pragma unroll
                        for (int d = 0; d < 16; d++) dst[d] = acc[d];
                    }
                    *reinterpret_cast<float2 *>(pg.part_ml + idx * 2) = make_float2(m_run, l_run);
                }
                m_run = NEG_INF;
                l_run = 0.0f;
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == W_MMA) {
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
                   int64_t groups) {
    auto fn = tc_encoder();
    if (!fn || rows <= 0 || rows >= (int64_t(1) << 31) || (reinterpret_cast<uintptr_t>(base) & 15)) return false;
    cuuint64_t dims[3] = {(cuuint64_t)elems, (cuuint64_t)rows, (cuuint64_t)groups};
    cuuint64_t strides[2] = {(cuuint64_t)elems * 2, (cuuint64_t)stride_rows * elems * 2};
    cuuint32_t box[3] = {64, 128, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void *>(base), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool fo_make_tc_maps(fo_decode_page *p, int64_t groups, int64_t tail_rows) {
    if (!tc_map(&p->tc_map, p->codes, FO_RECORD, p->prefix_len, p->prefix_stride, groups)) return false;
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
    a.n_units = (int64_t)pg.splits * groups;
    const unsigned grid = (unsigned)std::min<int64_t>(a.n_units, device_sms());
    fo::tc::decode_tc_kernel<FAST, R><<<grid, fo::tc::THREADS, fo::tc::SMEM, stream>>>(pg, a);
    return cudaGetLastError();
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
    if (e != cudaSuccess) return e;
    return fo_launch_decode_merge(page, groups, stream);
}
