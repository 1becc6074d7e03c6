// decode.cu -- split-KV decode and speculative-verify attention over the
// split cache (reference: SplitPrefix::attention_decode / attention_decode_rows,
// src/quant/kv.rs:565-972; per-group kernels pair / pair_rows,
// src/quant/kv/decode.rs:305-677; merge, src/quant/kv.rs:775-813).
//
// Work items are (page, split, group): FO_SPLIT positions of one KV group,
// for both heads of the group and every verification row, as the reference's
// pair_rows serves them (each record is read once and every row runs over
// it).  Persistent CTAs of four warp pairs walk the items; a pair owns whole
// items and streams each through NBUF buffers of 32-key chunks.  A chunk of
// prefix records arrives by one TMA tile copy through the cache's record
// tensor map, whose box is wider than a record so that the out-of-bounds fill
// pads every key's slot (consecutive keys start on different banks); a chunk
// that reaches the tail is copied record by record (cp.async.bulk).  Slots
// hold [T 32 | S0 32 | S1 32 | V 64] (a tail record's key fills both spatial
// halves).  The two warps of a pair compute on a chunk, one per head: logits
// with lane = key, the reference's online softmax per row over the chunk
// (chunk max, rescale, exp(s - max)), and O += P V with lane = two output
// dimensions, dequantizing exactly as the reference (fl(code * scale),
// decode.rs:151-187) with packed FP32 FMA (each half an ordinary fmaf).  Once
// both warps are done with a chunk, the copies NBUF chunks ahead are issued
// into its buffer, and the next item's records are prefetched into L2.  The
// chunks combine, in chunk order, into the split's unnormalized partial; a
// merge kernel, launched as a programmatic dependent, combines the splits in
// order and applies the sink.  Rows only see their own positions (row r:
// prefix + tail - rows + 1 + r, kv.rs:851-855) and every boundary and order
// is absolute, so each verification row equals its single-row decode bit for
// bit.
#include "fo_common.cuh"
#include "fo_kernels.h"
#include "sm100.cuh"

#include <cudaTypedefs.h>

#include <algorithm>
#include <atomic>
#include <type_traits>

namespace fo {

enum { DF32 = 0, DQ16 = 1, DQ8 = 2, DBF16 = 3, DQ4 = 4 };

// Per-format shape of a CTA: NPAIR pairs of warps; a pair owns whole items
// and streams their 32-key chunks through NBUF slot buffers; warp 2p + h of
// pair p computes head h of the item's KV group.
template <int F>
struct Shape {
    static constexpr int E = F == DF32 ? 4 : (F == DQ8 || F == DQ4 ? 1 : 2);  // bytes per TMA element
    static constexpr bool CODED = F == DQ16 || F == DQ8 || F == DQ4;
    // Bytes of n record elements (Q4: two codes per byte).
    static constexpr int bytes(int n) { return F == DQ4 ? n / 2 : n * E; }
    static constexpr int RB = bytes(FO_RECORD), TB = bytes(FO_TAIL_RECORD);
    static constexpr int CK = 32;                // keys per chunk (one per lane)
    static constexpr int KPL = 1;                // keys per lane
    static constexpr int NCH = FO_SPLIT / CK;    // chunks per item
    static constexpr int NPAIR = 4;
    // Slot buffers per pair: Q8 records are small enough for a third, which
    // keeps one more chunk in flight (single-row decode waits on its copies).
    static constexpr int NBUF = F == DQ8 || F == DQ4 ? 3 : 2;
    static constexpr int NW = 2 * NPAIR;
    static constexpr int THREADS = 32 * NW;
    static constexpr int MIN_CTAS = F == DF32 ? 1 : 2;
    // Padded slot: 16 bytes past the record, so consecutive keys start on
    // different banks (slot stride 4, 20 or 12 mod 32 words); a Q4 record
    // (80 bytes, 20 mod 32 words) needs no pad.
    static constexpr int SLOT = F == DQ4 ? RB : RB + 16;
    static_assert(NCH >= NBUF, "an item spans every buffer");
};

// Shared-memory layout of one instantiation (bytes).
template <int F, int R>
struct Smem {
    using S = Shape<F>;
    static constexpr int BUFS = S::NPAIR * S::NBUF;
    static constexpr int RECS = BUFS * S::CK * S::SLOT;                 // record slots per buffer
    static constexpr int SCL = S::CODED ? BUFS * S::CK * 5 * 4 : 0;    // decoded scales [key][T, S0, S1, V0, V1]
    static constexpr int Q = S::NW * R * FO_HD * 4;                     // per-warp q of its head [R][64]
    static constexpr int P = S::NW * R * S::CK * 4;                     // per-warp probabilities [R][CK]
    static constexpr int OFF_SCL = RECS;
    static constexpr int OFF_Q = OFF_SCL + SCL;
    static constexpr int OFF_P = OFF_Q + Q;
    static constexpr int OFF_BAR = (OFF_P + P + 7) / 8 * 8;
    static constexpr int OFF_FLAGS = OFF_BAR + BUFS * 8;
    static constexpr int BYTES = OFF_FLAGS + 16;
    static_assert(BYTES <= 227 * 1024, "shared memory per CTA");
};

// Two consecutive decoded values of a staged slot at element `e` (even).
template <int F>
__device__ __forceinline__ float2 slot_pair(const unsigned char *slot, int e, float scale) {
    if constexpr (F == DF32) {
        return *reinterpret_cast<const float2 *>(slot + 4 * e);
    } else if constexpr (F == DBF16) {
        const uint32_t w = *reinterpret_cast<const uint32_t *>(slot + 2 * e);
        return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xFFFF0000u));
    } else if constexpr (F == DQ16) {
        float lo, hi;
        s16x2_f32(*reinterpret_cast<const uint32_t *>(slot + 2 * e), lo, hi);
        return make_float2(__fmul_rn(lo, scale), __fmul_rn(hi, scale));
    } else if constexpr (F == DQ4) {
        float lo, hi;
        s4x2_f32(slot[e / 2], lo, hi);
        return make_float2(__fmul_rn(lo, scale), __fmul_rn(hi, scale));
    } else {
        float lo, hi;
        s8x2_f32(*reinterpret_cast<const uint16_t *>(slot + e), lo, hi);
        return make_float2(__fmul_rn(lo, scale), __fmul_rn(hi, scale));
    }
}

// 16 consecutive decoded values of a staged slot at element `e` (a multiple
// of 16, inside one 32-element scale block); with SCALED false, the codes of a
// coded format before their block scale.
template <int F, bool SCALED = true>
__device__ __forceinline__ void slot_span16(const unsigned char *slot, int e, float scale, float *out) {
    if constexpr (F == DF32) {
        const float4 *p = reinterpret_cast<const float4 *>(slot + 4 * e);
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const float4 x = p[i];
            out[4 * i] = x.x;
            out[4 * i + 1] = x.y;
            out[4 * i + 2] = x.z;
            out[4 * i + 3] = x.w;
        }
    } else if constexpr (F == DBF16 || F == DQ16) {
        const uint4 *p = reinterpret_cast<const uint4 *>(slot + 2 * e);
#pragma unroll
        for (int i = 0; i < 2; i++) {
            const uint4 x = p[i];
            const uint32_t w[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
            for (int c = 0; c < 4; c++) {
                if constexpr (F == DBF16) {
                    out[8 * i + 2 * c] = __uint_as_float(w[c] << 16);
                    out[8 * i + 2 * c + 1] = __uint_as_float(w[c] & 0xFFFF0000u);
                } else {
                    float lo, hi;
                    s16x2_f32(w[c], lo, hi);
                    out[8 * i + 2 * c] = SCALED ? __fmul_rn(lo, scale) : lo;
                    out[8 * i + 2 * c + 1] = SCALED ? __fmul_rn(hi, scale) : hi;
                }
            }
        }
    } else if constexpr (F == DQ4) {
        const uint2 x = *reinterpret_cast<const uint2 *>(slot + e / 2);
        const uint32_t w[2] = {x.x, x.y};
#pragma unroll
        for (int c = 0; c < 2; c++) {
            float f[8];
            s4x8_f32(w[c], f);
#pragma unroll
            for (int b = 0; b < 8; b++) out[8 * c + b] = SCALED ? __fmul_rn(f[b], scale) : f[b];
        }
    } else {
        const uint4 x = *reinterpret_cast<const uint4 *>(slot + e);
        const uint32_t w[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
        for (int c = 0; c < 4; c++) {
            float f[4];
            s8x4_f32(w[c], f);
#pragma unroll
            for (int b = 0; b < 4; b++) out[4 * c + b] = SCALED ? __fmul_rn(f[b], scale) : f[b];
        }
    }
}

// The values at dimensions e, e + 1 (e even) of two staged keys a and b, as
// (a[e], b[e]) and (a[e + 1], b[e + 1]): operands of the packed FMA whose two
// halves accumulate even and odd keys.
template <int F>
__device__ __forceinline__ void slot_vpair2(const unsigned char *sa, const unsigned char *sb, int e, float ca, float cb,
                                            float2 &lo, float2 &hi) {
    if constexpr (F == DF32) {
        lo = make_float2(*reinterpret_cast<const float *>(sa + 4 * e), *reinterpret_cast<const float *>(sb + 4 * e));
        hi = make_float2(*reinterpret_cast<const float *>(sa + 4 * e + 4),
                         *reinterpret_cast<const float *>(sb + 4 * e + 4));
    } else if constexpr (F == DBF16) {
        const uint32_t wa = *reinterpret_cast<const uint32_t *>(sa + 2 * e);
        const uint32_t wb = *reinterpret_cast<const uint32_t *>(sb + 2 * e);
        lo = make_float2(__uint_as_float(wa << 16), __uint_as_float(wb << 16));
        hi = make_float2(__uint_as_float(wa & 0xFFFF0000u), __uint_as_float(wb & 0xFFFF0000u));
    } else {
        float a0, a1, b0, b1;
        if constexpr (F == DQ16) {
            s16x2_f32(*reinterpret_cast<const uint32_t *>(sa + 2 * e), a0, a1);
            s16x2_f32(*reinterpret_cast<const uint32_t *>(sb + 2 * e), b0, b1);
        } else if constexpr (F == DQ4) {
            s4x2_f32(sa[e / 2], a0, a1);
            s4x2_f32(sb[e / 2], b0, b1);
        } else {
            s8x2_f32(*reinterpret_cast<const uint16_t *>(sa + e), a0, a1);
            s8x2_f32(*reinterpret_cast<const uint16_t *>(sb + e), b0, b1);
        }
        lo = make_float2(__fmul_rn(a0, ca), __fmul_rn(b0, cb));
        hi = make_float2(__fmul_rn(a1, ca), __fmul_rn(b1, cb));
    }
}

// Stages one key's record into its slot: a prefix record as it is, a tail
// record [K 64 | V 64] as [K | K[32:64] | V].
template <int F>
__device__ __forceinline__ void stage_key(const fo_decode_page &pg, int64_t g, int64_t pos, unsigned char *slot,
                                          uint64_t *bar) {
    using S = Shape<F>;
    if (pos < pg.prefix_len) {
        const int64_t r = g * pg.prefix_stride + pos;
        sm100::bulk_g2s(slot, reinterpret_cast<const unsigned char *>(pg.codes) + r * S::RB, S::RB, bar);
    } else {
        const int64_t r = g * pg.tail_stride + (pos - pg.prefix_len);
        const unsigned char *rec = reinterpret_cast<const unsigned char *>(pg.tail_codes) + r * S::TB;
        sm100::bulk_g2s(slot, rec, S::bytes(64), bar);
        sm100::bulk_g2s(slot + S::bytes(64), rec + S::bytes(32), S::bytes(32), bar);
        sm100::bulk_g2s(slot + S::bytes(96), rec + S::bytes(64), S::bytes(64), bar);
    }
}

// Coded formats: the decoded scales of this lane's key of chunk c of split s
// of group g, in slot order [T, S0, S1, V0, V1] (a tail key's spatial scale
// serves both heads).  Lanes past the chunk's keys load nothing.
template <int F>
__device__ __forceinline__ void load_chunk_scales(const fo_decode_page &pg, int64_t g, int s, int c, int lane,
                                                  float *sc) {
    const int64_t pos = (int64_t)s * FO_SPLIT + (int64_t)c * Shape<F>::CK + lane;
    if (pos >= min64((int64_t)(s + 1) * FO_SPLIT, pg.last)) return;
    if (pos < pg.prefix_len) {
        const uint16_t *p = pg.scales + (g * pg.prefix_stride + pos) * 5;
#pragma unroll
        for (int i = 0; i < 5; i++) sc[i] = bf16_f32(__ldg(p + i));
    } else {
        const uint16_t *p = pg.tail_scales + (g * pg.tail_stride + (pos - pg.prefix_len)) * 4;
        sc[0] = bf16_f32(__ldg(p));
        sc[1] = sc[2] = bf16_f32(__ldg(p + 1));
        sc[3] = bf16_f32(__ldg(p + 2));
        sc[4] = bf16_f32(__ldg(p + 3));
    }
}

// Bulk L2 prefetch of [addr, addr + bytes), trimmed inward to 16-byte
// boundaries (the prefetch's alignment rule); never reaches outside the range.
__device__ __forceinline__ void prefetch_l2(const void *addr, int64_t bytes) {
    const uint64_t a = reinterpret_cast<uint64_t>(addr);
    const uint64_t lo = (a + 15) & ~15ull, hi = (a + (uint64_t)bytes) & ~15ull;
    if (hi > lo)
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(lo), "r"((uint32_t)(hi - lo)) : "memory");
}

// Asks L2 for every record (and scale) of split s of group g, so that a
// later item's copies find their lines already on chip.
template <int F>
__device__ __forceinline__ void prefetch_item(const fo_decode_page &pg, int64_t g, int s) {
    using S = Shape<F>;
    const int64_t a = (int64_t)s * FO_SPLIT, b = min64(a + FO_SPLIT, pg.last);
    const int64_t pa = a, pb = min64(b, pg.prefix_len);
    if (pb > pa) {
        const int64_t r0 = g * pg.prefix_stride + pa;
        prefetch_l2(reinterpret_cast<const char *>(pg.codes) + r0 * S::RB, (pb - pa) * S::RB);
        if (S::CODED) prefetch_l2(pg.scales + r0 * 5, (pb - pa) * 10);
    }
    const int64_t ta = max64(a, pg.prefix_len), tb = b;
    if (tb > ta) {
        const int64_t r0 = g * pg.tail_stride + (ta - pg.prefix_len);
        prefetch_l2(reinterpret_cast<const char *>(pg.tail_codes) + r0 * S::TB, (tb - ta) * S::TB);
        if (S::CODED) prefetch_l2(pg.tail_scales + r0 * 4, (tb - ta) * 8);
    }
}

// Stages the records of chunk c of split s of group g (the issuing warp's
// lanes each arrive once on the chunk's barrier).  A chunk of prefix records
// only is one TMA tile load through the page's tensor map (rows padded to the
// slot by the box's out-of-bounds fill); a chunk that reaches the tail copies
// record by record.
template <int F>
__device__ __forceinline__ void stage_chunk(const fo_decode_page &pg, int64_t g, int s, int c, int lane,
                                            unsigned char *crec, uint64_t *bar) {
    using S = Shape<F>;
    const int64_t k0 = (int64_t)s * FO_SPLIT + (int64_t)c * S::CK;
    const int64_t w1 = min64(k0 + S::CK, min64((int64_t)s * FO_SPLIT + FO_SPLIT, pg.last));
    const int nk = (int)max64(0, w1 - k0);
    if (pg.has_map && nk > 0 && w1 <= pg.prefix_len) {
        const uint32_t bytes = lane == 0 ? (uint32_t)(S::CK * S::SLOT) : 0u;
        asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(sm100::smem_u32(bar)), "r"(bytes)
                     : "memory");
        if (lane == 0) sm100::tma_load_3d(crec, &pg.rec_map, bar, 0, (int)k0, (int)g);
        return;
    }
    const uint32_t bytes = lane < nk ? (uint32_t)S::RB : 0u;
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(sm100::smem_u32(bar)), "r"(bytes)
                 : "memory");
    if (lane < nk) stage_key<F>(pg, g, k0 + lane, crec + lane * S::SLOT, bar);
}

// rotate_query (rotation.rs:106-111: 2^-5 H D x) of a query head held as
// dimensions (2 lane, 2 lane + 1): lanes 0-15 hold the temporal block (kind
// 0), lanes 16-31 the spatial block (kind 1), element 2 (lane % 16) and the
// next.  The first butterfly stage pairs a lane's own two elements, the
// others pair lanes lane ^ 1, ^ 2, ^ 4, ^ 8 (inside the block's half-warp).
__device__ __forceinline__ float2 rotate_query_pair(float2 v, int lane) {
    const uint32_t signs = (lane >> 4) ? rotation_signs(1) : rotation_signs(0);
    const int i0 = 2 * (lane & 15);
    v.x = __uint_as_float(__float_as_uint(v.x) ^ (((signs >> i0) & 1u) << 31));
    v.y = __uint_as_float(__float_as_uint(v.y) ^ (((signs >> (i0 + 1)) & 1u) << 31));
    v = make_float2(__fadd_rn(v.x, v.y), __fsub_rn(v.x, v.y));
#pragma unroll
    for (int d = 1; d < 16; d <<= 1) {
        const float px = __shfl_xor_sync(0xffffffffu, v.x, d), py = __shfl_xor_sync(0xffffffffu, v.y, d);
        v = make_float2(butterfly(v.x, px, lane & d), butterfly(v.y, py, lane & d));
    }
    return make_float2(__fmul_rn(v.x, 0.03125f), __fmul_rn(v.y, 0.03125f));
}

// Waits on a pair's named barrier (id 1 + pair, 64 threads) and returns
// whether `ok` holds in both warps.
__device__ __forceinline__ bool pair_sync_and(int pair, bool ok) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.u32 p, %1, 0;\n\t"
        "barrier.red.and.pred q, %2, 64, p;\n\t"
        "selp.u32 %0, 1, 0, q;\n\t}"
        : "=r"(r)
        : "r"((uint32_t)ok), "r"(1 + pair)
        : "memory");
    return r != 0;
}

// Persistent CTAs: every pair of warps walks the work items (page, split,
// group) with a stride of all pairs of the grid.
template <int F, bool FAST, int R>
__global__ void __launch_bounds__(Shape<F>::THREADS, Shape<F>::MIN_CTAS)
    decode_kernel(const __grid_constant__ fo_decode_page page0, const fo_decode_page *pages, int64_t n_pages,
                  int64_t groups, int max_splits) {
    using S = Shape<F>;
    using L = Smem<F, R>;
    constexpr int CK = S::CK, NCH = S::NCH, NPAIR = S::NPAIR;
    extern __shared__ __align__(128) unsigned char dsm[];
    const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
    const int pair = warp >> 1, hd = warp & 1;
    const bool stager = hd == 0;  // the head-0 warp stages the pair's chunks
    uint64_t *bars = reinterpret_cast<uint64_t *>(dsm + L::OFF_BAR);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(dsm + L::OFF_FLAGS);
    // Buffer b of this pair: slots and decoded scales.
    auto brec = [&](int b) { return dsm + (size_t)(pair * S::NBUF + b) * CK * S::SLOT; };
    auto bscl = [&](int b) { return reinterpret_cast<float *>(dsm + L::OFF_SCL) + (pair * S::NBUF + b) * CK * 5; };
    uint64_t *pbar = bars + pair * S::NBUF;
    float(*qw)[FO_HD] = reinterpret_cast<float(*)[FO_HD]>(dsm + L::OFF_Q) + warp * R;
    float(*pw)[CK] = reinterpret_cast<float(*)[CK]>(dsm + L::OFF_P) + warp * R;
    const int64_t H = 2 * groups;
    const int64_t n_pairs = (int64_t)gridDim.x * NPAIR;
    // The work items are every page's own splits x groups, page-major, split
    // index next and group fastest (a page short of max_splits leaves no
    // empty items behind: the pairs share only real work).  The warp reads
    // the pages' split counts 32 at a time; `block` hands back lane's page
    // of the block starting at b, its inclusive prefix of splits and the
    // block's total.
    auto page_at = [&](int64_t p) -> const fo_decode_page * { return pages ? pages + p : &page0; };
    auto block = [&](int64_t b, int &s, int &incl) -> int64_t {
        const int64_t p = b + lane;
        s = p < n_pages ? page_at(p)->splits : 0;
        incl = s;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int x = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += x;
        }
        return __shfl_sync(0xffffffffu, incl, 31);
    };
    int64_t n_items = 0;
    for (int64_t b = 0; b < n_pages; b += 32) {
        int s, incl;
        n_items += block(b, s, incl);
    }
    n_items *= groups;

    if (t < NPAIR * S::NBUF) sm100::mbar_init(&bars[t], 32);
    if (t == 0) *abort_flag = 0;
    __syncthreads();
    // The merge kernel may launch now; it waits for this grid to finish.
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

    struct Item {
        const fo_decode_page *pp;  // the page (kernel parameter or device array; read in place)
        int s;
        int64_t g;
        int64_t it;
    };
    // Item it, if there is one (warp-uniform; the whole warp takes part).
    auto find = [&](Item &x, int64_t it) -> bool {
        if (it >= n_items) return false;
        x.g = it % groups;
        x.it = it;
        const int64_t k = it / groups;  // the split's index over all pages
        int64_t base = 0;               // splits of the pages before block b
        for (int64_t b = 0; b < n_pages; b += 32) {
            int s, incl;
            const int64_t total = block(b, s, incl);
            if (k < base + total) {
                const int l = __ffs(__ballot_sync(0xffffffffu, base + incl > k)) - 1;
                x.pp = page_at(b + l);
                x.s = (int)(k - base - __shfl_sync(0xffffffffu, incl - s, l));
                return true;
            }
            base += total;
        }
        return false;
    };
    // This warp's head rows of the item's queries: dims 2 lane, 2 lane + 1.
    auto load_q = [&](const Item &x, float2 *qv) {
#pragma unroll
        for (int r = 0; r < R; r++)
            qv[r] = __ldg(reinterpret_cast<const float2 *>(x.pp->q + (r * H + 2 * x.g + hd) * FO_HD) + lane);
        if (x.pp->rotated) {
#pragma unroll
            for (int r = 0; r < R; r++) qv[r] = rotate_query_pair(qv[r], lane);
        }
    };

    Item cur, nxt;
    // Pair ids run across the CTAs first, so that items spread over every SM.
    bool have = find(cur, (int64_t)pair * gridDim.x + blockIdx.x);
    bool have_n = have && find(nxt, cur.it + n_pairs);
    float2 qv[R];
    if (have) {
        load_q(cur, qv);  // ahead of the bulk copies in the memory queues
        if (stager) {
#pragma unroll
            for (int c = 0; c < S::NBUF; c++) {
                stage_chunk<F>(*cur.pp, cur.g, cur.s, c, lane, brec(c), &pbar[c]);
                if constexpr (S::CODED) {
                    float sc[5];
                    load_chunk_scales<F>(*cur.pp, cur.g, cur.s, c, lane, sc);
                    if (lane < min64(CK, cur.pp->last - (int64_t)cur.s * FO_SPLIT - (int64_t)c * CK))
#pragma unroll
                        for (int i = 0; i < 5; i++) bscl(c)[lane * 5 + i] = sc[i];
                }
            }
        }
    }
    pair_sync_and(pair, true);  // the first chunks' scales are visible
    uint32_t u = 0;             // chunks consumed by this pair
    bool ok = true;
    while (have && ok) {
#pragma unroll
        for (int r = 0; r < R; r++) *reinterpret_cast<float2 *>(&qw[r][2 * lane]) = qv[r];
        __syncwarp();
        const fo_decode_page &pg = *cur.pp;
        const int64_t p0 = (int64_t)cur.s * FO_SPLIT;
        const int64_t p_end = min64(p0 + FO_SPLIT, pg.last);
        // Row r sees positions [0, last - R + 1 + r) (kv.rs:851-855).
        const int64_t len0 = pg.last - R + 1;
        // Per row: the running max (warp-uniform), this lane's share of the
        // denominator, and this lane's output dimensions 2*lane (oa) and
        // 2*lane + 1 (ob), each as an (even keys, odd keys) pair of sums.
        float m_st[R], l_st[R];
        float2 oa[R], ob[R];
#pragma unroll
        for (int r = 0; r < R; r++) {
            m_st[r] = -INFINITY;
            l_st[r] = 0.0f;
            oa[r] = make_float2(0.0f, 0.0f);
            ob[r] = make_float2(0.0f, 0.0f);
        }
        for (int c = 0; c < NCH && ok; c++, u++) {
            const int b = (int)(u % S::NBUF);
            // The stager asks for chunk u + NBUF's scales now; they land while
            // this chunk computes and are published with its copies below.
            const int c2 = c + S::NBUF;
            const bool in_item = c2 < NCH;
            const Item &x2 = in_item ? cur : nxt;
            const bool has2 = in_item || have_n;
            float sc_pre[5];
            if constexpr (S::CODED) {
                if (stager && has2) load_chunk_scales<F>(*x2.pp, x2.g, x2.s, in_item ? c2 : c2 - NCH, lane, sc_pre);
            }
            const int64_t k0 = p0 + (int64_t)c * CK;
            const int64_t w1 = min64(k0 + CK, p_end);
            const int nk = (int)max64(0, w1 - k0);  // the chunk's keys (warp-uniform)
            const bool staged = sm100::mbar_wait(&pbar[b], (u / S::NBUF) & 1, abort_flag, pg.err);
            if (c == 0 && have_n && stager && lane == 0) {
                // The pair's next item streams into L2 while this one
                // computes (one item ahead: a whole batch of pages would
                // not fit in L2).
                prefetch_item<F>(*nxt.pp, nxt.g, nxt.s);
            }
            if (c == NCH - 1 && have_n) load_q(nxt, qv);  // the next item's queries, early
            const unsigned char *crec = brec(b);
            const float *cscl = bscl(b);
            if (nk > 0 && staged) {
                // Logit of this lane's key for each row of this warp's head.
                // The packed FMA pairs dimensions (d, d + 1) into (even, odd)
                // partial sums, each half an ordinary fmaf.
                const int key = min(lane, nk - 1);  // idle lanes read a staged key, masked below
                const unsigned char *ks = crec + key * S::SLOT;
                const float *kscl = cscl + key * 5;
                float lg[R];
                {
                    // Coded formats: the temporal (acc) and spatial (acs) blocks
                    // accumulate codes apart and take their scales once.
                    float2 acc[R], acs[R];
#pragma unroll
                    for (int r = 0; r < R; r++) acc[r] = acs[r] = make_float2(0.0f, 0.0f);
#pragma unroll
                    for (int part = 0; part < 4; part++) {  // T[0:16], T[16:32], S_h[0:16], S_h[16:32]
                        const int e = part < 2 ? 16 * part : 32 + 32 * hd + 16 * (part - 2);
                        float kv[16];
                        slot_span16<F, !S::CODED>(ks, e, 1.0f, kv);
#pragma unroll
                        for (int d = 0; d < 16; d += 4) {
#pragma unroll
                            for (int r = 0; r < R; r++) {
                                const float4 x = *reinterpret_cast<const float4 *>(&qw[r][16 * part + d]);
                                float2 &a = (S::CODED && part >= 2) ? acs[r] : acc[r];
                                a = __ffma2_rn(make_float2(x.x, x.y), make_float2(kv[d], kv[d + 1]), a);
                                a = __ffma2_rn(make_float2(x.z, x.w), make_float2(kv[d + 2], kv[d + 3]), a);
                            }
                        }
                    }
#pragma unroll
                    for (int r = 0; r < R; r++) {
                        if constexpr (S::CODED)
                            lg[r] = __fadd_rn(__fmul_rn(kscl[0], __fadd_rn(acc[r].x, acc[r].y)),
                                              __fmul_rn(kscl[1 + hd], __fadd_rn(acs[r].x, acs[r].y)));
                        else
                            lg[r] = __fadd_rn(acc[r].x, acc[r].y);
                    }
                }
                // Online softmax of the chunk per row (the reference's tile
                // step: chunk max, rescale, exp(s - max)), the rows interleaved
                // so their shuffles overlap.  Branch-free: a row with no
                // position in the chunk keeps its state.  Each lane keeps the
                // denominator of its own keys; the lanes add up once per item.
                // A full chunk (every row sees all of its keys) takes a path
                // without masks and with constant slot offsets.
                const bool full = nk == CK && k0 + CK <= len0;
                float ev[R], cm[R];
#pragma unroll
                for (int r = 0; r < R; r++) {
                    const int lim = full ? CK : (int)min64(nk, max64(0, len0 + r - k0));  // the row's keys: [0, lim)
                    ev[r] = lane < lim ? __fmul_rn(lg[r], 0.125f) : -INFINITY;
                    cm[r] = ev[r];
                }
#pragma unroll
                for (int o = 16; o > 0; o >>= 1)
#pragma unroll
                    for (int r = 0; r < R; r++) cm[r] = fmaxf(cm[r], __shfl_xor_sync(0xffffffffu, cm[r], o));
#pragma unroll
                for (int r = 0; r < R; r++) {
                    const bool empty = cm[r] == -INFINITY;
                    const float m_old = m_st[r];
                    const float m_new = rmax(m_old, cm[r]);
                    const float alpha = empty ? 1.0f : (m_old == -INFINITY ? 0.0f : expf(__fsub_rn(m_old, m_new)));
                    ev[r] = (ev[r] != -INFINITY && !empty) ? softmax_exp<FAST>(__fsub_rn(ev[r], m_new)) : 0.0f;
                    pw[r][lane] = ev[r];
                    m_st[r] = m_new;
                    l_st[r] = __fadd_rn(__fmul_rn(l_st[r], alpha), ev[r]);
                    oa[r] = __fmul2_rn(oa[r], make_float2(alpha, alpha));
                    ob[r] = __fmul2_rn(ob[r], make_float2(alpha, alpha));
                }
                __syncwarp();
                // O += P V in key order: even keys into the .x halves, odd
                // keys into the .y halves; this lane's two dimensions.  Keys
                // before len0 are visible to every row; the last R - 1
                // positions only to the rows that see them (a row never
                // touches a value it does not see, so a NaN there stays out).
                const int vblk = 3 + (lane >> 4);  // this lane's value scale block
                auto pv4 = [&](int j) {           // keys j .. j + 3, all rows
                    float2 va[2], vb[2];          // (key j + 2i, key j + 2i + 1) at dims 2 lane, 2 lane + 1
#pragma unroll
                    for (int i = 0; i < 2; i++)
                        slot_vpair2<F>(crec + (j + 2 * i) * S::SLOT, crec + (j + 2 * i + 1) * S::SLOT, 96 + 2 * lane,
                                       S::CODED ? cscl[(j + 2 * i) * 5 + vblk] : 1.0f,
                                       S::CODED ? cscl[(j + 2 * i + 1) * 5 + vblk] : 1.0f, va[i], vb[i]);
#pragma unroll
                    for (int r = 0; r < R; r++) {
                        const float4 p = *reinterpret_cast<const float4 *>(&pw[r][j]);
                        oa[r] = __ffma2_rn(make_float2(p.x, p.y), va[0], oa[r]);
                        ob[r] = __ffma2_rn(make_float2(p.x, p.y), vb[0], ob[r]);
                        oa[r] = __ffma2_rn(make_float2(p.z, p.w), va[1], oa[r]);
                        ob[r] = __ffma2_rn(make_float2(p.z, p.w), vb[1], ob[r]);
                    }
                };
                if (full) {
#pragma unroll
                    for (int j = 0; j < CK; j += 4) pv4(j);
                } else {
                    const int n_all = (int)max64(0, min64(w1, len0) - k0);
                    int j = 0;
                    for (; j + 4 <= n_all; j += 4) pv4(j);
                    for (; j < nk; j++) {
                        const float2 v =
                            slot_pair<F>(crec + j * S::SLOT, 96 + 2 * lane, S::CODED ? cscl[j * 5 + vblk] : 1.0f);
                        const bool all = j < n_all;
#pragma unroll
                        for (int r = 0; r < R; r++) {
                            if (all || k0 + j < len0 + r) {
                                const float p = pw[r][j];
                                if (j & 1) {
                                    oa[r].y = fmaf(p, v.x, oa[r].y);
                                    ob[r].y = fmaf(p, v.y, ob[r].y);
                                } else {
                                    oa[r].x = fmaf(p, v.x, oa[r].x);
                                    ob[r].x = fmaf(p, v.y, ob[r].x);
                                }
                            }
                        }
                    }
                }
                __syncwarp();
            }
            // Both warps are done with buffer b (and agree whether their
            // waits succeeded); the stager refills it with chunk u + NBUF and
            // its scales (read by both warps NBUF chunks later, after the
            // next pair barrier).
            ok = pair_sync_and(pair, staged);
            if (ok && stager && has2) {
                const int cc = in_item ? c2 : c2 - NCH;
                if constexpr (S::CODED) {
                    if (lane < min64(CK, x2.pp->last - (int64_t)x2.s * FO_SPLIT - (int64_t)cc * CK))
#pragma unroll
                        for (int i = 0; i < 5; i++) bscl(b)[lane * 5 + i] = sc_pre[i];
                }
                sm100::fence_proxy_async_smem();  // the slot reads before the copies' writes
                stage_chunk<F>(*x2.pp, x2.g, x2.s, cc, lane, brec(b), &pbar[b]);
            }
        }
        if (!ok) break;
        // This warp's head: the split's unnormalized partial (the lanes'
        // denominators added in a fixed order).
#pragma unroll
        for (int o = 16; o > 0; o >>= 1)
#pragma unroll
            for (int r = 0; r < R; r++) l_st[r] = __fadd_rn(l_st[r], __shfl_xor_sync(0xffffffffu, l_st[r], o));
#pragma unroll
        for (int r = 0; r < R; r++) {
            const int64_t row_head = (int64_t)r * H + 2 * cur.g + hd;
            *reinterpret_cast<float2 *>(pg.part_o + (row_head * pg.splits + cur.s) * FO_HD + 2 * lane) =
                make_float2(__fadd_rn(oa[r].x, oa[r].y), __fadd_rn(ob[r].x, ob[r].y));
            if (lane == 0)
                *reinterpret_cast<float2 *>(pg.part_ml + (row_head * pg.splits + cur.s) * 2) =
                    make_float2(m_st[r], l_st[r]);
        }
        have = have_n;
        if (have) {
            cur = nxt;
            have_n = find(nxt, cur.it + n_pairs);
        }
    }
    if (!ok && stager) {
        // A wait that gave up (error word raised) at chunk u - 1: let the
        // pair's copies in flight (chunks u - 1 .. u + NBUF - 2) land before
        // the CTA can exit; a phase that was never issued gives up after the
        // bound.
#pragma unroll
        for (int i = 0; i < S::NBUF; i++) {
            const uint32_t w = u - 1 + i;
            sm100::mbar_wait_drain(&pbar[w % S::NBUF], (w / S::NBUF) & 1);
        }
    }
}

// Merges the split partials of every (row, head) of a page, in split order,
// and applies the sink (the reference's merge and epilogue,
// kv.rs:775-813).  Launched as a programmatic dependent of the decode
// kernel: it starts early and waits (griddepcontrol.wait) until every
// partial is written.  CTA per (row, head): the splits' (max, denominator)
// pairs go to shared memory, then thread (4 dimensions, slice) sums the
// slice's splits k = slice, slice + SLICES, ... with its loads in flight
// together, and the slices add in order.  A split whose max is -inf saw no
// position and is skipped.  Everything depends only on the row's own length.
constexpr int MERGE_SLICES = 16;
constexpr int MERGE_THREADS = (FO_HD / 4) * MERGE_SLICES;

__global__ void __launch_bounds__(MERGE_THREADS) merge_kernel(const __grid_constant__ fo_decode_page page0,
                                                              const fo_decode_page *pages, int64_t H,
                                                              fo_append_page *advance) {
    extern __shared__ __align__(16) float msm[];
    asm volatile("griddepcontrol.wait;" ::: "memory");
    if (advance && blockIdx.x == 0 && threadIdx.x == 0) {
        // A batch plan's step: this page's append and decode are complete, so
        // its next append index moves on (a full tail keeps its capacity).
        fo_append_page &a = advance[blockIdx.y];
        if (a.first < a.tail_stride) a.first += 1;
    }
    const fo_decode_page *pp = pages ? pages + blockIdx.y : &page0;
    const int64_t row_head = blockIdx.x;
    const int64_t r = row_head / H, h = row_head % H;
    if (r >= pp->rows) return;
    if (pp->err && *reinterpret_cast<volatile unsigned *>(pp->err)) {
        // A bounded wait of the decode gave up: its partials are stale, so the
        // row is NaN rather than a plausible wrong answer.
        if (threadIdx.x < FO_HD) pp->out[row_head * FO_HD + threadIdx.x] = __int_as_float(0x7fc00000);
        return;
    }
    const int splits = pp->splits;
    const int64_t row_len = pp->last - pp->rows + 1 + r;
    // The row's partials: one per FO_SPLIT positions from 0, or (prefix_splits
    // set) one per `chunk` splits of the prefix and then of its tail.
    int n = (int)((row_len + FO_SPLIT - 1) / FO_SPLIT);
    if (pp->prefix_splits) {
        const int tail_splits = (int)((row_len - pp->prefix_len + FO_SPLIT - 1) / FO_SPLIT);
        n = (pp->prefix_splits + pp->chunk - 1) / pp->chunk + (tail_splits + pp->chunk - 1) / pp->chunk;
    }
    float *fk = msm;                                     // [splits] factors exp(m_k - M); -1 skips
    float *lk = msm + splits;                            // [splits] denominators
    float4 *part = reinterpret_cast<float4 *>(lk + splits + 4 - (2 * splits) % 4);  // [SLICES][16]
    const float *ml = pp->part_ml + row_head * splits * 2;
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
    // This thread's output slices of the first 8 * SLICES partials, loaded
    // now so that they are in flight with the (max, denominator) loads.
    const int dq = t % (FO_HD / 4), sl = t / (FO_HD / 4);
    const float4 *po = reinterpret_cast<const float4 *>(pp->part_o + row_head * splits * FO_HD) + dq;
    float4 o0[8];
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const int k = sl + i * MERGE_SLICES;
        o0[i] = k < n ? __ldcg(po + (int64_t)k * (FO_HD / 4)) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    __shared__ float wred[2][MERGE_THREADS / 32];
    // Row maximum over the splits: per thread, then per warp, then over the
    // warps (a maximum does not depend on the order).
    float m = -INFINITY;
    for (int k = t; k < n; k += MERGE_THREADS) {
        const float2 x = __ldcg(reinterpret_cast<const float2 *>(ml) + k);
        fk[k] = x.x;
        lk[k] = x.y;
        m = rmax(m, x.x);
    }
    m = warp_max(m);
    if (lane == 0) wred[0][warp] = m;
    __syncthreads();
#pragma unroll
    for (int w = 0; w < MERGE_THREADS / 32; w++) m = rmax(m, wred[0][w]);
    // Split factors exp(m_k - M) (-1 marks an empty split) and the
    // denominator: per thread over its splits, a butterfly per warp, then
    // the warps in order, so every call sums in the same order.
    float den = 0.0f;
    for (int k = t; k < n; k += MERGE_THREADS) {
        const float f = fk[k] == -INFINITY ? -1.0f : expf(fk[k] - m);
        fk[k] = f;
        if (f >= 0.0f) den = fmaf(lk[k], f, den);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) den = __fadd_rn(den, __shfl_xor_sync(0xffffffffu, den, o));
    if (lane == 0) wred[1][warp] = den;
    __syncthreads();
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int k0 = sl; k0 < n; k0 += 8 * MERGE_SLICES) {
        float4 o[8];
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const int k = k0 + i * MERGE_SLICES;
            o[i] = k0 == sl ? o0[i] : k < n ? __ldcg(po + (int64_t)k * (FO_HD / 4)) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const int k = k0 + i * MERGE_SLICES;
            if (k < n && fk[k] >= 0.0f) {
                acc.x = fmaf(o[i].x, fk[k], acc.x);
                acc.y = fmaf(o[i].y, fk[k], acc.y);
                acc.z = fmaf(o[i].z, fk[k], acc.z);
                acc.w = fmaf(o[i].w, fk[k], acc.w);
            }
        }
    }
    part[sl * (FO_HD / 4) + dq] = acc;
    __syncthreads();
    if (t < FO_HD) {
        den = 0.0f;
#pragma unroll
        for (int w = 0; w < MERGE_THREADS / 32; w++) den = __fadd_rn(den, wred[1][w]);
        const float *pf = reinterpret_cast<const float *>(part);
        float o = 0.0f;
#pragma unroll
        for (int i = 0; i < MERGE_SLICES; i++) o = __fadd_rn(o, pf[i * FO_HD + t]);
        const float lse = m + logf(den);
        float y = (o / den) * sink_scale(pp->sinks[h], lse);
        if (pp->rotated) {
            // unrotate (rotation.rs:113-119: 2^-5 D H x) of the output block
            // this warp holds, one element per lane: value 0..32 (kind 2) in
            // warp 0, value 32..64 (kind 3) in warp 1.
#pragma unroll
            for (int half = 1; half < 32; half <<= 1)
                y = butterfly(y, __shfl_xor_sync(0xffffffffu, y, half), lane & half);
            y = __uint_as_float(__float_as_uint(y) ^
                                ((((warp ? rotation_signs(3) : rotation_signs(2)) >> lane) & 1u) << 31));
            y = __fmul_rn(y, 0.03125f);
        }
        pp->out[row_head * FO_HD + t] = y;
    }
}

}  // namespace fo

static PFN_cuTensorMapEncodeTiled_v12000 record_map_encoder() {
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

template <int F>
static bool record_map(CUtensorMap *map, const void *codes, int64_t prefix_len, int64_t prefix_stride,
                       int64_t groups, CUtensorMapDataType type) {
    using S = fo::Shape<F>;
    auto fn = record_map_encoder();
    if (!fn || prefix_len <= 0 || prefix_len >= (int64_t(1) << 31)) return false;
    cuuint64_t dims[3] = {(cuuint64_t)(S::RB / S::E), (cuuint64_t)prefix_len, (cuuint64_t)groups};
    cuuint64_t strides[2] = {(cuuint64_t)S::RB, (cuuint64_t)prefix_stride * S::RB};
    cuuint32_t box[3] = {(cuuint32_t)(S::SLOT / S::E), (cuuint32_t)S::CK, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    return fn(map, type, 3, const_cast<void *>(codes), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
              CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) ==
           CUDA_SUCCESS;
}

bool fo_make_record_map(CUtensorMap *map, const void *codes, int format, int64_t prefix_len, int64_t prefix_stride,
                        int64_t groups) {
    if ((reinterpret_cast<uintptr_t>(codes) & 15) != 0) return false;
    switch (format & ~FO_KV_ROTATED_BIT) {
    case fo::DF32: return record_map<fo::DF32>(map, codes, prefix_len, prefix_stride, groups, CU_TENSOR_MAP_DATA_TYPE_FLOAT32);
    case fo::DQ16: return record_map<fo::DQ16>(map, codes, prefix_len, prefix_stride, groups, CU_TENSOR_MAP_DATA_TYPE_UINT16);
    case fo::DQ8: return record_map<fo::DQ8>(map, codes, prefix_len, prefix_stride, groups, CU_TENSOR_MAP_DATA_TYPE_UINT8);
    case fo::DQ4: return record_map<fo::DQ4>(map, codes, prefix_len, prefix_stride, groups, CU_TENSOR_MAP_DATA_TYPE_UINT8);
    case fo::DBF16: return record_map<fo::DBF16>(map, codes, prefix_len, prefix_stride, groups, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16);
    }
    return false;
}

// The merge kernel, as a programmatic dependent of the decode kernel just
// launched on `stream`.  Its dynamic shared memory (2 floats per split plus
// the slice sums) stays below 200 KB up to 25,000 splits (3.2M positions).
constexpr int MERGE_DSMEM_MAX = 200 * 1024;
static cudaError_t launch_merge(const fo_decode_page &page0, const fo_decode_page *dev_pages, int64_t n_pages,
                                int64_t groups, int max_splits, int rows, cudaStream_t stream,
                                fo_append_page *advance = nullptr) {
    // The attribute belongs to each device's context: set once per device.
    static std::atomic<unsigned long long> configured{0};
    int dev = 0;
    cudaGetDevice(&dev);
    const unsigned long long bit = 1ull << (dev & 63);
    if (!(configured.load() & bit)) {
        // The kernel's own static array sits beside the dynamic allowance.
        cudaError_t e =
            cudaFuncSetAttribute(fo::merge_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, MERGE_DSMEM_MAX);
        if (e != cudaSuccess) return e;
        configured.fetch_or(bit);
    }
    const size_t smem = (size_t)(2 * max_splits + 4 + fo::MERGE_SLICES * FO_HD) * sizeof(float);
    if (smem > MERGE_DSMEM_MAX) return cudaErrorInvalidValue;
    const int64_t H = 2 * groups;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(rows * H), (unsigned)n_pages);
    cfg.blockDim = dim3(fo::MERGE_THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, fo::merge_kernel, page0, dev_pages, H, advance);
}

// Launches one instantiation as persistent CTAs (as many as fit on the
// device at once, at most one per item), raising its dynamic shared-memory
// limit once.
template <int F, bool FAST, int R>
static cudaError_t launch_one(const fo_decode_page &page0, const fo_decode_page *dev_pages, int64_t n_pages,
                              int64_t groups, int max_splits, cudaStream_t stream, fo_append_page *advance) {
    constexpr int smem = fo::Smem<F, R>::BYTES;
    constexpr int threads = fo::Shape<F>::THREADS;
    // CTAs of this instantiation each device holds at once (the attribute and
    // the occupancy belong to each device's context: set up once per device).
    static std::atomic<int> resident[64];
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    int res = resident[dev & 63].load();
    if (!res) {
        e = cudaFuncSetAttribute(fo::decode_kernel<F, FAST, R>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return e;
        int sms = 0, per_sm = 0;
        if ((e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess) return e;
        e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fo::decode_kernel<F, FAST, R>, threads, smem);
        if (e != cudaSuccess) return e;
        res = std::max(1, sms * per_sm);
        resident[dev & 63].store(res);
    }
    const int64_t items = n_pages * (int64_t)max_splits * groups;
    const unsigned grid = (unsigned)std::min<int64_t>(items, res);
    fo::decode_kernel<F, FAST, R><<<grid, threads, smem, stream>>>(page0, dev_pages, n_pages, groups, max_splits);
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    return launch_merge(page0, dev_pages, n_pages, groups, max_splits, R, stream, advance);
}

template <int F, bool FAST>
static cudaError_t launch_rows(int rows, const fo_decode_page &page0, const fo_decode_page *dev_pages, int64_t n_pages,
                               int64_t groups, int max_splits, cudaStream_t stream, fo_append_page *advance) {
    switch (rows) {
    case 1: return launch_one<F, FAST, 1>(page0, dev_pages, n_pages, groups, max_splits, stream, advance);
    case 2: return launch_one<F, FAST, 2>(page0, dev_pages, n_pages, groups, max_splits, stream, advance);
    case 3: return launch_one<F, FAST, 3>(page0, dev_pages, n_pages, groups, max_splits, stream, advance);
    case 4: return launch_one<F, FAST, 4>(page0, dev_pages, n_pages, groups, max_splits, stream, advance);
    case 5: return launch_one<F, FAST, 5>(page0, dev_pages, n_pages, groups, max_splits, stream, advance);
    case 6: return launch_one<F, FAST, 6>(page0, dev_pages, n_pages, groups, max_splits, stream, advance);
    case 7: return launch_one<F, FAST, 7>(page0, dev_pages, n_pages, groups, max_splits, stream, advance);
    case 8: return launch_one<F, FAST, 8>(page0, dev_pages, n_pages, groups, max_splits, stream, advance);
    }
    return cudaErrorInvalidValue;
}

static cudaError_t launch_decode(const fo_decode_page &page0, const fo_decode_page *dev_pages, int64_t n_pages,
                                 int format, int64_t groups, int fast_exp, int64_t max_splits, int rows,
                                 cudaStream_t stream, fo_append_page *advance = nullptr) {
    if (n_pages <= 0 || max_splits <= 0) return cudaSuccess;
    const int ms = (int)max_splits;
    format &= ~FO_KV_ROTATED_BIT;  // rotation travels in the pages (fo_decode_page::rotated)
#define FO_DEC_CASE(FMT)                                                                        \
    case FMT:                                                                                   \
        return fast_exp ? launch_rows<FMT, true>(rows, page0, dev_pages, n_pages, groups, ms, stream, advance) \
                        : launch_rows<FMT, false>(rows, page0, dev_pages, n_pages, groups, ms, stream, advance);
    switch (format) {
        FO_DEC_CASE(fo::DF32)
        FO_DEC_CASE(fo::DQ16)
        FO_DEC_CASE(fo::DQ8)
        FO_DEC_CASE(fo::DQ4)
        FO_DEC_CASE(fo::DBF16)
    }
#undef FO_DEC_CASE
    return cudaErrorInvalidValue;
}

extern "C" cudaError_t fo_launch_decode_one(const fo_decode_page *page, int format, int64_t groups, int fast_exp,
                                            cudaStream_t stream) {
    if (page->prefix_splits) return fo_launch_decode_tc(page, groups, fast_exp, stream);
    return launch_decode(*page, nullptr, 1, format, groups, fast_exp, page->splits, page->rows, stream);
}

extern "C" cudaError_t fo_launch_decode_batch(const fo_decode_page *dev_pages, int64_t n_pages, int format,
                                              int64_t groups, int fast_exp, int64_t max_splits, int max_rows,
                                              fo_append_page *advance, cudaStream_t stream) {
    fo_decode_page none{};
    return launch_decode(none, dev_pages, n_pages, format, groups, fast_exp, max_splits, max_rows, stream, advance);
}

extern "C" cudaError_t fo_launch_decode_merge(const fo_decode_page *page, int64_t groups, cudaStream_t stream) {
    return launch_merge(*page, nullptr, 1, groups, page->splits, page->rows, stream);
}
