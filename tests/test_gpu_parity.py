"""GPU parity of the CUDA kernels against the CPU oracle and the reference's
golden fixtures, called through the C ABI (libfo_cuda.so).

Tolerances are the reference's: |a - b| <= tol * (1 + |b|) with tol 1e-5 for
FP32 paths (prefill64/tests.rs:80-85), the f64 tables' own bounds for the
golden cases, 1e-5 * (1 + |b|) between position partitions of a split
cache (src/quant/kv/tests.rs:253-280); integer codes are bit-exact."""

import os

import numpy as np
import pytest

import fo_cuda as F
import generators as G
import oracle as O

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

GOLD = np.load(os.path.join(os.path.dirname(__file__), "golden", "attention_golden.npz"))


@pytest.fixture(scope="module")
def ctx():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    c = F.Context(0)
    yield c
    c.close()


def dev(x):
    return torch.from_numpy(np.ascontiguousarray(x)).cuda()


def close(actual, expected, absolute, relative):
    a = np.asarray(actual, np.float64)
    b = np.asarray(expected, np.float64)
    err = np.abs(a - b) - (absolute + relative * np.abs(b))
    assert np.isfinite(a).all() == np.isfinite(b).all()
    assert (err <= 0).all(), f"{(err > 0).sum()} of {err.size} out of tolerance, worst excess {err.max():.3e}"


def run_attention(ctx, q, k, v, heads, kv_heads, dim, geometry, sinks, generated_k=None, options=None, mem="device"):
    ql = q.size // (heads * dim)
    if mem == "host":
        out = np.zeros(q.size, np.float32)
        F.attention_with(q, k, v, ql, geometry, sinks, out, heads, kv_heads, dim, generated_k=generated_k,
                         options=options, ctx=ctx)
        return out
    out = torch.zeros(q.size, dtype=torch.float32, device="cuda")
    gk = dev(generated_k) if generated_k is not None else None
    F.attention_with(dev(q), dev(k), dev(v), ql, geometry, dev(sinks), out, heads, kv_heads, dim, generated_k=gk,
                     options=options, ctx=ctx)
    torch.cuda.synchronize()
    return out.cpu().numpy()


# ------------------------------------------------------------------ prefill
def test_known_answer_image_boundaries_and_sink(ctx):
    """src/kernels/tests.rs:283-309, through the C ABI with host buffers."""
    qk = np.zeros(5, np.float32)
    out = run_attention(ctx, qk, qk, GOLD["kat5_values"], 1, 1, 1, (0, 1, 3), np.zeros(1, np.float32), mem="host")
    close(out, GOLD["kat5_expected"], 1e-6, 1e-7)
    out = run_attention(ctx, np.zeros(1, np.float32), np.zeros(1, np.float32), np.array([13.0], np.float32), 1, 1, 1,
                        (0, 0, 0), np.array([-np.inf], np.float32), mem="host")
    assert out.tolist() == [13.0]


@pytest.mark.parametrize("i", range(len(G.DENSE_TABLE)))
def test_dense_table(ctx, i):
    """src/kernels/tests.rs:250-281: 2e-6 absolute + 4e-6 relative of f64."""
    ql, kvl, h, d, off, st, en = G.DENSE_TABLE[i]
    q, k, v, s = (G.lcg_values(ql * h * d, 71), G.lcg_values(kvl * h * d, 83), G.lcg_values(kvl * h * d, 117),
                  G.lcg_values(h, 24))
    close(run_attention(ctx, q, k, v, h, h, d, (off, st, en), s), GOLD[f"dense_{i}"], 2e-6, 4e-6)


def test_extreme_logits_and_sinks(ctx):
    """src/kernels/tests.rs:311-345"""
    keys = np.array([1010.0 if i == 140 else -1000.0 for i in range(257)], np.float32)
    vals = np.array([np.float32(i) * np.float32(0.1) - np.float32(3.0) for i in range(257)], np.float32)
    for j, sink in enumerate([-10000.0, 10000.0, 1009.0, -np.inf]):
        out = run_attention(ctx, np.ones(1, np.float32), keys, vals, 1, 1, 1, (256, 0, 0),
                            np.array([sink], np.float32))
        close(out, GOLD[f"extreme_{j}"], 1e-6, 1e-6)
    out = run_attention(ctx, np.ones(4, np.float32), keys, vals, 1, 1, 1, (253, 0, 0), np.array([-1e4], np.float32))
    close(out, GOLD["extreme_multi"], 1e-6, 1e-6)


@pytest.mark.parametrize("case", G.PREFILL64_CASES)
@pytest.mark.parametrize("exp_fast", [False, True])
def test_fp32_tiles(ctx, case, exp_fast):
    """FP32 tiles (prefill64.rs) against f64 and the oracle: 1e-5 * (1 + |b|)."""
    ql, ist, ien = case
    q, k, v, s = G.prefill64_operands(ql)
    opts = F.PrefillOptions(F.EXP_FAST if exp_fast else F.EXP_EXACT, 0, F.SOFTMAX_ONLINE, F.SOFTMAX_ONLINE)
    out = run_attention(ctx, q, k, v, 16, 8, 64, (0, ist, ien), s, options=opts)
    close(G.sample_heads(out), GOLD[f"prefill64_{ql}"], 1e-5, 1e-5)
    close(out, O.prefill64(q, k, v, 16, 8, (0, ist, ien), s, exp_fast=exp_fast), 1e-5, 1e-5)


@pytest.mark.parametrize("i", range(len(G.STATIC_CASES)))
def test_fp32_static_shift_tiles(ctx, i):
    """prefill64/static_shift/tests.rs:372-394: within 1e-5 absolute of f64."""
    queries, total, off, ist, ien = G.STATIC_CASES[i]
    q, k, v, s = G.static_operands(queries, total)
    opts = F.PrefillOptions(F.EXP_FAST, 0, F.SOFTMAX_STATIC, F.SOFTMAX_STATIC)
    out = run_attention(ctx, q, k, v, 16, 8, 64, (off, ist, ien), s, options=opts)
    close(G.sample_heads(out), GOLD[f"static_{i}"], 1e-5, 0.0)


@pytest.mark.parametrize("case", [(4, 137, 141, 137, 1, 129), (9, 128, 137, 128, 1, 128), (33, 100, 133, 100, 1, 90),
                                  (40, 3, 43, 3, 1, 3), (5, 250, 300, 295, 0, 0), (2, 300, 302, 300, 5, 262),
                                  (1, 267, 268, 267, 1, 201)])
def test_mixed_caches(ctx, case):
    """Prefix keys per query head plus generated keys per KV head
    (src/kernels/attention/prefill64/tests.rs:96-103 shapes; image ends past
    the prefix are clamped to it, as CompactKv::validate requires,
    src/kernels/attention/mod.rs:184-187)."""
    ql, pl, tl, off, ist, ien = case
    q = G.prefill_values(ql * 16 * 64, 5 + ql, 3.0)
    pk = G.prefill_values(pl * 16 * 64, 7 + ql, 3.0)
    gk = G.prefill_values((tl - pl) * 8 * 64, 11 + ql, 3.0)
    v = G.prefill_values(tl * 8 * 64, 13 + ql, 3.0)
    s = G.prefill_values(16, 29, 2.0)
    out = run_attention(ctx, q, pk, v, 16, 8, 64, (off, ist, ien), s, generated_k=gk)
    ref = O.attention_online(q, pk, v, 16, 8, 64, (off, ist, ien), s, generated_k=gk)
    close(out, ref, 1e-5, 1e-5)
    close(out, G.attention_f64(q, pk, v, 16, 8, 64, (off, ist, ien), s, generated_k=gk), 1e-5, 1e-5)


def test_baseline_c1_causal_fp32(ctx):
    """1 x 16 x 1024 x 64 causal FP32, scale 1/8, N(0,1) seed 0."""
    rng = np.random.default_rng(0)
    q, k, v = (rng.standard_normal(1024 * 16 * 64).astype(np.float32) for _ in range(3))
    s = np.full(16, -np.inf, np.float32)  # the config has no sink
    out = run_attention(ctx, q, k, v, 16, 16, 64, (0, 0, 0), s)
    close(out, O.prefill64(q, k, v, 16, 16, (0, 0, 0), s), 1e-5, 1e-5)


# -------------------------------------------------------------- split cache
# The element formats, the rotated research formats (Q8Rot, Q4Rot) and the
# reference's test storages (unrotated Q4, rotated FP32).
FORMATS = [F.KV_F32, F.KV_Q16, F.KV_Q8, F.KV_BF16, F.KV_Q4, F.KV_Q8_ROT, F.KV_Q4_ROT, F.KV_F32 | F.KV_ROTATED]
CODED = (F.KV_Q16, F.KV_Q8, F.KV_Q4)


def sealed_pair(fmt, p, generated, seed, capacity=None, key_scale=None):
    k, v, q = G.kv_fixture(p, seed)
    if key_scale is not None:
        # per-position factors on every head's key (pairs stay shared)
        k = (k.reshape(p, -1) * key_scale.astype(np.float32)[:, None]).astype(np.float32).reshape(-1)
    capacity = capacity or p + max(generated, 1)
    ref = O.SplitCache(k, v, p, capacity, fmt=fmt)
    gpu = F.SplitPrefix.from_compact(dev(k), dev(v), p, capacity, fmt=fmt)
    tk, tv = G.kv_tail(generated)
    for t in range(generated):
        ku, vu = tk[t * 512:(t + 1) * 512], tv[t * 512:(t + 1) * 512]
        ref.push(ku, vu)
        # append takes expanded rows: both heads of a pair carry the group's key
        ke = np.repeat(ku.reshape(8, 1, 64), 2, axis=1).reshape(-1)
        ve = np.repeat(vu.reshape(8, 1, 64), 2, axis=1).reshape(-1)
        gpu.append(dev(ke), dev(ve))
    return ref, gpu, q


def d2h(ptr, n, dtype):
    """Copy n elements of device memory at `ptr` to a numpy array."""
    return F.device_to_host(ptr, n, dtype)


def device_records(gpu, fmt, groups):
    (codes, scales, tcodes, tscales), ps, ts = gpu.records()
    element = fmt & ~F.KV_ROTATED
    dt = {F.KV_F32: np.float32, F.KV_Q16: np.int16, F.KV_Q8: np.int8, F.KV_BF16: np.uint16, F.KV_Q4: np.uint8}[element]
    per = 2 if element == F.KV_Q4 else 1  # Q4: two codes per byte
    out = {"codes": d2h(codes, groups * ps * 160 // per, dt), "tail": d2h(tcodes, groups * max(ts, 1) * 128 // per, dt)}
    if element in CODED:
        out["scales"] = d2h(scales, groups * ps * 5, np.uint16)
        out["tail_scales"] = d2h(tscales, groups * max(ts, 1) * 4, np.uint16)
    return out


@pytest.mark.parametrize("fmt", FORMATS)
@pytest.mark.parametrize("p,generated", [(1, 1), (3, 2), (127, 1), (129, 17), (300, 130)])
def test_seal_and_append_are_bit_exact(ctx, fmt, p, generated):
    """Records, codes and BF16 scales equal the oracle's bit for bit
    (kv.rs:239-513, codec.rs)."""
    ref, gpu, _ = sealed_pair(fmt, p, generated, p)
    recs = device_records(gpu, fmt, 8)
    bits = lambda x: x.view(np.uint32) if x.dtype == np.float32 else x  # noqa: E731
    assert np.array_equal(bits(recs["codes"]), bits(ref.codes))
    width = 64 if fmt & ~F.KV_ROTATED == F.KV_Q4 else 128  # stored elements per tail record
    ta = recs["tail"].reshape(8, -1, width)[:, :generated]
    tb = ref.tail_codes.reshape(8, -1, width)[:, :generated]
    assert np.array_equal(bits(np.ascontiguousarray(ta)), bits(np.ascontiguousarray(tb)))
    if fmt & ~F.KV_ROTATED in CODED:
        assert np.array_equal(recs["scales"], ref.scales)
        assert np.array_equal(recs["tail_scales"].reshape(8, -1, 4)[:, :generated],
                              ref.tail_scales.reshape(8, -1, 4)[:, :generated])


@pytest.mark.parametrize("fmt", FORMATS)
def test_append_batch_equals_per_page_appends(ctx, fmt):
    """fo_kv_append_batch (the per-page appends of Model::decode_batch_next,
    src/model/mod.rs:760-852, in one launch) writes the same tail records,
    bit for bit, as one fo_kv_append per cache; capacity and duplicate
    refusals leave every cache as it was."""
    prefixes = [7, 128, 129, 300, 1000]
    cap = 12
    singles, batched = [], []
    for i, p in enumerate(prefixes):
        k, v, _ = G.kv_fixture(p, 11 + i)
        singles.append(F.SplitPrefix.from_compact(dev(k), dev(v), p, p + cap, fmt=fmt))
        batched.append(F.SplitPrefix.from_compact(dev(k), dev(v), p, p + cap, fmt=fmt))
    rng = np.random.default_rng(5)
    for step, rows in enumerate([1, 1, 3]):
        ks, vs = [], []
        for i in range(len(prefixes)):
            x = rng.standard_normal((2, rows, 8, 1, 64)).astype(np.float32)
            x = np.repeat(x, 2, axis=3).reshape(2, -1)  # expanded rows: pairs share the group's row
            if step == 1 and i == 2:
                x[1, 5] = np.nan  # a non-finite value gives a NaN block, batched or not
            ks.append(dev(x[0]))
            vs.append(dev(x[1]))
            singles[i].append(ks[i], vs[i])
        F.append_batch(batched, ks, vs, rows)
    torch.cuda.synchronize()
    bits = lambda x: x.view(np.uint32) if x.dtype == np.float32 else x  # noqa: E731
    width = 64 if fmt & ~F.KV_ROTATED == F.KV_Q4 else 128
    for a, b in zip(singles, batched):
        assert a.tail_len == b.tail_len == 5
        ra, rb = device_records(a, fmt, 8), device_records(b, fmt, 8)
        ta = np.ascontiguousarray(ra["tail"].reshape(8, -1, width)[:, :5])
        tb = np.ascontiguousarray(rb["tail"].reshape(8, -1, width)[:, :5])
        assert np.array_equal(bits(ta), bits(tb))
        if fmt & ~F.KV_ROTATED in CODED:
            assert np.array_equal(ra["tail_scales"].reshape(8, -1, 4)[:, :5], rb["tail_scales"].reshape(8, -1, 4)[:, :5])
    # one cache without room: nothing is written anywhere
    x = dev(np.zeros(8 * 16 * 64, np.float32))
    with pytest.raises(F.CapacityError):
        F.append_batch(batched, [x] * 5, [x] * 5, 8)
    assert [b.tail_len for b in batched] == [5] * 5
    with pytest.raises(F.FoError):
        F.append_batch([batched[0], batched[0]], [x] * 2, [x] * 2, 1)
    assert batched[0].tail_len == 5
    for c in singles + batched:
        c.close()


def plan_caches(fmt, ctx, room, prefixes=(7, 300, 1000)):
    out = []
    for i, p in enumerate(prefixes):
        k, v, _ = G.kv_fixture(p, 21 + i)
        out.append(F.SplitPrefix.from_compact(dev(k), dev(v), p, p + room, fmt=fmt, ctx=ctx))
    return out


def step_rows(rng, n):
    """One decode step's expanded K, V rows and queries for n pages."""
    kv = np.repeat(rng.standard_normal((n, 2, 8, 1, 64)).astype(np.float32), 2, axis=3).reshape(n, 2, -1)
    q = rng.standard_normal((n, 16 * 64)).astype(np.float32)
    return kv, q


@pytest.mark.parametrize("fmt", [F.KV_BF16, F.KV_Q8, F.KV_Q4_ROT])
def test_batch_plan_equals_per_step_calls(ctx, fmt):
    """fo_kv_plan_step (append + one-row decode per page from device-resident
    descriptors) gives, step by step, the outputs of fo_kv_append_batch +
    fo_kv_attention_decode_batch bit for bit, and leaves the same records."""
    a, b = plan_caches(fmt, ctx, 8), plan_caches(fmt, ctx, 8)
    n = len(a)
    kb = [torch.empty(1024, device="cuda") for _ in range(n)]
    vb = [torch.empty(1024, device="cuda") for _ in range(n)]
    qb = [torch.empty(1024, device="cuda") for _ in range(n)]
    ob = [torch.empty(1024, device="cuda") for _ in range(n)]
    sd = [dev(np.array([h * 0.3 - 2.0 for h in range(16)], np.float32))] * n
    plan = F.BatchPlan(b, kb, vb, qb, sd, ob)
    rng = np.random.default_rng(8)
    for step in range(5):
        kv, q = step_rows(rng, n)
        ks, vs, qs = [dev(kv[i, 0]) for i in range(n)], [dev(kv[i, 1]) for i in range(n)], [dev(q[i]) for i in range(n)]
        oa = [torch.empty(1024, device="cuda") for _ in range(n)]
        F.append_batch(a, ks, vs, 1)
        F.decode_batch(a, qs, sd, oa)
        for i in range(n):
            kb[i].copy_(ks[i])
            vb[i].copy_(vs[i])
            qb[i].copy_(qs[i])
        plan.step()
        torch.cuda.synchronize()
        for i in range(n):
            assert torch.equal(oa[i].view(torch.int32), ob[i].view(torch.int32)), (step, i)
    plan.finish()
    for x, y in zip(a, b):
        assert x.tail_len == y.tail_len == 5
        rx, ry = device_records(x, fmt, 8), device_records(y, fmt, 8)
        width = 64 if fmt & ~F.KV_ROTATED == F.KV_Q4 else 128
        assert np.array_equal(rx["tail"].reshape(8, -1, width)[:, :5], ry["tail"].reshape(8, -1, width)[:, :5])
    for c in a + b:
        c.close()


def test_batch_plan_replays_in_a_cuda_graph():
    """A plan step captured in a CUDA graph and replayed moves the pages on
    like eager steps (the descriptors live on the device)."""
    stream = torch.cuda.Stream()
    gctx = F.Context(0, stream=stream.cuda_stream)
    a, b = plan_caches(F.KV_BF16, gctx, 12), plan_caches(F.KV_BF16, gctx, 12)
    n = len(a)
    rng = np.random.default_rng(9)
    kv, q = step_rows(rng, n)
    sd = [dev(np.linspace(-1, 1, 16).astype(np.float32))] * n

    def bufs():
        return ([dev(kv[i, 0]) for i in range(n)], [dev(kv[i, 1]) for i in range(n)], [dev(q[i]) for i in range(n)],
                [torch.empty(1024, device="cuda") for _ in range(n)])
    ka, va, qa, oa = bufs()
    kb, vb, qb, ob = bufs()
    torch.cuda.synchronize()
    pa, pb = F.BatchPlan(a, ka, va, qa, sd, oa), F.BatchPlan(b, kb, vb, qb, sd, ob)
    with torch.cuda.stream(stream):
        for _ in range(7):
            pa.step()
        pb.step()  # one eager step before capture sets the launches up
    stream.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        pb.step()
        pb.step()
    for _ in range(3):
        g.replay()
    stream.synchronize()
    for i in range(n):
        assert torch.equal(oa[i].view(torch.int32), ob[i].view(torch.int32)), i
    del g
    pa.finish()
    pb.finish()
    assert [c.tail_len for c in a] == [c.tail_len for c in b] == [7] * n
    for c in a + b:
        c.close()
    gctx.close()


def test_batch_plan_stops_at_a_full_tail(ctx):
    """A plan step past a cache's capacity writes nothing more and finish
    reports FO_ERR_CAPACITY; the tail holds the rows it had room for."""
    caches = plan_caches(F.KV_BF16, ctx, 2)
    n = len(caches)
    bufs = [[torch.zeros(1024, device="cuda") for _ in range(n)] for _ in range(4)]
    sd = [dev(np.zeros(16, np.float32))] * n
    plan = F.BatchPlan(caches, bufs[0], bufs[1], bufs[2], sd, bufs[3])
    for _ in range(4):
        plan.step()
    with pytest.raises(F.CapacityError):
        plan.finish()
    assert [c.tail_len for c in caches] == [2] * n
    for c in caches:
        c.close()


def test_batch_plan_that_fills_its_tails_exactly_finishes_cleanly(ctx):
    """As many steps as the caches have room for: every row is written,
    finish reports no error, and the last step's output equals a decode of
    the full caches."""
    room = 3
    caches = plan_caches(F.KV_Q8, ctx, room)
    n = len(caches)
    rng = np.random.default_rng(12)
    kb = [torch.empty(1024, device="cuda") for _ in range(n)]
    vb = [torch.empty(1024, device="cuda") for _ in range(n)]
    qb = [torch.empty(1024, device="cuda") for _ in range(n)]
    ob = [torch.empty(1024, device="cuda") for _ in range(n)]
    sd = [dev(np.linspace(-1, 1, 16).astype(np.float32))] * n
    plan = F.BatchPlan(caches, kb, vb, qb, sd, ob)
    for _ in range(room):
        kv, q = step_rows(rng, n)
        for i in range(n):
            kb[i].copy_(dev(kv[i, 0]))
            vb[i].copy_(dev(kv[i, 1]))
            qb[i].copy_(dev(q[i]))
        plan.step()
    plan.finish()
    assert [c.tail_len for c in caches] == [room] * n
    for i, c in enumerate(caches):
        single = torch.empty(1024, device="cuda")
        c.attention_decode(qb[i], c.prefix_len + room, sd[i], single)
        torch.cuda.synchronize()
        assert torch.equal(single.view(torch.int32), ob[i].view(torch.int32)), i
        c.close()


def test_seal_errors(ctx):
    """kv.rs:248-295 and src/quant/kv/tests.rs:355-367"""
    k = np.zeros(16 * 64, np.float32)
    v = np.zeros(8 * 64, np.float32)
    k[64] = 1.0
    with pytest.raises(F.PairError):
        F.SplitPrefix.from_compact(k, v, 1, 2, fmt="f32")
    k[64] = 0.0
    F.SplitPrefix.from_compact(k, v, 1, 2, fmt="q8").close()
    v[5] = np.inf
    with pytest.raises(F.NonFiniteError):
        F.SplitPrefix.from_compact(k, v, 1, 2, fmt="q8")
    with pytest.raises(F.CapacityError):
        F.SplitPrefix.from_compact(k, v[:512] * 0, 1, 0, fmt="q8")
    # Values near FLT_MAX seal finitely: the rounded-up BF16 scale keeps
    # code * scale finite (kv.rs:328's check is defensive).
    vb = np.zeros(8 * 64, np.float32)
    vb[3] = np.finfo(np.float32).max
    F.SplitPrefix.from_compact(np.zeros(16 * 64, np.float32), vb, 1, 2, fmt="q8").close()


@pytest.mark.parametrize("fmt", FORMATS)
@pytest.mark.parametrize("p,generated", [(1, 1), (3, 2), (127, 1), (128, 5), (129, 17), (300, 130), (1000, 40)])
def test_decode_matches_oracle(ctx, fmt, p, generated):
    """attention_decode against the oracle at the reference's chunking bound."""
    ref, gpu, q = sealed_pair(fmt, p, generated, p)
    sinks = np.array([h * 0.25 - 1.0 for h in range(16)], np.float32)
    out = np.zeros(1024, np.float32)
    gpu.attention_decode(q, p + generated, sinks, out)
    close(out, ref.decode(q, sinks), 1e-5, 1e-5)
    gpu.with_fast_exp(True)
    ref.fast_exp = True
    gpu.attention_decode(q, p + generated, sinks, out)
    close(out, ref.decode(q, sinks), 1e-5, 1e-5)


@pytest.mark.parametrize("fmt", FORMATS)
def test_verification_rows_are_bitwise_single_rows(ctx, fmt):
    """src/quant/kv/tests.rs:26-69 on the GPU."""
    for (p, generated, rows) in [(300, 5, 5), (1000, 9, 8), (130, 3, 2), (7, 4, 4), (254, 6, 6), (250, 8, 8)]:
        ref, gpu, _ = sealed_pair(fmt, p, generated, p + 3)
        q = G.kv_rows_query(rows)
        sinks = np.array([h * 0.25 - 1.0 for h in range(16)], np.float32)
        joint = np.zeros(rows * 1024, np.float32)
        gpu.attention_decode_rows(q, rows, sinks, joint)
        close(joint, ref.decode_rows(q, rows, sinks), 1e-5, 1e-5)
        for r in reversed(range(rows)):
            gpu.truncate_tail(generated - (rows - 1 - r))
            single = np.zeros(1024, np.float32)
            gpu.attention_decode(q[r * 1024:(r + 1) * 1024], p + gpu.tail_len, sinks, single)
            assert np.array_equal(joint[r * 1024:(r + 1) * 1024].view(np.uint32), single.view(np.uint32)), (p, r)


@pytest.mark.parametrize("fmt", FORMATS)
def test_growing_logits_move_the_running_maximum(ctx, fmt):
    """Keys scaled per block of 128 positions so that the largest logit grows
    by about 10 (more than a factor e^8 in p) from one block to the next,
    within the runs of consecutive blocks a decode sums as one: the running
    sums are rescaled on the way and still match the oracle, and every verify
    row still equals its single-row decode bit for bit."""
    p, generated, rows = 8192, 6, 5
    scale = 1.0 + 30.0 * ((np.arange(p) // 128) % 4)
    ref, gpu, _ = sealed_pair(fmt, p, generated, 7, key_scale=scale)
    q = G.kv_rows_query(rows)
    sinks = np.array([h * 0.25 - 1.0 for h in range(16)], np.float32)
    joint = np.zeros(rows * 1024, np.float32)
    gpu.attention_decode_rows(q, rows, sinks, joint)
    close(joint, ref.decode_rows(q, rows, sinks), 1e-5, 1e-5)
    for r in reversed(range(rows)):
        gpu.truncate_tail(generated - (rows - 1 - r))
        single = np.zeros(1024, np.float32)
        gpu.attention_decode(q[r * 1024:(r + 1) * 1024], p + gpu.tail_len, sinks, single)
        assert np.array_equal(joint[r * 1024:(r + 1) * 1024].view(np.uint32), single.view(np.uint32)), r


@pytest.mark.parametrize("fmt", FORMATS)
def test_nonfinite_tail_values_reach_the_output(ctx, fmt):
    """src/quant/kv/tests.rs:306-324"""
    p = 130
    k, v, q = G.kv_fixture(p, 5)
    gpu = F.SplitPrefix.from_compact(k, v, p, p + 2, fmt=fmt)
    tail = np.full(16 * 64, 0.01, np.float32)
    gpu.append(tail, tail)
    tail[3] = np.nan
    tail[64 + 3] = np.nan  # expanded rows: both heads of the pair
    gpu.append(tail, tail)
    out = np.zeros(1024, np.float32)
    gpu.attention_decode(q, p + 2, np.full(16, 0.5, np.float32), out)
    assert np.isnan(out[:64]).all()
    assert np.isfinite(out[128:]).all()


@pytest.mark.parametrize("fmt", FORMATS)
def test_nonfinite_draft_reaches_only_the_rows_that_see_it(ctx, fmt):
    """A NaN value in the last drafted position: the verify rows before it do
    not see that position (kv.rs:851-855) and stay finite and equal to their
    single-row decodes; the last row is NaN on the pair's heads."""
    p, rows = 700, 4
    k, v, _ = G.kv_fixture(p, 5)
    gpu = F.SplitPrefix.from_compact(k, v, p, p + rows, fmt=fmt)
    tk, tv = G.kv_tail(rows)
    tk = np.repeat(tk.reshape(rows, 8, 1, 64), 2, axis=2).reshape(-1)
    tv = np.repeat(tv.reshape(rows, 8, 1, 64), 2, axis=2).reshape(-1)
    for x in (tk, tv):
        x[(rows - 1) * 1024 + 5] = np.nan
        x[(rows - 1) * 1024 + 64 + 5] = np.nan
    gpu.append(tk, tv)
    q = G.kv_rows_query(rows)
    sinks = np.full(16, 0.5, np.float32)
    joint = np.zeros(rows * 1024, np.float32)
    gpu.attention_decode_rows(q, rows, sinks, joint)
    assert np.isfinite(joint[:(rows - 1) * 1024]).all()
    assert np.isnan(joint[(rows - 1) * 1024:(rows - 1) * 1024 + 128]).all()
    assert np.isfinite(joint[(rows - 1) * 1024 + 128:]).all()
    for r in reversed(range(rows - 1)):
        gpu.truncate_tail(r + 1)
        single = np.zeros(1024, np.float32)
        gpu.attention_decode(q[r * 1024:(r + 1) * 1024], p + gpu.tail_len, sinks, single)
        assert np.array_equal(joint[r * 1024:(r + 1) * 1024].view(np.uint32), single.view(np.uint32)), r


@pytest.mark.parametrize("fmt", FORMATS)
def test_truncated_tails_take_new_positions_like_fresh_ones(ctx, fmt):
    """src/quant/kv/tests.rs:326-353"""
    p, generated, kept = 37, 6, 2
    k, v, q = G.kv_fixture(p, p + 5)
    rows = lambda seed: (((np.arange(generated * 1024) * seed) % 43).astype(np.float32) / np.float32(59.0)  # noqa
                         - np.float32(0.35)).astype(np.float32)
    old_k, old_v, new_k, new_v = rows(13), rows(17), rows(19), rows(23)
    # expanded rows with identical pairs: copy head 2g into 2g+1
    pairs = lambda x: np.repeat(x.reshape(-1, 8, 2, 64)[:, :, :1], 2, axis=2).reshape(-1)  # noqa
    old_k, old_v, new_k, new_v = pairs(old_k), pairs(old_v), pairs(new_k), pairs(new_v)
    split = kept * 1024
    sinks = np.array([h * 0.2 - 0.9 for h in range(16)], np.float32)
    reused = F.SplitPrefix.from_compact(k, v, p, p + generated, fmt=fmt)
    reused.append(old_k, old_v)
    reused.truncate_tail(kept)
    reused.append(new_k[split:], new_v[split:])
    fresh = F.SplitPrefix.from_compact(k, v, p, p + generated, fmt=fmt)
    fresh.append(np.concatenate([old_k[:split], new_k[split:]]), np.concatenate([old_v[:split], new_v[split:]]))
    a = np.zeros(1024, np.float32)
    b = np.zeros(1024, np.float32)
    reused.attention_decode(q, p + generated, sinks, a)
    fresh.attention_decode(q, p + generated, sinks, b)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


def test_research_formats_stay_close_to_fp32(ctx):
    """src/quant/kv/tests.rs:282-304 on the GPU: Q8Rot within 0.02 and Q4Rot
    within 0.05 of the compact FP32 attention (the golden output)."""
    p = 257
    k, v, q = G.kv_fixture(p, 9)
    tail = np.full(16 * 64, 0.02, np.float32)
    for fmt, bound in (("q8r", 0.02), ("q4r", 0.05)):
        gpu = F.SplitPrefix.from_compact(k, v, p, p + 1, fmt=fmt)
        gpu.append(tail, tail)
        out = np.zeros(1024, np.float32)
        gpu.attention_decode(q, p + 1, np.full(16, 0.5, np.float32), out)
        assert np.isfinite(out).all()
        assert np.all(np.abs(out - GOLD["kv_lowprec_expected"]) < bound), fmt


def test_rotated_seal_refuses_pairs_and_overflow(ctx):
    """kv/tests.rs:355-369 and kv.rs:289-293: the pair check sees the
    unrotated keys; a block whose rotation overflows is refused."""
    k = np.zeros(16 * 64, np.float32)
    v = np.zeros(8 * 64, np.float32)
    k[64] = 1.0
    with pytest.raises(F.PairError):
        F.SplitPrefix.from_compact(k, v, 1, 2, fmt="q8r")
    k[64] = 0.0
    k[:32] = k[64:96] = np.arange(32, dtype=np.float32)
    F.SplitPrefix.from_compact(k, v, 1, 2, fmt="q8r").close()
    with pytest.raises(F.FoError, match="rotated KV group overflows"):
        F.SplitPrefix.from_compact(np.full(16 * 64, 3e37, np.float32), v, 1, 2, fmt="q4r")
    with pytest.raises(F.FoError):
        F.SplitPrefix.from_compact(k, v, 1, 2, fmt=F.KV_BF16 | F.KV_ROTATED)


def test_decode_errors(ctx):
    k, v, q = G.kv_fixture(10, 1)
    gpu = F.SplitPrefix.from_compact(k, v, 10, 12, fmt="q8")
    out = np.zeros(1024, np.float32)
    with pytest.raises(F.FoError):
        gpu.attention_decode(q, 11, np.zeros(16, np.float32), out)  # total must be prefix + tail
    with pytest.raises(F.FoError):
        gpu.attention_decode_rows(np.zeros(2 * 1024, np.float32), 2, np.zeros(16, np.float32), np.zeros(2048,
                                                                                                         np.float32))
    row = np.zeros(1024, np.float32)
    gpu.append(row, row)
    gpu.append(row, row)
    with pytest.raises(F.CapacityError):
        gpu.append(row, row)
    with pytest.raises(F.FoError):
        gpu.truncate_tail(3)


@pytest.mark.parametrize("fmt", [F.KV_F32, F.KV_BF16])
@pytest.mark.parametrize("length", [6544, 12000, 16384])
def test_baseline_c3_verify_rows(ctx, fmt, length):
    """5 rows (1 accepted + 4 drafts) at 6,544/12,000/16,384,
    N(0,1) seed 2, temporal halves shared inside each pair."""
    rng = np.random.default_rng(2)
    p = length - 5  # the 5 query rows are the last 5 cached positions (kv.rs:851-855)
    k = rng.standard_normal((p, 16, 64)).astype(np.float32)
    k[:, 1::2, :32] = k[:, 0::2, :32]
    v = rng.standard_normal((p, 8, 64)).astype(np.float32)
    ref = O.SplitCache(k, v, p, length, fmt=fmt, chunks=4)
    gpu = F.SplitPrefix.from_compact(dev(k), dev(v), p, length, fmt=fmt)
    tk = rng.standard_normal((5, 8, 64)).astype(np.float32)
    tv = rng.standard_normal((5, 8, 64)).astype(np.float32)
    for t in range(5):
        ref.push(tk[t], tv[t])
    gpu.append(np.repeat(tk[:, :, None], 2, axis=2).reshape(-1), np.repeat(tv[:, :, None], 2, axis=2).reshape(-1))
    q = rng.standard_normal(5 * 1024).astype(np.float32)
    sinks = rng.standard_normal(16).astype(np.float32)
    out = np.zeros(5 * 1024, np.float32)
    gpu.attention_decode_rows(q, 5, sinks, out)
    close(out, ref.decode_rows(q, 5, sinks), 1e-5, 1e-5)


@pytest.mark.parametrize("fmt", ["q8", "q8r", "q4r"])
def test_batch_decode_equals_single_pages(ctx, fmt):
    """Page-parallel decode (call stack D): each page equals its own decode."""
    caches, qs, ss, outs, singles = [], [], [], [], []
    for i, p in enumerate([300, 1000, 17, 2049]):
        k, v, q = G.kv_fixture(p, 3 + i)
        c = F.SplitPrefix.from_compact(dev(k), dev(v), p, p + 1, fmt=fmt)
        caches.append(c)
        qs.append(dev(q))
        ss.append(dev(np.full(16, 0.3 * i, np.float32)))
        outs.append(torch.zeros(1024, device="cuda"))
        single = torch.zeros(1024, device="cuda")
        c.attention_decode(qs[-1], p, ss[-1], single)
        singles.append(single)
    F.decode_batch(caches, qs, ss, outs)
    torch.cuda.synchronize()
    for a, b in zip(outs, singles):
        assert torch.equal(a.view(torch.int32), b.view(torch.int32))


# ------------------------------------------------------------ bounded waits
def test_a_wait_that_runs_out_returns_an_error_and_the_context_survives(ctx):
    """A device wait on a barrier nothing completes gives up after its limit
    (1 ms here), raises the context's error word and returns; the host reads
    FO_ERR_CUDA and the same context then runs a decode correctly."""
    status = ctx.selftest_bounded_wait(1_000_000)
    assert status == F.ERR_CUDA
    assert "time limit" in F.lib().fo_last_error().decode()
    ref, gpu, q = sealed_pair(F.KV_Q8, 300, 2, 3)
    sinks = np.full(16, 0.5, np.float32)
    out = np.zeros(1024, np.float32)
    gpu.attention_decode(q, 302, sinks, out)
    close(out, ref.decode_rows(q, 1, sinks), 1e-5, 1e-5)
    gpu.close()
