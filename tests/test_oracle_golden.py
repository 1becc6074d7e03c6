"""Pins the CPU oracle (oracle/fo_oracle.c) to the reference's own tests:
known answers, f64 tolerance tables, codec rounding and the split cache's
structural invariants.  CPU only."""

import os

import numpy as np
import pytest

import generators as G
import oracle as O

GOLD = np.load(os.path.join(os.path.dirname(__file__), "golden", "attention_golden.npz"))


def close(actual, expected, absolute, relative):
    actual = np.asarray(actual, np.float64)
    expected = np.asarray(expected, np.float64)
    bad = np.abs(actual - expected) > absolute + relative * np.abs(expected)
    assert not bad.any(), f"{bad.sum()} mismatches, worst {np.abs(actual - expected).max():.3e}"


def test_known_answer_image_boundaries_and_sink():
    """src/kernels/tests.rs:283-309"""
    qk = np.zeros(5, np.float32)
    out = O.attention_online(qk, qk, GOLD["kat5_values"], 1, 1, 1, (0, 1, 3), [0.0])
    close(out, GOLD["kat5_expected"], 1e-6, 1e-7)
    out = O.attention_online([0.0], [0.0], [13.0], 1, 1, 1, (0, 0, 0), [-np.inf])
    assert out.tolist() == GOLD["kat5_nosink_expected"].tolist()
    # The FP32 tiles need 64-wide heads; the dense f64 oracle agrees too.
    close(O.attention_f64(qk, qk, GOLD["kat5_values"], 1, 1, 1, (0, 1, 3), [0.0]), GOLD["kat5_expected"], 1e-6, 1e-7)


@pytest.mark.parametrize("i", range(len(G.DENSE_TABLE)))
def test_dense_table(i):
    """src/kernels/tests.rs:250-281: 2e-6 absolute + 4e-6 relative."""
    ql, kvl, h, d, off, st, en = G.DENSE_TABLE[i]
    q, k, v, s = G.lcg_values(ql * h * d, 71), G.lcg_values(kvl * h * d, 83), G.lcg_values(kvl * h * d, 117), \
        G.lcg_values(h, 24)
    close(O.attention_online(q, k, v, h, h, d, (off, st, en), s), GOLD[f"dense_{i}"], 2e-6, 4e-6)
    close(O.attention_f64(q, k, v, h, h, d, (off, st, en), s), GOLD[f"dense_{i}"], 1e-12, 1e-12)


def test_extreme_logits_and_sinks():
    """src/kernels/tests.rs:311-345"""
    keys = np.array([1010.0 if i == 140 else -1000.0 for i in range(257)], np.float32)
    vals = np.array([np.float32(i) * np.float32(0.1) - np.float32(3.0) for i in range(257)], np.float32)
    for j, sink in enumerate([-10000.0, 10000.0, 1009.0, -np.inf]):
        out = O.attention_online([1.0], keys, vals, 1, 1, 1, (256, 0, 0), [sink])
        close(out, GOLD[f"extreme_{j}"], 1e-6, 1e-6)
        assert np.isfinite(out).all()
    out = O.attention_online(np.ones(4, np.float32), keys, vals, 1, 1, 1, (253, 0, 0), [-10000.0])
    close(out, GOLD["extreme_multi"], 1e-6, 1e-6)


@pytest.mark.parametrize("case", G.PREFILL64_CASES)
@pytest.mark.parametrize("exp_fast", [False, True])
def test_prefill64_tiles(case, exp_fast):
    """prefill64/tests.rs:66-89 bound 1e-5 * (1 + |b|), against f64."""
    ql, ist, ien = case
    q, k, v, s = G.prefill64_operands(ql)
    out = O.prefill64(q, k, v, 16, 8, (0, ist, ien), s, softmax_static=False, exp_fast=exp_fast)
    close(G.sample_heads(out), GOLD[f"prefill64_{ql}"], 1e-5, 1e-5)
    # the generic online head agrees with the tiles at the same bound
    ref = O.attention_online(q, k, v, 16, 8, 64, (0, ist, ien), s)
    close(out, ref, 1e-5, 1e-5)


@pytest.mark.parametrize("i", range(len(G.STATIC_CASES)))
def test_static_shift_tiles(i):
    """prefill64/static_shift/tests.rs:372-394: within 1e-5 absolute of f64."""
    queries, total, off, ist, ien = G.STATIC_CASES[i]
    q, k, v, s = G.static_operands(queries, total)
    out = O.prefill64(q, k, v, 16, 8, (off, ist, ien), s, softmax_static=True)
    close(G.sample_heads(out), GOLD[f"static_{i}"], 1e-5, 0.0)


@pytest.mark.parametrize("case", G.BF16_CASES)
def test_bf16_online_tiles(case):
    """prefill64/bf16.rs:851-926: within 3 * 2^-9 + 2e-3 of the BF16-operand f64."""
    ql, ist, ien = case
    q, k, v, s = G.bf16_operands(ql)
    out = O.prefill_bf16(q, k, v, 16, 8, (ist, ien), s, softmax_static=False)
    close(G.sample_heads(out), GOLD[f"bf16_{ql}"], 3 * 2.0 ** -9 + 2e-3, 0.0)


@pytest.mark.parametrize("case", G.BF16_CASES)
def test_bf16_static_tiles(case):
    """bf16/static_shift/tests.rs:234-285 on norm-8 operands made BF16-exact:
    within 3 * 2 * (2^-8 + 7.5e-5) + 1e-4 of f64."""
    ql, ist, ien = case
    q, k, v, s = G.static_operands(ql, ql)
    q, k, v = G.bf16_round(q), G.bf16_round(k), G.bf16_round(v)
    out = O.prefill_bf16(q, k, v, 16, 8, (ist, ien), s, softmax_static=True)
    ref = G.attention_f64(q, k, v, 16, 8, 64, (0, ist, ien), s)
    close(out, ref, 3 * 2 * (2.0 ** -8 + 7.5e-5) + 1e-4, 0.0)


def test_codes_round_ties_to_even():
    """src/quant/kv/tests.rs:568-612"""
    xs, limits, expected = GOLD["codes_x"], GOLD["codes_limit"], GOLD["codes_expected"]
    got = np.array([O.round_clamped(x, lim) for x, lim in zip(xs, limits)])
    assert np.array_equal(got, expected)
    assert np.isnan(O.round_clamped(np.nan, 127.0))
    for value, scale, c8, c16 in zip(GOLD["code_values"], GOLD["code_scales"], GOLD["code_q8"], GOLD["code_q16"]):
        assert O.q8_code(value, scale) == c8
        assert O.q16_code(value, scale) == c16
    assert O.q8_code(np.nan, 0.37) == 0 and O.q16_code(np.nan, 0.37) == 0


def test_bf16_up_is_smallest_bf16_at_or_above():
    """codec.rs:34-44 (q4_scales_round_up_to_bf16 asserts the same property)."""
    rng = np.random.default_rng(5)
    for x in np.abs(rng.standard_normal(2000)).astype(np.float32):
        b = O.bf16_up(x)
        assert O.bf16_f32(b) >= x and (O.bf16_f32(b - 1) < x or (b & 0x7FFF) == 0)
    assert O.bf16_up(np.nan) == 0x7FC0 and O.bf16_up(0.0) == 0


def test_exp_poly_domain():
    """exp.rs:232-258: NaN, underflow and overflow edges, accuracy on the softmax domain."""
    assert np.isnan(O.exp_poly(np.nan))
    assert O.exp_poly(-87.5) == 0.0 and O.exp_poly(88.5) == np.inf
    xs = np.linspace(-87, 0, 4001, dtype=np.float32)
    got = np.array([O.exp_poly(x) for x in xs])
    close(got, np.exp(xs.astype(np.float64)), 0.0, 3e-7)


def _sealed(fmt, p, generated, seed, chunks=None, fast_exp=False):
    k, v, q = G.kv_fixture(p, seed)
    c = O.SplitCache(k, v, p, p + max(generated, 1), fmt=fmt, chunks=chunks, fast_exp=fast_exp)
    assert c.status == O.OK
    tk, tv = G.kv_tail(generated)
    for t in range(generated):
        c.push(tk[t * 512:(t + 1) * 512], tv[t * 512:(t + 1) * 512])
    return c, k, v, q, tk, tv


@pytest.mark.parametrize("fmt", [O.F32, O.Q16, O.Q8, O.BF16])
@pytest.mark.parametrize("p,generated", [(1, 1), (3, 2), (127, 1), (128, 5), (129, 17), (300, 130)])
def test_records_decode_like_compact_over_their_values(fmt, p, generated):
    """src/quant/kv/tests.rs:198-250: one chunk, decode equals the online head
    over the dequantized compact cache (here to 1e-6: the orders match the
    reference, not each other's vector trees bit for bit)."""
    c, k, v, q, tk, tv = _sealed(fmt, p, generated, p, chunks=1)
    dk, dv = c.dequantized_compact()
    tail = c.decoded_tail().reshape(8, -1, 128)[:, :generated]
    gk = tail[:, :, :64].transpose(1, 0, 2).reshape(-1)
    gvv = tail[:, :, 64:].transpose(1, 0, 2).reshape(-1)
    if fmt == O.F32:
        assert np.array_equal(dk, k) and np.array_equal(dv, v)
        assert np.array_equal(gk, tk) and np.array_equal(gvv, tv)
    sinks = np.array([h * 0.25 - 1.0 for h in range(16)], np.float32)
    expected = O.attention_online(q, dk, np.concatenate([dv, gvv]), 16, 8, 64, (p + generated - 1, 0, p), sinks,
                                  generated_k=gk)
    close(c.decode(q, sinks), expected, 1e-6, 1e-6)


@pytest.mark.parametrize("fmt", [O.F32, O.Q16, O.Q8])
def test_position_chunks_change_rounding_only(fmt):
    """src/quant/kv/tests.rs:253-280: 1e-5 * (1 + |b|)."""
    p, generated = 1000, 40
    k, v, q = G.kv_fixture(p, 3)
    tail, _ = G.kv_tail(generated)
    sinks = np.full(16, 0.5, np.float32)
    outs = []
    for chunks in range(1, 5):
        c = O.SplitCache(k, v, p, p + generated, fmt=fmt, chunks=chunks)
        for t in range(generated):
            c.push(tail[t * 512:(t + 1) * 512], tail[t * 512:(t + 1) * 512])
        outs.append(c.decode(q, sinks))
    for o in outs[1:]:
        close(o, outs[0], 1e-5, 1e-5)


def test_low_precision_stays_close_to_fp32():
    """src/quant/kv/tests.rs:282-304: Q8 and Q16 within 0.02 of compact FP32."""
    p = 257
    k, v, q = G.kv_fixture(p, 9)
    tail = np.full(512, 0.02, np.float32)
    sinks = np.full(16, 0.5, np.float32)
    for fmt in (O.Q8, O.Q16, O.BF16):
        c = O.SplitCache(k, v, p, p + 1, fmt=fmt)
        c.push(tail, tail)
        out = c.decode(q, sinks)
        assert np.isfinite(out).all()
        assert np.all(np.abs(out - GOLD["kv_lowprec_expected"]) < 0.02)


@pytest.mark.parametrize("fmt", [O.F32, O.Q16, O.Q8, O.BF16])
def test_nonfinite_tail_values_reach_the_output(fmt):
    """src/quant/kv/tests.rs:306-324"""
    p = 130
    k, v, q = G.kv_fixture(p, 5)
    c = O.SplitCache(k, v, p, p + 2, fmt=fmt)
    tail = np.full(512, 0.01, np.float32)
    c.push(tail, tail)
    tail[3] = np.nan
    c.push(tail, tail)
    out = c.decode(q, np.full(16, 0.5, np.float32))
    assert np.isnan(out[:64]).all()


def test_refuses_nonidentical_temporal_keys_and_nonfinite():
    """src/quant/kv/tests.rs:355-367 and kv.rs:248-295"""
    k = np.zeros(16 * 64, np.float32)
    v = np.zeros(8 * 64, np.float32)
    k[64] = 1.0
    assert O.SplitCache(k, v, 1, 2, fmt=O.F32).status == O.ERR_PAIR
    k[64] = 0.0
    assert O.SplitCache(k, v, 1, 2, fmt=O.Q8).status == O.OK
    v[5] = np.inf
    assert O.SplitCache(k, v, 1, 2, fmt=O.Q8).status == O.ERR_NONFINITE
    assert O.SplitCache(k, v[:0], 0, 2, fmt=O.Q8).status == O.ERR_CAPACITY


@pytest.mark.parametrize("fmt", [O.F32, O.Q8])
def test_verification_rows_are_single_rows(fmt):
    """src/quant/kv/tests.rs:26-69: row r of a verify step equals the single-row
    decode after truncating the tail to its length."""
    for (p, generated, rows) in [(300, 5, 5), (130, 3, 2), (7, 4, 4)]:
        c, k, v, _, tk, tv = _sealed(fmt, p, generated, p + 3, chunks=2)
        q = G.kv_rows_query(rows)
        sinks = np.array([h * 0.25 - 1.0 for h in range(16)], np.float32)
        joint = c.decode_rows(q, rows, sinks)
        for r in reversed(range(rows)):
            c.truncate_tail(generated - (rows - 1 - r))
            single = c.decode(q[r * 1024:(r + 1) * 1024], sinks)
            assert np.array_equal(joint[r * 1024:(r + 1) * 1024].view(np.uint32), single.view(np.uint32))
