"""Pins the oracle's rotated and 4-bit record formats to the
reference's own tests: src/quant/rotation.rs:139-217 (sign words, the
Sylvester matrix, exact round trips, NaN spreading) and
src/quant/kv/tests.rs:156-250, 282-304, 355-369, 634-662 (rotated storages
decode as a pre/post transform, error bounds against FP32, the pair check
on unrotated keys, rotated FP32 changes rounding only).  CPU only."""

import os

import numpy as np
import pytest

import generators as G
import oracle as O

GOLD = np.load(os.path.join(os.path.dirname(__file__), "golden", "attention_golden.npz"))
KINDS = range(4)


def _values(seed):
    """Deterministic values in [-1, 1) (rotation.rs:142-145 uses its own
    generator; any spread of magnitude ~1 serves these properties)."""
    return np.random.default_rng(seed).uniform(-1.0, 1.0, 32).astype(np.float32)


def test_sign_words_are_the_documented_splitmix_outputs():
    """rotation.rs:163-170"""
    assert [O.rotation_signs(k) for k in KINDS] == [0x04DCF6B7, 0x871F5F8B, 0x489CE13C, 0x4A81CBCB]
    for k in KINDS:
        assert 8 <= bin(O.rotation_signs(k)).count("1") <= 24


def test_fwht_is_the_sylvester_hadamard_matrix():
    """rotation.rs:150-161"""
    for j in range(32):
        x = np.zeros(32, np.float32)
        x[j] = 1.0
        h = O.fwht32(x)
        expected = [1.0 if bin(i & j).count("1") % 2 == 0 else -1.0 for i in range(32)]
        assert h.tolist() == expected


def test_unrotate_inverts_rotate():
    """rotation.rs:172-195: integers come back exactly; general values within 1e-5."""
    integers = np.array([((i * 37 + 11) % 23) - 11.0 for i in range(32)], np.float32)
    for kind in KINDS:
        x = O.rotate(integers, kind)
        assert np.all(x == np.round(x))
        assert np.array_equal(O.unrotate(x, kind), integers)
        for seed in range(64):
            original = _values(seed)
            back = O.unrotate(O.rotate(original, kind), kind)
            assert np.max(np.abs(back - original)) <= 1e-5


def test_rotated_query_dots_equal_the_original_dots():
    """rotation.rs:197-216"""
    for kind in KINDS:
        for seed in range(64):
            q, k = _values(2 * seed), _values(2 * seed + 1)
            rq, rk = O.rotate_query(q, kind), O.rotate(k, kind)
            expected = float(np.dot(q.astype(np.float64), k.astype(np.float64)))
            rotated = float(np.dot(rq.astype(np.float64), rk.astype(np.float64)))
            assert abs(rotated - expected) <= 1e-5
            assert np.array_equal(rq.view(np.uint32), (O.rotate(q, kind) / np.float32(32)).view(np.uint32))


def test_a_nonfinite_value_spreads_over_its_block():
    """rotation.rs:207-216"""
    x = _values(3)
    x[5] = np.nan
    assert np.isnan(O.rotate(x, 2)).all()
    x = _values(4)
    x[0] = np.inf
    assert not np.isfinite(O.rotate(x, 0)).any()


def test_nibbles_and_q4_blocks():
    """codec.rs:87-129: codes -7..7 two per byte (element 2i low), a NaN
    block scale for a non-finite block, zero codes and scale for zeros."""
    assert [O.lib().fo_or_nibble(0xF7, h) for h in (0, 1)] == [7, -1]
    assert [O.lib().fo_or_nibble(0x89, h) for h in (0, 1)] == [-7, -8]
    vals = np.linspace(-3.0, 3.5, 32).astype(np.float32)
    bits, codes = O.q4_block(vals)
    scale = O.bf16_f32(bits)
    assert bits == O.bf16_up(np.float32(np.float64(3.5) / 7.0))
    dec = np.array([O.lib().fo_or_nibble(int(codes[i // 2]), i % 2) for i in range(32)])
    assert np.all(np.abs(dec) <= 7)
    want = [int(O.round_clamped(float(x) / scale, 7.0)) for x in vals]
    assert dec.tolist() == want
    vals[9] = np.nan
    bits, codes = O.q4_block(vals)
    assert bits == 0x7FC0 and not codes.any()
    bits, codes = O.q4_block(np.zeros(32, np.float32))
    assert bits == 0 and not codes.any()


STORAGES = [O.FORMATS[n] for n in ("f32", "f32r", "q8", "q8r", "q4", "q4r", "q16")]


def _rotated_blocks(values, kinds, rotated):
    if not rotated:
        return values
    out = values.reshape(-1, len(kinds), 32).copy()
    for i, kind in enumerate(kinds):
        for row in range(out.shape[0]):
            out[row, i] = O.rotate(out[row, i], kind)
    return out.reshape(-1)


@pytest.mark.parametrize("fmt", STORAGES)
@pytest.mark.parametrize("p,generated", [(1, 1), (3, 2), (129, 17), (300, 130)])
def test_rotated_storages_decode_as_a_pre_and_post_transform(fmt, p, generated):
    """kv/tests.rs:198-250: FP32 records hold exactly the (rotated) values;
    every storage's decode equals the online head over its dequantized
    records with the rotated query, its output un-rotated (here to 1e-6)."""
    rotated = bool(fmt & O.ROTATED)
    k, v, q = G.kv_fixture(p, p)
    c = O.SplitCache(k, v, p, p + generated, fmt=fmt, chunks=1)
    assert c.status == O.OK
    tk, tv = G.kv_tail(generated)
    for t in range(generated):
        c.push(tk[t * 512:(t + 1) * 512], tv[t * 512:(t + 1) * 512])
    dk, dv = c.dequantized_compact()
    tail = c.decoded_tail().reshape(8, -1, 128)[:, :generated]
    gk = tail[:, :, :64].transpose(1, 0, 2).reshape(-1)
    gvv = tail[:, :, 64:].transpose(1, 0, 2).reshape(-1)
    if fmt & ~O.ROTATED == O.F32:
        assert np.array_equal(dk, _rotated_blocks(k, (0, 1), rotated))
        assert np.array_equal(dv, _rotated_blocks(v, (2, 3), rotated))
        assert np.array_equal(gk, _rotated_blocks(tk, (0, 1), rotated))
        assert np.array_equal(gvv, _rotated_blocks(tv, (2, 3), rotated))
    sinks = np.array([h * 0.25 - 1.0 for h in range(16)], np.float32)
    rq = q.reshape(16, 2, 32).copy()
    if rotated:
        for h in range(16):
            rq[h, 0], rq[h, 1] = O.rotate_query(rq[h, 0], 0), O.rotate_query(rq[h, 1], 1)
    expected = O.attention_online(rq.reshape(-1), dk, np.concatenate([dv, gvv]), 16, 8, 64,
                                  (p + generated - 1, 0, p), sinks, generated_k=gk).reshape(16, 2, 32)
    if rotated:
        for h in range(16):
            expected[h, 0], expected[h, 1] = O.unrotate(expected[h, 0], 2), O.unrotate(expected[h, 1], 3)
    out = c.decode(q, sinks)
    bad = np.abs(out - expected.reshape(-1)) > 1e-6 * (1 + np.abs(expected.reshape(-1)))
    assert not bad.any(), np.abs(out - expected.reshape(-1)).max()


def test_research_formats_stay_close_to_fp32():
    """kv/tests.rs:282-304: Q8Rot within 0.02, Q4Rot within 0.05 of compact FP32."""
    p = 257
    k, v, q = G.kv_fixture(p, 9)
    tail = np.full(512, 0.02, np.float32)
    sinks = np.full(16, 0.5, np.float32)
    for name, bound in (("q8r", 0.02), ("q4r", 0.05)):
        c = O.SplitCache(k, v, p, p + 1, fmt=name)
        assert c.status == O.OK
        c.push(tail, tail)
        out = c.decode(q, sinks)
        assert np.isfinite(out).all()
        assert np.all(np.abs(out - GOLD["kv_lowprec_expected"]) < bound), name


def test_rotated_fp32_records_change_rounding_only():
    """kv/tests.rs:634-662: 1e-6 * (1 + |b|) against unrotated FP32 records."""
    worst = 0.0
    for p, generated in [(1, 1), (129, 17), (1000, 40)]:
        k, v, q = G.kv_fixture(p, 7)
        tk, tv = G.kv_tail(generated)
        sinks = np.array([h * 0.25 - 1.0 for h in range(16)], np.float32)
        outs = []
        for fmt in ("f32", "f32r"):
            c = O.SplitCache(k, v, p, p + generated, fmt=fmt)
            for t in range(generated):
                c.push(tk[t * 512:(t + 1) * 512], tv[t * 512:(t + 1) * 512])
            outs.append(c.decode(q, sinks))
        worst = max(worst, float(np.max(np.abs(outs[1] - outs[0]) / (1 + np.abs(outs[0])))))
    assert worst <= 1e-6, worst


def test_rotated_storage_checks_the_pair_on_unrotated_keys():
    """kv/tests.rs:355-369"""
    k = np.zeros(16 * 64, np.float32)
    v = np.zeros(8 * 64, np.float32)
    k[64] = 1.0
    assert O.SplitCache(k, v, 1, 2, fmt="q8r").status == O.ERR_PAIR
    k[64] = 0.0
    k[:32] = k[64:96] = np.arange(32, dtype=np.float32)
    assert O.SplitCache(k, v, 1, 2, fmt="q8r").status == O.OK
    big = np.full(16 * 64, 3e37, np.float32)
    assert O.SplitCache(big, v, 1, 2, fmt="q4r").status == O.ERR_ROTATED


@pytest.mark.parametrize("fmt", ["q4", "q8r", "q4r"])
def test_nonfinite_tail_values_reach_the_output(fmt):
    """kv/tests.rs:306-324 (rotation spreads the NaN over its block first)."""
    p = 130
    k, v, q = G.kv_fixture(p, 5)
    c = O.SplitCache(k, v, p, p + 2, fmt=fmt)
    tail = np.full(512, 0.01, np.float32)
    c.push(tail, tail)
    tail[3] = np.nan
    c.push(tail, tail)
    out = c.decode(q, np.full(16, 0.5, np.float32))
    assert np.isnan(out[:64]).all()
