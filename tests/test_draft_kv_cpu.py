"""Pins the oracle's draft-head KV (src/draft_head.rs:177-220
`Kv::Q8` / `quantize_row`, :548-759 `attend` / `group_q8`) to the reference's
own test `int8_attention_and_window` (draft_head.rs:794-870): int8
attention within 0.03 of a double-precision reference over the newest
`window` verified rows and the FP32 chain rows.  CPU only."""

import numpy as np
import pytest

import oracle as O

ROWS, CHAIN, WIDTH = 300, 2, 512


def x(i):
    """draft_head.rs:799: ((i * 7919 % 1009) - 504) / 250."""
    i = np.asarray(i, np.int64)
    return (((i * 7919) % 1009).astype(np.float32) - np.float32(504.0)) / np.float32(250.0)


def fixture():
    keys = x(3 * np.arange(ROWS * WIDTH) + 1)
    values = x(5 * np.arange(ROWS * WIDTH) + 2)
    q = x(7 * np.arange(16 * 64) + 3)  # the query heads of the QKV row
    chain_keys = x(11 * np.arange(CHAIN * WIDTH) + 4)
    chain_values = x(13 * np.arange(CHAIN * WIDTH) + 5)
    return keys, values, q, chain_keys, chain_values


def reference_f64(keys, values, q, chain_keys, chain_values, start):
    """The test's double-precision attention over positions start..rows+chain."""
    k = np.concatenate([keys, chain_keys]).reshape(-1, 8, 64).astype(np.float64)
    v = np.concatenate([values, chain_values]).reshape(-1, 8, 64).astype(np.float64)
    out = np.zeros((16, 64))
    for h in range(16):
        g = h // 2
        s = k[start:, g] @ q[h * 64:(h + 1) * 64].astype(np.float64) / 8.0
        w = np.exp(s - s.max())
        out[h] = (w / w.sum()) @ v[start:, g]
    return out.reshape(-1)


def test_quantize_row_rounds_half_away_and_clamps():
    """draft_head.rs:213-220"""
    row = np.linspace(-2.0, 1.0, 64).astype(np.float32)
    codes = np.zeros(64, np.int8)
    scale = O.lib().fo_or_draft_quantize_row(O._p(row), O._p(codes))
    assert scale == np.float32(2.0) / np.float32(127.0)
    inv = np.float32(127.0) / np.float32(2.0)
    want = np.clip(np.sign(row * inv) * np.floor(np.abs(row * inv) + 0.5), -127, 127).astype(np.int8)
    assert np.array_equal(codes, want)
    row[:] = 0.0
    row[3] = np.nan
    scale = O.lib().fo_or_draft_quantize_row(O._p(row), O._p(codes))
    assert scale == 0.0 and not codes.any()


@pytest.mark.parametrize("window", [0, 1, 64, ROWS, 1000])
def test_int8_attention_and_window(window):
    """draft_head.rs:794-870: int8 within 0.03 of f64 over the newest window."""
    keys, values, q, ck, cv = fixture()
    kv = O.DraftKv(ROWS + 8)
    kv.push(keys[:100 * WIDTH], values[:100 * WIDTH])
    kv.push(keys[100 * WIDTH:], values[100 * WIDTH:])
    start = 0 if window == 0 else max(ROWS - window, 0)
    expected = reference_f64(keys, values, q, ck, cv, start)
    got = kv.attend(q, ROWS, window, ck, cv)
    assert np.max(np.abs(got - expected)) < 0.03


def test_window_attends_exactly_the_newest_rows():
    """A window of w equals a cache holding only the newest w rows."""
    keys, values, q, ck, cv = fixture()
    full = O.DraftKv(ROWS)
    full.push(keys, values)
    for w in (1, 7, 64):
        tail = O.DraftKv(w)
        tail.push(keys[(ROWS - w) * WIDTH:], values[(ROWS - w) * WIDTH:])
        a = full.attend(q, ROWS, w, ck, cv)
        b = tail.attend(q, w, 0, ck, cv)
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
