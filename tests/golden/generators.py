"""Deterministic input generators of the reference's own attention tests,
restated in numpy, plus an independent numpy f64 dense attention.

These build the inputs the reference's tests use, so the golden fixtures
(tests/golden/*.npz, written by make_golden.py) and the tests that read them
regenerate identical operands.  Citations are to the reference project.
"""

from __future__ import annotations

import numpy as np

_A, _C, _M = 1664525, 1013904223, (1 << 32) - 1


def lcg_states(n: int, seed: int) -> np.ndarray:
    """u32 states of `state = state * 1664525 + 1013904223` (wrapping), the
    generator of src/kernels/tests.rs:6-14 and prefill64/tests.rs:4-19."""
    if n == 0:
        return np.zeros(0, np.uint64)
    block = 1024
    first = np.empty(min(n, block), np.uint64)
    s = seed & _M
    for i in range(first.size):
        s = (s * _A + _C) & _M
        first[i] = s
    if n <= block:
        return first
    # jump ahead by `block` steps: s -> A*s + C (mod 2^32)
    a_j, c_j = 1, 0
    for _ in range(block):
        a_j, c_j = (a_j * _A) & _M, (c_j * _A + _C) & _M
    out = np.empty(((n + block - 1) // block) * block, np.uint64)
    out[:block] = first
    cur = first.copy()
    for b in range(1, out.size // block):
        cur = (cur * np.uint64(a_j) + np.uint64(c_j)) & np.uint64(_M)
        out[b * block:(b + 1) * block] = cur
    return out[:n]


def lcg_values(n: int, seed: int) -> np.ndarray:
    """src/kernels/tests.rs:6-14: values in [-1, 1)."""
    s = lcg_states(n, seed)
    return ((s >> np.uint64(8)).astype(np.float64) / 16777216.0 * 2.0 - 1.0).astype(np.float32)


def prefill_values(n: int, seed: int, rng: float) -> np.ndarray:
    """prefill64/tests.rs:4-19: scaled LCG values with -0.0, +0.0 and a
    subnormal (bits 3) at every index i % 97 in {0, 1, 2}."""
    s = lcg_states(n, seed)
    x = (((s >> np.uint64(8)).astype(np.float64) / 16777216.0 * 2.0 - 1.0).astype(np.float32) * np.float32(rng))
    i = np.arange(n) % 97
    x[i == 0] = np.float32(-0.0)
    x[i == 1] = np.float32(0.0)
    x[i == 2] = np.array([3], np.uint32).view(np.float32)[0]
    return x.astype(np.float32)


def scaled_values(n: int, seed: int, rng: float) -> np.ndarray:
    """prefill64/test_data.rs:4-11: kernels::test_values scaled by `rng`."""
    return (lcg_values(n, seed) * np.float32(rng)).astype(np.float32)


def normalized(n: int, seed: int) -> np.ndarray:
    """prefill64/test_data.rs:13-23: heads scaled to norm 8 (f32 sequential sum)."""
    x = scaled_values(n, seed, 1.0).reshape(-1, 64)
    norm = np.sqrt(np.cumsum(x * x, axis=1, dtype=np.float32)[:, -1]).astype(np.float32)
    factor = (np.float32(8.0) / norm).astype(np.float32)
    return (x * factor[:, None]).astype(np.float32).reshape(-1)


def bf16_round(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even to BF16 (half::bf16::from_f32), as float32."""
    u = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16
    r = np.where(nan, ((u >> 16) | 0x40) << 16, r)
    return r.astype(np.uint32).view(np.float32)


def bf16_values(n: int, seed: int, rng: float) -> np.ndarray:
    """prefill64/bf16.rs:671-681: scaled LCG values made BF16-exact."""
    return bf16_round(lcg_values(n, seed) * np.float32(rng))


def kv_fixture(p: int, seed: int, heads: int = 16, groups: int = 8):
    """src/quant/kv/tests.rs:71-89: modular keys whose temporal halves are
    shared inside each GQA pair, values and one query row."""
    t = np.arange(p)[:, None, None]
    h = np.arange(heads)[None, :, None]
    d = np.arange(64)[None, None, :]
    identity = np.where(d < 32, h // 2, h)
    k = (((t * 31 + identity * 17 + d * 7 + seed) % 101).astype(np.float32) / np.float32(151.0)
         - np.float32(0.3)).astype(np.float32)
    i = np.arange(p * groups * 64)
    v = (((i + seed) % 73).astype(np.float32) / np.float32(97.0) - np.float32(0.2)).astype(np.float32)
    j = np.arange(heads * 64)
    q = (((j * 7 + seed) % 61).astype(np.float32) / np.float32(21.0) - np.float32(1.4)).astype(np.float32)
    return k.reshape(-1), v, q


def kv_tail(generated: int, groups: int = 8):
    """src/quant/kv/tests.rs:30-35: generated keys and values [generated][G][64]."""
    i = np.arange(generated * groups * 64)
    tk = (((i * 13) % 37).astype(np.float32) / np.float32(53.0) - np.float32(0.3)).astype(np.float32)
    tv = (((i * 11) % 41).astype(np.float32) / np.float32(67.0) - np.float32(0.3)).astype(np.float32)
    return tk, tv


def kv_rows_query(rows: int, heads: int = 16):
    """src/quant/kv/tests.rs:36-38: verification queries."""
    i = np.arange(rows * heads * 64)
    return (((i * 7 + 3) % 61).astype(np.float32) / np.float32(21.0) - np.float32(1.4)).astype(np.float32)


def attention_f64(q, prefix_k, v, heads, kv_heads, dim, geometry, sinks, generated_k=None, bf16_operands=False):
    """Dense f64 attention with the sink folded into the denominator
    (src/kernels/tests.rs:204-248), over a compact cache (mod.rs:78-157).
    Independent numpy restatement (the C oracle has its own)."""
    offset, image_start, image_end = geometry
    q = np.asarray(q, np.float64).reshape(-1, heads, dim)
    pk = np.asarray(prefix_k, np.float64).reshape(-1, heads, dim)
    vv = np.asarray(v, np.float64).reshape(-1, kv_heads, dim)
    if bf16_operands:
        q = bf16_round(q.astype(np.float32)).astype(np.float64)
        pk = bf16_round(pk.astype(np.float32)).astype(np.float64)
        vv = bf16_round(vv.astype(np.float32)).astype(np.float64)
    total = vv.shape[0]
    repeat = heads // kv_heads
    keys = np.empty((total, heads, dim))
    keys[:pk.shape[0]] = pk
    if total > pk.shape[0]:
        gk = np.asarray(generated_k, np.float64).reshape(-1, kv_heads, dim)
        if bf16_operands:
            gk = bf16_round(gk.astype(np.float32)).astype(np.float64)
        keys[pk.shape[0]:] = np.repeat(gk, repeat, axis=1)
    values = np.repeat(vv, repeat, axis=1)  # [T][H][d]
    ql = q.shape[0]
    absolute = offset + np.arange(ql)[:, None]
    key = np.arange(total)[None, :]
    in_img = lambda p: (p >= image_start) & (p < image_end)
    allowed = (key <= absolute) | (in_img(absolute) & in_img(key))  # [Q][T]
    scores = np.einsum("qhd,thd->hqt", q, keys) / np.sqrt(dim)
    scores = np.where(allowed[None], scores, -np.inf)
    sinks = np.asarray(sinks, np.float64)[:, None, None]
    mx = np.maximum(scores.max(axis=2, keepdims=True), sinks)
    e = np.exp(scores - mx)
    denom = np.exp(sinks - mx) + e.sum(axis=2, keepdims=True)
    out = np.einsum("hqt,thd->qhd", e / denom, values)
    return out.reshape(-1)


# Case tables of the reference's tests.
DENSE_TABLE = [  # src/kernels/tests.rs:252-262 (qlen, kvlen, heads, dim, offset, start, end)
    (7, 7, 2, 7, 0, 1, 5),
    (5, 5, 3, 17, 0, 0, 0),
    (1, 267, 16, 64, 266, 1, 201),
    (3, 260, 2, 33, 257, 2, 193),
    (33, 267, 2, 64, 234, 2, 252),
    (133, 133, 2, 64, 0, 16, 98),
    (129, 129, 2, 8, 0, 0, 129),
    (1, 1, 1, 1, 0, 0, 0),
]
PREFILL64_CASES = [(70, 3, 65), (300, 5, 262), (257, 0, 257), (160, 16, 144), (129, 1, 128), (40, 0, 3),
                   (95, 10, 90)]  # prefill64/tests.rs:36-44
STATIC_CASES = [(70, 70, 0, 3, 65), (300, 300, 0, 5, 262), (257, 257, 0, 0, 257), (160, 160, 0, 16, 144),
                (129, 129, 0, 1, 128), (40, 40, 0, 0, 3), (95, 95, 0, 10, 90), (5, 5, 0, 1, 3),
                (37, 300, 263, 5, 262), (100, 230, 130, 1, 129)]  # static_shift/tests.rs:53-64
BF16_CASES = [(70, 3, 65), (300, 5, 262), (257, 0, 257), (129, 1, 128), (40, 0, 3),
              (95, 10, 90)]  # bf16.rs:860-867, bf16/static_shift/tests.rs:88-95


def prefill64_operands(query_len):
    """prefill64/tests.rs:25-33"""
    return (prefill_values(query_len * 16 * 64, 17 + query_len, 3.0),
            prefill_values(query_len * 16 * 64, 19 + query_len, 3.0),
            prefill_values(query_len * 8 * 64, 23 + query_len, 3.0),
            prefill_values(16, 29, 2.0))


def static_operands(queries, total):
    """prefill64/test_data.rs:25-34"""
    seed = 17 + total
    return (normalized(queries * 16 * 64, seed), normalized(total * 16 * 64, seed + 2),
            scaled_values(total * 8 * 64, seed + 6, 3.0), scaled_values(16, 29, 2.0))


def bf16_operands(query_len):
    """prefill64/bf16.rs:869-872 (BF16-exact inputs)"""
    return (bf16_values(query_len * 16 * 64, 17 + query_len, 3.0),
            bf16_values(query_len * 16 * 64, 19 + query_len, 3.0),
            bf16_values(query_len * 8 * 64, 23 + query_len, 3.0),
            bf16_values(16, 29, 2.0))


# Heads whose outputs the large fixtures keep (one even, one odd head of
# different GQA groups) to keep the committed files small.
SAMPLE_HEADS = (0, 9)


def sample_heads(out, heads=16, dim=64):
    return np.asarray(out).reshape(-1, heads, dim)[:, list(SAMPLE_HEADS), :].reshape(-1)


def rope_interleaved(x: np.ndarray, theta: float = 10000.0) -> np.ndarray:
    """Rotate interleaved pairs (2i, 2i+1) of every 64-wide head of
    x [S][H][64] by position * theta^(-2i/64), as src/model/rope.rs:55-67
    applies its [cos, sin] factors."""
    s = x.shape[0]
    i = np.arange(32, dtype=np.float64)
    angle = np.arange(s, dtype=np.float64)[:, None] * theta ** (-2.0 * i / 64.0)[None, :]
    cos = np.cos(angle).astype(np.float32)[:, None, :]
    sin = np.sin(angle).astype(np.float32)[:, None, :]
    a, b = x[..., 0::2], x[..., 1::2]
    out = np.empty_like(x)
    out[..., 0::2] = a * cos - b * sin
    out[..., 1::2] = a * sin + b * cos
    return out


def c2_inputs(seed: int = 1, seq: int = 6544, image_end: int = 4096, heads: int = 16, kv_heads: int = 8):
    """full-page prefill, 4,096 bidirectional image tokens
    then causal text; Q, K ~ N(0, 0.5) (0.5 is the variance) rotated by RoPE
    theta 10,000 at their positions; V ~ N(0, 1); sinks ~ N(0, 1)."""
    rng = np.random.default_rng(seed)
    q = rope_interleaved((rng.standard_normal((seq, heads, 64)) * np.sqrt(0.5)).astype(np.float32))
    k = rope_interleaved((rng.standard_normal((seq, heads, 64)) * np.sqrt(0.5)).astype(np.float32))
    v = rng.standard_normal((seq, kv_heads, 64)).astype(np.float32)
    sinks = rng.standard_normal(heads).astype(np.float32)
    return q, k, v, sinks, (0, 0, image_end)
