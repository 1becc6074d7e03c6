"""ctypes wrapper of the CPU oracle (oracle/fo_oracle.c).

TEST INFRASTRUCTURE ONLY.  This module is the checker: tests/,
__graft_entry__.smoke() and bench.py's cpu_baseline / reference arm use it
to compute what the reference's CPU attention returns on the same inputs.
The product (falcon-ocr-cpu_b200/) never imports it.

The C library restates the reference Rust crate's arithmetic; see the
file:line citations in fo_oracle.c.  Parity is pinned by the reference's own
known answers and tolerance tables (tests/golden/).
"""

from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
BUILD = os.path.join(HERE, "_build")

F32, Q16, Q8, BF16, Q4 = 0, 1, 2, 3, 4
# Flag: every 32-element block stored rotated (src/quant/rotation.rs); with
# F32, Q8 or Q4.  Q8 | ROTATED is Kv::Q8Rot, Q4 | ROTATED Kv::Q4Rot.
ROTATED = 16
FORMATS = {"f32": F32, "q16": Q16, "q8": Q8, "bf16": BF16, "q4": Q4, "q8r": Q8 | ROTATED, "q4r": Q4 | ROTATED,
           "f32r": F32 | ROTATED}
# Record codes dtype per element format (src/quant/kv.rs:98-118; BF16 is
# new here); Q4 packs two codes per byte.
CODE_DTYPES = {F32: np.float32, Q16: np.int16, Q8: np.int8, BF16: np.uint16, Q4: np.uint8}

OK, ERR_PAIR, ERR_NONFINITE, ERR_OVERFLOW, ERR_SHAPE, ERR_CAPACITY, ERR_ROTATED = range(7)

RECORD, TAIL_RECORD = 160, 128

_lib = None


def _cpu_has_avx512() -> bool:
    try:
        with open("/proc/cpuinfo") as f:
            flags = f.read()
        return " avx512f" in flags and " avx512bw" in flags and " avx512vl" in flags
    except OSError:
        return False


def build() -> None:
    """Compile the oracle (make in oracle/)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is not None:
        return _lib
    name = "libfo_oracle_v4.so" if _cpu_has_avx512() else "libfo_oracle_v3.so"
    path = os.path.join(BUILD, name)
    if not os.path.exists(path):
        build()
    L = ctypes.CDLL(path)
    P, I64, I, F = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_float
    sig = {
        "fo_or_bf16_up": (ctypes.c_uint16, [F]),
        "fo_or_bf16_f32": (F, [ctypes.c_uint16]),
        "fo_or_bf16_rne": (ctypes.c_uint16, [F]),
        "fo_or_q8_scale": (F, [P, I64]),
        "fo_or_q16_scale": (F, [P, I64]),
        "fo_or_round_clamped": (ctypes.c_double, [ctypes.c_double, ctypes.c_double]),
        "fo_or_q8_code": (ctypes.c_int8, [F, F]),
        "fo_or_q16_code": (ctypes.c_int16, [F, F]),
        "fo_or_exp_poly": (F, [F]),
        "fo_or_exp_poly_unchecked": (F, [F]),
        "fo_or_attention_f64": (None, [P, P, P, P] + [I64] * 9 + [P, I, P]),
        "fo_or_attention_online": (None, [P, P, P, P] + [I64] * 9 + [P, I, P]),
        "fo_or_prefill64": (None, [P, P, P] + [I64] * 6 + [P, I, I, P]),
        "fo_or_prefill_bf16": (None, [P, P, P] + [I64] * 5 + [P, I, I, P]),
        "fo_or_kv_seal": (I, [P, P] + [I64] * 5 + [I, P, P]),
        "fo_or_kv_push": (None, [P, P, I64, I, I64, I64, P, P]),
        "fo_or_kv_value": (F, [P, P, I, I64, I64, I64]),
        "fo_or_kv_decode_rows": (None, [P, P, P, P, I] + [I64] * 5 + [P, I64, P, I64, I, P]),
        "fo_or_qkv_rows": (None, [P, P, I64, I64, I64, P, P, P]),
        "fo_or_rotation_signs": (ctypes.c_uint32, [I]),
        "fo_or_fwht32": (None, [P]),
        "fo_or_rotate": (None, [P, I]),
        "fo_or_rotate_query": (None, [P, I]),
        "fo_or_unrotate": (None, [P, I]),
        "fo_or_q4_block": (ctypes.c_uint16, [P, P]),
        "fo_or_nibble": (ctypes.c_int8, [ctypes.c_uint8, I]),
        "fo_or_draft_quantize_row": (F, [P, P]),
        "fo_or_draft_push": (None, [P, P, I64, I64, I64, P, P, P, P]),
        "fo_or_draft_attend": (None, [P, P, P, P, I64, P, I64, I64, P, P, I64, P]),
        "fo_or_set_threads": (None, [I]),
        "fo_or_max_threads": (I, []),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    _lib = L
    return L


def _p(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def set_threads(n: int) -> None:
    lib().fo_or_set_threads(int(n))


def max_threads() -> int:
    return int(lib().fo_or_max_threads())


# ---------------------------------------------------------------- codec
def bf16_up(x: float) -> int:
    return int(lib().fo_or_bf16_up(float(x)))


def bf16_f32(bits: int) -> float:
    return float(lib().fo_or_bf16_f32(int(bits)))


def bf16_rne(x: float) -> int:
    return int(lib().fo_or_bf16_rne(float(x)))


def round_clamped(x: float, limit: float) -> float:
    return float(lib().fo_or_round_clamped(float(x), float(limit)))


def q8_code(value: float, scale: float) -> int:
    return int(lib().fo_or_q8_code(float(value), float(scale)))


def q16_code(value: float, scale: float) -> int:
    return int(lib().fo_or_q16_code(float(value), float(scale)))


def q8_scale(values) -> float:
    v = _f32(values)
    return float(lib().fo_or_q8_scale(_p(v), v.size))


def q16_scale(values) -> float:
    v = _f32(values)
    return float(lib().fo_or_q16_scale(_p(v), v.size))


def exp_poly(x: float) -> float:
    return float(lib().fo_or_exp_poly(float(x)))


# ------------------------------------------------------------ attention
def _compact(q, prefix_k, generated_k, v, n_heads, n_kv_heads, head_dim):
    q, prefix_k, v = _f32(q), _f32(prefix_k), _f32(v)
    generated_k = _f32(generated_k if generated_k is not None else np.zeros(0, np.float32))
    prefix_len = prefix_k.size // (n_heads * head_dim)
    total_len = v.size // (n_kv_heads * head_dim)
    query_len = q.size // (n_heads * head_dim)
    return q, prefix_k, generated_k, v, query_len, prefix_len, total_len


def attention_f64(q, prefix_k, v, n_heads, n_kv_heads, head_dim, geometry, sinks, generated_k=None,
                  bf16_operands=False):
    """Dense f64 attention (src/kernels/tests.rs:204-248); returns float64."""
    q, pk, gk, v, ql, pl, tl = _compact(q, prefix_k, generated_k, v, n_heads, n_kv_heads, head_dim)
    out = np.zeros(q.size, np.float64)
    sinks = _f32(sinks)
    lib().fo_or_attention_f64(_p(q), _p(pk), _p(gk), _p(v), ql, pl, tl, n_heads, n_kv_heads, head_dim,
                              geometry[0], geometry[1], geometry[2], _p(sinks), int(bf16_operands), _p(out))
    return out


def attention_online(q, prefix_k, v, n_heads, n_kv_heads, head_dim, geometry, sinks, generated_k=None,
                     exp_fast=False):
    """The online head, any head width (src/kernels/attention/online.rs:89-169)."""
    q, pk, gk, v, ql, pl, tl = _compact(q, prefix_k, generated_k, v, n_heads, n_kv_heads, head_dim)
    out = np.zeros(q.size, np.float32)
    sinks = _f32(sinks)
    lib().fo_or_attention_online(_p(q), _p(pk), _p(gk), _p(v), ql, pl, tl, n_heads, n_kv_heads, head_dim,
                                 geometry[0], geometry[1], geometry[2], _p(sinks), int(exp_fast), _p(out))
    return out


def prefill64(q, k, v, n_heads, n_kv_heads, geometry, sinks, softmax_static=False, exp_fast=False):
    """FP32 prefill tiles over a pure prefix (prefill64.rs, static_shift.rs)."""
    q, k, v, sinks = _f32(q), _f32(k), _f32(v), _f32(sinks)
    ql = q.size // (n_heads * 64)
    out = np.zeros(q.size, np.float32)
    lib().fo_or_prefill64(_p(q), _p(k), _p(v), ql, n_heads, n_kv_heads, geometry[0], geometry[1], geometry[2],
                          _p(sinks), int(softmax_static), int(exp_fast), _p(out))
    return out


def prefill_bf16(q, k, v, n_heads, n_kv_heads, image, sinks, softmax_static=True, exp_fast=False):
    """BF16 prefill tiles (prefill64/bf16.rs, bf16/static_shift.rs); query_offset 0."""
    q, k, v, sinks = _f32(q), _f32(k), _f32(v), _f32(sinks)
    ql = q.size // (n_heads * 64)
    out = np.zeros(q.size, np.float32)
    lib().fo_or_prefill_bf16(_p(q), _p(k), _p(v), ql, n_heads, n_kv_heads, image[0], image[1], _p(sinks),
                             int(softmax_static), int(exp_fast), _p(out))
    return out


# ---------------------------------------------------------- split cache
def rotation_signs(kind: int) -> int:
    """D's bit pattern of block kind 0..3 (rotation.rs:42-61)."""
    return int(lib().fo_or_rotation_signs(int(kind)))


def _block_op(name, x, kind):
    x = _f32(x).copy()
    assert x.size == 32
    getattr(lib(), name)(_p(x), int(kind))
    return x


def fwht32(x):
    x = _f32(x).copy()
    lib().fo_or_fwht32(_p(x))
    return x


def rotate(x, kind):
    return _block_op("fo_or_rotate", x, kind)


def rotate_query(x, kind):
    return _block_op("fo_or_rotate_query", x, kind)


def unrotate(x, kind):
    return _block_op("fo_or_unrotate", x, kind)


def q4_block(values):
    """(BF16 scale bits, 16 packed code bytes) of one 32-value block."""
    values = _f32(values)
    codes = np.zeros(16, np.uint8)
    bits = lib().fo_or_q4_block(_p(values), _p(codes))
    return int(bits), codes


def qkv_rows(qkv, rope, rows, heads=16, groups=8):
    """fo_or_qkv_rows: the fused split + per-head RMS norm + RoPE of the
    projection rows (src/model/fused.rs:96-116).  Returns q, k [rows][heads][64]
    and v [rows][groups][64] as flat float32 arrays."""
    qkv, rope = _f32(qkv), _f32(rope)
    q = np.zeros(rows * heads * 64, np.float32)
    k = np.zeros(rows * heads * 64, np.float32)
    v = np.zeros(rows * groups * 64, np.float32)
    lib().fo_or_qkv_rows(_p(qkv), _p(rope), rows, heads, groups, _p(q), _p(k), _p(v))
    return q, k, v


class SplitCache:
    """The reference's SplitPrefix (src/quant/kv.rs:155-174) over numpy arrays:
    prefix records [G][P][160], scales [G][P][5]; tail [G][cap][128], [G][cap][4]."""

    def __init__(self, k, v, prefix_len, capacity, heads=16, groups=8, fmt=F32, chunks=None, fast_exp=False):
        self.fmt = fmt if isinstance(fmt, int) else FORMATS[fmt]
        self.element, self.rotated = self.fmt & ~ROTATED, bool(self.fmt & ROTATED)
        self.prefix_len, self.capacity, self.heads, self.groups = prefix_len, capacity, heads, groups
        self.tail_capacity = capacity - prefix_len
        self.tail_len = 0
        # default_chunks (kv.rs:188-197): F32 one scan, coded caches four.
        self.chunks = chunks if chunks else (1 if self.element in (F32,) else 4)
        self.fast_exp = bool(fast_exp)
        dt = CODE_DTYPES[self.element]
        per = 2 if self.element == Q4 else 1  # codes per stored element
        self.codes = np.zeros(max(groups * prefix_len * RECORD // per, 1), dt)
        self.scales = np.zeros(max(groups * prefix_len * 5, 1), np.uint16)
        self.tail_codes = np.zeros(max(groups * self.tail_capacity * TAIL_RECORD // per, 1), dt)
        self.tail_scales = np.zeros(max(groups * self.tail_capacity * 4, 1), np.uint16)
        k, v = _f32(k), _f32(v)
        self.status = lib().fo_or_kv_seal(_p(k), _p(v), prefix_len, capacity, heads, groups, 64, self.fmt,
                                          _p(self.codes), _p(self.scales))

    def push(self, k_unique, v_unique):
        """One generated position, [G][64] keys and values (kv.rs:456-513)."""
        assert self.tail_len < self.tail_capacity, "split tail capacity"
        k_unique, v_unique = _f32(k_unique), _f32(v_unique)
        lib().fo_or_kv_push(_p(k_unique), _p(v_unique), self.groups, self.fmt, self.tail_capacity, self.tail_len,
                            _p(self.tail_codes), _p(self.tail_scales))
        self.tail_len += 1

    def append(self, k, v):
        """Expanded rows [rows][heads][64]: the pair's first head per group (kv.rs:430-449)."""
        width = self.heads * 64
        k, v = _f32(k).reshape(-1, width), _f32(v).reshape(-1, width)
        for kr, vr in zip(k, v):
            ku = kr.reshape(self.groups, 2, 64)[:, 0, :]
            vu = vr.reshape(self.groups, 2, 64)[:, 0, :]
            self.push(ku, vu)

    def truncate_tail(self, tail_len):
        assert tail_len <= self.tail_len, "cannot grow the tail by truncation"
        self.tail_len = tail_len

    def decode_rows(self, q, rows, sinks):
        q, sinks = _f32(q), _f32(sinks)
        out = np.zeros(rows * self.heads * 64, np.float32)
        lib().fo_or_kv_decode_rows(_p(self.codes), _p(self.scales), _p(self.tail_codes), _p(self.tail_scales),
                                   self.fmt, self.prefix_len, self.tail_capacity, self.tail_len, self.heads,
                                   self.groups, _p(q), rows, _p(sinks), self.chunks, int(self.fast_exp), _p(out))
        return out

    def decode(self, q, sinks):
        return self.decode_rows(q, 1, sinks)

    def dequantized_compact(self):
        """Compact keys [P][heads][64] and values [P][G][64] the records decode to."""
        L = lib()
        P, G = self.prefix_len, self.groups
        rec = self.decoded_records()
        k = np.zeros((P, self.heads, 64), np.float32)
        vv = np.zeros((P, G, 64), np.float32)
        r = rec.reshape(G, P, RECORD)
        for pair in range(2):
            k[:, pair::2, :32] = r[:, :, 0:32].transpose(1, 0, 2)
            k[:, pair::2, 32:] = r[:, :, 32 + 32 * pair:64 + 32 * pair].transpose(1, 0, 2)
        vv[:] = r[:, :, 96:160].transpose(1, 0, 2)
        del L
        return k.reshape(-1), vv.reshape(-1)

    def decoded_records(self):
        return decode_records(self.codes, self.scales, self.fmt)

    def decoded_tail(self):
        return decode_records(self.tail_codes, self.tail_scales, self.fmt)


def decode_records(codes, scales, fmt):
    """Vectorised kv.rs:209-219: fl(code * bf16 scale) (rotated records stay
    in the rotated basis)."""
    fmt &= ~ROTATED
    if fmt == Q4:
        lo = ((codes.astype(np.uint8) << 4).view(np.int8) >> 4).astype(np.int8)
        hi = (codes.view(np.int8) >> 4).astype(np.int8)
        codes = np.stack([lo, hi], axis=-1).reshape(-1)
        fmt = Q8
    if fmt == F32:
        return codes.astype(np.float32)
    if fmt == BF16:
        return (codes.astype(np.uint32) << 16).view(np.float32)
    sc = (scales.astype(np.uint32) << 16).view(np.float32)
    per = np.repeat(sc, 32)[: codes.size]
    return (codes.astype(np.float32) * per).astype(np.float32)


class DraftKv:
    """The draft head's int8 key/value cache (src/draft_head.rs:177-220):
    codes [8][capacity][64] with one FP32 scale per 64-value row."""

    def __init__(self, capacity):
        self.capacity, self.len = capacity, 0
        self.key_codes = np.zeros(8 * capacity * 64, np.int8)
        self.value_codes = np.zeros(8 * capacity * 64, np.int8)
        self.key_scales = np.zeros(8 * capacity, np.float32)
        self.value_scales = np.zeros(8 * capacity, np.float32)

    def push(self, keys, values):
        """Rows [rows][512] of keys and values (Kv::push, draft_head.rs:194-210)."""
        keys, values = _f32(keys), _f32(values)
        rows = keys.size // 512
        assert self.len + rows <= self.capacity
        lib().fo_or_draft_push(_p(keys), _p(values), rows, self.capacity, self.len, _p(self.key_codes),
                               _p(self.key_scales), _p(self.value_codes), _p(self.value_scales))
        self.len += rows

    def attend(self, q, bases, window=0, chain_keys=None, chain_values=None):
        """attend + group_q8 (draft_head.rs:548-759): out [16][64]."""
        q = _f32(q)
        chain = 0 if chain_keys is None else _f32(chain_keys).size // 512
        ck = _f32(chain_keys) if chain else np.zeros(1, np.float32)
        cv = _f32(chain_values) if chain else np.zeros(1, np.float32)
        out = np.zeros(16 * 64, np.float32)
        lib().fo_or_draft_attend(_p(self.key_codes), _p(self.key_scales), _p(self.value_codes), _p(self.value_scales),
                                 self.capacity, _p(q), bases, window, _p(ck), _p(cv), chain, _p(out))
        return out
