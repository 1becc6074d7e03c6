"""ctypes wrapper of the CPU baseline (oracle/fo_cpu_simd.c).

BENCHMARK AND TEST INFRASTRUCTURE ONLY.  bench.py's reference arm and its
cpu_baseline leg time these functions on the host cores; tests check them
against the scalar restatement (oracle.py).  The product never imports it.

fo_cpu_simd.c restates the reference's production CPU kernels with the same
x86 vector instructions: the AVX-512 BF16 static-shift prefill tiles
(prefill64/bf16.rs, bf16/static_shift.rs) and the AVX2 verify decode over F32
split records (quant/kv/decode.rs pair_rows, kv.rs merge).
"""

from __future__ import annotations

import ctypes
import os
import platform
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
PATH = os.path.join(HERE, "_build", "libfo_cpu_simd.so")

_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(PATH):
        subprocess.run(["make", "-s", "-C", HERE], check=True)
    L = ctypes.CDLL(PATH)
    P, I64, I = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int
    sig = {
        "fo_cpu_set_threads": (None, [I]),
        "fo_cpu_max_threads": (I, []),
        "fo_cpu_has_bf16": (I, []),
        "fo_cpu_has_avx2": (I, []),
        "fo_cpu_prefill_bf16_static": (I, [P, P, P, I64, I64, I64, I64, I64, P, P]),
        "fo_cpu_decode_rows_f32": (I, [P, P, I64, I64, I64, I64, I64, P, I64, P, I64, P]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    _lib = L
    return L


def _p(a):
    return a.ctypes.data_as(ctypes.c_void_p)


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def has_bf16() -> bool:
    return bool(lib().fo_cpu_has_bf16())


def has_avx2() -> bool:
    return bool(lib().fo_cpu_has_avx2())


def set_threads(n: int) -> None:
    lib().fo_cpu_set_threads(int(n))


def max_threads() -> int:
    return int(lib().fo_cpu_max_threads())


def prefill_bf16_static(q, k, v, n_heads, n_kv_heads, image, sinks, out=None):
    """The reference's fast-mode prefill (BF16 static-shift tiles, AVX-512
    BF16) of a pure prefix; None when the host lacks AVX512-BF16."""
    q, k, v, sinks = _f32(q), _f32(k), _f32(v), _f32(sinks)
    total = q.size // (n_heads * 64)
    if out is None:
        out = np.empty(q.size, np.float32)
    st = lib().fo_cpu_prefill_bf16_static(_p(q), _p(k), _p(v), total, n_heads, n_kv_heads, image[0], image[1],
                                          _p(sinks), _p(out))
    return None if st != 0 else out


def decode_rows_f32(cache, q, rows, sinks, out=None):
    """attention_decode_rows over the F32 records of an oracle SplitCache,
    AVX2 (the reference's pair_rows); None when the host lacks AVX2/FMA."""
    assert cache.fmt == 0, "F32 records only"
    q, sinks = _f32(q), _f32(sinks)
    if out is None:
        out = np.empty(rows * cache.heads * 64, np.float32)
    st = lib().fo_cpu_decode_rows_f32(_p(cache.codes), _p(cache.tail_codes), cache.prefix_len, cache.prefix_len,
                                      cache.tail_len, cache.tail_capacity, cache.groups, _p(q), rows, _p(sinks),
                                      cache.chunks, _p(out))
    return None if st != 0 else out


def host_description() -> dict:
    """CPU model, logical and physical core counts and the vector flags the
    baseline uses (from lscpu / /proc/cpuinfo)."""
    model, flags, physical = platform.processor() or "", set(), None
    try:
        text = open("/proc/cpuinfo").read()
        for line in text.splitlines():
            if line.startswith("model name") and not model.strip(" x86_64"):
                model = line.split(":", 1)[1].strip()
            if line.startswith("flags"):
                flags = set(line.split(":", 1)[1].split())
        cores = {(blk.split("physical id")[1].split("\n")[0], blk.split("core id")[1].split("\n")[0])
                 for blk in text.split("\n\n") if "core id" in blk and "physical id" in blk}
        physical = len(cores) or None
    except (OSError, IndexError):
        pass
    try:
        lscpu = subprocess.run(["lscpu"], capture_output=True, text=True, timeout=10).stdout
        for line in lscpu.splitlines():
            if line.startswith("Model name:"):
                model = line.split(":", 1)[1].strip()
    except (OSError, subprocess.SubprocessError):
        pass
    return {"model": model, "logical": os.cpu_count(), "physical": physical,
            "flags": sorted(f for f in flags if f in ("avx2", "fma", "avx512f", "avx512bw", "avx512_bf16",
                                                       "amx_bf16"))}
