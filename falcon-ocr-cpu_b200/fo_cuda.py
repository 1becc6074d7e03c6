"""ctypes binding of libfo_cuda.so (include/fo_attention.h), mirroring the
reference's attention operator interface for tests and benchmarks:

* ``attention_with``          kernels::attention_with (src/kernels/attention/mod.rs:256-311)
* ``attention_prefill_bf16``  kernels::attention_prefill_bf16 (mod.rs:321-349)
* ``SplitPrefix``             quant::kv::SplitPrefix (src/quant/kv.rs:155-972):
  ``from_compact``, ``append``, ``truncate_tail``, ``tail_len``, ``bytes``,
  ``attention_decode``, ``attention_decode_rows``; ``decode_batch`` for pages.

Arrays may be numpy (host memory: the call copies to and from the device) or
CUDA torch tensors (device memory, read and written in place).  Shape errors
raise ``FoError`` as the reference's asserts panic; seal errors raise the
matching subclass as the reference returns an ``anyhow`` error.  There is no
CPU fallback: importing this module without the built library raises.
"""

from __future__ import annotations

import ctypes
import os
from typing import Optional, Sequence

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "lib", "libfo_cuda.so")

OK, ERR_INVALID, ERR_PAIR, ERR_NONFINITE, ERR_OVERFLOW, ERR_CAPACITY, ERR_CUDA, ERR_DECLINED = range(8)
MEM_DEVICE, MEM_HOST = 0, 1
KV_F32, KV_Q16, KV_Q8, KV_BF16, KV_Q4 = 0, 1, 2, 3, 4
KV_ROTATED = 16  # flag: blocks stored rotated (src/quant/rotation.rs); with F32, Q8, Q4
KV_Q8_ROT, KV_Q4_ROT = KV_Q8 | KV_ROTATED, KV_Q4 | KV_ROTATED  # Kv::Q8Rot, Kv::Q4Rot
KV_FORMATS = {"f32": KV_F32, "q16": KV_Q16, "q8": KV_Q8, "bf16": KV_BF16, "q4": KV_Q4, "q8r": KV_Q8_ROT,
              "q4r": KV_Q4_ROT, "f32r": KV_F32 | KV_ROTATED}
EXP_EXACT, EXP_FAST = 0, 1
SOFTMAX_ONLINE, SOFTMAX_STATIC = 0, 1


class FoError(RuntimeError):
    status = ERR_INVALID


class PairError(FoError):
    status = ERR_PAIR


class NonFiniteError(FoError):
    status = ERR_NONFINITE


class OverflowKvError(FoError):
    status = ERR_OVERFLOW


class CapacityError(FoError):
    status = ERR_CAPACITY


class CudaError(FoError):
    status = ERR_CUDA


class Declined(FoError):
    status = ERR_DECLINED


_ERRORS = {c.status: c for c in (FoError, PairError, NonFiniteError, OverflowKvError, CapacityError, CudaError,
                                  Declined)}


class Geometry(ctypes.Structure):
    """src/kernels/attention/mod.rs:35-76"""
    _fields_ = [("query_offset", ctypes.c_int64), ("image_start", ctypes.c_int64), ("image_end", ctypes.c_int64)]


class CompactKv(ctypes.Structure):
    """src/kernels/attention/mod.rs:78-97"""
    _fields_ = [("prefix_k", ctypes.c_void_p), ("generated_k", ctypes.c_void_p), ("v", ctypes.c_void_p),
                ("prefix_len", ctypes.c_int64), ("total_len", ctypes.c_int64), ("n_heads", ctypes.c_int64),
                ("n_kv_heads", ctypes.c_int64), ("head_dim", ctypes.c_int64)]


class PrefillOptions(ctypes.Structure):
    """src/kernels/attention/mod.rs:204-221"""
    _fields_ = [("exp", ctypes.c_int32), ("profile", ctypes.c_int32), ("softmax", ctypes.c_int32),
                ("fp32_softmax", ctypes.c_int32)]

    @classmethod
    def exact(cls):
        return cls(EXP_EXACT, 0, SOFTMAX_ONLINE, SOFTMAX_ONLINE)


EXPORTS = [
    "fo_version", "fo_last_error", "fo_ctx_create", "fo_ctx_destroy", "fo_ctx_synchronize", "fo_ctx_last_ms",
    "fo_attention", "fo_attention_prefill_bf16", "fo_convert_bf16", "fo_kv_seal", "fo_kv_destroy",
    "fo_kv_set_fast_exp", "fo_kv_append", "fo_kv_truncate_tail", "fo_kv_tail_len", "fo_kv_prefix_len",
    "fo_kv_bytes", "fo_kv_records", "fo_kv_attention_decode", "fo_kv_attention_decode_rows",
    "fo_kv_attention_decode_batch", "fo_kv_append_batch", "fo_qkv_prefix_rows", "fo_kv_append_qkv",
    "fo_sharded_prefill_bf16", "fo_nccl_unique_id", "fo_nccl_comm_init", "fo_nccl_comm_destroy", "fo_kv_seal_layer",
    "fo_kv_plan_create", "fo_kv_plan_step", "fo_kv_plan_finish",
    "fo_decode_rows_static_scratch", "fo_decode_static_scratch_status",
    "fo_selftest_bounded_wait",
    "fo_attention_prefill_bf16_rows", "fo_attention_prefill_bf16_rows_split", "fo_i8_seal", "fo_i8_destroy", "fo_i8_bytes", "fo_i8_records",
    "fo_i8_decode_batch", "fo_draft_kv_create", "fo_draft_kv_destroy", "fo_draft_kv_push", "fo_draft_kv_len",
    "fo_draft_kv_bytes", "fo_draft_kv_records", "fo_draft_attend", "fo_peer_block_register",
    "fo_peer_block_destroy", "fo_sharded_prefill_bf16_peers",
]

_lib: Optional[ctypes.CDLL] = None


def lib() -> ctypes.CDLL:
    """The loaded library; raises if it was not built (no fallback exists)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise ImportError(f"{LIB_PATH} is missing: run `python falcon-ocr-cpu_b200/build.py` (no CPU fallback)")
    L = ctypes.CDLL(LIB_PATH)
    P, I32, I64, I = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64, ctypes.c_int
    PP = ctypes.POINTER(ctypes.c_void_p)
    sigs = {
        "fo_version": (I, []),
        "fo_last_error": (ctypes.c_char_p, []),
        "fo_ctx_create": (I, [I, P, ctypes.POINTER(P)]),
        "fo_ctx_destroy": (I, [P]),
        "fo_ctx_synchronize": (I, [P]),
        "fo_ctx_last_ms": (I, [P, ctypes.POINTER(ctypes.c_float)]),
        "fo_attention": (I, [P, P, ctypes.POINTER(CompactKv), I64, Geometry, P, P, PrefillOptions, I]),
        "fo_attention_prefill_bf16": (I, [P, P, ctypes.POINTER(CompactKv), I64, Geometry, P, P, P, P,
                                          PrefillOptions, I]),
        "fo_convert_bf16": (I, [P, P, P, I64]),
        "fo_kv_seal": (I, [P, P, P, I64, I64, I64, I64, I64, I32, I32, I, ctypes.POINTER(P)]),
        "fo_kv_destroy": (I, [P]),
        "fo_kv_set_fast_exp": (I, [P, I32]),
        "fo_kv_append": (I, [P, P, P, I64, I]),
        "fo_kv_truncate_tail": (I, [P, I64]),
        "fo_kv_tail_len": (I64, [P]),
        "fo_kv_prefix_len": (I64, [P]),
        "fo_kv_bytes": (I64, [P]),
        "fo_kv_records": (I, [P, PP, PP, PP, PP, ctypes.POINTER(I64), ctypes.POINTER(I64)]),
        "fo_kv_attention_decode": (I, [P, P, I64, P, P, I]),
        "fo_kv_attention_decode_rows": (I, [P, P, I64, P, P, I]),
        "fo_kv_attention_decode_batch": (I, [PP, I64, PP, PP, PP]),
        "fo_kv_append_batch": (I, [PP, I64, PP, PP, I64]),
        "fo_qkv_prefix_rows": (I, [P, P, P, I64, I64, I64, P, P, P, P, P]),
        "fo_kv_append_qkv": (I, [P, P, P, I64, P]),
        "fo_sharded_prefill_bf16": (I, [P, P, I32, I32, P, P, P, I64, I64, I64, Geometry, P, PrefillOptions, I32,
                                        I32, P]),
        "fo_nccl_unique_id": (I, [P]),
        "fo_nccl_comm_init": (I, [P, I32, I32, P, ctypes.POINTER(P)]),
        "fo_nccl_comm_destroy": (I, [P]),
        "fo_kv_plan_create": (I, [PP, I64, PP, PP, PP, PP, PP, ctypes.POINTER(P)]),
        "fo_kv_plan_step": (I, [P]),
        "fo_kv_plan_finish": (I, [P]),
        "fo_kv_seal_layer": (I, [P, I32, ctypes.c_uint64, I32, I32, I32, P, P, I64, I64, I64, I64, I64, I32,
                                 ctypes.POINTER(P)]),
        "fo_decode_rows_static_scratch": (I, [P, P, P, P, I32, I64, I64, I64, I64, I64, I64, P, I64, P, I32, P, P]),
        "fo_decode_static_scratch_status": (I, [P]),
        "fo_selftest_bounded_wait": (I, [P, ctypes.c_uint64]),
        "fo_attention_prefill_bf16_rows": (I, [P, P, P, P, I64, I64, I64, Geometry, P, P, I64, I64, PrefillOptions]),
        "fo_attention_prefill_bf16_rows_split": (I, [P, P, P, P, I64, I64, I64, Geometry, P, P, I32, I64, I64,
                                                     PrefillOptions, I]),
        "fo_i8_seal": (I, [P, P, P, I64, I64, I, ctypes.POINTER(P)]),
        "fo_i8_destroy": (I, [P]),
        "fo_i8_bytes": (I64, [P]),
        "fo_i8_records": (I, [P, PP, PP, PP, PP]),
        "fo_i8_decode_batch": (I, [PP, I64, PP, PP, PP, I32]),
        "fo_draft_kv_create": (I, [P, I64, ctypes.POINTER(P)]),
        "fo_draft_kv_destroy": (I, [P]),
        "fo_draft_kv_push": (I, [P, P, P, I64, I]),
        "fo_draft_kv_len": (I64, [P]),
        "fo_draft_kv_bytes": (I64, [P]),
        "fo_draft_kv_records": (I, [P, PP, PP, PP, PP]),
        "fo_draft_attend": (I, [P, P, I64, I64, P, P, I64, P, I]),
        "fo_peer_block_register": (I, [P, P, I32, I32, P, I64, ctypes.POINTER(P)]),
        "fo_peer_block_destroy": (I, [P]),
        "fo_sharded_prefill_bf16_peers": (I, [P, P, P, P, P, I64, I64, I64, Geometry, P, PrefillOptions, I32]),
    }
    for name, (res, args) in sigs.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    _lib = L
    return L


def check(status: int) -> None:
    if status != OK:
        msg = lib().fo_last_error().decode(errors="replace")
        raise _ERRORS.get(status, FoError)(f"fo status {status}: {msg}")


def _is_torch(x) -> bool:
    return type(x).__module__.startswith("torch")


def _on_device(a) -> bool:
    return _is_torch(a) and a.is_cuda


def _ptr_mem(arrays):
    """Pointers of a call's arrays and its memory mode: all host (numpy
    arrays or CPU torch tensors, e.g. pinned) or all device (CUDA tensors)."""
    kinds = {_on_device(a) for a in arrays if a is not None}
    if len(kinds) > 1:
        raise FoError("mix of host and device arrays in one call")
    device = kinds == {True}
    ptrs = []
    for a in arrays:
        if a is None:
            ptrs.append(None)
        elif _is_torch(a):
            if not a.is_contiguous():
                raise FoError("arrays must be contiguous")
            ptrs.append(a.data_ptr())
        else:
            if not (a.flags["C_CONTIGUOUS"]):
                raise FoError("host arrays must be C-contiguous")
            ptrs.append(a.ctypes.data)
    return ptrs, (MEM_DEVICE if device else MEM_HOST)


def _f32(a):
    if a is None or _is_torch(a):
        return a
    return np.ascontiguousarray(a, dtype=np.float32)


class Context:
    """A device and a stream (fo_ctx)."""

    def __init__(self, device: int = 0, stream: Optional[int] = None):
        h = ctypes.c_void_p()
        check(lib().fo_ctx_create(device, stream, ctypes.byref(h)))
        self.handle = h
        self.device = device

    def close(self):
        if self.handle:
            lib().fo_ctx_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def synchronize(self):
        check(lib().fo_ctx_synchronize(self.handle))

    def last_ms(self) -> float:
        v = ctypes.c_float()
        check(lib().fo_ctx_last_ms(self.handle, ctypes.byref(v)))
        return v.value

    def selftest_bounded_wait(self, limit_ns: int) -> int:
        """fo_selftest_bounded_wait: the raw status (FO_ERR_CUDA when the
        device wait gave up after limit_ns, as designed)."""
        return lib().fo_selftest_bounded_wait(self.handle, limit_ns)


_default: Optional[Context] = None


def default_context() -> Context:
    global _default
    if _default is None:
        _default = Context(0)
    return _default


def attention_with(q, prefix_k, v, query_len, geometry, sinks, output, n_heads, n_kv_heads, head_dim,
                   generated_k=None, prefix_len=None, total_len=None, options=None, ctx=None):
    """kernels::attention_with: `output` is overwritten."""
    ctx = ctx or default_context()
    q, prefix_k, v, sinks, generated_k = _f32(q), _f32(prefix_k), _f32(v), _f32(sinks), _f32(generated_k)
    (pq, ppk, pgk, pv, ps, po), mem = _ptr_mem([q, prefix_k, generated_k, v, sinks, output])
    if prefix_len is None:
        prefix_len = prefix_k.numel() // (n_heads * head_dim) if _is_torch(prefix_k) else prefix_k.size // (
            n_heads * head_dim)
    if total_len is None:
        total_len = (v.numel() if _is_torch(v) else v.size) // (n_kv_heads * head_dim)
    kv = CompactKv(ppk, pgk, pv, prefix_len, total_len, n_heads, n_kv_heads, head_dim)
    g = Geometry(*geometry)
    check(lib().fo_attention(ctx.handle, pq, ctypes.byref(kv), query_len, g, ps, po, options or PrefillOptions.exact(),
                             mem))
    return output


def attention_prefill_bf16(q, k, v, geometry, sinks, output, n_heads, n_kv_heads, keys_bf16=None, values_bf16=None,
                           options=None, ctx=None):
    """kernels::attention_prefill_bf16 over a pure prefix; raises Declined for other shapes."""
    ctx = ctx or default_context()
    q, k, v, sinks = _f32(q), _f32(k), _f32(v), _f32(sinks)
    (pq, pk, pv, ps, po), mem = _ptr_mem([q, k, v, sinks, output])
    total = (q.numel() if _is_torch(q) else q.size) // (n_heads * 64)
    kv = CompactKv(pk, None, pv, total, total, n_heads, n_kv_heads, 64)
    kb = keys_bf16.data_ptr() if keys_bf16 is not None else None
    vb = values_bf16.data_ptr() if values_bf16 is not None else None
    if options is None:
        options = PrefillOptions(EXP_FAST, 0, SOFTMAX_STATIC, SOFTMAX_ONLINE)
    check(lib().fo_attention_prefill_bf16(ctx.handle, pq, ctypes.byref(kv), total, Geometry(*geometry), ps, po, kb, vb,
                                          options, mem))
    return output


def attention_prefill_bf16_rows(q, keys_bf16, values_bf16, geometry, sinks, output, n_heads, n_kv_heads, query_begin,
                                query_end, options=None, ctx=None, kv_splits=1):
    """fo_attention_prefill_bf16_rows: the BF16 prefill of query rows
    [query_begin, query_end) of a pure prefix (CUDA tensors; BF16 keys and
    values already converted).  Rows outside the range are left as they are.
    kv_splits > 1 cuts each query pair's keys into that many ranges, and a
    BF16 `output` takes the rounded result directly
    (fo_attention_prefill_bf16_rows_split)."""
    ctx = ctx or default_context()
    for a in (q, keys_bf16, values_bf16, sinks, output):
        if not _on_device(a) or not a.is_contiguous():
            raise FoError("fo_attention_prefill_bf16_rows takes contiguous CUDA tensors")
    total = q.numel() // (n_heads * 64)
    if options is None:
        options = PrefillOptions(EXP_FAST, 0, SOFTMAX_STATIC, SOFTMAX_ONLINE)
    out_bf16 = 1 if str(output.dtype) == "torch.bfloat16" else 0
    if kv_splits == 1 and not out_bf16:
        check(lib().fo_attention_prefill_bf16_rows(ctx.handle, q.data_ptr(), keys_bf16.data_ptr(),
                                                   values_bf16.data_ptr(), total, n_heads, n_kv_heads,
                                                   Geometry(*geometry), sinks.data_ptr(), output.data_ptr(),
                                                   query_begin, query_end, options))
    else:
        check(lib().fo_attention_prefill_bf16_rows_split(ctx.handle, q.data_ptr(), keys_bf16.data_ptr(),
                                                         values_bf16.data_ptr(), total, n_heads, n_kv_heads,
                                                         Geometry(*geometry), sinks.data_ptr(), output.data_ptr(),
                                                         out_bf16, query_begin, query_end, options, kv_splits))
    return output


class SplitPrefix:
    """quant::kv::SplitPrefix on the device (src/quant/kv.rs:155-972)."""

    def __init__(self, handle, ctx, heads):
        self.handle = handle
        self.ctx = ctx
        self.heads = heads

    @classmethod
    def from_compact(cls, k, v, prefix_len, capacity, fmt="f32", heads=16, kv_heads=8, head_dim=64, chunks=0,
                     ctx=None):
        ctx = ctx or default_context()
        fmt = KV_FORMATS[fmt] if isinstance(fmt, str) else fmt
        k, v = _f32(k), _f32(v)
        (pk, pv), mem = _ptr_mem([k, v])
        h = ctypes.c_void_p()
        check(lib().fo_kv_seal(ctx.handle, pk, pv, prefix_len, capacity, heads, kv_heads, head_dim, fmt, chunks, mem,
                               ctypes.byref(h)))
        return cls(h, ctx, heads)

    @classmethod
    def seal_layer(cls, layer, k, v, filled, prefix_len, capacity, mode="bf16", kv_q8_layers=0, fast_exps=False,
                   decode_fast_exp=None, heads=16, kv_heads=8, chunks=0, ctx=None):
        """fo_kv_seal_layer (model::cache::seal_layer, src/model/cache.rs:218-276)
        on device tensors k, v: Q8 records where bit `layer` of kv_q8_layers is
        set, `mode` otherwise."""
        ctx = ctx or default_context()
        mode = KV_FORMATS[mode] if isinstance(mode, str) else mode
        req = -1 if decode_fast_exp is None else int(bool(decode_fast_exp))
        h = ctypes.c_void_p()
        check(lib().fo_kv_seal_layer(ctx.handle, layer, kv_q8_layers, mode, int(bool(fast_exps)), req, k.data_ptr(),
                                     v.data_ptr(), filled, prefix_len, capacity, heads, kv_heads, chunks,
                                     ctypes.byref(h)))
        return cls(h, ctx, heads)

    def close(self):
        if self.handle:
            lib().fo_kv_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def with_fast_exp(self, fast: bool = True) -> "SplitPrefix":
        check(lib().fo_kv_set_fast_exp(self.handle, int(bool(fast))))
        return self

    def append(self, k, v):
        k, v = _f32(k), _f32(v)
        (pk, pv), mem = _ptr_mem([k, v])
        n = (k.numel() if _is_torch(k) else k.size) // (self.heads * 64)
        check(lib().fo_kv_append(self.handle, pk, pv, n, mem))

    def truncate_tail(self, tail_len: int):
        check(lib().fo_kv_truncate_tail(self.handle, tail_len))

    @property
    def tail_len(self) -> int:
        return int(lib().fo_kv_tail_len(self.handle))

    @property
    def prefix_len(self) -> int:
        return int(lib().fo_kv_prefix_len(self.handle))

    def bytes(self) -> int:
        return int(lib().fo_kv_bytes(self.handle))

    def records(self):
        """(codes, scales, tail_codes, tail_scales) device pointers and strides."""
        ptrs = [ctypes.c_void_p() for _ in range(4)]
        ps, ts = ctypes.c_int64(), ctypes.c_int64()
        check(lib().fo_kv_records(self.handle, *[ctypes.byref(p) for p in ptrs], ctypes.byref(ps), ctypes.byref(ts)))
        return [p.value for p in ptrs], ps.value, ts.value

    def attention_decode(self, q, total_len, sinks, output):
        q, sinks = _f32(q), _f32(sinks)
        (pq, ps, po), mem = _ptr_mem([q, sinks, output])
        check(lib().fo_kv_attention_decode(self.handle, pq, total_len, ps, po, mem))
        return output

    def attention_decode_rows(self, q, rows, sinks, output):
        q, sinks = _f32(q), _f32(sinks)
        (pq, ps, po), mem = _ptr_mem([q, sinks, output])
        check(lib().fo_kv_attention_decode_rows(self.handle, pq, rows, ps, po, mem))
        return output


def decode_batch(caches: Sequence[SplitPrefix], qs, sinks, outputs):
    """One single-row decode per page in one launch (device tensors)."""
    n = len(caches)
    arr = lambda xs: (ctypes.c_void_p * n)(*xs)  # noqa: E731
    check(lib().fo_kv_attention_decode_batch(arr([c.handle.value for c in caches]), n, arr([q.data_ptr() for q in qs]),
                                             arr([s.data_ptr() for s in sinks]),
                                             arr([o.data_ptr() for o in outputs])))


def append_batch(caches: Sequence[SplitPrefix], ks, vs, rows: int):
    """fo_kv_append_batch: `rows` expanded rows into each cache in one launch
    (device tensors ks[i], vs[i] of [rows][heads][64])."""
    n = len(caches)
    arr = lambda xs: (ctypes.c_void_p * n)(*xs)  # noqa: E731
    check(lib().fo_kv_append_batch(arr([c.handle.value for c in caches]), n, arr([k.data_ptr() for k in ks]),
                                   arr([v.data_ptr() for v in vs]), rows))


def qkv_prefix_rows(qkv, rope, rows: int, q, k, v, k_bf16=None, v_bf16=None, heads: int = 16, kv_heads: int = 8,
                    ctx=None):
    """fo_qkv_prefix_rows on device tensors: the fused split + per-head RMS
    norm + RoPE of projection rows into q, k (and their BF16 copies)."""
    ctx = ctx or default_context()
    ptr = lambda t: None if t is None else t.data_ptr()  # noqa: E731
    check(lib().fo_qkv_prefix_rows(ctx.handle, qkv.data_ptr(), rope.data_ptr(), rows, heads, kv_heads, q.data_ptr(),
                                   k.data_ptr(), v.data_ptr(), ptr(k_bf16), ptr(v_bf16)))


def append_qkv(cache: SplitPrefix, qkv, rope, rows: int, q):
    """fo_kv_append_qkv on device tensors: decode rows' queries into q, their
    keys and values appended to the cache's tail."""
    check(lib().fo_kv_append_qkv(cache.handle, qkv.data_ptr(), rope.data_ptr(), rows, q.data_ptr()))


class BatchPlan:
    """fo_kv_plan_*: the append of one row and the one-row decode of every
    cache as one device-resident step (graph-capturable).  ks, vs, qs, sinks
    and outs are device tensors the plan reads and writes at every step."""

    def __init__(self, caches, ks, vs, qs, sinks, outs):
        n = len(caches)
        arr = lambda xs: (ctypes.c_void_p * n)(*xs)  # noqa: E731
        h = ctypes.c_void_p()
        check(lib().fo_kv_plan_create(arr([c.handle.value for c in caches]), n, arr([t.data_ptr() for t in ks]),
                                      arr([t.data_ptr() for t in vs]), arr([t.data_ptr() for t in qs]),
                                      arr([t.data_ptr() for t in sinks]), arr([t.data_ptr() for t in outs]),
                                      ctypes.byref(h)))
        self.handle = h
        self._keep = (ks, vs, qs, sinks, outs)

    def step(self):
        check(lib().fo_kv_plan_step(self.handle))

    def finish(self):
        if self.handle:
            h, self.handle = self.handle, None
            check(lib().fo_kv_plan_finish(h))


class NcclComm:
    """An NCCL communicator from the library's NCCL (fo_nccl_comm_init); rank 0
    makes the id with nccl_unique_id() and the caller shares it."""

    def __init__(self, world: int, rank: int, uid: bytes, ctx=None):
        ctx = ctx or default_context()
        if len(uid) != 128:
            raise FoError("an NCCL unique id is 128 bytes")
        buf = (ctypes.c_uint8 * 128).from_buffer_copy(uid)
        h = ctypes.c_void_p()
        check(lib().fo_nccl_comm_init(ctx.handle, world, rank, buf, ctypes.byref(h)))
        self.handle, self.world, self.rank = h, world, rank

    def close(self):
        if self.handle:
            check(lib().fo_nccl_comm_destroy(self.handle))
            self.handle = None


def nccl_unique_id() -> bytes:
    buf = (ctypes.c_uint8 * 128)()
    check(lib().fo_nccl_unique_id(buf))
    return bytes(buf)


def sharded_prefill_bf16(comm: NcclComm, q, keys_bf16, values_bf16, geometry, sinks, gathered, n_heads, n_kv_heads,
                         n_bands=1, kv_splits=0, options=None, ctx=None):
    """fo_sharded_prefill_bf16 on this rank's heads (contiguous CUDA tensors);
    `gathered` BF16 holds the bands' rank-major blocks one after another."""
    ctx = ctx or default_context()
    total = q.numel() // (n_heads * 64)
    if options is None:
        options = PrefillOptions(EXP_FAST, 0, SOFTMAX_STATIC, SOFTMAX_ONLINE)
    check(lib().fo_sharded_prefill_bf16(ctx.handle, comm.handle, comm.rank, comm.world, q.data_ptr(),
                                        keys_bf16.data_ptr(), values_bf16.data_ptr(), total, n_heads, n_kv_heads,
                                        Geometry(*geometry), sinks.data_ptr(), options, n_bands, kv_splits,
                                        gathered.data_ptr()))
    return gathered


class DraftKv:
    """The draft head's int8 key/value cache on the device (fo_draft_kv_*:
    DraftState's Kv::Q8 and attend, src/draft_head.rs:177-220, 548-759)."""

    def __init__(self, capacity, ctx=None):
        ctx = ctx or default_context()
        h = ctypes.c_void_p()
        check(lib().fo_draft_kv_create(ctx.handle, capacity, ctypes.byref(h)))
        self.handle, self.capacity, self.ctx = h, capacity, ctx

    @property
    def len(self) -> int:
        return lib().fo_draft_kv_len(self.handle)

    def push(self, keys, values):
        """Rows [rows][512] of keys and values (numpy: host; CUDA tensors: device)."""
        keys, values = _f32(keys), _f32(values)
        (pk, pv), mem = _ptr_mem([keys, values])
        n = keys.numel() if _is_torch(keys) else keys.size
        check(lib().fo_draft_kv_push(self.handle, pk, pv, n // 512, mem))

    def attend(self, q, bases, output, window=0, chain_keys=None, chain_values=None):
        """Attention of q [16][64] over the verified rows (the newest `window`
        of the first `bases`; 0: all) and the chain rows [chain][512]."""
        chain = 0
        if chain_keys is not None:
            chain = (chain_keys.numel() if _is_torch(chain_keys) else np.asarray(chain_keys).size) // 512
        q = _f32(q)
        ck = _f32(chain_keys) if chain else None
        cv = _f32(chain_values) if chain else None
        (pq, pk, pv, po), mem = _ptr_mem([q, ck, cv, output])
        check(lib().fo_draft_attend(self.handle, pq, bases, window, pk, pv, chain, po, mem))
        return output

    def records(self):
        """Device pointers (key_codes, key_scales, value_codes, value_scales)."""
        ptrs = [ctypes.c_void_p() for _ in range(4)]
        check(lib().fo_draft_kv_records(self.handle, *[ctypes.byref(p) for p in ptrs]))
        return tuple(p.value for p in ptrs)

    def close(self):
        if self.handle:
            lib().fo_draft_kv_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class PeerBlock:
    """fo_peer_block_register: every rank's gathered buffer mapped into this
    process (collective over the communicator's ranks)."""

    def __init__(self, comm: "NcclComm", gathered, ctx=None):
        ctx = ctx or default_context()
        h = ctypes.c_void_p()
        nbytes = gathered.numel() * gathered.element_size()
        check(lib().fo_peer_block_register(ctx.handle, comm.handle, comm.rank, comm.world, gathered.data_ptr(), nbytes,
                                           ctypes.byref(h)))
        self.handle, self.gathered = h, gathered

    def close(self):
        if self.handle:
            lib().fo_peer_block_destroy(self.handle)
            self.handle = None


def sharded_prefill_bf16_peers(block: PeerBlock, q, keys_bf16, values_bf16, geometry, sinks, n_heads, n_kv_heads,
                               kv_splits=0, options=None, ctx=None):
    """fo_sharded_prefill_bf16_peers: this rank's heads, every finished row
    stored by the kernels into all ranks' registered blocks."""
    ctx = ctx or default_context()
    total = q.numel() // (n_heads * 64)
    if options is None:
        options = PrefillOptions(EXP_FAST, 0, SOFTMAX_STATIC, SOFTMAX_ONLINE)
    check(lib().fo_sharded_prefill_bf16_peers(ctx.handle, block.handle, q.data_ptr(), keys_bf16.data_ptr(),
                                              values_bf16.data_ptr(), total, n_heads, n_kv_heads, Geometry(*geometry),
                                              sinks.data_ptr(), options, kv_splits))
    return block.gathered


class Int8Cache:
    """BASELINE config 4's INT8 KV format on the device (fo_i8_seal): keys
    and values [len][heads][64] quantized per (head, 64-position group)."""

    def __init__(self, k, v, heads=16, ctx=None):
        ctx = ctx or default_context()
        k, v = _f32(k), _f32(v)
        (pk, pv), mem = _ptr_mem([k, v])
        n = k.numel() if _is_torch(k) else k.size
        self.len, self.heads, self.ctx = n // (heads * 64), heads, ctx
        h = ctypes.c_void_p()
        check(lib().fo_i8_seal(ctx.handle, pk, pv, self.len, heads, mem, ctypes.byref(h)))
        self.handle = h

    def bytes(self) -> int:
        return lib().fo_i8_bytes(self.handle)

    def records(self):
        """Device pointers (k_codes, k_scales, v_codes, v_scales)."""
        ptrs = [ctypes.c_void_p() for _ in range(4)]
        check(lib().fo_i8_records(self.handle, *[ctypes.byref(p) for p in ptrs]))
        return tuple(p.value for p in ptrs)

    def close(self):
        if self.handle:
            lib().fo_i8_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def int8_decode_batch(caches: Sequence[Int8Cache], qs, sinks, outputs, fast_exp=False):
    """One decode row per page in one launch (CUDA tensors)."""
    n = len(caches)
    arr = lambda xs: (ctypes.c_void_p * n)(*xs)  # noqa: E731
    check(lib().fo_i8_decode_batch(arr([c.handle.value for c in caches]), n, arr([q.data_ptr() for q in qs]),
                                   arr([s.data_ptr() for s in sinks]), arr([o.data_ptr() for o in outputs]),
                                   int(bool(fast_exp))))


def decode_rows_static_scratch(cache: SplitPrefix, fmt, q, rows, sinks, output, fast_exp=False, stream=None):
    """fo_decode_rows_static_scratch over a sealed cache's records: the decode
    for callers that cannot allocate device memory (q, sinks and output are
    CUDA tensors; the partials live in the library's static array)."""
    fmt = KV_FORMATS[fmt] if isinstance(fmt, str) else fmt
    (codes, scales, tcodes, tscales), ps, ts = cache.records()
    check(lib().fo_decode_rows_static_scratch(codes, scales, tcodes, tscales, fmt, cache.prefix_len, ps,
                                              cache.tail_len, ts, cache.heads, cache.heads // 2, q.data_ptr(), rows,
                                              sinks.data_ptr(), int(bool(fast_exp)), output.data_ptr(), stream))
    return output


def static_scratch_status(stream=None):
    """fo_decode_static_scratch_status: raises CudaError if a bounded device
    wait of a static-scratch decode gave up since the last check."""
    check(lib().fo_decode_static_scratch_status(stream))


class _DeviceArray:
    """A raw device pointer as a CUDA array (__cuda_array_interface__)."""

    def __init__(self, ptr, n, dtype):
        self.__cuda_array_interface__ = {"shape": (n,), "typestr": np.dtype(dtype).str, "data": (ptr, False),
                                         "version": 3, "strides": None}


def device_to_host(ptr, n, dtype):
    """n elements of device memory at `ptr` (e.g. from SplitPrefix.records)
    copied to a numpy array through torch (tests and tooling)."""
    import torch
    torch.cuda.synchronize()
    return torch.as_tensor(_DeviceArray(ptr, n, dtype), device="cuda").cpu().numpy().copy()
