"""The C ABI on CPU: libfo_cuda.so loads, exports every entry point that
include/fo_attention.h declares, and validates shapes with the reference's
rules before touching the GPU (no compute calls here)."""

import ctypes
import os
import re

import numpy as np
import pytest

import fo_cuda as F

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "fo_attention.h")


def declared():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"^\s*(?:const\s+)?(?:int|int64_t|char)\s*\*?\s*(fo_[a-z0-9_]+)\(", text, re.M)))


def test_library_exports_every_declared_entry_point():
    names = declared()
    assert len(names) >= 20
    lib = F.lib()
    for name in names:
        assert hasattr(lib, name), name
    assert set(names) == set(F.EXPORTS)
    assert lib.fo_version() == 100


def test_library_is_built_for_sm100a():
    # The cubin's target is recorded in the ELF; cuobjdump --list-elf only prints names.
    import subprocess
    out = subprocess.run(["cuobjdump", "--list-elf", F.LIB_PATH], capture_output=True, text=True)
    assert out.returncode == 0 and "sm_100a" in out.stdout


def kv(prefix_len=8, total_len=8, heads=2, kv_heads=1, dim=64, null=False):
    a = np.zeros(max(total_len, 1) * heads * dim, np.float32)
    p = None if null else a.ctypes.data
    return F.CompactKv(p, p, p, prefix_len, total_len, heads, kv_heads, dim), a


def call_attention(q_len, kvs, geometry, ctx=None):
    q = np.zeros(max(q_len, 1) * 2 * 64, np.float32)
    s = np.zeros(2, np.float32)
    return F.lib().fo_attention(ctx, q.ctypes.data, ctypes.byref(kvs), q_len, F.Geometry(*geometry), s.ctypes.data,
                                q.ctypes.data, F.PrefillOptions.exact(), F.MEM_HOST)


def last_error():
    return F.lib().fo_last_error().decode()


@pytest.mark.parametrize("mutate,message", [
    (dict(heads=0), "head dimensions must be positive"),
    (dict(heads=3, kv_heads=2), "GQA grouping"),
    (dict(prefix_len=9, total_len=8), "prefix length"),
])
def test_compact_shape_asserts(mutate, message):
    """CompactKv::validate (src/kernels/attention/mod.rs:159-195)."""
    kvs, _keep = kv(**mutate)
    assert call_attention(4, kvs, (0, 0, 0)) == F.ERR_INVALID
    assert message in last_error()


def test_geometry_asserts():
    kvs, _keep = kv()
    assert call_attention(4, kvs, (0, 2, 9)) == F.ERR_INVALID
    assert "image must be inside the prefix" in last_error()
    assert call_attention(4, kvs, (5, 0, 0)) == F.ERR_INVALID
    assert "query interval" in last_error()
    kvs, _keep = kv(null=True)
    assert call_attention(4, kvs, (0, 0, 0)) == F.ERR_INVALID
    assert "pointer is null" in last_error()
    # A valid shape reaches the context check.
    kvs, _keep = kv()
    assert call_attention(4, kvs, (0, 0, 0)) == F.ERR_INVALID
    assert last_error() == "null context"


def test_bf16_prefill_declines_shapes_outside_its_scope():
    """attention_prefill_bf16 returns false for mixed caches, offsets, short
    queries and other head widths (src/kernels/attention/mod.rs:333-349)."""
    q = np.zeros(8 * 2 * 64, np.float32)
    s = np.zeros(2, np.float32)
    for (ql, pl, tl, off, dim) in [(3, 3, 3, 0, 64), (8, 8, 8, 0, 32), (4, 8, 8, 4, 64), (8, 4, 8, 0, 64)]:
        kvs, _keep = kv(prefix_len=pl, total_len=tl, dim=dim)
        st = F.lib().fo_attention_prefill_bf16(None, q.ctypes.data, ctypes.byref(kvs), ql, F.Geometry(off, 0, 0),
                                               s.ctypes.data, q.ctypes.data, None, None, F.PrefillOptions.exact(),
                                               F.MEM_HOST)
        assert st == F.ERR_DECLINED, (ql, pl, tl, off, dim)


def test_seal_argument_errors():
    """SplitPrefix::seal's ensure! checks (src/quant/kv.rs:248-263)."""
    k = np.zeros(16 * 64, np.float32)
    v = np.zeros(8 * 64, np.float32)
    out = ctypes.c_void_p()
    seal = F.lib().fo_kv_seal
    assert seal(None, k.ctypes.data, v.ctypes.data, 1, 2, 16, 8, 32, 0, 0, F.MEM_HOST, ctypes.byref(out)) \
        == F.ERR_INVALID
    assert "paired GQA heads" in last_error()
    assert seal(None, k.ctypes.data, v.ctypes.data, 1, 2, 16, 4, 64, 0, 0, F.MEM_HOST, ctypes.byref(out)) \
        == F.ERR_INVALID
    assert seal(None, k.ctypes.data, v.ctypes.data, 0, 2, 16, 8, 64, 0, 0, F.MEM_HOST, ctypes.byref(out)) \
        == F.ERR_CAPACITY
    assert seal(None, k.ctypes.data, v.ctypes.data, 2, 1, 16, 8, 64, 0, 0, F.MEM_HOST, ctypes.byref(out)) \
        == F.ERR_CAPACITY
    assert seal(None, k.ctypes.data, v.ctypes.data, 1, 2, 16, 8, 64, 9, 0, F.MEM_HOST, ctypes.byref(out)) \
        == F.ERR_INVALID
    assert seal(None, k.ctypes.data, v.ctypes.data, 1, 2, 16, 8, 64, 0, 0, F.MEM_HOST, ctypes.byref(out)) \
        == F.ERR_INVALID
    assert last_error() == "null context"


def test_null_handles_are_rejected():
    L = F.lib()
    assert L.fo_kv_truncate_tail(None, 0) == F.ERR_INVALID
    assert L.fo_kv_append(None, None, None, 1, F.MEM_HOST) == F.ERR_INVALID
    assert L.fo_kv_attention_decode_rows(None, None, 1, None, None, F.MEM_HOST) == F.ERR_INVALID
    assert L.fo_kv_tail_len(None) == -1 and L.fo_kv_bytes(None) == -1
    assert L.fo_ctx_destroy(None) == F.OK and L.fo_kv_destroy(None) == F.OK
    assert L.fo_selftest_bounded_wait(None, 1000) == F.ERR_INVALID
    assert L.fo_i8_seal(None, None, None, 1, 16, F.MEM_HOST, ctypes.byref(ctypes.c_void_p())) == F.ERR_INVALID
    assert L.fo_i8_decode_batch(None, 1, None, None, None, 0) == F.ERR_INVALID
    assert L.fo_i8_bytes(None) == -1 and L.fo_i8_destroy(None) == F.OK
    assert L.fo_draft_kv_create(None, 8, ctypes.byref(ctypes.c_void_p())) == F.ERR_INVALID
    assert L.fo_draft_kv_push(None, None, None, 1, F.MEM_HOST) == F.ERR_INVALID
    assert L.fo_draft_attend(None, None, 1, 0, None, None, 0, None, F.MEM_HOST) == F.ERR_INVALID
    assert L.fo_draft_kv_len(None) == -1 and L.fo_draft_kv_destroy(None) == F.OK
    assert L.fo_peer_block_register(None, None, 0, 2, None, 16, ctypes.byref(ctypes.c_void_p())) == F.ERR_INVALID
    assert L.fo_peer_block_destroy(None) == F.OK
    opts = F.PrefillOptions(F.EXP_FAST, 0, F.SOFTMAX_STATIC, F.SOFTMAX_ONLINE)
    assert L.fo_sharded_prefill_bf16_peers(None, None, None, None, None, 4096, 2, 1, F.Geometry(0, 0, 0), None, opts,
                                           0) == F.ERR_INVALID
    h = ctypes.c_void_p()
    assert L.fo_ctx_create(-1, None, ctypes.byref(h)) != F.OK


def test_batched_and_fused_entries_reject_bad_arguments():
    """fo_kv_append_batch, fo_qkv_prefix_rows and fo_kv_append_qkv refuse
    null handles and bad shapes before touching a device."""
    L = F.lib()
    arr = (ctypes.c_void_p * 1)(None)
    assert L.fo_kv_append_batch(None, 1, arr, arr, 1) == F.ERR_INVALID
    assert L.fo_kv_append_batch(arr, 1, arr, arr, 1) == F.ERR_INVALID  # a null cache
    assert L.fo_kv_append_batch(arr, -1, arr, arr, 1) == F.ERR_INVALID
    assert L.fo_kv_append_batch(arr, 0, arr, arr, 1) == F.OK  # nothing to do
    assert L.fo_qkv_prefix_rows(None, None, None, 4, 16, 8, None, None, None, None, None) == F.ERR_INVALID
    assert L.fo_kv_append_qkv(None, None, None, 1, None) == F.ERR_INVALID
    assert L.fo_kv_append_qkv(None, None, None, -1, None) == F.ERR_INVALID
    out = ctypes.c_void_p()
    seal = L.fo_kv_seal_layer
    assert seal(None, 0, 0, F.KV_BF16, 0, -1, None, None, 8, 8, 9, 16, 8, 0, None) == F.ERR_INVALID
    assert seal(None, 0, 0, 7, 0, -1, None, None, 8, 8, 9, 16, 8, 0, ctypes.byref(out)) == F.ERR_INVALID
    # rotation only with F32, Q8 or Q4 records (Storage, kv.rs:128-152)
    for mode in (F.KV_BF16 | F.KV_ROTATED, F.KV_Q16 | F.KV_ROTATED, 32):
        assert seal(None, 0, 0, mode, 0, -1, None, None, 8, 8, 9, 16, 8, 0, ctypes.byref(out)) == F.ERR_INVALID
        assert "unknown mode" in last_error()
    assert seal(None, 0, 0, F.KV_BF16, 0, -1, None, None, 7, 8, 9, 16, 8, 0, ctypes.byref(out)) == F.ERR_INVALID
    assert "complete prefix" in last_error()
    assert seal(None, -1, 0, F.KV_BF16, 0, -1, None, None, 8, 8, 9, 16, 8, 0, ctypes.byref(out)) == F.ERR_INVALID


def test_row_band_entries_reject_a_null_context():
    """The row-band prefill entries (whole and split) refuse a null context
    before touching a device, whatever the number of key ranges."""
    L = F.lib()
    opts = F.PrefillOptions(F.EXP_FAST, 0, F.SOFTMAX_STATIC, F.SOFTMAX_ONLINE)
    g = F.Geometry(0, 0, 0)
    assert L.fo_attention_prefill_bf16_rows(None, None, None, None, 256, 16, 8, g, None, None, 0, 256,
                                            opts) == F.ERR_INVALID
    for splits in (1, 0, 65):
        assert L.fo_attention_prefill_bf16_rows_split(None, None, None, None, 256, 16, 8, g, None, None, 1, 0, 256,
                                                      opts, splits) == F.ERR_INVALID


def test_static_scratch_decode_refuses_misaligned_pointers_before_any_device_call():
    """fo_decode_rows_static_scratch stages records with bulk copies from
    16-byte aligned addresses and reads q two floats at a time: misaligned
    pointers are refused on the host (this runs without a GPU)."""
    buf = np.zeros(4096, np.float32)
    base = (buf.ctypes.data + 15) & ~15
    L = F.lib()
    for codes, tail, q in ((base + 8, base, base), (base, base + 4, base), (base, base, base + 4)):
        st = L.fo_decode_rows_static_scratch(codes, base, tail, base, F.KV_Q8, 10, 10, 2, 2, 16, 8, q, 2, base, 0,
                                             base, None)
        assert st == F.ERR_INVALID
        assert "aligned" in last_error()
