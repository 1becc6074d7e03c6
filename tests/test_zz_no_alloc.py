"""The decode entry point that allocates no device memory
(fo_decode_rows_static_scratch), against the regular verify-row decode.

Callers that own all device memory through their own pool, or that must not
call cudaMalloc/cudaFree while decoding (those calls can synchronize the
whole device), use this entry point: its scratch is a fixed static array in
the library.  Both entry points run the same kernels over the same split
partition, so the outputs must be equal bit for bit.  This file is named so
that pytest collects it last; it creates its own context, so it also passes
alone in a fresh process."""

import ctypes

import numpy as np
import pytest

import fo_cuda as F
import generators as G

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

SINKS = np.array([h * 0.25 - 1.0 for h in range(16)], np.float32)


def sealed(fmt, p, generated, seed, ctx):
    k, v, _ = G.kv_fixture(p, seed)
    cache = F.SplitPrefix.from_compact(torch.from_numpy(k).cuda(), torch.from_numpy(v).cuda(), p, p + generated,
                                       fmt=fmt, ctx=ctx)
    tk, tv = G.kv_tail(generated)
    ke = np.repeat(tk.reshape(generated, 8, 1, 64), 2, axis=2).reshape(-1)
    ve = np.repeat(tv.reshape(generated, 8, 1, 64), 2, axis=2).reshape(-1)
    cache.append(torch.from_numpy(ke).cuda(), torch.from_numpy(ve).cuda())
    return cache


def both(cache, fmt, rows, stream=None):
    """(static-scratch output, regular decode output) for one query set."""
    sinks = torch.from_numpy(SINKS).cuda()
    q = torch.from_numpy(G.kv_rows_query(rows)).cuda()
    expected = torch.zeros(rows * 1024, device="cuda")
    cache.attention_decode_rows(q, rows, sinks, expected)
    got = torch.full((rows * 1024,), float("nan"), device="cuda")
    torch.cuda.synchronize()
    if stream is None:
        F.decode_rows_static_scratch(cache, fmt, q, rows, sinks, got)
    else:
        with torch.cuda.stream(stream):
            F.decode_rows_static_scratch(cache, fmt, q, rows, sinks, got, stream=stream.cuda_stream)
        stream.synchronize()
    torch.cuda.synchronize()
    F.static_scratch_status()
    return got, expected


@pytest.mark.parametrize("fmt", ["q8", "q16", "f32", "bf16", "q4", "q8r", "q4r"])
def test_static_scratch_decode_equals_decode_rows_twice(fmt):
    """Two calls in a row (a long cache with 5 rows, then a short one with 2
    rows, which runs over the array the first call left behind), each equal
    bit for bit to fo_kv_attention_decode_rows; the second on a non-default
    stream."""
    assert torch.cuda.is_available()
    ctx = F.Context(0)
    side = torch.cuda.Stream()
    for (p, generated, rows), stream in (((9000, 6, 5), None), ((700, 3, 2), side)):
        cache = sealed(fmt, p, generated, p, ctx)
        got, expected = both(cache, fmt, rows, stream)
        assert torch.equal(got, expected), (fmt, p, float((got - expected).abs().max()))
        cache.close()
    ctx.close()


def test_static_scratch_decode_at_its_limit():
    """The largest accepted call: 8 rows, 16 heads, 16,384 positions."""
    ctx = F.Context(0)
    cache = sealed("bf16", 16384 - 8, 8, 3, ctx)
    got, expected = both(cache, "bf16", 8)
    assert torch.equal(got, expected)
    cache.close()
    ctx.close()


def test_static_scratch_decode_refuses_sizes_beyond_its_limit():
    ctx = F.Context(0)
    p = 16384  # with one generated position: 16,385 > the 16,384-position limit
    k = torch.zeros(p * 16 * 64, device="cuda")
    v = torch.zeros(p * 8 * 64, device="cuda")
    cache = F.SplitPrefix.from_compact(k, v, p, p + 1, fmt="q8", ctx=ctx)
    row = torch.zeros(16 * 64, device="cuda")
    cache.append(row, row)
    q = torch.zeros(1024, device="cuda")
    with pytest.raises(F.CapacityError, match="exceed the static scratch limit"):
        F.decode_rows_static_scratch(cache, "q8", q, 1, torch.zeros(16, device="cuda"), torch.zeros(1024,
                                                                                                       device="cuda"))
    cache.close()
    ctx.close()


def test_static_scratch_decode_refuses_misaligned_records():
    """Records are staged with bulk copies from 16-byte aligned addresses;
    a misaligned pointer is refused before anything launches."""
    ctx = F.Context(0)
    cache = sealed("q8", 300, 2, 1, ctx)
    (codes, scales, tcodes, tscales), ps, ts = cache.records()
    q = torch.zeros(2 * 1024, device="cuda")
    s = torch.zeros(16, device="cuda")
    out = torch.zeros(2 * 1024, device="cuda")
    L = F.lib()
    for c, t, qq in ((codes + 8, tcodes, q.data_ptr()), (codes, tcodes + 4, q.data_ptr()),
                     (codes, tcodes, q.data_ptr() + 4)):
        st = L.fo_decode_rows_static_scratch(c, scales, t, tscales, F.KV_Q8, 300, ps, 2, ts, 16, 8, qq, 2,
                                             s.data_ptr(), 0, out.data_ptr(), None)
        assert st == F.ERR_INVALID
        assert b"aligned" in L.fo_last_error()
    cache.close()
    ctx.close()
