"""The decode entry point that allocates no device memory
(fo_decode_rows_static_scratch), against the regular verify-row decode.

Callers that own all device memory through their own pool, or that must not
call cudaMalloc/cudaFree while decoding (those calls can synchronize the
whole device), use this entry point: its scratch is a fixed static array in
the library.  This file is named so that pytest collects it last; it creates
its own context, so it also passes alone in a fresh process."""

import numpy as np
import pytest

import fo_cuda as F
import generators as G

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def sealed(fmt, p, generated, seed, ctx):
    k, v, _ = G.kv_fixture(p, seed)
    cache = F.SplitPrefix.from_compact(torch.from_numpy(k).cuda(), torch.from_numpy(v).cuda(), p, p + generated,
                                       fmt=fmt, ctx=ctx)
    tk, tv = G.kv_tail(generated)
    ke = np.repeat(tk.reshape(generated, 8, 1, 64), 2, axis=2).reshape(-1)
    ve = np.repeat(tv.reshape(generated, 8, 1, 64), 2, axis=2).reshape(-1)
    cache.append(torch.from_numpy(ke).cuda(), torch.from_numpy(ve).cuda())
    return cache


def test_static_scratch_decode_matches_decode_rows_twice():
    assert torch.cuda.is_available()
    ctx = F.Context(0)
    sinks = torch.from_numpy(np.array([h * 0.25 - 1.0 for h in range(16)], np.float32)).cuda()
    # Two calls in a row: a long Q8 cache with 5 rows, then a short FP32 cache
    # with 2 rows, which runs over the array the first call left behind.
    for fmt, p, generated, rows in (("q8", 9000, 6, 5), ("f32", 700, 3, 2)):
        cache = sealed(fmt, p, generated, p, ctx)
        q = torch.from_numpy(G.kv_rows_query(rows)).cuda()
        expected = torch.zeros(rows * 1024, device="cuda")
        cache.attention_decode_rows(q, rows, sinks, expected)
        got = torch.full((rows * 1024,), float("nan"), device="cuda")
        F.decode_rows_static_scratch(cache, fmt, q, rows, sinks, got)
        torch.cuda.synchronize()
        a, b = got.cpu().numpy().astype(np.float64), expected.cpu().numpy().astype(np.float64)
        assert np.all(np.abs(a - b) <= 1e-5 * (1.0 + np.abs(b))), (fmt, np.abs(a - b).max())
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
