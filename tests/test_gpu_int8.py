"""GPU parity of BASELINE config 4's INT8 KV format (fo_i8_seal,
fo_i8_decode_batch) with its numpy restatement (oracle/baseline_int8.py):
codes and scales bit-exact; decode within FP32 rounding (1e-5 * (1 + |b|))
of the float64 attention over the dequantized cache, and within BASELINE's
INT8 tolerance (2e-2 * (1 + |b|)) of attention over the unquantized keys and
values."""

import numpy as np
import pytest

import baseline_int8 as B
import fo_cuda as F

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def d2h(ptr, n, dtype):
    """Copy n elements of device memory at `ptr` to a numpy array."""
    return F.device_to_host(ptr, n, dtype)


@pytest.fixture(scope="module")
def ctx():
    c = F.Context(0)
    yield c
    c.close()


def page(length, seed, heads=16):
    rng = np.random.default_rng(seed)
    k = rng.standard_normal((length, heads, 64)).astype(np.float32)
    v = rng.standard_normal((length, heads, 64)).astype(np.float32)
    q = rng.standard_normal((heads, 64)).astype(np.float32)
    sinks = rng.standard_normal(heads).astype(np.float32)
    k[: min(length, 64), 3] = 0.0  # a whole zero group: scale 0, codes 0
    return k, v, q, sinks


@pytest.mark.parametrize("length", [1, 63, 64, 1000, 1025, 4160])
def test_codes_and_scales_are_bit_exact(ctx, length):
    k, v, _, _ = page(length, length)
    cache = F.Int8Cache(k, v, ctx=ctx)
    kc, ks, vc, vs = cache.records()
    groups = (length + 63) // 64
    for x, codes, scales in ((k, kc, ks), (v, vc, vs)):
        want_c, want_s = B.quantize(x)
        assert np.array_equal(d2h(codes, 16 * length * 64, np.int8).reshape(16, length, 64), want_c)
        assert np.array_equal(d2h(scales, 16 * groups, np.float32).reshape(16, groups).view(np.uint32),
                              want_s.view(np.uint32))
    assert cache.bytes() == 2 * 16 * length * 64 + 2 * 16 * groups * 4
    cache.close()


@pytest.mark.parametrize("fast_exp", [False, True])
def test_decode_batch_matches_the_oracle(ctx, fast_exp):
    lengths = [16384, 700, 1025, 64, 3000]
    caches, qs, ss, outs, want, exact = [], [], [], [], [], []
    for i, length in enumerate(lengths):
        k, v, q, sinks = page(length, 100 + i)
        caches.append(F.Int8Cache(torch.from_numpy(k).cuda(), torch.from_numpy(v).cuda(), ctx=ctx))
        qs.append(torch.from_numpy(q).cuda())
        ss.append(torch.from_numpy(sinks).cuda())
        outs.append(torch.full((16 * 64,), float("nan"), device="cuda"))
        kc, ks = B.quantize(k)
        vc, vs = B.quantize(v)
        want.append(B.decode(q, kc, ks, vc, vs, sinks))
        exact.append(_dense(q, k, v, sinks))
    F.int8_decode_batch(caches, qs, ss, outs, fast_exp=fast_exp)
    torch.cuda.synchronize()
    for i in range(len(lengths)):
        got = outs[i].cpu().numpy().reshape(16, 64).astype(np.float64)
        tol = 1e-4 if fast_exp else 1e-5
        assert np.all(np.abs(got - want[i]) <= tol * (1 + np.abs(want[i]))), (lengths[i], np.abs(got - want[i]).max())
        assert np.all(np.abs(got - exact[i]) <= 2e-2 * (1 + np.abs(exact[i])))
    for c in caches:
        c.close()


def _dense(q, k, v, sinks):
    """float64 attention over the unquantized keys and values."""
    k, v = k.astype(np.float64).transpose(1, 0, 2), v.astype(np.float64).transpose(1, 0, 2)
    s = np.einsum("hd,hpd->hp", q.astype(np.float64), k) / 8.0
    m = s.max(axis=1, keepdims=True)
    e = np.exp(s - m)
    den = e.sum(axis=1, keepdims=True)
    lse = m[:, 0] + np.log(den[:, 0])
    return np.einsum("hp,hpd->hd", e, v) / den / (1.0 + np.exp(sinks.astype(np.float64) - lse))[:, None]


def test_a_cache_twice_in_one_batch_is_refused(ctx):
    k, v, q, sinks = page(100, 1)
    c = F.Int8Cache(k, v, ctx=ctx)
    qd, sd, od = torch.from_numpy(q).cuda(), torch.from_numpy(sinks).cuda(), torch.empty(1024, device="cuda")
    with pytest.raises(F.FoError):
        F.int8_decode_batch([c, c], [qd, qd], [sd, sd], [od, od])
    c.close()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_one_process_decodes_on_a_second_device():
    """Launch attributes (the INT8 kernel's 64 KB of shared memory, the split
    merge's allowance) belong to each device: a process that decodes on
    device 0 and then on device 1 gets the same results on both."""
    k, v, q, sinks = page(3000, 7)
    outs = []
    for d in (0, 1):
        c = F.Context(d)
        with torch.cuda.device(d):
            cache = F.Int8Cache(torch.from_numpy(k).to(d), torch.from_numpy(v).to(d), ctx=c)
            out = torch.zeros(16 * 64, device=d)
            F.int8_decode_batch([cache], [torch.from_numpy(q).to(d)], [torch.from_numpy(sinks).to(d)], [out])
            kk = k.copy()  # a split cache needs each pair's temporal halves equal
            kk[:, 1::2, :32] = kk[:, 0::2, :32]
            vv = np.ascontiguousarray(v[:, :8])
            split = F.SplitPrefix.from_compact(torch.from_numpy(kk).to(d), torch.from_numpy(vv).to(d), 3000, 3001,
                                               fmt="q8", ctx=c)
            o2 = torch.zeros(16 * 64, device=d)
            split.attention_decode(torch.from_numpy(q.reshape(-1)).to(d), 3000, torch.from_numpy(sinks).to(d), o2)
            torch.cuda.synchronize(d)
            outs.append((out.cpu(), o2.cpu()))
            split.close()
            cache.close()
        c.close()
    assert torch.equal(outs[0][0], outs[1][0]) and torch.equal(outs[0][1], outs[1][1])
