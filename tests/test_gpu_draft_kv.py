"""GPU parity of the draft head's int8 KV (fo_draft_kv_*, draft.cu) against
the oracle restatement of src/draft_head.rs:177-220 and :548-759: codes and
scales bit-exact; attention within 1e-5 * (1 + |b|) of the oracle and within
the reference's own 0.03 of a double-precision attention
(draft_head.rs:794-870); a window equals a cache of only the newest rows,
bit for bit."""

import numpy as np
import pytest

import fo_cuda as F
import oracle as O
from test_draft_kv_cpu import CHAIN, ROWS, fixture, reference_f64

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def dev(x):
    return torch.from_numpy(np.ascontiguousarray(x)).cuda()


def records(kv, n, capacity):
    kc, ks, vc, vs = kv.records()
    rows = 8 * capacity
    return (F.device_to_host(kc, rows * 64, np.int8).reshape(8, capacity, 64)[:, :n],
            F.device_to_host(ks, rows, np.float32).reshape(8, capacity)[:, :n],
            F.device_to_host(vc, rows * 64, np.int8).reshape(8, capacity, 64)[:, :n],
            F.device_to_host(vs, rows, np.float32).reshape(8, capacity)[:, :n])


def pair(capacity, keys, values, device):
    ref, gpu = O.DraftKv(capacity), F.DraftKv(capacity)
    ref.push(keys, values)
    gpu.push(dev(keys) if device else keys, dev(values) if device else values)
    return ref, gpu


@pytest.mark.parametrize("device", [False, True])
def test_push_is_bit_exact(device):
    keys, values, _, _, _ = fixture()
    keys = keys.copy()
    keys[5] = np.nan  # a NaN value codes 0 (Rust's `as i8`)
    keys[512 * 7:512 * 7 + 64] = 0.0  # an all-zero row: scale 0, codes 0
    cap = ROWS + 3
    ref, gpu = pair(cap, keys, values, device)
    assert gpu.len == ROWS
    kc, ks, vc, vs = records(gpu, ROWS, cap)
    assert np.array_equal(kc, ref.key_codes.reshape(8, cap, 64)[:, :ROWS])
    assert np.array_equal(vc, ref.value_codes.reshape(8, cap, 64)[:, :ROWS])
    assert np.array_equal(ks.view(np.uint32), ref.key_scales.reshape(8, cap)[:, :ROWS].view(np.uint32))
    assert np.array_equal(vs.view(np.uint32), ref.value_scales.reshape(8, cap)[:, :ROWS].view(np.uint32))
    gpu.close()


@pytest.mark.parametrize("window", [0, 1, 64, ROWS, 1000])
@pytest.mark.parametrize("chain", [0, CHAIN])
@pytest.mark.parametrize("device", [False, True])
def test_attend_matches_oracle_and_f64(window, chain, device):
    keys, values, q, ck, cv = fixture()
    ref, gpu = pair(ROWS, keys, values, device)
    ck, cv = ck[:chain * 512], cv[:chain * 512]
    if device:
        out = torch.zeros(1024, device="cuda")
        gpu.attend(dev(q), ROWS, out, window, dev(ck) if chain else None, dev(cv) if chain else None)
        torch.cuda.synchronize()
        got = out.cpu().numpy()
    else:
        got = gpu.attend(q, ROWS, np.zeros(1024, np.float32), window, ck if chain else None, cv if chain else None)
    expected = ref.attend(q, ROWS, window, ck if chain else None, cv if chain else None)
    assert np.all(np.abs(got - expected) <= 1e-5 * (1 + np.abs(expected))), np.abs(got - expected).max()
    if chain == CHAIN:
        start = 0 if window == 0 else max(ROWS - window, 0)
        assert np.max(np.abs(got - reference_f64(keys, values, q, ck, cv, start))) < 0.03
    gpu.close()


def test_window_equals_a_cache_of_the_newest_rows():
    keys, values, q, ck, cv = fixture()
    _, full = pair(ROWS, keys, values, True)
    for w in (1, 7, 64, 257):
        _, tail = pair(w, keys[(ROWS - w) * 512:], values[(ROWS - w) * 512:], True)
        a = full.attend(q, ROWS, np.zeros(1024, np.float32), w, ck, cv)
        b = tail.attend(q, w, np.zeros(1024, np.float32), 0, ck, cv)
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32)), w
        tail.close()
    full.close()


def test_long_caches_and_growing_pushes():
    """1,500 verified positions (the reference's profiling size) pushed in
    uneven batches, attended at several prefixes."""
    rng = np.random.default_rng(3)
    keys = rng.standard_normal(1500 * 512).astype(np.float32)
    values = rng.standard_normal(1500 * 512).astype(np.float32)
    q = rng.standard_normal(1024).astype(np.float32)
    ref, gpu = O.DraftKv(1600), F.DraftKv(1600)
    at = 0
    for n in (1, 17, 300, 682, 500):
        ref.push(keys[at * 512:(at + n) * 512], values[at * 512:(at + n) * 512])
        gpu.push(dev(keys[at * 512:(at + n) * 512]), dev(values[at * 512:(at + n) * 512]))
        at += n
        for bases in (at, max(at - 5, 1)):
            for window in (0, 256, 1024):
                got = gpu.attend(q, bases, np.zeros(1024, np.float32), window)
                want = ref.attend(q, bases, window)
                assert np.all(np.abs(got - want) <= 1e-5 * (1 + np.abs(want))), (at, bases, window)
    gpu.close()


def test_errors():
    keys, values, q, ck, cv = fixture()
    gpu = F.DraftKv(4)
    with pytest.raises(F.CapacityError):
        gpu.push(keys[:5 * 512], values[:5 * 512])
    assert gpu.len == 0
    gpu.push(keys[:2 * 512], values[:2 * 512])
    out = np.zeros(1024, np.float32)
    with pytest.raises(F.FoError):
        gpu.attend(q, 3, out)  # beyond the pushed rows
    with pytest.raises(F.FoError):
        gpu.attend(q, 0, out)  # nothing to attend to
    big = np.zeros(65 * 512, np.float32)
    with pytest.raises(F.FoError):
        gpu.attend(q, 2, out, 0, big, big)  # more chain rows than the scratch holds
    gpu.attend(q, 0, out, 0, ck, cv)  # chain rows alone
    assert np.isfinite(out).all()
    gpu.close()
