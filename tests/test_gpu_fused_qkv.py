"""GPU parity of the fused QKV rows (fo_qkv_prefix_rows, fo_kv_append_qkv)
against the oracle's restatement of src/model/fused.rs:96-116 and
src/model/rope.rs:15-85: bit for bit, through the C ABI."""

import numpy as np
import pytest

import fo_cuda as F
import oracle as O
from test_fused_qkv_cpu import fixture

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

HEADS, GROUPS = 16, 8
WIDTH = HEADS * 64 + 2 * GROUPS * 64


@pytest.fixture(scope="module")
def ctx():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    c = F.Context(0)
    yield c
    c.close()


def dev(x):
    return torch.from_numpy(np.ascontiguousarray(x)).cuda()


def bits(x):
    return np.asarray(x).view(np.uint32)


def same(a, b):
    """Bit for bit where not NaN, NaN where NaN (payloads differ by device)."""
    a, b = np.asarray(a, np.float32), np.asarray(b, np.float32)
    na, nb = np.isnan(a), np.isnan(b)
    return np.array_equal(na, nb) and np.array_equal(bits(a[~na]), bits(b[~nb]))


def bf16_rne(x):
    """Round to nearest even (half::bf16::from_f32), NaN kept quiet."""
    u = np.asarray(x, np.float32).view(np.uint32).astype(np.uint64)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    return np.where(nan, ((u >> 16) | 0x40).astype(np.uint16), r)


@pytest.mark.parametrize("rows", [1, 23, 6544])
def test_prefix_rows_are_the_oracle_bit_for_bit(ctx, rows):
    qkv, rope = fixture(rows, seed=100 + rows)
    q_ref, k_ref, v_ref = O.qkv_rows(qkv, rope, rows)
    q = torch.empty(rows * HEADS * 64, device="cuda")
    k = torch.empty_like(q)
    v = torch.empty(rows * GROUPS * 64, device="cuda")
    kb = torch.empty(rows * HEADS * 64, dtype=torch.bfloat16, device="cuda")
    vb = torch.empty(rows * GROUPS * 64, dtype=torch.bfloat16, device="cuda")
    F.qkv_prefix_rows(dev(qkv), dev(rope), rows, q, k, v, kb, vb, ctx=ctx)
    torch.cuda.synchronize()
    assert np.array_equal(bits(q.cpu().numpy()), bits(q_ref))
    assert np.array_equal(bits(k.cpu().numpy()), bits(k_ref))
    assert np.array_equal(bits(v.cpu().numpy()), bits(v_ref))
    assert np.array_equal(kb.view(torch.int16).cpu().numpy().view(np.uint16), bf16_rne(k_ref))
    assert np.array_equal(vb.view(torch.int16).cpu().numpy().view(np.uint16), bf16_rne(v_ref))


FORMATS = [F.KV_F32, F.KV_Q16, F.KV_Q8, F.KV_BF16, F.KV_Q4, F.KV_Q8_ROT, F.KV_Q4_ROT]


@pytest.mark.parametrize("fmt", FORMATS)
def test_decode_rows_append_what_the_oracle_pushes(ctx, fmt):
    """fo_kv_append_qkv: the queries equal the oracle's, and the tail records
    equal the oracle's push of the pair's first key head and the group's
    value (what SplitPrefix::append keeps of split_norm_rope's rows)."""
    import generators as G
    p, gen = 130, 5
    k0, v0, _ = G.kv_fixture(p, 9)
    ref = O.SplitCache(k0, v0, p, p + gen + 1, fmt=fmt)
    gpu = F.SplitPrefix.from_compact(dev(k0), dev(v0), p, p + gen + 1, fmt=fmt, ctx=ctx)
    qkv, rope = fixture(gen, seed=31)
    qkv[2 * WIDTH + 5] = np.nan  # a non-finite query value stays in its own row
    q_ref, k_ref, v_ref = O.qkv_rows(qkv, rope, gen)
    q = torch.empty(gen * HEADS * 64, device="cuda")
    F.append_qkv(gpu, dev(qkv[:2 * WIDTH]), dev(rope[:2 * HEADS * 64]), 2, q[:2 * HEADS * 64])
    F.append_qkv(gpu, dev(qkv[2 * WIDTH:]), dev(rope[2 * HEADS * 64:]), gen - 2, q[2 * HEADS * 64:])
    torch.cuda.synchronize()
    assert gpu.tail_len == gen
    assert same(q.cpu().numpy(), q_ref)
    assert np.isnan(q_ref.reshape(gen, HEADS, 64)[2, 0]).all() and np.isfinite(q_ref.reshape(gen, HEADS, 64)[3]).all()
    kr = k_ref.reshape(gen, HEADS, 64)[:, 0::2]  # the pair's first head
    vr = v_ref.reshape(gen, GROUPS, 64)
    for t in range(gen):
        ref.push(np.ascontiguousarray(kr[t]).reshape(-1), np.ascontiguousarray(vr[t]).reshape(-1))
    (codes, scales, tcodes, tscales), ps, ts = gpu.records()
    element = fmt & ~F.KV_ROTATED
    dt = {F.KV_F32: np.float32, F.KV_Q16: np.int16, F.KV_Q8: np.int8, F.KV_BF16: np.uint16, F.KV_Q4: np.uint8}[element]
    width = 64 if element == F.KV_Q4 else 128  # stored elements per tail record
    tail = F.device_to_host(tcodes, GROUPS * ts * width, dt).reshape(GROUPS, ts, width)[:, :gen]
    want = ref.tail_codes.reshape(GROUPS, -1, width)[:, :gen]
    b = (lambda x: x.view(np.uint32)) if dt == np.float32 else (lambda x: x)
    assert np.array_equal(b(np.ascontiguousarray(tail)), b(np.ascontiguousarray(want)))
    if element in (F.KV_Q16, F.KV_Q8, F.KV_Q4):
        got = F.device_to_host(tscales, GROUPS * ts * 4, np.uint16).reshape(GROUPS, ts, 4)[:, :gen]
        assert np.array_equal(got, ref.tail_scales.reshape(GROUPS, -1, 4)[:, :gen])
    with pytest.raises(F.CapacityError):
        F.append_qkv(gpu, dev(qkv[:2 * WIDTH]), dev(rope[:2 * HEADS * 64]), 2, q[:2 * HEADS * 64])
    assert gpu.tail_len == gen
    gpu.close()


def test_fused_prefill_operands_give_the_same_attention(ctx):
    """A C2-shaped page whose Q, K, V and BF16 copies come from
    fo_qkv_prefix_rows attends exactly as one whose operands were built from
    the oracle's rows and converted separately."""
    rows = 6544
    qkv, rope = fixture(rows, seed=3)
    q_ref, k_ref, v_ref = O.qkv_rows(qkv, rope, rows)
    q = torch.empty(rows * HEADS * 64, device="cuda")
    k, v = torch.empty_like(q), torch.empty(rows * GROUPS * 64, device="cuda")
    kb = torch.empty(rows * HEADS * 64, dtype=torch.bfloat16, device="cuda")
    vb = torch.empty(rows * GROUPS * 64, dtype=torch.bfloat16, device="cuda")
    F.qkv_prefix_rows(dev(qkv), dev(rope), rows, q, k, v, kb, vb, ctx=ctx)
    sinks = dev(np.linspace(-1, 1, HEADS).astype(np.float32))
    geo = (0, 0, 4096)
    opts = F.PrefillOptions(F.EXP_FAST, 0, F.SOFTMAX_STATIC, F.SOFTMAX_ONLINE)
    out_a = torch.empty_like(q)
    F.attention_prefill_bf16(q, k, v, geo, sinks, out_a, HEADS, GROUPS, keys_bf16=kb, values_bf16=vb, options=opts,
                             ctx=ctx)
    qr, kr, vr = dev(q_ref), dev(k_ref), dev(v_ref)
    out_b = torch.empty_like(q)
    F.attention_prefill_bf16(qr, kr, vr, geo, sinks, out_b, HEADS, GROUPS, keys_bf16=kr.to(torch.bfloat16),
                             values_bf16=vr.to(torch.bfloat16), options=opts, ctx=ctx)
    torch.cuda.synchronize()
    assert torch.equal(out_a.view(torch.int32), out_b.view(torch.int32))


@pytest.mark.parametrize("mode,fast", [("bf16", False), ("q8", True), ("q4r", True)])
def test_layer_flow_stays_on_the_device(ctx, mode, fast):
    """Three layers of one page with no host round trip (seal_layer,
    src/model/cache.rs:218-276): fused QKV rows -> prefill attention ->
    fo_kv_seal_layer (Q8 records on the layer kv_q8_layers names, `mode`
    elsewhere; fast exp from the cache's mode) -> fused decode rows appended ->
    verify decode.  Each layer equals the oracle's flow within 1e-5."""
    T, gen, mask = 300, 3, 0b010
    qkv_all, rope = fixture(T + gen, seed=77)
    # The temporal half of the rotation (pairs 0..15) depends on the position
    # only (rope.rs:99-103), so paired heads keep equal temporal keys.
    rope = rope.reshape(T + gen, HEADS, 32, 2)
    rope[:, :, :16] = rope[:, :1, :16]
    rope = np.ascontiguousarray(rope).reshape(-1)
    sinks = np.array([h * 0.2 - 1.0 for h in range(HEADS)], np.float32)
    sd = dev(sinks)
    for layer in range(3):
        qkv = (qkv_all * np.float32(1.0 + 0.25 * layer)).astype(np.float32)
        pre, dec = qkv[:T * WIDTH], qkv[T * WIDTH:]
        rp, rd = rope[:T * HEADS * 64], rope[T * HEADS * 64:]
        q = torch.empty(T * HEADS * 64, device="cuda")
        k, v = torch.empty_like(q), torch.empty(T * GROUPS * 64, device="cuda")
        F.qkv_prefix_rows(dev(pre), dev(rp), T, q, k, v, ctx=ctx)
        out = torch.empty_like(q)
        F.attention_with(q, k, v, T, (0, 0, 0), sd, out, HEADS, GROUPS, 64, ctx=ctx)
        cache = F.SplitPrefix.seal_layer(layer, k, v, T, T, T + gen, mode=mode, kv_q8_layers=mask, fast_exps=fast,
                                         ctx=ctx)
        qd = torch.empty(gen * HEADS * 64, device="cuda")
        F.append_qkv(cache, dev(dec), dev(rd), gen, qd)
        dec_out = torch.empty(gen * HEADS * 64, device="cuda")
        cache.attention_decode_rows(qd, gen, sd, dec_out)
        torch.cuda.synchronize()
        # the oracle's flow
        q_ref, k_ref, v_ref = O.qkv_rows(pre, rp, T)
        want = O.prefill64(q_ref, k_ref, v_ref, HEADS, GROUPS, (0, 0, 0), sinks)
        got = out.cpu().numpy()
        assert (np.abs(got - want) <= 1e-5 * (1 + np.abs(want))).all()
        fmt = "q8" if (mask >> layer) & 1 else mode
        ref = O.SplitCache(k_ref, v_ref, T, T + gen, fmt=fmt)
        ref.fast_exp = fast and mode in ("q8", "q8r", "q4r")  # default_fast_exp (kv.rs:182-184)
        qd_ref, kd_ref, vd_ref = O.qkv_rows(dec, rd, gen)
        kr = kd_ref.reshape(gen, HEADS, 64)[:, 0::2]
        for t in range(gen):
            ref.push(np.ascontiguousarray(kr[t]).reshape(-1), np.ascontiguousarray(vd_ref.reshape(gen, GROUPS, 64)[t])
                     .reshape(-1))
        want = ref.decode_rows(qd_ref, gen, sinks)
        got = dec_out.cpu().numpy()
        assert (np.abs(got - want) <= 1e-5 * (1 + np.abs(want))).all(), layer
        cache.close()
    with pytest.raises(F.FoError):  # only a complete prefix is sealed
        F.SplitPrefix.seal_layer(0, k, v, T - 1, T, T + gen, ctx=ctx)
