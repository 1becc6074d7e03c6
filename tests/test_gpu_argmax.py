"""Greedy-argmax parity over a synthetic logit head: the attention outputs of
the CUDA path and of the CPU restatement of the reference, on the same seeded
inputs, go through one random-init head W [65,536][1,024], W ~ N(0, 1/1024)
(torch generator seed 5, float64, on the device), and the argmax of the
logits must agree on at least 99.9 % of the steps.

A step is one output row (a query row of a prefill page, one verify row of a
decode call, one page of a batched INT8 decode step).  The reference's model
feeds attention outputs through its projections before its LM head; W stands
in for that whole stack, so the gate measures how often an output difference
flips the greedy choice."""

import numpy as np
import pytest

import fo_cuda as F
import generators as G
import oracle as O
import baseline_int8 as B

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

VOCAB, HIDDEN = 65536, 1024
AGREE = 0.999


@pytest.fixture(scope="module")
def ctx():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    c = F.Context(0)
    yield c
    c.close()


@pytest.fixture(scope="module")
def head():
    g = torch.Generator(device="cuda").manual_seed(5)
    return torch.randn(VOCAB, HIDDEN, generator=g, device="cuda", dtype=torch.float64) / 32.0


def agreement(head, a, b) -> float:
    """Fraction of rows whose logits W x have the same argmax for a and b."""
    a = torch.as_tensor(np.asarray(a, np.float64).reshape(-1, HIDDEN), device="cuda")
    b = torch.as_tensor(np.asarray(b, np.float64).reshape(-1, HIDDEN), device="cuda")
    same = 0
    for i in range(0, a.shape[0], 1024):
        same += int((torch.argmax(a[i:i + 1024] @ head.T, 1) == torch.argmax(b[i:i + 1024] @ head.T, 1)).sum())
    return same / a.shape[0]


def dev(x):
    return torch.from_numpy(np.ascontiguousarray(x)).cuda()


def test_c2_prefill_rows_fp32(ctx, head):
    """BASELINE config 2 (6,544 rows, 4,096-token image prefix, seed 1), FP32
    exact tiles."""
    q, k, v, s, geo = G.c2_inputs()
    out = torch.zeros(q.size, dtype=torch.float32, device="cuda")
    F.attention_with(dev(q), dev(k), dev(v), 6544, geo, dev(s), out, 16, 8, 64, ctx=ctx)
    ref = O.prefill64(q, k, v, 16, 8, geo, s)
    torch.cuda.synchronize()
    agree = agreement(head, out.cpu().numpy(), ref)
    print(f"argmax agreement C2 fp32: {agree:.5f} of 6544 rows")
    assert agree >= AGREE


SEEDS = range(1, 9)


@pytest.mark.parametrize("mode", ["bf16_static", "bf16_online"])
def test_c2_prefill_rows_bf16_eight_seeds(ctx, head, mode):
    """BASELINE config 2 pages from eight seeds (6,544 rows each, 4,096-token
    image prefix), BF16 static shift and online softmax: every page must
    pass the gate on its own."""
    static = mode == "bf16_static"
    opts = F.PrefillOptions(F.EXP_FAST, 0, F.SOFTMAX_STATIC if static else F.SOFTMAX_ONLINE, F.SOFTMAX_ONLINE)
    agrees = {}
    for seed in SEEDS:
        q, k, v, s, geo = G.c2_inputs(seed=seed)
        out = torch.zeros(q.size, dtype=torch.float32, device="cuda")
        F.attention_prefill_bf16(dev(q), dev(k), dev(v), geo, dev(s), out, 16, 8, options=opts, ctx=ctx)
        ref = O.prefill_bf16(q, k, v, 16, 8, geo[1:], s, softmax_static=static)
        torch.cuda.synchronize()
        agrees[seed] = agreement(head, out.cpu().numpy(), ref)
        print(f"argmax agreement C2 {mode} seed {seed}: {agrees[seed]:.5f} of 6544 rows")
    print(f"argmax agreement C2 {mode}: worst {min(agrees.values()):.5f}, mean "
          f"{sum(agrees.values()) / len(agrees):.5f} over {len(agrees)} seeds")
    assert min(agrees.values()) >= AGREE


@pytest.mark.parametrize("fmt", [F.KV_F32, F.KV_BF16, F.KV_Q8])
def test_c3_verify_steps(ctx, head, fmt):
    """BASELINE config 3 at 6,544 positions: 64 verify calls of 5 rows each
    against one sealed page (N(0,1), seed 2)."""
    rng = np.random.default_rng(2)
    length, rows, calls = 6544, 5, 64
    p = length - rows
    k = rng.standard_normal((p, 16, 64)).astype(np.float32)
    k[:, 1::2, :32] = k[:, 0::2, :32]
    v = rng.standard_normal((p, 8, 64)).astype(np.float32)
    ref = O.SplitCache(k, v, p, length, fmt=fmt)
    gpu = F.SplitPrefix.from_compact(dev(k), dev(v), p, length, fmt=fmt, ctx=ctx)
    tk = rng.standard_normal((rows, 8, 64)).astype(np.float32)
    tv = rng.standard_normal((rows, 8, 64)).astype(np.float32)
    for t in range(rows):
        ref.push(tk[t], tv[t])
    gpu.append(np.repeat(tk[:, :, None], 2, axis=2).reshape(-1), np.repeat(tv[:, :, None], 2, axis=2).reshape(-1))
    got, want = [], []
    for _ in range(calls):
        q = rng.standard_normal(rows * 1024).astype(np.float32)
        sinks = rng.standard_normal(16).astype(np.float32)
        out = np.zeros(rows * 1024, np.float32)
        gpu.attention_decode_rows(q, rows, sinks, out)
        got.append(out)
        want.append(ref.decode_rows(q, rows, sinks))
    gpu.close()
    agree = agreement(head, np.concatenate(got), np.concatenate(want))
    print(f"argmax agreement C3 format {fmt}: {agree:.5f} of {calls * rows} rows")
    assert agree >= AGREE


def int8_decode_f64(q, kd, vd, sinks):
    """The INT8 format's decode (baseline_int8.decode) in float64 on the
    device: kd, vd [heads][positions][64] dequantized (code * scale, FP32)."""
    q = torch.as_tensor(q, device="cuda", dtype=torch.float64).reshape(kd.shape[0], 64)
    s = torch.einsum("hd,hpd->hp", q, kd) / 8.0
    m = s.max(dim=1, keepdim=True).values
    e = torch.exp(s - m)
    den = e.sum(dim=1, keepdim=True)
    o = torch.einsum("hp,hpd->hd", e, vd) / den
    lse = m[:, 0] + torch.log(den[:, 0])
    sk = torch.as_tensor(sinks, device="cuda", dtype=torch.float64)
    return (o / (1.0 + torch.exp(sk - lse))[:, None]).reshape(-1)


def test_c4_int8_steps(ctx, head):
    """8 pages of 16,384 positions in the INT8 format,
    32 single-row steps (N(0,1), seed 3), against the format's restatement
    (its float64 decode, run on the device for speed; the first step is also
    checked against baseline_int8.decode itself)."""
    rng = np.random.default_rng(3)
    pages, length, steps = 8, 16384, 32
    caches, deq, first = [], [], None
    for _ in range(pages):
        k = rng.standard_normal((length, 16, 64)).astype(np.float32)
        v = rng.standard_normal((length, 16, 64)).astype(np.float32)
        caches.append(F.Int8Cache(dev(k), dev(v), ctx=ctx))
        kc, ks = B.quantize(k)
        vc, vs = B.quantize(v)
        if first is None:
            first = (kc, ks, vc, vs)
        deq.append((dev(B.dequantize(kc, ks)).double(), dev(B.dequantize(vc, vs)).double()))
    got, want = [], []
    for step in range(steps):
        qs = [rng.standard_normal((16, 64)).astype(np.float32) for _ in range(pages)]
        ss = [rng.standard_normal(16).astype(np.float32) for _ in range(pages)]
        outs = [torch.zeros(1024, device="cuda") for _ in range(pages)]
        F.int8_decode_batch(caches, [dev(x) for x in qs], [dev(x) for x in ss], outs)
        torch.cuda.synchronize()
        for i in range(pages):
            got.append(outs[i].cpu().numpy())
            want.append(int8_decode_f64(qs[i], deq[i][0], deq[i][1], ss[i]).cpu().numpy())
        if step == 0:
            ref = B.decode(qs[0], *first, ss[0]).reshape(-1)
            assert np.allclose(want[0], ref, rtol=1e-12, atol=1e-12)
            assert np.all(np.abs(got[0] - ref) <= 1e-5 * (1 + np.abs(ref)))
    for c in caches:
        c.close()
    agree = agreement(head, np.stack(got), np.stack(want))
    print(f"argmax agreement C4 int8: {agree:.5f} of {steps * pages} rows")
    assert agree >= AGREE
