"""The CPU baseline (oracle/fo_cpu_simd.c: the reference's production SIMD
kernels restated with the same x86 instructions) against the scalar
restatement of the reference (oracle/fo_oracle.c) on the reference tests'
inputs.  Both restate the same operation sequence, so they agree bit for
bit; the benchmark times the SIMD one."""

import numpy as np
import pytest

import cpu_simd as C
import generators as G
import oracle as O


@pytest.mark.parametrize("case", G.BF16_CASES)
def test_bf16_static_prefill_equals_the_scalar_restatement(case):
    if not C.has_bf16():
        pytest.skip("host lacks AVX512-BF16")
    n, image_start, image_end = case
    q, k, v, s = G.bf16_operands(n)
    got = C.prefill_bf16_static(q, k, v, 16, 8, (image_start, image_end), s)
    want = O.prefill_bf16(q, k, v, 16, 8, (image_start, image_end), s, softmax_static=True)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), float(np.abs(got - want).max())


def test_bf16_static_prefill_on_a_c2_shaped_page():
    """A 1,100-token page with a 700-token image prefix and RoPE inputs
    (BASELINE config 2's generator, shortened)."""
    if not C.has_bf16():
        pytest.skip("host lacks AVX512-BF16")
    q, k, v, s, _ = G.c2_inputs(seed=3, seq=1100, image_end=700)
    got = C.prefill_bf16_static(q, k, v, 16, 8, (0, 700), s)
    want = O.prefill_bf16(q, k, v, 16, 8, (0, 700), s, softmax_static=True)
    assert np.array_equal(got, want)


@pytest.mark.parametrize("p,generated,rows", [(600, 5, 5), (1000, 8, 8), (257, 2, 2), (130, 3, 1)])
def test_f32_verify_decode_equals_the_scalar_restatement(p, generated, rows):
    if not C.has_avx2():
        pytest.skip("host lacks AVX2/FMA")
    k, v, _ = G.kv_fixture(p, 7)
    cache = O.SplitCache(k, v, p, p + generated, fmt=O.F32)
    tk, tv = G.kv_tail(generated)
    for t in range(generated):
        cache.push(tk[t * 512:(t + 1) * 512], tv[t * 512:(t + 1) * 512])
    q = G.kv_rows_query(rows)
    sinks = np.array([h * 0.25 - 1.0 for h in range(16)], np.float32)
    got = C.decode_rows_f32(cache, q, rows, sinks)
    want = cache.decode_rows(q, rows, sinks)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), float(np.abs(got - want).max())


def test_host_description_names_the_cpu():
    d = C.host_description()
    assert d["logical"] >= 1 and isinstance(d["flags"], list)
