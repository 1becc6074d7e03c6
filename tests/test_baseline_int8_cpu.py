"""The numpy restatement of BASELINE config 4's INT8 format (test
infrastructure) against hand-checked properties: ties to even, the clamp,
zero groups, dequantization error at most half a step."""

import numpy as np

import baseline_int8 as B


def test_ties_round_to_even_and_codes_clamp():
    x = np.zeros((64, 1, 64), np.float32)
    x[0, 0, 0] = 127.0          # scale 1.0
    x[1, 0, :4] = [0.5, 1.5, 2.5, -0.5]
    x[2, 0, 0] = -127.0
    codes, scales = B.quantize(x)
    assert scales.tolist() == [[1.0]]
    assert codes[0, 1, :4].tolist() == [0, 2, 2, 0]
    assert codes[0, 0, 0] == 127 and codes[0, 2, 0] == -127


def test_zero_groups_and_partial_groups():
    rng = np.random.default_rng(0)
    x = rng.standard_normal((100, 2, 64)).astype(np.float32)
    x[:64, 1] = 0.0
    codes, scales = B.quantize(x)
    assert codes.shape == (2, 100, 64) and scales.shape == (2, 2)
    assert scales[1, 0] == 0.0 and not codes[1, :64].any()
    back = B.dequantize(codes, scales)
    step = np.repeat(scales, 64, axis=1)[:, :100, None]
    assert np.all(np.abs(back - x.transpose(1, 0, 2)) <= 0.5 * step + 1e-7)


def test_decode_of_a_single_position_is_its_value_times_the_sink_factor():
    v = np.full((1, 1, 64), 0.5, np.float32)
    k = np.ones((1, 1, 64), np.float32)
    kc, ks = B.quantize(k)
    vc, vs = B.quantize(v)
    out = B.decode(np.zeros((1, 64), np.float32), kc, ks, vc, vs, np.array([-np.inf]))
    assert np.allclose(out, 0.5)
