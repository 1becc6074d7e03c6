"""Writes tests/golden/attention_golden.npz: the reference's own known answers
and f64 expectations for the inputs its attention tests use.

Run from the repository root:  python tests/golden/make_golden.py

Contents (all restated from the reference project's tests):
* kat5_*            the hand-computed 5-token image/sink answer and the
                    sink = -inf identity (src/kernels/tests.rs:283-309);
* dense_<i>         f64 outputs for the dense tolerance table
                    (src/kernels/tests.rs:250-281);
* extreme_<j>       large-logit / large-sink cases (src/kernels/tests.rs:311-345);
* prefill64_<n>     f64 outputs of the FP32 tile cases (prefill64/tests.rs:36-44),
                    heads 0 and 9 only, stored as float32 (the
                    tolerances are >= 1e-5);
* static_<i>        f64 outputs of the static-shift cases
                    (prefill64/static_shift/tests.rs:53-64), heads 0 and 9;
* bf16_<n>          f64 outputs on BF16 operands (prefill64/bf16.rs:851-926),
                    heads 0 and 9;
* kv_lowprec_*      the compact FP32 decode the Q8/Q16 records must stay within
                    0.02 of (src/quant/kv/tests.rs:282-304);
* codes_*           round-ties-even code table (src/quant/kv/tests.rs:568-612).
"""

from __future__ import annotations

import os
import sys

import numpy as np

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
import generators as G  # noqa: E402

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "attention_golden.npz")


def main() -> None:
    data = {}
    # -- known answer: src/kernels/tests.rs:283-309
    data["kat5_expected"] = np.array([0.5, 27.75, 27.75, 222.2, 1851.8334], np.float64)
    data["kat5_values"] = np.array([1.0, 10.0, 100.0, 1000.0, 10000.0], np.float32)
    data["kat5_nosink_expected"] = np.array([13.0], np.float32)

    # -- dense table: src/kernels/tests.rs:250-281
    for i, (ql, kvl, h, d, off, st, en) in enumerate(G.DENSE_TABLE):
        q = G.lcg_values(ql * h * d, 71)
        k = G.lcg_values(kvl * h * d, 83)
        v = G.lcg_values(kvl * h * d, 117)
        s = G.lcg_values(h, 24)
        data[f"dense_{i}"] = G.attention_f64(q, k, v, h, h, d, (off, st, en), s)

    # -- extreme logits: src/kernels/tests.rs:311-345
    keys = np.array([1010.0 if i == 140 else -1000.0 for i in range(257)], np.float32)
    vals = np.array([np.float32(i) * np.float32(0.1) - np.float32(3.0) for i in range(257)], np.float32)
    for j, sink in enumerate([-10000.0, 10000.0, 1009.0, -np.inf]):
        data[f"extreme_{j}"] = G.attention_f64(np.array([1.0], np.float32), keys, vals, 1, 1, 1, (256, 0, 0),
                                               np.array([sink], np.float32))
    data["extreme_multi"] = G.attention_f64(np.ones(4, np.float32), keys, vals, 1, 1, 1, (253, 0, 0),
                                            np.array([-10000.0], np.float32))

    # -- FP32 tiles: prefill64/tests.rs:36-89
    for (ql, ist, ien) in G.PREFILL64_CASES:
        q, k, v, s = G.prefill64_operands(ql)
        data[f"prefill64_{ql}"] = G.sample_heads(G.attention_f64(q, k, v, 16, 8, 64, (0, ist, ien), s)).astype(np.float32)

    # -- static shift: prefill64/static_shift/tests.rs:53-64, 372-394
    for i, (queries, total, off, ist, ien) in enumerate(G.STATIC_CASES):
        q, k, v, s = G.static_operands(queries, total)
        data[f"static_{i}"] = G.sample_heads(G.attention_f64(q, k, v, 16, 8, 64, (off, ist, ien), s)).astype(np.float32)

    # -- BF16 operands: prefill64/bf16.rs:851-926
    for (ql, ist, ien) in G.BF16_CASES:
        q, k, v, s = G.bf16_operands(ql)
        data[f"bf16_{ql}"] = G.sample_heads(G.attention_f64(q, k, v, 16, 8, 64, (0, ist, ien), s)).astype(np.float32)

    # -- Q8/Q16 vs compact FP32: src/quant/kv/tests.rs:282-304
    p = 257
    k, v, q = G.kv_fixture(p, 9)
    tail = np.full(8 * 64, 0.02, np.float32)
    sinks = np.full(16, 0.5, np.float32)
    vall = np.concatenate([v, tail])
    data["kv_lowprec_expected"] = G.attention_f64(q, k, vall, 16, 8, 64, (p, 0, p), sinks, generated_k=tail)

    # -- code rounding: src/quant/kv/tests.rs:568-612
    xs, limits, expect = [], [], []
    for limit in (7.0, 127.0, 32767.0):
        vals = [0.0, -0.0, np.inf, -np.inf, 1e-300, -1e-300, 1e300, -1e300]
        for kk in range(-int(limit) - 3, int(limit) + 4):
            for base in (float(kk), kk + 0.5):
                vals += [base, np.nextafter(base, np.inf), np.nextafter(base, -np.inf), base + 0.25, base - 0.25]
        for x in vals:
            xs.append(x)
            limits.append(limit)
            expect.append(float(np.clip(np.round(x), -limit, limit)))  # numpy rounds half to even
    data["codes_x"] = np.array(xs, np.float64)
    data["codes_limit"] = np.array(limits, np.float64)
    data["codes_expected"] = np.array(expect, np.float64)
    cv, cs, c8, c16 = [], [], [], []
    for scale in (0.0, 1e-3, 0.37, float(np.array([1], np.uint32).view(np.float32)[0])):
        for value in (0.0, -0.0, 0.25, -1.5, 3.7, 1e3, -1e3):
            x = np.float64(np.float32(value)) / np.float64(np.float32(scale)) if scale != 0.0 else 0.0
            cv.append(value)
            cs.append(scale)
            c8.append(0 if scale == 0.0 else int(np.clip(np.round(x), -127, 127)))
            c16.append(0 if scale == 0.0 else int(np.clip(np.round(x), -32767, 32767)))
    data["code_values"] = np.array(cv, np.float32)
    data["code_scales"] = np.array(cs, np.float32)
    data["code_q8"] = np.array(c8, np.int64)
    data["code_q16"] = np.array(c16, np.int64)

    np.savez_compressed(OUT, **data)
    print(f"wrote {OUT}: {len(data)} arrays, {os.path.getsize(OUT) / 1e6:.2f} MB")


if __name__ == "__main__":
    main()
