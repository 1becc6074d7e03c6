"""TEST INFRASTRUCTURE ONLY (the checker, never the product): a numpy
restatement of the INT8 KV format BASELINE's config 4 names, and of single-row
decode attention over it.

The reference (falcon-ocr-cpu) has no such format; its INT8 KV is the Q8
record format of src/quant/kv.rs (one BF16 scale per 32-element block).  This
one is BASELINE's: keys and values of every head stored separately as int8
codes, [head][position][64], with one FP32 scale per (head, 64-position
group), for keys and values apart.  Codes are round-to-nearest-even of
x / scale clamped to [-127, 127], as the reference's codec rounds
(src/quant/kv/codec.rs:60-83); scale = max |x| over the group / 127 (a group
of zeros has scale 0 and codes 0).  A decoded element is code * scale (FP32).

Decode attention of one query row against a page: every head sees every
position; scores q.k / 8, softmax with the sink folded into the denominator
(src/kernels/attention/online.rs:145-149), in float64.
"""

from __future__ import annotations

import numpy as np

GROUP = 64


def quantize(x: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """x [positions][heads][64] FP32 -> codes [heads][positions][64] int8 and
    scales [heads][ceil(positions / 64)] FP32."""
    x = np.asarray(x, np.float32)
    p, h, d = x.shape
    xh = np.ascontiguousarray(x.transpose(1, 0, 2))  # [h][p][64]
    groups = (p + GROUP - 1) // GROUP
    pad = groups * GROUP - p
    xp = np.concatenate([xh, np.zeros((h, pad, d), np.float32)], axis=1) if pad else xh
    absmax = np.abs(xp.reshape(h, groups, GROUP * d)).max(axis=2)
    scales = (absmax / np.float32(127.0)).astype(np.float32)
    safe = np.where(scales > 0, scales, np.float32(1.0)).astype(np.float32)
    q = xp.reshape(h, groups, GROUP, d) / safe[:, :, None, None]
    codes = np.clip(np.rint(q), -127, 127).astype(np.int8)
    codes = np.where(scales[:, :, None, None] > 0, codes, 0).astype(np.int8)
    return codes.reshape(h, groups * GROUP, d)[:, :p], scales


def dequantize(codes: np.ndarray, scales: np.ndarray) -> np.ndarray:
    """-> [heads][positions][64] FP32 (code * scale)."""
    h, p, d = codes.shape
    s = np.repeat(scales, GROUP, axis=1)[:, :p]
    return (codes.astype(np.float32) * s[:, :, None]).astype(np.float32)


def decode(q: np.ndarray, k_codes, k_scales, v_codes, v_scales, sinks) -> np.ndarray:
    """One query row q [heads][64] -> output [heads][64] (float64 math)."""
    k = dequantize(k_codes, k_scales).astype(np.float64)
    v = dequantize(v_codes, v_scales).astype(np.float64)
    q = np.asarray(q, np.float64).reshape(k.shape[0], 64)
    s = np.einsum("hd,hpd->hp", q, k) / 8.0
    m = s.max(axis=1, keepdims=True)
    e = np.exp(s - m)
    den = e.sum(axis=1, keepdims=True)
    o = np.einsum("hp,hpd->hd", e, v) / den
    lse = m[:, 0] + np.log(den[:, 0])
    return (o / (1.0 + np.exp(np.asarray(sinks, np.float64) - lse))[:, None])
