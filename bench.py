"""Benchmark of the B200 attention hot path (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Headline: full-page prefill attention, 6,544 tokens =
4,096-token bidirectional image prefix + 2,448 causal text tokens, 16 query
heads and 8 KV heads of 64, Q/K ~ N(0, 0.5) with RoPE, V ~ N(0, 1), through
fo_attention_prefill_bf16 (tcgen05, static-shift softmax: the reference's
fast-mode default).  A step is one prefill of one page; `value` is tokens/s
over all ranks with inputs resident in HBM (6 distinct input sets rotate, so
every step reads from DRAM, not L2).  `e2e` times the same call with FP32
host buffers (pinned): H2D of Q/K/V, BF16 conversion, attention, D2H of the
output.  `decode` times 5-row speculative-verify decode
at 16,384 KV positions over BF16 and FP32 split records, rotating over more
than 4x L2 of distinct caches.  Pages shard across ranks with no collective
on the data path (weak scaling); timing is the max over ranks of CUDA-event
time, bracketed by barriers and synchronizes.

--impl reference times the reference's algorithm on the host cores instead:
the reference's production CPU kernels restated in C with the same x86
vector instructions (oracle/fo_cpu_simd.c: AVX-512 BF16 static-shift prefill
tiles on all logical cores, AVX2 verify decode over F32 records on the
physical cores), since the Rust reference cannot be built here.  Prefill
pages and decode steps interleave; each reports the median.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "falcon-ocr-cpu_b200"))
sys.path.insert(0, os.path.join(ROOT, "tests", "golden"))

METRIC = "prefill attn tok/s @6,544 ctx; decode attn µs/step @16,384 KV; % of roofline"
SEQ, IMAGE_END, HEADS, KV_HEADS = 6544, 4096, 16, 8
# Visible (query, key) pairs per head: 4096^2 + sum_{t=4097}^{6544} t.
VISIBLE_PAIRS = IMAGE_END * IMAGE_END + sum(range(IMAGE_END + 1, SEQ + 1))
FLOP_PER_CALL = 4 * 64 * VISIBLE_PAIRS * HEADS  # QK and PV multiply-adds, 2 FLOP each
DECODE_L, DECODE_ROWS = 16384, 5
SHARDED_T = 16384  # C5b page
C4_L, C4_PAGES = 16384, 8
# Prefix record bytes per position, all groups, codes and BF16 scales (tail
# records are smaller: TAIL_BYTES per group).
RECORD_BYTES = {"bf16": 8 * 160 * 2, "f32": 8 * 160 * 4, "q8": 8 * (160 + 10), "q8r": 8 * (160 + 10),
                "q4r": 8 * (80 + 10)}
TAIL_BYTES = {"bf16": 256, "f32": 512, "q8": 136, "q8r": 136, "q4r": 72}


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            p = json.load(f)
        return {"hbm_gbs": p["hbm_gbs"], "bf16_tflops": p["bf16_tflops"],
                "bf16_tflops_sustained": p.get("bf16_tflops_sustained"), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


def load_traffic():
    """Per-launch DRAM bytes from the committed ncu summaries (or None)."""
    path = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(path):
        with open(path) as f:
            return json.load(f)
    return {}


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.device), f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.thread.join(timeout=2)
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax = float(parts[2])
            except ValueError:
                continue
            for name, flag in zip(names, parts[5:9]):
                if flag.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax, "samples": len(sm),
                "reasons": sorted(reasons)}


def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def host_cores():
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


# ------------------------------------------------------------------ CPU arm
CPU_SAMPLE_S = 10.0  # the cpu_baseline leg repeats whole pages for at least this long


def bench_config(world):
    """The workload both arms time (identical config keys and values)."""
    return {"workload": "C2 full-page prefill attention, 6,544 tokens (4,096 image + 2,448 text), 16 heads x 64, "
                        "8 KV heads, BF16 static-shift softmax, one page per step",
            "global_batch": world, "seq_len": SEQ, "parallelism": f"pages x{world}",
            "l2": "inputs rotate over more than 3x L2"}


class CpuReference:
    """The reference's CPU path on the host cores: oracle/fo_cpu_simd.c (its
    production SIMD kernels restated with the same instructions; bitwise
    equal to the scalar restatement, tests/test_cpu_baseline.py).  Prefill:
    BF16 static-shift tiles (AVX-512 BF16) over all logical cores, or the
    scalar restatement when the host lacks AVX512-BF16.  Decode: 5-row verify
    over F32 split records at 16,384 positions (AVX2) on the physical cores,
    as the reference's thread policy has it."""

    def __init__(self):
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import cpu_simd as C
        import generators as G
        import oracle as O
        self.C, self.O = C, O
        self.host = C.host_description()
        self.logical = C.max_threads()
        self.physical = self.host.get("physical") or self.logical
        self.q, self.k, self.v, self.sinks, _ = G.c2_inputs(seed=1)
        self.out = np.empty(self.q.size, np.float32)
        self.simd = C.has_bf16()
        rng = np.random.default_rng(2)
        p = DECODE_L - DECODE_ROWS
        kp = rng.standard_normal((p, HEADS, 64)).astype(np.float32)
        kp[:, 1::2, :32] = kp[:, 0::2, :32]
        vp = rng.standard_normal((p, KV_HEADS, 64)).astype(np.float32)
        self.cache = O.SplitCache(kp, vp, p, DECODE_L, fmt=O.F32)
        tail = rng.standard_normal((DECODE_ROWS, KV_HEADS, 64)).astype(np.float32)
        for t in range(DECODE_ROWS):
            self.cache.push(tail[t], tail[t])
        self.dq = rng.standard_normal(DECODE_ROWS * HEADS * 64).astype(np.float32)
        self.ds = rng.standard_normal(HEADS).astype(np.float32)
        self.dout = np.empty(DECODE_ROWS * HEADS * 64, np.float32)
        self.decode_ok = C.has_avx2()

    def prefill_page(self):
        C = self.C
        C.set_threads(self.logical)
        t0 = time.perf_counter()
        if self.simd:
            C.prefill_bf16_static(self.q, self.k, self.v, HEADS, KV_HEADS, (0, IMAGE_END), self.sinks, self.out)
        else:
            self.O.prefill_bf16(self.q, self.k, self.v, HEADS, KV_HEADS, (0, IMAGE_END), self.sinks,
                                softmax_static=True)
        return time.perf_counter() - t0

    def decode_step(self):
        if not self.decode_ok:
            return None
        C = self.C
        C.set_threads(self.physical)
        t0 = time.perf_counter()
        C.decode_rows_f32(self.cache, self.dq, DECODE_ROWS, self.ds, self.dout)
        dt = time.perf_counter() - t0
        C.set_threads(self.logical)
        return dt

    def run(self, steps, warmup, min_seconds=0.0):
        """Interleaved prefill pages and decode steps: warmup of each, then
        at least `steps` of each (and at least min_seconds of prefill)."""
        for _ in range(warmup):
            self.prefill_page()
            self.decode_step()
        pre, dec = [], []
        while len(pre) < steps or sum(pre) < min_seconds:
            pre.append(self.prefill_page())
            d = self.decode_step()
            if d is not None:
                dec.append(d)
        return pre, dec

    def describe(self, pre, dec):
        med = statistics.median(pre)
        kind = "AVX-512 BF16 static-shift tiles" if self.simd else "scalar restatement (host lacks AVX512-BF16)"
        out = {"value": round(SEQ / med, 1), "unit": "tok/s", "cores": self.logical, "kind": "port",
               "sample": f"median of {len(pre)} interleaved full C2 pages ({med:.3f} s each, {sum(pre):.1f} s in "
                         f"all), {kind}, {self.logical} threads; C restatement of the reference's prefill64/bf16 "
                         f"kernels (oracle/fo_cpu_simd.c)",
               "host": {"model": self.host.get("model"), "logical": self.logical, "physical": self.physical,
                        "flags": self.host.get("flags")}}
        if dec:
            out["decode_us_per_step"] = round(statistics.median(dec) * 1e6, 1)
            out["decode_sample"] = (f"median of {len(dec)} interleaved C3 steps: 5 verify rows over F32 records at "
                                    f"{DECODE_L:,} positions, AVX2 pair_rows on {self.physical} threads")
        return out


def run_reference(args, world, rank):
    """--impl reference: the reference algorithm on the host cores (rank 0)."""
    if rank != 0:
        return
    ref = CpuReference()
    pre, dec = ref.run(args.steps, args.warmup)
    cpu = ref.describe(pre, dec)
    med = statistics.median(pre)
    value = SEQ / med
    line = {
        "metric": METRIC, "value": round(value, 1), "unit": "tok/s", "impl": "reference", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(med * 1e3, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic", "config": bench_config(world),
        "cpu_baseline": cpu,
        "e2e": {"value": round(value, 1), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    if dec:
        line["decode"] = {"f32": {"us_per_step": cpu["decode_us_per_step"]}, "kv_len": DECODE_L,
                          "rows": DECODE_ROWS}
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ GPU arm
class Runner:
    """One rank's device, context and timing helpers."""

    def __init__(self, world, rank, local):
        import torch
        import fo_cuda as F
        self.torch, self.F = torch, F
        self.world, self.rank, self.local = world, rank, local
        torch.cuda.set_device(local)
        self.dev = torch.device("cuda", local)
        if world > 1:
            import datetime
            import torch.distributed as dist
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=self.dev)
        self.ctx = F.Context(local)  # default stream: ordered with torch's allocations and events
        self.peaks = load_peaks()
        self.traffic = load_traffic()

    def barrier(self):
        self.torch.cuda.synchronize()
        if self.world > 1:
            import torch.distributed as dist
            dist.barrier()
        self.torch.cuda.synchronize()

    def max_over_ranks(self, x: float) -> float:
        if self.world == 1:
            return x
        import torch.distributed as dist
        t = self.torch.tensor([x], dtype=self.torch.float64, device=self.dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def timed(self, step, steps, clocks=False):
        """Device milliseconds of `steps` calls of step(i), max over ranks."""
        torch = self.torch
        sampler = ClockSampler(self.local) if clocks else None
        if sampler:
            sampler.start()
            time.sleep(0.3)
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        self.barrier()
        start.record()
        for i in range(steps):
            step(i)
        end.record()
        self.barrier()
        ms = self.max_over_ranks(start.elapsed_time(end))
        return ms, (sampler.stop() if sampler else None)

    def close(self):
        self.ctx.close()
        if self.world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


def prefill_inputs(rank):
    import generators as G
    return G.c2_inputs(seed=1 + rank)  # each rank prefills its own page


def time_prefill(run, args, inputs, n_sets):
    """Device time of the BF16 prefill with Q (FP32) and BF16 K/V resident."""
    torch, F = run.torch, run.F
    q, k, v, sinks, geo = inputs
    sets = []
    for i in range(n_sets):
        qd = torch.from_numpy(q).to(run.dev)
        if i:
            qd = qd * (1.0 + 1e-3 * i)
        kd, vd = torch.from_numpy(k).to(run.dev), torch.from_numpy(v).to(run.dev)
        sets.append(dict(q=qd.contiguous(), k=kd, v=vd, kb=kd.to(torch.bfloat16), vb=vd.to(torch.bfloat16),
                         out=torch.empty(SEQ * HEADS * 64, device=run.dev)))
    sd = torch.from_numpy(sinks).to(run.dev)
    opts = F.PrefillOptions(F.EXP_FAST, 0, F.SOFTMAX_STATIC, F.SOFTMAX_ONLINE)

    def step(i):
        s = sets[i % n_sets]
        F.attention_prefill_bf16(s["q"], s["k"], s["v"], geo, sd, s["out"], HEADS, KV_HEADS, keys_bf16=s["kb"],
                                 values_bf16=s["vb"], options=opts, ctx=run.ctx)

    for i in range(max(args.warmup, 3)):
        step(i)
    ms, clocks = run.timed(step, args.steps, clocks=True)
    ms_per_step = ms / args.steps
    achieved = FLOP_PER_CALL / (ms_per_step / 1e3) / 1e12
    peak = run.peaks["bf16_tflops"]
    roof = {"bound": "tensor", "achieved": round(achieved, 1), "peak": peak, "unit": "TFLOP/s",
            "frac": round(achieved / peak, 4), "traffic": run.traffic.get("prefill_bf16_static"),
            "note": f"{FLOP_PER_CALL / 1e9:.2f} GFLOP algorithmic per launch (476.83M visible scores x 256 FLOP); "
                    f"peak = {run.peaks['source']} burst bf16 (of measured)"}
    value = run.world * args.steps * SEQ / (ms / 1e3)
    del sets
    torch.cuda.empty_cache()
    return value, ms_per_step, roof, clocks


def time_e2e(run, args, inputs):
    """The same call through the C ABI with pinned FP32 host buffers: H2D of
    Q/K/V/sinks, BF16 conversion, attention, D2H of the output."""
    torch, F = run.torch, run.F
    q, k, v, sinks, geo = inputs
    qh = torch.from_numpy(q.reshape(-1)).pin_memory()
    kh = torch.from_numpy(k.reshape(-1)).pin_memory()
    vh = torch.from_numpy(v.reshape(-1)).pin_memory()
    oh = torch.empty(SEQ * HEADS * 64, dtype=torch.float32).pin_memory()
    sh = torch.from_numpy(sinks).clone()
    opts = F.PrefillOptions(F.EXP_FAST, 0, F.SOFTMAX_STATIC, F.SOFTMAX_ONLINE)

    def step(_):
        F.attention_prefill_bf16(qh, kh, vh, geo, sh, oh, HEADS, KV_HEADS, options=opts, ctx=run.ctx)

    for i in range(3):
        step(i)
    steps = max(3, min(args.steps, 20))
    ms, _ = run.timed(step, steps)
    ms /= steps
    h2d = (q.size + k.size + v.size + sinks.size) * 4
    return {"value": round(run.world * SEQ / (ms / 1e3), 1), "unit": "tok/s", "h2d_bytes_per_step": int(h2d),
            "d2h_bytes_per_step": int(SEQ * HEADS * 64 * 4), "ms_per_step": round(ms, 3)}


def time_e2e_fused(run, args):
    """The C2 page from the QKV projection's output: per step the rows
    [6,544][16*64 + 2*8*64] FP32 go host -> device (pinned), fo_qkv_prefix_rows
    splits, normalizes and rotates them into Q, K, V and the BF16 copies on
    the device, the BF16 prefill attends, and the output comes back.  The
    RoPE table [6,544][16][32] {cos, sin} is per-page state shared by every
    layer, so it stays resident (uploaded once, outside the timed region).
    Synthetic projection rows N(0, 1), seed 1; RoPE theta 10,000 by position."""
    torch, F = run.torch, run.F
    rng = np.random.default_rng(1)
    width = HEADS * 64 + 2 * KV_HEADS * 64
    qkv_h = torch.from_numpy(rng.standard_normal(SEQ * width).astype(np.float32)).pin_memory()
    inv = 10000.0 ** (-np.arange(32) * 2.0 / 64.0)
    ang = np.arange(SEQ)[:, None] * inv[None, :]
    rope = np.stack([np.cos(ang), np.sin(ang)], -1).astype(np.float32)  # [SEQ][32][2]
    rope_d = torch.from_numpy(np.repeat(rope[:, None], HEADS, axis=1).reshape(-1)).to(run.dev)
    sinks = torch.from_numpy(np.random.default_rng(2).standard_normal(HEADS).astype(np.float32)).to(run.dev)
    qkv_d = torch.empty(SEQ * width, device=run.dev)
    q = torch.empty(SEQ * HEADS * 64, device=run.dev)
    k, v = torch.empty_like(q), torch.empty(SEQ * KV_HEADS * 64, device=run.dev)
    kb = torch.empty(SEQ * HEADS * 64, dtype=torch.bfloat16, device=run.dev)
    vb = torch.empty(SEQ * KV_HEADS * 64, dtype=torch.bfloat16, device=run.dev)
    out = torch.empty_like(q)
    out_h = torch.empty(SEQ * HEADS * 64, dtype=torch.float32).pin_memory()
    opts = F.PrefillOptions(F.EXP_FAST, 0, F.SOFTMAX_STATIC, F.SOFTMAX_ONLINE)
    geo = (0, 0, IMAGE_END)

    def step(_):
        qkv_d.copy_(qkv_h, non_blocking=True)
        F.qkv_prefix_rows(qkv_d, rope_d, SEQ, q, k, v, kb, vb, ctx=run.ctx)
        F.attention_prefill_bf16(q, k, v, geo, sinks, out, HEADS, KV_HEADS, keys_bf16=kb, values_bf16=vb,
                                 options=opts, ctx=run.ctx)
        out_h.copy_(out, non_blocking=True)

    for i in range(3):
        step(i)
    steps = max(3, min(args.steps, 20))
    ms, _ = run.timed(step, steps)
    ms /= steps
    return {"value": round(run.world * SEQ / (ms / 1e3), 1), "unit": "tok/s", "ms_per_step": round(ms, 3),
            "h2d_bytes_per_step": int(SEQ * width * 4), "d2h_bytes_per_step": int(SEQ * HEADS * 64 * 4),
            "path": "QKV projection rows in: fo_qkv_prefix_rows + fo_attention_prefill_bf16 (BF16 static shift)",
            "gpu_launches_per_step": 2}


def time_c4(run, args):
    """C4: one decode row per page over 8 independent pages of 16,384
    positions, in one batched call: the reference's Q8 records (1,360 B per
    position) and BASELINE's INT8 format (int8 per head, FP32 scale per head
    and 64 positions; 2,048 B + scales per position).  BF16-valued queries,
    seed 3; two page sets rotate (> 2x L2 each step)."""
    torch, F = run.torch, run.F
    rng = np.random.default_rng(3 + run.rank)
    L, n_pages = C4_L, C4_PAGES
    out = {}
    stream = torch.cuda.Stream(device=run.dev)
    dctx = F.Context(run.local, stream=stream.cuda_stream)

    def bf16_round(x):
        return torch.from_numpy(x).to(torch.bfloat16).float()

    qs = [bf16_round(rng.standard_normal(HEADS * 64).astype(np.float32)).to(run.dev) for _ in range(n_pages)]
    ss = [torch.from_numpy(rng.standard_normal(HEADS).astype(np.float32)).to(run.dev) for _ in range(n_pages)]
    os_ = [torch.empty(HEADS * 64, device=run.dev) for _ in range(n_pages)]
    for fmt in ("q8", "int8"):
        sets = []
        for _ in range(2):
            pages = []
            for _ in range(n_pages):
                k = torch.randn(L, HEADS, 64, device=run.dev)
                v = torch.randn(L, HEADS if fmt == "int8" else KV_HEADS, 64, device=run.dev)
                if fmt == "q8":
                    k[:, 1::2, :32] = k[:, 0::2, :32]
                    pages.append(F.SplitPrefix.from_compact(k, v, L, L, fmt="q8", ctx=dctx))
                else:
                    pages.append(F.Int8Cache(k, v, ctx=dctx))
                del k, v
            sets.append(pages)
        torch.cuda.synchronize()

        def step(i):
            pages = sets[i % 2]
            if fmt == "q8":
                F.decode_batch(pages, qs, ss, os_)
            else:
                F.int8_decode_batch(pages, qs, ss, os_)

        with torch.cuda.stream(stream):
            for i in range(max(args.warmup, 3)):
                step(i)
            stream.synchronize()
            steps = max(args.steps, 20)
            start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            run.barrier()
            start.record(stream)
            for i in range(steps):
                step(i)
            end.record(stream)
            run.barrier()
        us = run.max_over_ranks(start.elapsed_time(end)) * 1e3 / steps
        if fmt == "q8":
            bytes_step = n_pages * L * 8 * (160 + 10)
        else:
            bytes_step = n_pages * (L * HEADS * 128 + 2 * HEADS * ((L + 63) // 64) * 4)
        gbs = bytes_step / (us * 1e-6) / 1e9
        out[fmt] = {"us_per_step": round(us, 2), "pages": n_pages, "kv_len": L, "rows": 1,
                    "bytes_per_step": int(bytes_step),
                    "format": "reference Q8 records (BF16 block scales)" if fmt == "q8"
                              else "BASELINE int8 (per head, FP32 scale per 64 positions)",
                    "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": run.peaks["hbm_gbs"],
                                 "unit": "GB/s", "frac": round(gbs / run.peaks["hbm_gbs"], 4),
                                 "traffic": run.traffic.get(f"c4_{fmt}")},
                    "gpu_launches_per_step": 2, "timing": "back-to-back batched calls (no host sync)"}
        for pages in sets:
            for c in pages:
                c.close()
        del sets
        torch.cuda.empty_cache()
    dctx.close()
    return out


def time_sharded(run, args):
    """C5b: one 16,384-token causal prefill (BF16 static shift, seed 4)
    sharded by KV group over the ranks through the C ABI.  With more than one
    rank the headline path is fo_sharded_prefill_bf16_peers: the kernels store
    every finished BF16 row into all ranks' registered blocks over NVLink
    (plain peer stores, overlapped with the computation), between two one-word
    NCCL barriers.  The NCCL all-gather path (fo_sharded_prefill_bf16: each
    band stored into this rank's slot, then all-gathered in place) is timed
    beside it.  Every rank builds the same page and keeps its own heads."""
    import generators as G
    import sharded as S
    torch, F = run.torch, run.F
    T = SHARDED_T
    q, k, v, sinks, geo = G.c2_inputs(seed=4, seq=T, image_end=0)
    qd = torch.from_numpy(q.reshape(T, HEADS, 64)).to(run.dev)
    kd = torch.from_numpy(k.reshape(T, HEADS, 64)).to(run.dev)
    vd = torch.from_numpy(v.reshape(T, KV_HEADS, 64)).to(run.dev)
    sd = torch.from_numpy(sinks).to(run.dev)
    g0, g1 = S.group_range(run.rank, run.world, KV_HEADS)
    h0, h1 = 2 * g0, 2 * g1
    h = h1 - h0
    q_r = qd[:, h0:h1].contiguous()
    kb_r = kd[:, h0:h1].to(torch.bfloat16).contiguous()
    vb_r = vd[:, g0:g1].to(torch.bfloat16).contiguous()
    s_r = sd[h0:h1].contiguous()
    uid = [F.nccl_unique_id() if run.rank == 0 else None]
    if run.world > 1:
        import torch.distributed as dist
        dist.broadcast_object_list(uid, src=0)
    comm = F.NcclComm(run.world, run.rank, uid[0], ctx=run.ctx)
    gathered = torch.empty(run.world * T * h * 64, dtype=torch.bfloat16, device=run.dev)
    n_bands = args.bands
    steps = max(3, min(args.steps, 20))

    def nccl_step(_):
        F.sharded_prefill_bf16(comm, q_r, kb_r, vb_r, geo, s_r, gathered, h, g1 - g0, n_bands=n_bands,
                               kv_splits=args.kv_splits, ctx=run.ctx)

    for i in range(max(args.warmup, 3)):
        nccl_step(i)
    ms_nccl, _ = run.timed(nccl_step, steps)
    ms_nccl /= steps
    ms, path, block, layout = ms_nccl, "nccl all-gather", None, S.bands(T, n_bands)
    peer_error = None
    if run.world > 1:
        # Registration exchanges handles collectively, then maps the peers'
        # buffers locally; every rank must succeed before any uses the path
        # (its barriers are collectives), else all keep the NCCL gather.
        try:
            block = F.PeerBlock(comm, gathered, ctx=run.ctx)
        except F.FoError as e:
            peer_error = str(e)
        if run.max_over_ranks(0.0 if block is not None else 1.0) > 0.0:
            if block is not None:
                block.close()
                block = None
            peer_error = peer_error or "another rank could not map the peers' buffers"

    if block is not None:

        def peer_step(_):
            F.sharded_prefill_bf16_peers(block, q_r, kb_r, vb_r, geo, s_r, h, g1 - g0, kv_splits=args.kv_splits,
                                         ctx=run.ctx)

        for i in range(max(args.warmup, 3)):
            peer_step(i)
        ms_peer, _ = run.timed(peer_step, steps)
        ms_peer /= steps
        ms, path, layout = ms_peer, "kernel peer stores (NVLink)", [(0, T)]
    flop = S.flops(T, HEADS, geo)
    # Parity of the gathered page (the headline path's) with the whole page
    # on one GPU (bitwise when both use one key range: every head's
    # arithmetic is the same).
    check = None
    if run.rank == 0:
        kb, vb = kd.to(torch.bfloat16), vd.to(torch.bfloat16)
        whole = torch.empty(T * HEADS * 64, device=run.dev)
        F.attention_prefill_bf16(qd, kd, vd, geo, sd, whole, HEADS, KV_HEADS, keys_bf16=kb, values_bf16=vb,
                                 ctx=run.ctx)
        parts, off = [], 0
        for b, e in layout:
            n = run.world * (e - b) * h * 64
            parts.append(gathered[off:off + n].view(run.world, e - b, h, 64))
            off += n
        got = S.token_major(parts).float()
        check = float((got - whole.view(T, HEADS, 64).to(torch.bfloat16).float()).abs().max().item())
    run.barrier()
    if block is not None:
        block.close()
    comm.close()
    gathered_bytes = T * HEADS * 64 * 2
    achieved = flop / (ms / 1e3) / 1e12
    out = {"workload": "C5b: 16,384-token causal prefill, heads sharded by KV group, BF16 output gathered on every "
                       "rank",
           "tokens": T, "ranks": run.world, "gather": path, "bands": len(layout),
           "kv_splits": args.kv_splits or "auto", "ms_per_step": round(ms, 4),
           "tok_per_s": round(T / (ms / 1e3), 1), "gflop": round(flop / 1e9, 1), "tflops": round(achieved, 1),
           "frac_of_world_peak": round(achieved / (run.world * run.peaks["bf16_tflops"]), 4),
           "gather_bytes": gathered_bytes, "max_abs_diff_vs_one_gpu": check}
    if run.world > 1:
        out["nccl_gather_ms_per_step"] = round(ms_nccl, 4)
    if peer_error:
        out["peer_gather_unavailable"] = peer_error
    del qd, kd, vd, gathered
    torch.cuda.empty_cache()
    return out


def time_decode(run, args, lengths=(DECODE_L,)):
    """5-row verify decode over BF16 and FP32 records at each cache length,
    and over the 8-bit, rotated 8-bit and rotated 4-bit records (Kv::Q8,
    Kv::Q8Rot, Kv::Q4Rot) at DECODE_L, rotating distinct caches (together
    more than 4x L2).  The K calls are
    captured once in a CUDA graph on the caches' own stream and replayed, so
    the device time is not bounded by the Python launch path (a serving loop
    replays a graph the same way).  Returns {length: {format: line}}."""
    torch, F = run.torch, run.F
    rng = np.random.default_rng(2 + run.rank)
    sd = torch.from_numpy(rng.standard_normal(HEADS).astype(np.float32)).to(run.dev)
    stream = torch.cuda.Stream(device=run.dev)
    dctx = F.Context(run.local, stream=stream.cuda_stream)
    l2 = getattr(torch.cuda.get_device_properties(run.dev), "L2_cache_size", 126 << 20) or (126 << 20)
    res = {}
    plan = [(n, f) for n in lengths for f in ("bf16", "f32")]
    if DECODE_L in lengths:
        plan += [(DECODE_L, f) for f in ("q8", "q8r", "q4r")]
    for length, fmt in plan:
        out = res.setdefault(length, {})
        p = length - DECODE_ROWS
        n_caches = max(2, -(-4 * l2 // (p * RECORD_BYTES[fmt])))
        kp = rng.standard_normal((p, HEADS, 64)).astype(np.float32)
        kp[:, 1::2, :32] = kp[:, 0::2, :32]
        vp = rng.standard_normal((p, KV_HEADS, 64)).astype(np.float32)
        kd, vd = torch.from_numpy(kp).to(run.dev), torch.from_numpy(vp).to(run.dev)
        tail = np.repeat(rng.standard_normal((DECODE_ROWS, KV_HEADS, 1, 64)).astype(np.float32), 2, axis=2)
        td = torch.from_numpy(tail.reshape(-1)).to(run.dev)
        torch.cuda.synchronize()
        caches = []
        for i in range(n_caches):
            kk = kd if i == 0 else kd * (1 + 1e-3 * i)
            torch.cuda.synchronize()
            c = F.SplitPrefix.from_compact(kk, vd, p, length, fmt=fmt, ctx=dctx)
            c.append(td, td)
            caches.append(c)
        torch.cuda.synchronize()
        del kd, vd
        qd = torch.from_numpy(rng.standard_normal(DECODE_ROWS * HEADS * 64).astype(np.float32)).to(run.dev)
        od = torch.empty_like(qd)
        torch.cuda.synchronize()

        def step(i):
            caches[i % n_caches].attention_decode_rows(qd, DECODE_ROWS, sd, od)

        for i in range(max(args.warmup, 3)):
            step(i)
        torch.cuda.synchronize()
        steps = max(args.steps, 50) if args.mode == "full" else args.steps
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            for i in range(steps):
                step(i)
        graph.replay()
        run.barrier()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            start.record()
            graph.replay()
            end.record()
        run.barrier()
        us = run.max_over_ranks(start.elapsed_time(end)) * 1e3 / steps
        bytes_step = p * RECORD_BYTES[fmt] + DECODE_ROWS * KV_HEADS * TAIL_BYTES[fmt]
        gbs = bytes_step / (us * 1e-6) / 1e9
        out[fmt] = {"us_per_step": round(us, 2), "rows": DECODE_ROWS, "kv_len": length,
                    "bytes_per_step": int(bytes_step),
                    "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": run.peaks["hbm_gbs"],
                                 "unit": "GB/s", "frac": round(gbs / run.peaks["hbm_gbs"], 4),
                                 "traffic": run.traffic.get(f"decode_{fmt}") if length == DECODE_L else None},
                    "caches_rotated": n_caches,
                    # the decode kernel (tensor-core for BF16 records, CUDA-core
                    # for the others) and its split-merge kernel
                    "gpu_launches_per_step": 2, "timing": "CUDA graph of the steps"}
        del graph
        for c in caches:
            c.close()
        torch.cuda.empty_cache()
    dctx.close()
    return res


FP32_NOMINAL_TFLOPS = 148 * 128 * 2 * 1.965e9 / 1e12  # 148 SMs x 128 FP32 FMA/clk x 1.965 GHz


PAGES = 64  # BASELINE config 5(a): independent pages, sharded by page
PAGE_STEPS = 2048  # single-row decode steps per page after its prefill


DRAFT_ROWS, DRAFT_CHAIN = 1500, 4  # verified positions (draft_head.rs's profile size), chain rows


def time_draft(run, args):
    """The draft head's int8 KV attention (draft_head.rs:548-759)
    over 1,500 verified positions and 4 FP32 chain rows, full and with the
    reference profile's windows of 1,024 and 256 positions: CUDA-event time
    of a graph of calls on the cache's stream, and the oracle restatement of
    the same call on one host core beside it."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    torch, F = run.torch, run.F
    rng = np.random.default_rng(6 + run.rank)
    keys = rng.standard_normal(DRAFT_ROWS * 512).astype(np.float32)
    values = rng.standard_normal(DRAFT_ROWS * 512).astype(np.float32)
    q = rng.standard_normal(1024).astype(np.float32)
    ck = rng.standard_normal(DRAFT_CHAIN * 512).astype(np.float32)
    cv = rng.standard_normal(DRAFT_CHAIN * 512).astype(np.float32)
    stream = torch.cuda.Stream(device=run.dev)
    dctx = F.Context(run.local, stream=stream.cuda_stream)
    kv = F.DraftKv(DRAFT_ROWS, ctx=dctx)
    kd, vd = torch.from_numpy(keys).to(run.dev), torch.from_numpy(values).to(run.dev)
    qd, ckd, cvd = (torch.from_numpy(x).to(run.dev) for x in (q, ck, cv))
    od = torch.empty(1024, device=run.dev)
    torch.cuda.synchronize()
    kv.push(kd, vd)
    ref = None
    if run.rank == 0:
        ref = O.DraftKv(DRAFT_ROWS)
        ref.push(keys, values)
    res = {"workload": f"draft-head int8 KV attention, {DRAFT_ROWS} verified positions + {DRAFT_CHAIN} chain rows, "
                       "16 heads x 64, 8 KV groups"}
    for window in (0, 1024, 256):
        n = DRAFT_ROWS if window == 0 else min(window, DRAFT_ROWS)
        with torch.cuda.stream(stream):
            for _ in range(3):
                kv.attend(qd, DRAFT_ROWS, od, window, ckd, cvd)
        stream.synchronize()
        steps = 200
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            for _ in range(steps):
                kv.attend(qd, DRAFT_ROWS, od, window, ckd, cvd)
        graph.replay()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            start.record()
            graph.replay()
            end.record()
        stream.synchronize()
        us = start.elapsed_time(end) * 1e3 / steps
        # codes and scales of n rows for keys and values, plus the chain rows
        nbytes = 8 * n * 2 * (64 + 4) + 2 * DRAFT_CHAIN * 512 * 4
        gbs = nbytes / (us * 1e-6) / 1e9
        line = {"us_per_call": round(us, 2), "positions": n, "bytes_per_call": nbytes,
                "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": run.peaks["hbm_gbs"], "unit": "GB/s",
                             "frac": round(gbs / run.peaks["hbm_gbs"], 4),
                             "note": "a cache this small is launch- and latency-bound: CTAs split the positions "
                                     "of each KV group, then the last one merges"},
                "gpu_launches_per_call": 1}
        if ref is not None:
            O.set_threads(1)
            t0, k = time.perf_counter(), 0
            while k < 20 or time.perf_counter() - t0 < 0.5:
                ref.attend(q, DRAFT_ROWS, window, ck, cv)
                k += 1
            line["cpu_baseline"] = {"value": round((time.perf_counter() - t0) / k * 1e6, 1), "unit": "us/call",
                                    "cores": 1, "kind": "port",
                                    "sample": f"{k} calls of the same attention (oracle restatement)"}
            O.set_threads(0)
        res[f"window_{window}" if window else "full"] = line
        del graph
    kv.close()
    dctx.close()
    return res


def time_pages(run, args):
    """BASELINE config 5(a): 64 independent pages, each a 6,544-token
    prefix-LM prefill (C2, BF16 static shift) and then 2,048 single-row
    decode steps against its own growing BF16 split cache (KV 6,545 ->
    8,592), pages round-robin over the ranks with no collective.  A step
    appends the new row to every page of the rank and decodes one row per
    page, as Model::decode_batch_next does per layer
    (src/model/mod.rs:760-852), through a batch plan (fo_kv_plan_*: the
    descriptors stay on the device and move on by one position per step), so
    the 2,048 steps run as 32 replays of a CUDA graph of 64 steps.  The caches
    are allocated and sealed from the pages' K/V before the timed region
    (allocation is not a per-page cost); the timed job is every prefill,
    append and decode of the rank's pages, device time max over ranks.
    Synthetic pages: C2's inputs (seed 4) with each GQA pair's temporal key
    half shared, as the split cache's records require."""
    import generators as G
    torch, F = run.torch, run.F
    mine = list(range(run.rank, PAGES, run.world))
    n = len(mine)
    q, k, v, sinks, geo = G.c2_inputs(seed=4)
    k = k.copy()
    k[:, 1::2, :32] = k[:, 0::2, :32]
    stream = torch.cuda.Stream(device=run.dev)
    pctx = F.Context(run.local, stream=stream.cuda_stream)  # a capturable stream
    qd, kd, vd = (torch.from_numpy(x).to(run.dev) for x in (q, k, v))
    kb, vb = kd.to(torch.bfloat16), vd.to(torch.bfloat16)
    sd = torch.from_numpy(sinks).to(run.dev)
    outs = [torch.empty(SEQ * HEADS * 64, device=run.dev) for _ in range(2)]
    opts = F.PrefillOptions(F.EXP_FAST, 0, F.SOFTMAX_STATIC, F.SOFTMAX_ONLINE)
    warm, chunk = 4, 64
    torch.cuda.synchronize()
    caches = [F.SplitPrefix.from_compact(kd, vd, SEQ, SEQ + PAGE_STEPS + warm, fmt="bf16", ctx=pctx) for _ in mine]
    rng = np.random.default_rng(40 + run.rank)
    row = rng.standard_normal((2, 1, KV_HEADS, 1, 64)).astype(np.float32)
    row = torch.from_numpy(np.repeat(row, 2, axis=3).reshape(2, -1)).to(run.dev)  # expanded K, V rows
    qrow = torch.from_numpy(rng.standard_normal(HEADS * 64).astype(np.float32)).to(run.dev)
    dec_out = torch.empty((n, HEADS * 64), device=run.dev)
    torch.cuda.synchronize()

    def prefill(i):
        F.attention_prefill_bf16(qd, kd, vd, geo, sd, outs[i & 1], HEADS, KV_HEADS, keys_bf16=kb, values_bf16=vb,
                                 options=opts, ctx=pctx)

    def new_plan():
        return F.BatchPlan(caches, [row[0]] * n, [row[1]] * n, [qrow] * n, [sd] * n, [dec_out[i] for i in range(n)])

    with torch.cuda.stream(stream):
        plan = new_plan()
        for i in range(warm):  # untimed: warm both paths, then give the tails back
            prefill(i)
            plan.step()
        plan.finish()
        for c in caches:
            c.truncate_tail(0)
        plan = new_plan()
    stream.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for _ in range(chunk):
            plan.step()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
    run.barrier()
    with torch.cuda.stream(stream):
        ev[0].record()
        for i in range(n):
            prefill(i)
        ev[1].record()
        for _ in range(PAGE_STEPS // chunk):
            graph.replay()
        ev[2].record()
    stream.synchronize()
    run.barrier()
    plan.finish()
    assert all(c.tail_len == PAGE_STEPS for c in caches)
    total_ms = run.max_over_ranks(ev[0].elapsed_time(ev[2]))
    prefill_ms = run.max_over_ranks(ev[0].elapsed_time(ev[1]))
    decode_ms = run.max_over_ranks(ev[1].elapsed_time(ev[2]))
    # per step the rank's decode reads every page's records once
    pos = sum(SEQ + s + 1 for s in range(PAGE_STEPS)) / PAGE_STEPS
    step_bytes = n * pos * RECORD_BYTES["bf16"]
    gbs = step_bytes / (decode_ms / PAGE_STEPS * 1e-3) / 1e9
    res = {"workload": f"C5a: {PAGES} pages x (C2 prefill + {PAGE_STEPS} single-row decode steps), BF16 cache, "
                       "pages round-robin over ranks, no collective",
           "pages_per_s": round(PAGES / (total_ms / 1e3), 2), "seconds": round(total_ms / 1e3, 4),
           "pages_per_rank": n, "prefill_ms": round(prefill_ms, 3), "decode_ms": round(decode_ms, 3),
           "decode_us_per_step": round(decode_ms * 1e3 / PAGE_STEPS, 2),
           "decode_roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": run.peaks["hbm_gbs"], "unit": "GB/s",
                               "frac": round(gbs / run.peaks["hbm_gbs"], 4),
                               "note": "record bytes of every page per step (prefix records 2,560 B per position; "
                                       "tail records counted at the same size)"},
           "gpu_launches": n + 3 * PAGE_STEPS, "scaling": "weak per page, strong per job",
           "note": "caches sealed before the timed region; per step one append (which also sets every page's "
                   "decode length), one decode and one merge launch (which moves every page's append index on), "
                   "replayed from a CUDA graph of 64 steps"}
    del graph
    for c in caches:
        c.close()
    pctx.close()
    del outs, dec_out
    torch.cuda.empty_cache()
    return res


def time_prefill_rows(run, args, inputs):
    """Secondary prefill rows of the C2 page: the FP32 exact tiles
    (fo_attention, platform-exact exp; bound by FP32 CUDA cores) and the
    reference probe's geometry (image_end 6,534: every row but the last ten
    bidirectional) on the BF16 static-shift tiles."""
    torch, F = run.torch, run.F
    q, k, v, sinks, geo = inputs
    qd, kd, vd = (torch.from_numpy(x).to(run.dev) for x in (q, k, v))
    kb, vb = kd.to(torch.bfloat16), vd.to(torch.bfloat16)
    sd = torch.from_numpy(sinks).to(run.dev)
    out = torch.empty(SEQ * HEADS * 64, device=run.dev)
    res = {}
    steps = max(3, min(args.steps, 10))

    def fp32(_):
        F.attention_with(qd, kd, vd, SEQ, geo, sd, out, HEADS, KV_HEADS, 64, ctx=run.ctx)

    for i in range(2):
        fp32(i)
    ms, _ = run.timed(fp32, steps)
    ms /= steps
    tf = FLOP_PER_CALL / (ms / 1e3) / 1e12
    res["fp32_exact"] = {"ms_per_step": round(ms, 4), "tok_per_s": round(SEQ / (ms / 1e3), 1),
                         "roofline": {"bound": "fp32", "achieved": round(tf, 1), "peak": round(FP32_NOMINAL_TFLOPS, 1),
                                      "unit": "TFLOP/s", "frac": round(tf / FP32_NOMINAL_TFLOPS, 4),
                                      "note": "peak = nominal FP32 FMA rate (no measured FP32 figure)"}}
    probe = (0, 0, 6534)
    pairs = 6534 * 6534 + sum(t + 1 for t in range(6534, SEQ))  # rows < 6534 see 6,534 keys, the rest t + 1
    flop = 4.0 * 64 * pairs * HEADS
    opts = F.PrefillOptions(F.EXP_FAST, 0, F.SOFTMAX_STATIC, F.SOFTMAX_ONLINE)

    def bf16_probe(_):
        F.attention_prefill_bf16(qd, kd, vd, probe, sd, out, HEADS, KV_HEADS, keys_bf16=kb, values_bf16=vb,
                                 options=opts, ctx=run.ctx)

    for i in range(3):
        bf16_probe(i)
    ms, _ = run.timed(bf16_probe, max(args.steps, 10))
    ms /= max(args.steps, 10)
    tf = flop / (ms / 1e3) / 1e12
    res["bf16_probe_geometry"] = {"image_end": 6534, "ms_per_step": round(ms, 4),
                                  "tok_per_s": round(SEQ / (ms / 1e3), 1), "gflop": round(flop / 1e9, 2),
                                  "roofline": {"bound": "tensor", "achieved": round(tf, 1),
                                               "peak": run.peaks["bf16_tflops"], "unit": "TFLOP/s",
                                               "frac": round(tf / run.peaks["bf16_tflops"], 4)}}
    return res


def compact_decode(d):
    """One length's decode lines, short enough that the whole JSON line's
    tail (where the decode headline sits) survives truncated logs."""
    out = {}
    for fmt, x in d.items():
        r = x["roofline"]
        out[fmt] = {"us_per_step": x["us_per_step"], "gbs": r["achieved"], "frac": r["frac"],
                    "bytes_per_step": x["bytes_per_step"]}
        if r.get("traffic"):
            out[fmt]["traffic"] = r["traffic"]
    any_line = next(iter(d.values()))
    out.update(rows=any_line["rows"], caches_rotated=any_line["caches_rotated"], timing=any_line["timing"])
    return out


def run_ours(args, world, rank, local):
    run = Runner(world, rank, local)
    inputs = prefill_inputs(rank)
    line = {"metric": METRIC, "value": None, "unit": "tok/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": None, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic", "config": bench_config(world)}
    extra, dec = {}, None
    if args.mode in ("full", "prefill"):
        value, ms_per_step, roof, clocks = time_prefill(run, args, inputs, 6 if args.mode == "full" else 1)
        line.update(value=round(value, 1), ms_per_step=round(ms_per_step, 4), roofline=roof, clocks=clocks,
                    gpu_launches=args.steps)
    if args.mode == "full":
        line["e2e"] = time_e2e(run, args, inputs)
        line["e2e_from_qkv"] = time_e2e_fused(run, args)
    if args.mode in ("full", "decode"):
        lengths = (DECODE_L, 6544, 12000) if args.mode == "full" else (DECODE_L,)
        dec = time_decode(run, args, lengths)
    if args.mode in ("full", "c4"):
        extra["decode_c4"] = time_c4(run, args)
    if args.mode in ("full", "sharded"):
        extra["sharded_prefill"] = time_sharded(run, args)
    if args.mode in ("full", "pages"):
        extra["pages"] = time_pages(run, args)
    if args.mode in ("full", "draft"):
        extra["draft"] = time_draft(run, args)
    if args.mode == "full":
        extra["prefill_rows"] = time_prefill_rows(run, args, inputs)
    cpu_decode_us = None
    if args.mode == "full" and rank == 0 and world == 1:
        ref = CpuReference()
        pre, cdec = ref.run(steps=8, warmup=1, min_seconds=CPU_SAMPLE_S)
        line["cpu_baseline"] = ref.describe(pre, cdec)
        cpu_decode_us = line["cpu_baseline"].get("decode_us_per_step")
    line.update(extra)
    if dec is not None:
        # The decode headline (BASELINE config 3 at 16,384 positions) goes last.
        if len(dec) > 1:
            line["decode_lengths"] = {str(n): compact_decode(dec[n]) for n in dec if n != DECODE_L}
        line["decode"] = dict(kv_len=DECODE_L, peak_gbs=run.peaks["hbm_gbs"], **compact_decode(dec[DECODE_L]))
        if cpu_decode_us is not None:
            line["decode"]["cpu_f32_us_per_step"] = cpu_decode_us
    if rank == 0:
        print(json.dumps(line), flush=True)
    run.close()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--kv-splits", type=int, default=0,
                    help="key ranges per query pair in the sharded prefill (0: chosen from the CTA count)")
    ap.add_argument("--bands", type=int, default=1,
                    help="query-row bands of the sharded prefill (C5b); one band measured fastest at 2 ranks")
    ap.add_argument("--mode", choices=["full", "prefill", "decode", "c4", "sharded", "pages", "draft"], default="full",
                    help="full: the contract line; prefill/decode: only that part (profiling runs)")
    args = ap.parse_args()
    world, rank, local = dist_setup()
    if args.impl == "reference":
        run_reference(args, world, rank)
    else:
        run_ours(args, world, rank, local)


if __name__ == "__main__":
    main()
