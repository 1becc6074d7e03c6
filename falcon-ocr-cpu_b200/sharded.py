"""Head-sharded prefill of one long page over the ranks of a process group
(one process per GPU), with the output gathered over NCCL.

The page's KV groups are split evenly over the ranks: rank i computes the
query heads of its groups with the BF16 tensor-core prefill (no inter-GPU
traffic while it computes; each rank reads only its own heads' Q, K and V)
and the outputs meet in one all-gather.  The output is produced in bands of
query rows so that the gather of a finished band overlaps the computation of
the next: each band's kernel runs on the compute stream, and its all-gather is
issued on a separate stream that waits for that band's event.  Bands run
latest rows first: under a causal or prefix-LM mask later rows see more keys,
so the heavy band computes while nothing waits on it and the light band last
leaves the shortest gather exposed.  Each band
gathers into its own rank-major buffer ``[world][rows][heads_per_rank][64]``
(every rank's block contiguous, so the gather needs neither packing nor a
copy afterwards); ``token_major`` assembles ``[T][H][64]`` for a consumer
that wants it.

Peers' tiles reach a GPU only through NCCL into its own memory; no kernel
here reads another GPU's memory.

There is no counterpart in the reference, which prefills a page on one host;
the per-rank computation is ``kernels::attention_prefill_bf16``
(src/kernels/attention/mod.rs:321-349) on a subset of heads.
"""

from __future__ import annotations

from typing import Callable, Optional, Sequence

import torch
import torch.distributed as dist


def group_range(rank: int, world: int, n_kv_heads: int) -> tuple[int, int]:
    """KV groups [begin, end) of `rank`; the groups divide evenly."""
    if world < 1 or n_kv_heads % world:
        raise ValueError(f"{n_kv_heads} KV groups do not split over {world} ranks")
    per = n_kv_heads // world
    return rank * per, (rank + 1) * per


def bands(total: int, n_bands: int) -> list[tuple[int, int]]:
    """Query-row bands [begin, end) of about equal size, boundaries on
    multiples of 256 (the BF16 kernel's query-pair granularity)."""
    pairs = (total + 255) // 256
    n_bands = max(1, min(n_bands, pairs))
    out = []
    for i in range(n_bands):
        b = (pairs * i // n_bands) * 256
        e = min(total, (pairs * (i + 1) // n_bands) * 256)
        if e > b:
            out.append((b, e))
    return out


def token_major(band_buffers: Sequence[torch.Tensor]) -> torch.Tensor:
    """The bands' [world][rows][h][64] buffers as one [T][world * h][64]
    tensor (head w * h + j of a token comes from rank w)."""
    parts = [b.permute(1, 0, 2, 3).reshape(b.shape[1], b.shape[0] * b.shape[2], b.shape[3]) for b in band_buffers]
    return torch.cat(parts, 0)


def kv_splits_for(pairs: int, heads: int, sms: int) -> int:
    """Key ranges per query pair so that a launch of `pairs` x `heads` CTAs
    has at least one per SM (a rank holding few heads would otherwise wait on
    its longest pairs): the smallest power of two up to 8.  Measured on a
    16,384-token causal page: at 2 heads per rank (128 CTAs) two ranges take
    the rank from 0.184 to 0.109 ms; at 4 heads (256 CTAs) any split is slower
    (each range reloads its queries and a merge pass follows)."""
    k = 1
    while k < 8 and pairs * heads * k < sms:
        k *= 2
    return k


def cuda_band(q, kb, vb, sinks, geometry, heads, groups, begin, end, out, ctx=None, options=None, kv_splits=1):
    """The CUDA computation of one band on one rank (fo_attention_prefill_bf16_rows)."""
    import fo_cuda as F

    F.attention_prefill_bf16_rows(q, kb, vb, geometry, sinks, out, heads, groups, begin, end, options=options, ctx=ctx,
                                  kv_splits=kv_splits)


class ShardedPrefill:
    """The per-rank state of a head-sharded prefill: this rank's Q, BF16 K and
    V and sinks (its heads only), its output and the gathered output.

    `compute(q, kb, vb, sinks, geometry, heads, groups, begin, end, out)`
    fills rows [begin, end) of `out` ([T][heads][64]); the default is the
    CUDA kernel (a rank without a GPU fails loudly there)."""

    def __init__(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, sinks: torch.Tensor,
                 geometry: Sequence[int], n_heads: int, n_kv_heads: int, rank: int, world: int,
                 group: Optional[dist.ProcessGroup] = None, n_bands: int = 4,
                 compute: Optional[Callable] = None, out_dtype: torch.dtype = torch.bfloat16, ctx=None,
                 stream: Optional["torch.cuda.Stream"] = None, kv_splits: Optional[int] = None):
        """q [T][H][64], k [T][H][64], v [T][G][64] hold either the whole page
        (this rank slices its heads) or only this rank's heads.  On GPUs,
        `ctx` must be bound to `stream` (both are created when not given)."""
        g0, g1 = group_range(rank, world, n_kv_heads)
        hpg = n_heads // n_kv_heads
        self.heads, self.groups = (g1 - g0) * hpg, g1 - g0
        self.total = q.shape[0]
        self.rank, self.world, self.group = rank, world, group
        self.geometry = tuple(geometry)
        sl_h = slice(g0 * hpg, g1 * hpg) if q.shape[1] == n_heads else slice(None)
        sl_g = slice(g0, g1) if v.shape[1] == n_kv_heads else slice(None)
        self.q = q[:, sl_h].contiguous()
        self.kb = k[:, sl_h].to(torch.bfloat16).contiguous()
        self.vb = v[:, sl_g].to(torch.bfloat16).contiguous()
        self.sinks = (sinks[sl_h] if sinks.shape[0] == n_heads else sinks).contiguous()
        self.out = torch.empty(self.total, self.heads, 64, dtype=torch.float32, device=q.device)
        self.out_lp = torch.empty(self.total, self.heads, 64, dtype=out_dtype, device=q.device)
        self.bands = bands(self.total, n_bands)
        self.gathered = [torch.empty(world, e - b, self.heads, 64, dtype=out_dtype, device=q.device)
                         for b, e in self.bands]
        self.compute = compute or cuda_band
        self.cuda = q.is_cuda
        self.kv_splits = 1
        if self.cuda:
            # The kernels run on the context's stream; the gathers on their own.
            import fo_cuda as F

            if kv_splits is None:
                sms = torch.cuda.get_device_properties(q.device).multi_processor_count
                pairs = min((e - b + 255) // 256 for b, e in self.bands)
                kv_splits = kv_splits_for(pairs, self.heads, sms)

            self.kv_splits = kv_splits
            self.compute_stream = stream or torch.cuda.Stream(device=q.device)
            self.ctx = ctx or F.Context(q.device.index, stream=self.compute_stream.cuda_stream)
            self.comm_stream = torch.cuda.Stream(device=q.device)
        else:
            self.ctx = ctx

    def _gather(self, i: int, b: int, e: int) -> None:
        part = self.out_lp[b:e]
        if self.world == 1:
            self.gathered[i][0].copy_(part)
        elif self.cuda:
            dist.all_gather_into_tensor(self.gathered[i], part, group=self.group)
        else:
            dist.all_gather(list(self.gathered[i].unbind(0)), part.contiguous(), group=self.group)

    def run(self) -> list:
        """Computes this rank's heads band by band and gathers every band;
        returns the bands' rank-major buffers (complete for the caller's
        current stream on return)."""
        kwargs = {"ctx": self.ctx, "kv_splits": self.kv_splits} if self.compute is cuda_band else {}
        if not self.cuda:
            for i in reversed(range(len(self.bands))):
                b, e = self.bands[i]
                self.compute(self.q, self.kb, self.vb, self.sinks, self.geometry, self.heads, self.groups, b, e,
                             self.out, **kwargs)
                self.out_lp[b:e].copy_(self.out[b:e])
                self._gather(i, b, e)
            return self.gathered
        caller = torch.cuda.current_stream(self.q.device)
        self.compute_stream.wait_stream(caller)
        # The CUDA kernel stores BF16 rows itself (no conversion pass).
        direct = self.compute is cuda_band and self.out_lp.dtype == torch.bfloat16
        for i in reversed(range(len(self.bands))):
            b, e = self.bands[i]
            with torch.cuda.stream(self.compute_stream):
                self.compute(self.q, self.kb, self.vb, self.sinks, self.geometry, self.heads, self.groups, b, e,
                             self.out_lp if direct else self.out, **kwargs)
                if not direct:
                    self.out_lp[b:e].copy_(self.out[b:e])
                ev = torch.cuda.Event()
                ev.record(self.compute_stream)
            with torch.cuda.stream(self.comm_stream):
                self.comm_stream.wait_event(ev)
                self._gather(i, b, e)
        caller.wait_stream(self.compute_stream)
        caller.wait_stream(self.comm_stream)
        return self.gathered


def flops(total: int, n_heads: int, geometry: Sequence[int] = (0, 0, 0)) -> float:
    """Algorithmic FLOPs of a pure-prefix prefill: 4 * 64 per visible
    (query, key) pair per head."""
    _, image_start, image_end = geometry
    pairs = 0
    for t in range(total):
        pairs += image_end if image_start <= t < image_end else t + 1
    return 4.0 * 64 * pairs * n_heads
