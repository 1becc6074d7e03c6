"""The head-sharded prefill's host logic on CPU ranks (gloo, world size 2
and 4): group ranges, row bands, the band-by-band all-gather and the
rank-major layout.  The per-rank computation is the CPU oracle here (the
checker); on GPUs it is the tcgen05 kernel."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import generators as G
import oracle as O
import sharded as S


def test_group_ranges_and_bands():
    assert [S.group_range(r, 4, 8) for r in range(4)] == [(0, 2), (2, 4), (4, 6), (6, 8)]
    with pytest.raises(ValueError):
        S.group_range(0, 3, 8)
    assert S.bands(16384, 4) == [(0, 4096), (4096, 8192), (8192, 12288), (12288, 16384)]
    assert S.bands(300, 4) == [(0, 256), (256, 300)]
    assert S.bands(1000, 1) == [(0, 1000)]


def test_key_range_splits_fill_the_gpu():
    """One CTA per SM at least, in powers of two up to 8: C5b's 64 query
    pairs on 148 SMs split only at 8 ranks (2 heads each)."""
    assert S.kv_splits_for(64, 16, 148) == 1
    assert S.kv_splits_for(64, 8, 148) == 1
    assert S.kv_splits_for(64, 4, 148) == 1
    assert S.kv_splits_for(64, 2, 148) == 2
    assert S.kv_splits_for(1, 2, 148) == 8


def oracle_band(q, kb, vb, sinks, geometry, heads, groups, begin, end, out):
    """Rows [begin, end) of the BF16 static-shift tiles on this rank's heads."""
    full = O.prefill_bf16(q.numpy().reshape(-1), kb.float().numpy().reshape(-1), vb.float().numpy().reshape(-1),
                          heads, groups, (geometry[1], geometry[2]), sinks.numpy(), softmax_static=True)
    out[begin:end] = torch.from_numpy(full.reshape(out.shape))[begin:end]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, result_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        q, k, v, s = (torch.from_numpy(x) for x in G.bf16_operands(300))
        geometry = (0, 5, 262)
        sp = S.ShardedPrefill(q.view(300, 16, 64), k.view(300, 16, 64), v.view(300, 8, 64), s, geometry, 16, 8, rank,
                              world, n_bands=2, compute=oracle_band, out_dtype=torch.float32)
        gathered = sp.run()
        np.save(os.path.join(result_dir, f"rank{rank}.npy"), S.token_major(gathered).numpy())
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_sharded_prefill_gathers_every_head(tmp_path, world):
    port = _free_port()
    mp.start_processes(_rank_main, args=(world, port, str(tmp_path)), nprocs=world, start_method="spawn")
    q, k, v, s = G.bf16_operands(300)
    whole = O.prefill_bf16(q, k, v, 16, 8, (5, 262), s, softmax_static=True).reshape(300, 16, 64)
    for rank in range(world):
        got = np.load(tmp_path / f"rank{rank}.npy").reshape(300, 16, 64)
        assert np.array_equal(got, whole), rank
