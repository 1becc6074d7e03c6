"""The head-sharded prefill through the C ABI (fo_sharded_prefill_bf16 over an
NCCL communicator from fo_nccl_comm_init), one process per GPU: every rank's
gathered page equals, bit for bit, the whole page computed on one GPU with
the same key-range split and rounded to BF16.  Needs two GPUs (skipped on
fewer)."""

import multiprocessing as mp

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

T, HEADS, GROUPS = 4096, 16, 8


def worker(rank, world, uid, kv_splits, bands, result):
    import fo_cuda as F
    import generators as G
    import sharded as S
    torch.cuda.set_device(rank)
    ctx = F.Context(rank)
    comm = F.NcclComm(world, rank, uid, ctx=ctx)
    try:
        q, k, v, sinks, geo = G.c2_inputs(seed=4, seq=T, image_end=2048)
        qd = torch.from_numpy(q.reshape(T, HEADS, 64)).cuda()
        kb = torch.from_numpy(k.reshape(T, HEADS, 64)).cuda().to(torch.bfloat16)
        vb = torch.from_numpy(v.reshape(T, GROUPS, 64)).cuda().to(torch.bfloat16)
        sd = torch.from_numpy(sinks).cuda()
        g0, g1 = S.group_range(rank, world, GROUPS)
        h0, h1 = 2 * g0, 2 * g1
        h = h1 - h0
        gathered = torch.empty(world * T * h * 64, dtype=torch.bfloat16, device="cuda")
        F.sharded_prefill_bf16(comm, qd[:, h0:h1].contiguous(), kb[:, h0:h1].contiguous(),
                               vb[:, g0:g1].contiguous(), geo, sd[h0:h1].contiguous(), gathered, h, g1 - g0,
                               n_bands=bands, kv_splits=kv_splits, ctx=ctx)
        whole = torch.empty(T * HEADS * 64, dtype=torch.bfloat16, device="cuda")
        F.attention_prefill_bf16_rows(qd.reshape(-1), kb.reshape(-1), vb.reshape(-1), geo, sd, whole, HEADS, GROUPS,
                                      0, T, ctx=ctx, kv_splits=kv_splits)
        torch.cuda.synchronize()
        parts, off = [], 0
        for b, e in S.bands(T, bands):
            n = world * (e - b) * h * 64
            parts.append(gathered[off:off + n].view(world, e - b, h, 64))
            off += n
        page = S.token_major(parts)
        same = torch.equal(page.view(torch.int16), whole.view(T, HEADS, 64).view(torch.int16))
        result.put((rank, bool(same)))
    finally:
        comm.close()
        ctx.close()


@pytest.mark.parametrize("kv_splits,bands", [(1, 3), (2, 2)])
def test_sharded_prefill_through_the_c_abi_equals_one_gpu(kv_splits, bands):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import fo_cuda as F
    world = 2
    uid = F.nccl_unique_id()
    ctx = mp.get_context("spawn")
    result = ctx.Queue()
    procs = [ctx.Process(target=worker, args=(r, world, uid, kv_splits, bands, result)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    codes = [p.exitcode for p in procs]
    for p in procs:
        if p.is_alive():
            p.kill()
    assert codes == [0] * world, codes
    got = dict(result.get(timeout=10) for _ in range(world))
    assert got == {r: True for r in range(world)}


def peer_worker(rank, world, uid, kv_splits, result):
    import fo_cuda as F
    import generators as G
    import sharded as S
    torch.cuda.set_device(rank)
    ctx = F.Context(rank)
    comm = F.NcclComm(world, rank, uid, ctx=ctx)
    block = None
    try:
        q, k, v, sinks, geo = G.c2_inputs(seed=5, seq=T, image_end=2048)
        qd = torch.from_numpy(q.reshape(T, HEADS, 64)).cuda()
        kb = torch.from_numpy(k.reshape(T, HEADS, 64)).cuda().to(torch.bfloat16)
        vb = torch.from_numpy(v.reshape(T, GROUPS, 64)).cuda().to(torch.bfloat16)
        sd = torch.from_numpy(sinks).cuda()
        g0, g1 = S.group_range(rank, world, GROUPS)
        h0, h1 = 2 * g0, 2 * g1
        h = h1 - h0
        args = (qd[:, h0:h1].contiguous(), kb[:, h0:h1].contiguous(), vb[:, g0:g1].contiguous(), geo,
                sd[h0:h1].contiguous())
        via_nccl = torch.empty(world * T * h * 64, dtype=torch.bfloat16, device="cuda")
        F.sharded_prefill_bf16(comm, *args, via_nccl, h, g1 - g0, n_bands=1, kv_splits=kv_splits, ctx=ctx)
        peers = torch.full((world * T * h * 64,), float("nan"), dtype=torch.bfloat16, device="cuda")
        block = F.PeerBlock(comm, peers, ctx=ctx)
        same_runs = []
        for _ in range(3):  # later calls overwrite the previous page behind the opening barrier
            F.sharded_prefill_bf16_peers(block, *args, h, g1 - g0, kv_splits=kv_splits, ctx=ctx)
            torch.cuda.synchronize()
            same_runs.append(torch.equal(peers.view(torch.int16), via_nccl.view(torch.int16)))
        whole = torch.empty(T * HEADS * 64, dtype=torch.bfloat16, device="cuda")
        F.attention_prefill_bf16_rows(qd.reshape(-1), kb.reshape(-1), vb.reshape(-1), geo, sd, whole, HEADS, GROUPS,
                                      0, T, ctx=ctx, kv_splits=kv_splits)
        torch.cuda.synchronize()
        page = S.token_major([peers.view(world, T, h, 64)])
        same_one = torch.equal(page.view(torch.int16), whole.view(T, HEADS, 64).view(torch.int16))
        result.put((rank, all(same_runs) and bool(same_one)))
    finally:
        if block is not None:
            block.close()
        comm.close()
        ctx.close()


@pytest.mark.parametrize("kv_splits", [1, 2])
def test_peer_store_gather_equals_the_nccl_gather_and_one_gpu(kv_splits):
    """fo_sharded_prefill_bf16_peers: the kernels store every row into all
    ranks' registered blocks over NVLink; three calls in a row give, bit for
    bit, the NCCL path's gathered page and the whole page on one GPU."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import fo_cuda as F
    world = 2
    uid = F.nccl_unique_id()
    ctx = mp.get_context("spawn")
    result = ctx.Queue()
    procs = [ctx.Process(target=peer_worker, args=(r, world, uid, kv_splits, result)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    codes = [p.exitcode for p in procs]
    for p in procs:
        if p.is_alive():
            p.kill()
    assert codes == [0] * world, codes
    got = dict(result.get(timeout=10) for _ in range(world))
    assert got == {r: True for r in range(world)}
