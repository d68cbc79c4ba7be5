"""Head sharding + gather-to-root host logic on 2 CPU ranks (gloo), checked with the oracle."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from usagi_b200 import patterns as P
from usagi_b200 import shard


def test_shard_range_partitions():
    for n in [1, 5, 32, 128, 129]:
        for world in [1, 2, 3, 4, 8]:
            spans = [shard.shard_range(n, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            assert all(spans[i][1] == spans[i + 1][0] for i in range(world - 1))
            sizes = [e - s for s, e in spans]
            assert max(sizes) - min(sizes) <= 1


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q, kind):
    import torch.distributed as dist
    from oracle.bsattn_oracle import attn_blockwise
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        if kind == "retrieval":
            B, H, T = 2, 3, 512
            pat = P.retrieval_pattern(B, H, T, 4, seed=1)
            sl = torch.tensor([512, 300], dtype=torch.int32)
        else:  # the scaling mix's head-dependent families; 4 heads over 3 ranks are uneven
            B, H, T = 1, 4, 2048
            pat = P.mixed_pattern(B, H, T)
            sl = None
        g = torch.Generator().manual_seed(0)
        qq, kk, vv = [torch.randn(B, H, T, 128, generator=g).half() for _ in range(3)]
        sq, sk, sv, srp, sci, ssl, (s0, s1) = shard.shard_problem(qq, kk, vv, pat.row_ptr,
                                                                  pat.col_idx, sl, world, rank)
        o_shard, _ = attn_blockwise(sq, sk, sv, srp, sci, ssl)
        full = shard.gather_to_root(o_shard.reshape(s1 - s0, T, 128), B * H, world, rank)
        if rank == 0:
            ref, _ = attn_blockwise(qq, kk, vv, pat.row_ptr, pat.col_idx, sl)
            q.put(float((full.reshape(B, H, T, 128) - ref).abs().max()))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,kind", [(2, "retrieval"), (3, "mixed")])
def test_sharded_oracle_gathers_to_full_result(world, kind):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q, kind)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    assert q.get(timeout=5) == 0.0


def _pipelined_worker(rank, world, port, q, chunks):
    import torch.distributed as dist
    from oracle.bsattn_oracle import attn_blockwise
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        B, H, T = 1, 5, 1024  # 5 heads over 3 ranks: shards of 2, 2, 1; some chunks are empty
        pat = P.mixed_pattern(B, H, T)
        g = torch.Generator().manual_seed(0)
        qq, kk, vv = [torch.randn(B, H, T, 128, generator=g).half() for _ in range(3)]
        sq, sk, sv, srp, sci, _, (s0, s1) = shard.shard_problem(qq, kk, vv, pat.row_ptr,
                                                               pat.col_idx, None, world, rank)

        def compute_chunk(c, a, b, dst):
            o, _ = attn_blockwise(sq[a:b], sk[a:b], sv[a:b], srp[a:b], sci[a:b], None)
            dst.copy_(o.reshape(b - a, T, 128))

        root = torch.full((B * H, T, 128), float("nan")) if rank == 0 else None
        local = torch.empty((s1 - s0, T, 128)) if rank != 0 else None
        works = shard.compute_and_gather(compute_chunk, chunks, B * H, world, rank, root, local)
        for w in works:
            w.wait()
        if rank == 0:
            ref, _ = attn_blockwise(qq, kk, vv, pat.row_ptr, pat.col_idx, None)
            q.put(float((root.reshape(B, H, T, 128) - ref).abs().max()))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("chunks", [1, 2, 3])
def test_pipelined_compute_and_gather_places_every_chunk(chunks):
    """compute_and_gather: each rank's chunks land in their own rows of rank 0's output (rank 0's
    own chunks computed in place), whatever the chunk count, including empty chunks."""
    world = 3
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_pipelined_worker, args=(r, world, port, q, chunks))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    assert q.get(timeout=5) == 0.0
