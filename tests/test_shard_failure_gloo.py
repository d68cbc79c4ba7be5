"""Failure detection of the multi-GPU gather, on CPU ranks (gloo): when one rank dies or stalls
before handing over its heads, the ranks that wait for it must end their gather with an error
within the process group's timeout instead of hanging.  The failure is made on the host (a rank
that exits abruptly, or one that never enters the collective); nothing here touches a GPU.

The reference has no multi-GPU code; these cover the head-sharded gather of this build
(``shard.gather_to_root`` and the pipelined ``shard.compute_and_gather``).
"""
import datetime
import os
import socket
import time

import pytest
import torch
import torch.multiprocessing as mp

from usagi_b200 import shard

PG_TIMEOUT_S = 5  # short, so that a rank that waits for a stalled peer gives up quickly
N_HEADS, T, D = 4, 256, 128


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _report_and_exit(q, item):
    """Hand the result to the test and leave without tearing the process group down (its
    destructor may wait for the peer that is gone)."""
    q.put(item)
    q.close()
    q.join_thread()
    os._exit(0)


def _worker(rank, world, port, q, failure, path):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=PG_TIMEOUT_S))
    s0, s1 = shard.shard_range(N_HEADS, world, rank)
    local = torch.full((s1 - s0, T, D), float(rank + 1), dtype=torch.float16)
    dist.barrier()  # every rank is up; the failure below happens between steps
    if rank == world - 1:
        if failure == "exit":
            os._exit(3)  # dies without a word
        time.sleep(2 * PG_TIMEOUT_S)  # alive, but never enters the gather
        os._exit(0)
    t0 = time.monotonic()
    try:
        if path == "collective":
            shard.gather_to_root(local, N_HEADS, world, rank)
        else:
            root = torch.zeros((N_HEADS, T, D), dtype=torch.float16) if rank == 0 else None

            def compute_chunk(c, a, b, dst):
                dst.copy_(local[a:b])

            works = shard.compute_and_gather(compute_chunk, 2, N_HEADS, world, rank, root,
                                             None if rank == 0 else local)
            for w in works:
                w.wait()
        _report_and_exit(q, (rank, "completed", time.monotonic() - t0))
    except Exception as e:  # noqa: BLE001 - the error itself is what the test checks
        _report_and_exit(q, (rank, type(e).__name__, time.monotonic() - t0))


@pytest.mark.parametrize("failure", ["exit", "stall"])
@pytest.mark.parametrize("path", ["collective", "pipelined"])
def test_gather_ends_with_an_error_when_a_rank_is_gone(failure, path):
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q, failure, path))
             for r in range(world)]
    for p in procs:
        p.start()
    try:
        rank, outcome, elapsed = q.get(timeout=120)
    finally:
        for p in procs:
            p.join(timeout=2 * PG_TIMEOUT_S + 10)
            if p.is_alive():
                p.kill()  # the exact child this test started
                p.join()
    print(f"{failure}/{path}: rank 0 ended with {outcome} after {elapsed:.1f} s")
    assert rank == 0
    assert outcome != "completed", "rank 0 finished a gather whose peer never sent its heads"
    # The error arrives no later than about the process group's timeout (gloo reports a peer
    # that exited as soon as its connection closes, a stalled one when the timeout runs out).
    assert elapsed < 6 * PG_TIMEOUT_S, (outcome, elapsed)
