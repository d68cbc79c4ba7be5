"""shard.PeerGather on one GPU: two processes play rank 0 and rank 1 (gloo for the host side).

Rank 0 exports its output buffer through the library's IPC entry points; rank 1 maps it into its
own context.  Either rank 1 copies its finished chunks into rank 0's rows with copy-engine copies
(``run``), or rank 1's attention kernel writes its output tiles straight into those rows
(``run_fused`` with ``block_sparse_attn_fwd_into``).  Rank 0's stream waits on rank 1's
interprocess event.  Rank 0 then checks every head of the gathered output against its own
single-process computation of the whole problem, bit for bit.  On one GPU the writes stay in the
same memory, but the code path (export, open in the writing process's context, copies or kernel
stores through the mapping, event ordering, close) is the one the multi-GPU gather runs.  Nothing
in either process waits on the other inside a kernel: only memory and events are shared.
"""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q, mode, chunks):
    import torch.distributed as dist
    import usagi_b200 as ub
    from usagi_b200 import patterns as P
    from usagi_b200 import shard
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        dev = torch.device("cuda", 0)
        torch.cuda.set_device(dev)
        ub.setup(device="cuda:0")
        B, H, T = 1, 5, 2048  # 5 heads over 2 ranks: shards of 3 and 2
        pat = P.mixed_pattern(B, H, T)
        g = torch.Generator(device=dev).manual_seed(41)
        qq, kk, vv = [torch.randn(B, H, T, 128, generator=g, device=dev).half() for _ in range(3)]
        sq, sk, sv, srp, sci, _, (s0, s1) = shard.shard_problem(qq, kk, vv, pat.row_ptr,
                                                               pat.col_idx, None, world, rank)
        sq, sk, sv = sq.contiguous(), sk.contiguous(), sv.contiguous()
        srp, sci = srp.to(dev), sci.to(dev)
        n = s1 - s0
        lse = torch.empty((n, 1, T), device=dev)
        local = torch.empty((n, T, 128), device=dev, dtype=torch.float16) if rank else None

        def compute_chunk(c, a, b, dst):
            ub.block_sparse_attn_fwd(sq[a:b], sk[a:b], sv[a:b], srp[a:b], sci[a:b], None,
                                     out=dst.view(b - a, 1, T, 128), lse_out=lse[a:b])

        peer = shard.PeerGather((B * H, T, 128), torch.float16, B * H, world, rank, dev)
        ok = True
        for _ in range(2):  # twice: the buffer and the events are reused across calls
            if rank == 0:
                peer.root.fill_(float("nan"))
            torch.cuda.synchronize()
            dist.barrier()
            if mode == "fused":
                peer.run_fused(lambda ptr: ub.block_sparse_attn_fwd_into(
                    ptr, sq, sk, sv, srp, sci, None, lse_out=lse))
            else:
                peer.run(compute_chunk, chunks, local)
            torch.cuda.synchronize()
            dist.barrier()
            if rank == 0:
                ref, _ = ub.block_sparse_attn_fwd(qq, kk, vv, pat.row_ptr.to(dev),
                                                  pat.col_idx.to(dev), None)
                ok = ok and torch.equal(peer.root, ref.reshape(B * H, T, 128))
        ub.check_errors(dev)
        peer.close()
        if rank == 0:
            q.put(bool(ok))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("mode,chunks", [("copy", 1), ("copy", 2), ("fused", 1)])
def test_peer_gather_two_processes_one_gpu(mode, chunks):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q, mode, chunks)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    codes = [p.exitcode for p in procs]
    for p in procs:
        if p.is_alive():
            p.kill()
    assert codes == [0, 0], codes
    assert q.get(timeout=5) is True
