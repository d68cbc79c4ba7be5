"""Head sharding across the GPUs of one node (one process per GPU).

Every (batch, head) pair of block-sparse attention is independent, so a problem is split by
flattened head index bh = b*H + h into contiguous, near-equal ranges -- no exchange on the data
path.  When the caller wants all outputs on one device, ``gather_to_root`` collects the o shards
on rank 0 with one NCCL (or gloo, on CPU) collective.  The reference has no multi-GPU code; this
is the partitioning its (B*H, T/128) grid (kernels/v4_leaderboard_0740ms.py:166-167) implies.
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch

__all__ = ["shard_range", "shard_problem", "gather_to_root", "timed_gather_to_root",
           "chunk_range", "compute_and_gather", "PeerGather",
           "PeerGatherUnavailable"]


def shard_range(n: int, world: int, rank: int) -> Tuple[int, int]:
    """Contiguous [start, end) slice of n units for `rank`; sizes differ by at most one."""
    if world < 1 or not (0 <= rank < world):
        raise ValueError(f"bad world/rank {world}/{rank}")
    base, rem = divmod(n, world)
    start = rank * base + min(rank, rem)
    return start, start + base + (1 if rank < rem else 0)


def shard_problem(q, k, v, row_ptr, col_idx, seq_lens: Optional[torch.Tensor], world: int,
                  rank: int):
    """Slice one rank's heads out of a [B, H, T, D] problem.

    Returns (q, k, v, row_ptr, col_idx, seq_lens, (start, end)) where the tensors are shaped as a
    problem with B' = end - start heads of one "batch entry" each (H' = 1), so per-head seq_lens
    follow the heads they belong to.
    """
    B, H, T, D = q.shape
    start, end = shard_range(B * H, world, rank)
    n = end - start

    def heads(t):
        return t.reshape(B * H, *t.shape[2:])[start:end].reshape(n, 1, *t.shape[2:])

    def meta(t):
        if t.dim() == 1:  # one shared row for every head
            return t
        if t.dim() == 2:
            return t[start:end].reshape(n, 1, -1)
        return t.reshape(B * H, -1)[start:end].reshape(n, 1, -1)

    sl = None
    if seq_lens is not None:
        sl = seq_lens.reshape(B).repeat_interleave(H)[start:end].contiguous()
    return heads(q), heads(k), heads(v), meta(row_ptr), meta(col_idx), sl, (start, end)


def gather_to_root(o_shard: torch.Tensor, total_heads: int, world: int, rank: int,
                   group=None) -> Optional[torch.Tensor]:
    """Gather per-rank o shards ([n_r, ...] heads) into [total_heads, ...] on rank 0.

    Shards are padded to the largest shard so the collective sees equal sizes. Returns the
    gathered tensor on rank 0 and None elsewhere.  Every rank must call this.
    """
    import torch.distributed as dist
    per = -(-total_heads // world)
    flat = o_shard.reshape(o_shard.shape[0], -1)
    if flat.shape[0] < per:
        pad = torch.zeros((per - flat.shape[0], flat.shape[1]), dtype=flat.dtype, device=flat.device)
        flat = torch.cat([flat, pad], 0)
    flat = flat.contiguous()
    out_list = [torch.empty_like(flat) for _ in range(world)] if rank == 0 else None
    dist.gather(flat, gather_list=out_list, dst=0, group=group)
    if rank != 0:
        return None
    parts = []
    for r in range(world):
        s, e = shard_range(total_heads, world, r)
        parts.append(out_list[r][: e - s])
    return torch.cat(parts, 0).reshape(total_heads, *o_shard.shape[1:])


def timed_gather_to_root(o_shard: torch.Tensor, world: int, rank: int, device) -> float:
    """Device time (ms, max over ranks) of gathering every rank's o shard onto rank 0."""
    import torch.distributed as dist
    total = o_shard.shape[0] * world
    gather_to_root(o_shard, total, world, rank)  # warm-up (communicator setup)
    torch.cuda.synchronize(device)
    dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    gather_to_root(o_shard, total, world, rank)
    e1.record()
    torch.cuda.synchronize(device)
    t = torch.tensor([e0.elapsed_time(e1)], device=device, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def chunk_range(n: int, chunks: int, c: int) -> Tuple[int, int]:
    """[start, end) of chunk c when n units are cut into `chunks` contiguous near-equal pieces
    (empty pieces when n < chunks)."""
    return shard_range(n, chunks, c)


def compute_and_gather(compute_chunk, chunks: int, total_heads: int, world: int, rank: int,
                       root_out: Optional[torch.Tensor], local_out: Optional[torch.Tensor],
                       comm_stream=None, group=None) -> list:
    """Compute this rank's heads chunk by chunk and stream every finished chunk to rank 0 while
    the next one computes.

    ``compute_chunk(c, a, b, dst)`` enqueues, on the current stream, the computation of heads
    [a, b) of this rank's shard (``shard_range(total_heads, world, rank)``) into ``dst``, a
    [b - a, ...] view.  On rank 0, ``dst`` is the matching slice of ``root_out``
    ([total_heads, ...]): rank 0's own heads are written in place.  On the other ranks ``dst`` is
    a slice of ``local_out`` ([n_local, ...]); once the chunk's kernel has finished, a
    ``comm_stream`` waits for it and sends the slice to rank 0, which receives it directly into
    its place in ``root_out`` -- no gather buffer and no concatenation.  Every rank uses the same
    number of chunks, so chunk c of every rank travels in one NCCL group on rank 0.  Nothing
    waits on the host; returns the communication work handles (the caller synchronises the
    compute stream and ``comm_stream``).
    """
    import contextlib
    import torch.distributed as dist
    ref = root_out if rank == 0 else local_out
    on_gpu = ref is not None and ref.is_cuda  # gloo (CPU tensors): no streams, same protocol
    cur = torch.cuda.current_stream(ref.device) if on_gpu else None
    comm = (comm_stream if comm_stream is not None else torch.cuda.Stream(ref.device)) \
        if on_gpu else None
    on_comm = (lambda: torch.cuda.stream(comm)) if on_gpu else contextlib.nullcontext
    s0, s1 = shard_range(total_heads, world, rank)
    works = []
    for c in range(chunks):
        a, b = chunk_range(s1 - s0, chunks, c)
        if rank == 0:
            dst = root_out[s0 + a:s0 + b]
            ops = []
            for r in range(1, world):
                rs, re = shard_range(total_heads, world, r)
                ra, rb = chunk_range(re - rs, chunks, c)
                if rb > ra:
                    ops.append(dist.P2POp(dist.irecv, root_out[rs + ra:rs + rb], r, group))
            if ops:  # the receives do not depend on rank 0's own compute
                with on_comm():
                    works += dist.batch_isend_irecv(ops)
            if b > a:
                compute_chunk(c, a, b, dst)
        else:
            dst = local_out[a:b]
            if b > a:
                compute_chunk(c, a, b, dst)
                if on_gpu:
                    done = torch.cuda.Event()
                    done.record(cur)
                    comm.wait_event(done)
                with on_comm():
                    works += dist.batch_isend_irecv([dist.P2POp(dist.isend, dst, 0, group)])
    return works


class PeerGatherUnavailable(RuntimeError):
    """Raised on every rank when any rank could not map rank 0's buffer (the caller falls back to
    a kernel-based gather)."""


class PeerGather:
    """Rank 0's [total_heads, ...] output buffer, written by every rank, either with copy-engine
    peer copies of finished chunks (``run``) or directly by each rank's attention kernel
    (``run_fused``).

    Why not NCCL for the overlapped gather: NCCL moves data with kernels, and the attention
    kernel is persistent -- one CTA per SM holding the whole register file and most of shared
    memory -- so an NCCL kernel queued on another stream only runs between attention launches.
    A device-to-peer copy is a DMA on a copy engine and needs no SM, so it runs while the next
    chunk computes.  Rank 0 exports its buffer once with CUDA IPC (bsattn_ipc_export); every
    other rank maps it into its own device's context (bsattn_ipc_open, peer access over NVLink)
    and copies each finished chunk straight into its rows (bsattn_peer_copy).  Completion reaches
    rank 0 through one interprocess CUDA event per rank, which rank 0's stream waits on after a
    host barrier (gloo) that orders the event records before the waits.  Construct collectively
    on every rank after the NCCL process group exists; ``close`` collectively before freeing.
    """

    def __init__(self, shape, dtype, total_heads: int, world: int, rank: int, device):
        import ctypes
        import torch.distributed as dist
        from . import _lib
        self.lib = _lib.load()
        self.world, self.rank, self.total_heads = world, rank, total_heads
        self.device = torch.device(device)
        self.host = dist.new_group(backend="gloo")  # host-side ordering only
        self.row_bytes = 1
        for d in shape[1:]:
            self.row_bytes *= int(d)
        self.row_bytes *= torch.empty((), dtype=dtype).element_size()
        obj = [None]
        self.root = None
        self.remote = None  # rank != 0: mapped address of rank 0's buffer
        self.event = None
        err = ""
        if rank == 0:
            try:
                self.root = torch.empty(shape, dtype=dtype, device=self.device)
                handle = ctypes.create_string_buffer(64)
                off = ctypes.c_uint64(0)
                with torch.cuda.device(self.device):
                    rc = self.lib.bsattn_ipc_export(self.root.data_ptr(), handle, ctypes.byref(off))
                if rc != 0:
                    raise RuntimeError(f"bsattn_ipc_export: {_lib.strerror(rc)}")
                obj = [(handle.raw, off.value)]
            except Exception as e:  # noqa: BLE001 -- reported to every rank below
                err = f"rank 0: {e}"
        dist.broadcast_object_list(obj, src=0, group=self.host)
        handle = None
        if rank != 0 and obj[0] is not None:
            try:
                raw, self.offset = obj[0]
                ptr = ctypes.c_void_p(0)
                with torch.cuda.device(self.device):
                    rc = self.lib.bsattn_ipc_open(raw, self.offset, ctypes.byref(ptr))
                    if rc != 0:
                        raise RuntimeError(f"bsattn_ipc_open: {_lib.strerror(rc)}")
                    self.remote = ptr.value
                    self.event = torch.cuda.Event(interprocess=True)
                    self.event.record(torch.cuda.current_stream(self.device))
                    handle = self.event.ipc_handle()
            except Exception as e:  # noqa: BLE001
                err = f"rank {rank}: {e}"
        elif rank != 0:
            err = f"rank {rank}: no handle from rank 0"
        # Every rank learns whether every rank is set up, so all take the same path.
        status = [None] * world
        dist.all_gather_object(status, (err, handle), group=self.host)
        errors = [e for e, _ in status if e]
        if errors:
            if self.remote is not None:
                with torch.cuda.device(self.device):
                    self.lib.bsattn_ipc_close(self.remote, self.offset)
                self.remote = None
            dist.barrier(group=self.host)
            raise PeerGatherUnavailable("; ".join(errors))
        self.peer_events = []
        if rank == 0:
            with torch.cuda.device(self.device):
                self.peer_events = [torch.cuda.Event.from_ipc_handle(self.device, h)
                                    for _, h in status[1:]]
        self.comm = torch.cuda.Stream(self.device)

    def run(self, compute_chunk, chunks: int, local_out: Optional[torch.Tensor]) -> None:
        """One compute + gather: ``compute_chunk(c, a, b, dst)`` as in ``compute_and_gather``.
        Rank 0 computes into its rows of ``self.root``; the other ranks compute into
        ``local_out`` (contiguous [n_local, ...]) and push each finished chunk to rank 0 on the
        copy stream.  On return rank 0's current stream is ordered after every rank's copies (it
        waited on their events); the other ranks' current streams after their own copies."""
        import torch.distributed as dist
        from . import _lib
        cur = torch.cuda.current_stream(self.device)
        s0, s1 = shard_range(self.total_heads, self.world, self.rank)
        for c in range(chunks):
            a, b = chunk_range(s1 - s0, chunks, c)
            if b <= a:
                continue
            if self.rank == 0:
                compute_chunk(c, a, b, self.root[s0 + a:s0 + b])
                continue
            src = local_out[a:b]
            compute_chunk(c, a, b, src)
            done = torch.cuda.Event()
            done.record(cur)
            self.comm.wait_event(done)
            rc = self.lib.bsattn_peer_copy(self.remote + (s0 + a) * self.row_bytes, src.data_ptr(),
                                           (b - a) * self.row_bytes, self.comm.cuda_stream)
            if rc != 0:
                raise RuntimeError(f"bsattn_peer_copy: {_lib.strerror(rc)}")
        if self.rank != 0:
            self.event.record(self.comm)
            cur.wait_stream(self.comm)
        dist.barrier(group=self.host)  # every rank has recorded its event
        if self.rank == 0:
            for ev in self.peer_events:
                cur.wait_event(ev)

    def out_ptr(self) -> int:
        """Device address of this rank's rows ([n_local, ...] starting at its first head) in rank
        0's buffer, valid on this rank's GPU: rank 0's own memory, or the mapping of it."""
        s0, _ = shard_range(self.total_heads, self.world, self.rank)
        base = self.root.data_ptr() if self.rank == 0 else self.remote
        return base + s0 * self.row_bytes

    def run_fused(self, launch) -> None:
        """Compute and gather in one step: ``launch(ptr)`` enqueues, on the current stream, the
        computation of this rank's whole share with its output at device address ``ptr``
        (``out_ptr()``, e.g. through ``block_sparse_attn_fwd_into``).  On ranks other than 0
        that address is rank 0's memory, so each output tile crosses NVLink as the kernel's
        epilogue stores it, overlapped with the rest of the computation tile by tile, and no
        copy follows.  Ordering is as in ``run``: on return rank 0's current stream waits on
        every rank's interprocess event, recorded after its kernel."""
        import torch.distributed as dist
        cur = torch.cuda.current_stream(self.device)
        s0, s1 = shard_range(self.total_heads, self.world, self.rank)
        if s1 > s0:
            launch(self.out_ptr())
        if self.rank != 0:
            self.event.record(cur)
        dist.barrier(group=self.host)  # every rank has recorded its event
        if self.rank == 0:
            for ev in self.peer_events:
                cur.wait_event(ev)

    def close(self) -> None:
        """Unmap rank 0's buffer on the other ranks before rank 0 may free it (collective)."""
        import torch.distributed as dist
        torch.cuda.synchronize(self.device)
        if self.rank != 0 and self.remote is not None:
            with torch.cuda.device(self.device):
                self.lib.bsattn_ipc_close(self.remote, self.offset)
            self.remote = None
        dist.barrier(group=self.host)
