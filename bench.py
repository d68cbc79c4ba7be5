"""Benchmark: block-sparse causal attention forward on B200.

Metric: ms/call and live-block TFLOP/s at B=2, H=16, T=8192, D=128 against the
B200 fp16 tensor-core peak.  One *step* = one call for each of the three sparsity families
(sliding window 8, global prefix 4 + window 4, retrieval 8 random), fp16 inputs ~N(0,1),
synthetic (seeded) data.  ``value`` is whole-job live-block TFLOP/s = live tiles x 4*128^3 FLOP
summed over the three calls and all ranks, divided by the max-over-ranks device time.

Multi-GPU: one process per GPU (torchrun); every rank runs the same per-GPU workload on its own
(batch, head) shard -- B = 2 per rank of a global batch 2N -- with no collective on the data path
(weak scaling).  The optional NCCL gather of one family's o to rank 0 is timed separately
(``gather_ms``).

Every line also carries ``mix``: the head-sharded scaling configuration, one B=4, H=32, T=32768
problem whose heads cycle through window16 / prefix8+window8 / retrieval(2+16), its 128 (batch,
head) pairs split contiguously across the N ranks (strong scaling: the total work is fixed).  It
reports the kernel time (max over ranks) and the time until rank 0 holds every head, with each
rank's output tiles stored straight into rank 0's buffer over NVLink by the kernel's own epilogue
(the default, ``--mix-transport fused``), or its heads computed in chunks with every finished chunk
copied into rank 0's output while the next one computes (copy-engine peer copies with
``--mix-transport copy``, NCCL send/recv with ``--mix-transport nccl``), and rank 0's bit-exact check
of the first and last head of every rank's share.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload families|mix|dense] [--mix-transport fused|copy|nccl] [--no-mix]

``--workload mix`` prints the scaling configuration as its own line (with an end-to-end leg);
``--workload dense`` prints a comparison line: this kernel on dense causal attention next to torch
SDPA (cuDNN, flash) and flash_attn 2 on the same inputs.

``--impl reference`` times the reference's CPU path (the dense-masked fp32 restatement in
oracle/, the reference having no CPU implementation of its own) on the host cores, rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
import threading
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

FAMILIES = ["window8", "prefix4+window4", "retrieval8"]
B_PER_RANK, H, T, D = 2, 16, 8192, 128
METRIC = "ms/call + live-block TFLOP/s (B=2,H=16,T=8192,D=128) vs B200 fp16 TC peak"
FALLBACK_PEAKS = {"bf16_tflops": 1590.0, "hbm_gbs": 6650.0, "source": "fallback"}


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return {"bf16_tflops": float(d["bf16_tflops"]), "hbm_gbs": float(d["hbm_gbs"]),
                "source": "measured"}
    except Exception:
        return dict(FALLBACK_PEAKS)


def kernel_source_sha256() -> str:
    """sha256 over the kernel's source files (the capture in profiles/ names the one it measured)."""
    import hashlib
    h = hashlib.sha256()
    for name in ("bsattn_fwd.cu", "sm100_ptx.cuh"):
        with open(os.path.join(ROOT, "usagi_b200", "csrc", name), "rb") as f:
            h.update(f.read())
    return h.hexdigest()


def load_traffic():
    """Per-launch DRAM bytes of the kernel from the committed ncu summary, or None.  The summary
    carries the sha256 of the kernel source it was captured from; when the source has changed
    since, the number no longer describes this kernel and is not reported."""
    path = os.path.join(ROOT, "profiles", "bsattn_fwd_traffic.txt")
    try:
        out = {}
        with open(path) as f:
            for line in f:
                if ":" in line and not line.startswith("#"):
                    k, v = line.split(":", 1)
                    out[k.strip()] = v.strip()
    except Exception:
        return None
    if out.get("kernel_source_sha256") != kernel_source_sha256():
        return {"note": "stale: the committed DRAM capture was taken from another kernel source "
                        "(sha256 mismatch), so no traffic is reported"}
    return out


class ClockSampler:
    """Samples SM clock and throttle reasons while the timed region runs (NVML in a thread at a
    few-millisecond period; nvidia-smi as a fallback when NVML is unavailable)."""

    REASONS = {  # NVML clocks-event reason bits
        "hw_slowdown": 0x0000000000000008,
        "sw_thermal_slowdown": 0x0000000000000020,
        "hw_thermal_slowdown": 0x0000000000000040,
        "sw_power_cap": 0x0000000000000004,
    }

    def __init__(self, gpu_index: int, period_s: float = 0.002):
        self.gpu = gpu_index
        self.period = period_s
        self.samples = []
        self.max_mhz = None
        self._stop = threading.Event()
        self._thread = None
        self._nvml = None

    def __enter__(self):
        try:
            import pynvml
            pynvml.nvmlInit()
            self._nvml = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByIndex(self.gpu)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
            self._thread = threading.Thread(target=self._run_nvml, daemon=True)
            self._thread.start()
        except Exception:
            self._nvml = None
        return self

    def _run_nvml(self):
        pn = self._nvml
        getr = getattr(pn, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
            getattr(pn, "nvmlDeviceGetCurrentClocksThrottleReasons")
        while not self._stop.is_set():
            try:
                mhz = pn.nvmlDeviceGetClockInfo(self._h, pn.NVML_CLOCK_SM)
                reasons = getr(self._h)
                self.samples.append((mhz, reasons))
            except Exception:
                pass
            time.sleep(self.period)

    def __exit__(self, *a):
        self._stop.set()
        if self._thread is not None:
            self._thread.join(timeout=2)

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0,
                    "source": "nvml" if self._nvml else "unavailable"}
        reasons = set()
        for _, r in self.samples:
            for name, bit in self.REASONS.items():
                if r & bit:
                    reasons.add(name)
        return {"sm_mhz": statistics.median(m for m, _ in self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(reasons), "samples": len(self.samples), "source": "nvml"}


def numa_info(gpu_index: int) -> dict:
    """NUMA node of the GPU (sysfs, through its PCI bus id) and of the CPUs this process may run
    on: where pinned host buffers land relative to the GPU's PCIe root."""
    out = {"gpu_numa_node": None, "process_cpu_numa_nodes": None}
    try:
        import pynvml
        pynvml.nvmlInit()
        bus = pynvml.nvmlDeviceGetPciInfo(pynvml.nvmlDeviceGetHandleByIndex(gpu_index)).busId
        bus = bus.decode() if isinstance(bus, bytes) else bus
        dom, rest = bus.lower().split(":", 1)
        path = f"/sys/bus/pci/devices/{dom[-4:]}:{rest}/numa_node"
        with open(path) as f:
            out["gpu_numa_node"] = int(f.read().strip())
    except Exception:
        pass
    try:
        cpus = os.sched_getaffinity(0)
        nodes = set()
        base = "/sys/devices/system/node"
        for name in os.listdir(base):
            if not name.startswith("node"):
                continue
            with open(os.path.join(base, name, "cpulist")) as f:
                spec = f.read().strip()
            ids = set()
            for part in spec.split(","):
                if "-" in part:
                    a, b = part.split("-")
                    ids.update(range(int(a), int(b) + 1))
                elif part:
                    ids.add(int(part))
            if ids & cpus:
                nodes.add(int(name[4:]))
        out["process_cpu_numa_nodes"] = sorted(nodes)
    except Exception:
        pass
    return out


def make_inputs(device):
    """q, k, v of the benchmark configurations: B=2, H=16, T=8192, D=128,
    N(0,1) fp32 from CPU seed 0 drawn in the order q, k, v, cast to fp16.  The three families use
    these same tensors, and they are the draw the full-size reference fixtures were made from
    (tests/golden/cases.full_inputs).  Every rank holds the same problem (weak scaling)."""
    g = torch.Generator().manual_seed(0)
    shape = (B_PER_RANK, H, T, D)
    return [torch.randn(shape, generator=g).half().to(device) for _ in range(3)]


def cpu_reference_throughput(budget_s: float, threads: int):
    """Dense-masked fp32 CPU path on a bounded sample of the same workload.

    Runs whole heads of the three families (B=2, H=16, T=8192) round-robin until ``budget_s``
    elapsed (at least one head per family); returns live-block TFLOP/s of the sampled heads.
    """
    from oracle.bsattn_oracle import attn_dense_masked
    from usagi_b200 import patterns as P
    torch.set_num_threads(threads)
    pats = {f: P.family_pattern(f, B_PER_RANK, H, T) for f in FAMILIES}
    g = torch.Generator().manual_seed(7)
    q = torch.randn(1, 1, T, D, generator=g)
    k = torch.randn(1, 1, T, D, generator=g)
    v = torch.randn(1, 1, T, D, generator=g)
    flops, n_heads, t_used, per_fam = 0, 0, 0.0, {f: 0 for f in FAMILIES}
    t_start = time.perf_counter()
    i = 0
    while True:
        fam = FAMILIES[i % len(FAMILIES)]
        bh = (i // 3) % (B_PER_RANK * H)
        pat = pats[fam]
        rp = pat.row_ptr.reshape(-1, T // 128 + 1)[bh:bh + 1].reshape(1, 1, -1)
        ci = pat.col_idx.reshape(B_PER_RANK * H, -1)[bh:bh + 1].reshape(1, 1, -1)
        t0 = time.perf_counter()
        attn_dense_masked(q, k, v, rp, ci)
        t_used += time.perf_counter() - t0
        n = rp.reshape(-1).to(torch.int64)
        lens = n[1:] - n[:-1]
        flops += int(((lens - 1).clamp(min=0) + 1).sum()) * 4 * 128 ** 3
        n_heads += 1
        per_fam[fam] += 1
        i += 1
        if i >= len(FAMILIES) and time.perf_counter() - t_start >= budget_s:
            break
    tflops = flops / t_used / 1e12
    return {
        "value": tflops,
        "unit": "TFLOP/s",
        "cores": threads,
        "kind": "port",
        "sample": (f"dense-masked fp32 torch CPU path (oracle/bsattn_oracle.attn_dense_masked) on "
                   f"{n_heads} whole heads (T=8192) of the 3 families ({per_fam}); "
                   f"{t_used:.1f}s; live-block FLOPs of the sampled heads / CPU time"),
        "ms_per_head": 1e3 * t_used / n_heads,
        "heads": n_heads,
        "seconds": t_used,
    }


def cpu_config0(threads: int, reps: int = 5) -> dict:
    """The reference's CPU-runnable configuration itself: B=1, H=2, T=1024, D=128, window of 4
    blocks, q, k, v ~ N(0,1) fp32 from seed 0 (drawn in q, k, v order), through the same
    dense-masked fp32 path; median of `reps` warm calls."""
    from oracle.bsattn_oracle import attn_dense_masked
    from usagi_b200 import patterns as P
    torch.set_num_threads(threads)
    g = torch.Generator().manual_seed(0)
    q, k, v = [torch.randn(1, 2, 1024, D, generator=g) for _ in range(3)]
    pat = P.window_pattern(1, 2, 1024, 4, shared=False)
    attn_dense_masked(q, k, v, pat.row_ptr, pat.col_idx)  # first call: allocation, threads
    ts = []
    for _ in range(reps):
        t0 = time.perf_counter()
        attn_dense_masked(q, k, v, pat.row_ptr, pat.col_idx)
        ts.append(time.perf_counter() - t0)
    ms = 1e3 * statistics.median(ts)
    flops = pat.live_blocks() * 4 * 128 ** 3
    return {"config": "B=1,H=2,T=1024,D=128, window 4, fp32, seed 0 (BASELINE config 0)",
            "ms_per_call": ms, "value": flops / (ms * 1e-3) / 1e12, "unit": "TFLOP/s",
            "live_blocks": pat.live_blocks(), "cores": threads, "reps": reps}


def run_reference(args, rank, world):
    """The reference arm: the reference's CPU path (its dense-masked fp32 restatement in
    oracle/) on the host cores, rank 0 only.  A step is a bounded sample of the 3-family step:
    whole heads, round robin over the families, for about --ref-budget seconds (at least one head
    of each); its value is the sample's live-block FLOPs over its CPU time, and ms_per_step is
    the measured wall time of that sample -- not a full 96-head step, which would take ~15 s."""
    if rank != 0:
        return 0
    threads = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count()
    per_step, wall = [], []
    base = None
    # keep the whole --steps/--warmup run within a few minutes of CPU time
    budget = min(args.ref_budget, 150.0 / (args.warmup + args.steps))
    for s in range(args.warmup + args.steps):
        t0 = time.perf_counter()
        r = cpu_reference_throughput(budget_s=budget if s >= args.warmup else 0.0, threads=threads)
        if s >= args.warmup:
            per_step.append(r)
            wall.append(time.perf_counter() - t0)
        base = r
    vals = [r["value"] for r in per_step]
    v = statistics.median(vals)
    heads = statistics.median(r["heads"] for r in per_step)
    line = {
        "impl": "reference",
        "metric": METRIC,
        "value": v,
        "unit": "TFLOP/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": 1e3 * statistics.median(wall),
        "ms_per_step_note": (f"measured wall time of one sampled step: about {heads:.0f} of the "
                             f"{3 * B_PER_RANK * H} heads of a 3-family step (whole heads, round "
                             "robin over the families); value is the sample's live-block FLOPs "
                             "over its CPU time"),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic (seeded N(0,1))",
        "config": {"workload": "3 families (window8, prefix4+window4, retrieval8) B=2,H=16,T=8192,D=128",
                   "parallelism": "host cores, rank 0 only"},
        "cpu_baseline": {"value": v, "unit": "TFLOP/s", "cores": base["cores"], "kind": "port",
                         "sample": base["sample"], "config0": cpu_config0(threads)},
        "e2e": {"value": v, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


_FLOPS_CACHE = {}


def _pattern_flops(fam):
    from usagi_b200 import patterns as P
    if fam not in _FLOPS_CACHE:
        _FLOPS_CACHE[fam] = P.family_pattern(fam, B_PER_RANK, H, T).live_blocks() * 4 * 128 ** 3
    return _FLOPS_CACHE[fam]


MIX_B, MIX_H, MIX_T = 4, 32, 32768
MIX_METRIC = ("ms/call + live-block TFLOP/s, head-sharded scaling mix (B=4,H=32,T=32768,D=128) "
              "vs B200 fp16 TC peak")


def init_distributed(world, device):
    """NCCL process group for world > 1.  NCCL announces itself on stdout when the communicator is
    created; that goes to stderr so stdout carries only the JSON line."""
    import datetime
    import torch.distributed as dist
    if world <= 1:
        return
    sys.stdout.flush()
    saved_fd = os.dup(1)
    os.dup2(2, 1)
    try:
        dist.init_process_group("nccl", device_id=device, timeout=datetime.timedelta(seconds=120))
        dist.barrier()
        torch.cuda.synchronize()
    finally:
        sys.stdout.flush()
        os.dup2(saved_fd, 1)
        os.close(saved_fd)


MIX_CHUNKS = 4  # chunks per rank in the pipelined compute + gather of the scaling mix


def measure_mix(args, rank, world, device, peaks):
    """The head-sharded scaling configuration, strong scaling over the N ranks.

    One B=4, H=32, T=32768 problem (heads cycle window16 / prefix8+window8 / retrieval 2+16); its
    128 (batch, head) pairs are split contiguously across the ranks.  Two measurements:
      * kernel: one call per rank on its whole share; ms = max over ranks of the device time;
      * kernel + gather: ms = max over ranks from the first launch until rank 0 holds every
        head in its [B*H, T, D] output.  With the default transport (fused) each rank runs one
        kernel whose epilogue stores its output tiles straight into its rows of rank 0's buffer
        (CUDA IPC mapping), so the transfer overlaps the computation tile by tile.  The other
        transports compute each share in MIX_CHUNKS chunks and move every finished chunk while
        the next one computes: copy-engine peer copies (copy) or NCCL send/recv (nccl).  At
        N = 1 there is nothing to send: the chunked kernels alone.
    Rank 0 then recomputes the first and last head of every rank's share on its own GPU and
    checks that the gathered rows equal them bit for bit.  Returns (dict, extra) where extra
    holds the tensors the standalone mix line needs for its end-to-end leg.
    """
    import torch.distributed as dist
    import usagi_b200 as ub
    from usagi_b200 import patterns as P
    from usagi_b200 import shard

    pat = P.mixed_pattern(MIX_B, MIX_H, MIX_T)  # host, identical on every rank (seed 1)
    total_heads = MIX_B * MIX_H
    g = torch.Generator(device=device).manual_seed(11)
    shape = (MIX_B, MIX_H, MIX_T, D)
    full = [torch.randn(shape, generator=g, device=device, dtype=torch.float32).half()
            for _ in range(3)]  # the same problem on every rank; each keeps its heads
    q, k, v, rp, ci, _, (h0, h1) = shard.shard_problem(*full, pat.row_ptr, pat.col_idx, None,
                                                       world, rank)
    q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
    if rank != 0:
        del full
        full = None
    n = h1 - h0
    rp_d, ci_d = rp.to(device), ci.to(device)
    plan = ub.make_plan(rp, ci, n, 1, MIX_T, device=device)
    o = torch.empty_like(q)
    lse = torch.empty((n, 1, MIX_T), device=device, dtype=torch.float32)
    rp_bh = pat.row_ptr.reshape(total_heads, -1).to(torch.int64)
    live_rank = int((rp_bh[h0:h1, -1] - rp_bh[h0:h1, 0]).sum())
    flops_total = pat.live_blocks() * 4 * 128 ** 3
    flops_rank = live_rank * 4 * 128 ** 3
    steps = max(3, min(args.steps, 20))

    def call():
        ub.block_sparse_attn_fwd(q, k, v, rp_d, ci_d, None, out=o, lse_out=lse, plan=plan)

    for _ in range(3):
        call()
    torch.cuda.synchronize()
    ub.check_errors(device)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(steps)]
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    for a, b in ev:
        a.record()
        call()
        b.record()
    torch.cuda.synchronize()
    rank_ms = sum(a.elapsed_time(b) for a, b in ev) / steps
    t = torch.tensor([rank_ms], device=device, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())

    # ---- pipelined: chunked kernels with the gather to rank 0 overlapped
    chunk_plans = {}
    for c in range(MIX_CHUNKS):
        a, b = shard.chunk_range(n, MIX_CHUNKS, c)
        if b > a:
            chunk_plans[c] = ub.make_plan(rp[a:b], ci[a:b], b - a, 1, MIX_T, device=device)
    local_out = o.reshape(n, MIX_T, D) if rank != 0 else None
    cur = torch.cuda.current_stream(device)
    transport = args.mix_transport if world > 1 else "none"
    peer = None
    fallback = None
    if transport in ("copy", "fused"):
        try:
            peer = shard.PeerGather((total_heads, MIX_T, D), torch.float16, total_heads, world,
                                    rank, device)
        except shard.PeerGatherUnavailable as e:  # raised on every rank together
            fallback, transport = str(e), "nccl"
    if peer is not None:
        root_out = peer.root if rank == 0 else None
    else:
        root_out = torch.empty((total_heads, MIX_T, D), device=device, dtype=torch.float16) \
            if rank == 0 else None
        comm = torch.cuda.Stream(device)

    def compute_chunk(c, a, b, dst):
        ub.block_sparse_attn_fwd(q[a:b], k[a:b], v[a:b], rp_d[a:b], ci_d[a:b], None,
                                 out=dst.view(b - a, 1, MIX_T, D), lse_out=lse[a:b],
                                 plan=chunk_plans[c])

    def pipelined():
        if peer is not None and transport == "fused":
            peer.run_fused(lambda ptr: ub.block_sparse_attn_fwd_into(
                ptr, q, k, v, rp_d, ci_d, None, lse_out=lse, plan=plan))
            return []
        if peer is not None:
            peer.run(compute_chunk, MIX_CHUNKS, local_out)
            return []
        works = shard.compute_and_gather(compute_chunk, MIX_CHUNKS, total_heads, world, rank,
                                         root_out, local_out, comm_stream=comm)
        cur.wait_stream(comm)
        return works

    for _ in range(2):  # warm-up: creates the point-to-point communicators / peer mappings
        for w in pipelined():
            w.wait()
        torch.cuda.synchronize()
    p_steps = max(3, min(args.steps, 10))
    pev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(p_steps)]
    p_ms = []
    for a, b in pev:
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        a.record()
        works = pipelined()
        b.record()
        for w in works:
            w.wait()
        torch.cuda.synchronize()
        p_ms.append(a.elapsed_time(b))
    tp = torch.tensor([sum(p_ms) / p_steps], device=device, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(tp, op=dist.ReduceOp.MAX)
    pipe_ms = float(tp.item())
    ub.check_errors(device)
    if world > 1:
        dist.barrier()

    # ---- rank 0 checks the gathered rows of every rank's share against a local recompute
    checked, max_diff, heads_checked = None, None, []
    if rank == 0:
        fq, fk, fv = [t.reshape(total_heads, 1, MIX_T, D) for t in full]
        frp = pat.row_ptr.reshape(total_heads, 1, -1)
        fci = pat.col_idx.reshape(total_heads, 1, -1)
        checked, max_diff = True, 0.0
        for r in range(world):
            rs, re = shard.shard_range(total_heads, world, r)
            for h in sorted({rs, re - 1}):
                oh, _ = ub.block_sparse_attn_fwd(fq[h:h + 1], fk[h:h + 1], fv[h:h + 1],
                                                 frp[h:h + 1].to(device), fci[h:h + 1].to(device),
                                                 None)
                d = (oh[0, 0].float() - root_out[h].float()).abs().max().item()
                max_diff = max(max_diff, d)
                checked = checked and torch.equal(oh[0, 0], root_out[h])
                heads_checked.append(h)
        torch.cuda.synchronize()
        ub.check_errors(device)
    if peer is not None:
        peer.close()
    res = {
        "workload": "scaling mix B=4,H=32,T=32768,D=128: heads cycle window16 / prefix8+window8 / "
                    "retrieval(2+16); 128 (batch, head) pairs split contiguously over the ranks",
        "scaling": "strong",
        "heads_per_rank": n,
        "live_blocks": pat.live_blocks(),
        "ms": ms,
        "value": flops_total / (ms * 1e-3) / 1e12,
        "unit": "TFLOP/s",
        "frac_per_rank": flops_rank / (rank_ms * 1e-3) / 1e12 / peaks["bf16_tflops"],
        "kernel_plus_gather_ms": pipe_ms,
        "value_with_gather": flops_total / (pipe_ms * 1e-3) / 1e12,
        "gather": ("none (one GPU)" if world == 1 else
                   "one kernel per rank whose epilogue stores every output tile straight into "
                   "rank 0's buffer over NVLink (CUDA IPC mapping, TMA tensor stores), so the "
                   "transfer overlaps the computation tile by tile; no copy follows"
                   if transport == "fused" else
                   f"{MIX_CHUNKS} chunks per rank; each finished chunk copied to rank 0 while the "
                   "next one computes, in place (no concatenation), by " +
                   ("copy-engine peer copies over NVLink into rank 0's buffer (CUDA IPC), which "
                    "need no SMs" if transport == "copy" else "NCCL send/recv on a second stream")),
        "gather_transport": transport,
        "gather_fallback_reason": fallback,
        "gather_checked": checked,
        "gather_max_abs_diff": max_diff,
        "gather_heads_checked": heads_checked,
        "timed_steps": steps,
    }
    extra = dict(q=q, k=k, v=v, rp_d=rp_d, ci_d=ci_d, plan=plan, o=o, lse=lse,
                 flops_total=flops_total, flops_rank=flops_rank, rank_ms=rank_ms, n=n, pat=pat)
    return res, extra


DENSE_CASES = [(2, 16, 8192), (1, 8, 32768)]
DENSE_METRIC = "dense causal attention forward TFLOP/s (4*B*H*D*T(T+1)/2 FLOP per call), D=128 fp16"


def run_dense(args, rank, world, local_rank):
    """``--workload dense``: a comparison point for the roofline fraction.  This kernel runs a
    dense causal pattern (every block at or below the diagonal: the window family with a window as
    long as the sequence) next to the dense causal attention of torch's SDPA (cuDNN and flash
    backends) and of flash_attn 2, on identical inputs.  Those library kernels serve only as
    comparison points here; nothing in the package calls them.  FLOPs are the exact causal count
    for every implementation.  Each call is timed alone with CUDA events, L2 flushed before it;
    the kernel of this build is timed before and after the libraries and reported as the median
    over both blocks.  Rank 0 alone runs it."""
    if rank != 0:
        return 0
    import torch.nn.functional as F
    from torch.nn.attention import SDPBackend, sdpa_kernel
    import usagi_b200 as ub
    from usagi_b200 import patterns as P

    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    ub.setup(device=str(device))
    peaks = load_peaks()
    flush = torch.empty(512 * 1024 * 1024, dtype=torch.uint8, device=device)
    n = max(10, min(args.steps, 50))

    def time_calls(fn):
        for _ in range(max(args.warmup, 3)):
            flush.zero_()
            fn()
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
               for _ in range(n)]
        for a, b in evs:
            flush.zero_()
            a.record()
            fn()
            b.record()
        torch.cuda.synchronize()
        return [a.elapsed_time(b) for a, b in evs]

    cases = []
    with ClockSampler(local_rank) as clk:
        for (b, h, t) in DENSE_CASES:
            g = torch.Generator().manual_seed(0)
            q, k, v = [torch.randn((b, h, t, D), generator=g).half().to(device) for _ in range(3)]
            nqb = t // 128
            pat = P.window_pattern(b, h, t, window=nqb)
            rp, ci = pat.row_ptr.to(device), pat.col_idx.to(device)
            plan = ub.make_plan(pat.row_ptr, pat.col_idx, b, h, t, device=device)
            o = torch.empty_like(q)
            lse = torch.empty((b, h, t), device=device, dtype=torch.float32)

            def ours():
                ub.block_sparse_attn_fwd(q, k, v, rp, ci, None, out=o, lse_out=lse, plan=plan)

            times = {"usagi_b200": time_calls(ours)}
            ub.check_errors(device)
            flops = 4.0 * b * h * D * t * (t + 1) / 2
            res, errors, maxdiff = {}, {}, {}
            for name, be in (("torch_sdpa_cudnn", SDPBackend.CUDNN_ATTENTION),
                             ("torch_sdpa_flash", SDPBackend.FLASH_ATTENTION)):
                try:
                    with sdpa_kernel([be]):
                        ref = F.scaled_dot_product_attention(q, k, v, is_causal=True)
                        times[name] = time_calls(
                            lambda: F.scaled_dot_product_attention(q, k, v, is_causal=True))
                    maxdiff[name] = float((ref.float() - o.float()).abs().max())
                    del ref
                except Exception as e:  # noqa: BLE001 - a backend missing on this box
                    errors[name] = f"{type(e).__name__}: {str(e)[:160]}"
            try:
                from flash_attn import flash_attn_func
                qt, kt, vt = (x.transpose(1, 2).contiguous() for x in (q, k, v))
                ref = flash_attn_func(qt, kt, vt, causal=True)
                times["flash_attn2"] = time_calls(lambda: flash_attn_func(qt, kt, vt, causal=True))
                maxdiff["flash_attn2"] = float((ref.transpose(1, 2).float() - o.float()).abs().max())
                del qt, kt, vt, ref
            except Exception as e:  # noqa: BLE001
                errors["flash_attn2"] = f"{type(e).__name__}: {str(e)[:160]}"
            times["usagi_b200"] += time_calls(ours)
            for name, ts in times.items():
                ms = statistics.median(ts)
                tf = flops / (ms * 1e-3) / 1e12
                res[name] = {"ms": round(ms, 4), "tflops": round(tf, 1),
                             "frac_of_peak": round(tf / peaks["bf16_tflops"], 3)}
            for name, d in maxdiff.items():
                assert d < 1e-2, (name, d)  # same attention, fp16 outputs
            cases.append({"B": b, "H": h, "T": t, "D": D, "flops": flops, "results": res,
                          "max_abs_diff_vs_usagi_b200": maxdiff, "errors": errors})
            del q, k, v, o, lse
            torch.cuda.empty_cache()
    print(json.dumps({
        "metric": DENSE_METRIC, "unit": "TFLOP/s", "impl": "ours", "workload": "dense",
        "higher_is_better": True, "n_gpus": 1, "calls_per_case": n, "dtype": "fp16",
        "data": "synthetic: N(0,1) fp32 from CPU seed 0 in the order q, k, v, cast to fp16",
        "pattern": "usagi_b200: CSR rows of every block 0..qb (window = T/128); libraries: is_causal",
        "l2": "flushed (512 MB write) before every timed call",
        "peak": {"value": peaks["bf16_tflops"], "unit": "TFLOP/s", "source": peaks["source"]},
        "cases": cases, "clocks": clk.summary()}), flush=True)
    return 0


def run_mix(args, rank, world, local_rank):
    """``--workload mix``: the scaling configuration as its own JSON line (with an end-to-end leg
    through the public API on each rank's share)."""
    import torch.distributed as dist
    import usagi_b200 as ub

    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    init_distributed(world, device)
    ub.setup(device=str(device))
    peaks = load_peaks()
    with ClockSampler(local_rank) as clk:
        mix, x = measure_mix(args, rank, world, device, peaks)
    q, k, v, rp_d, ci_d, plan, o, lse = (x[key] for key in
                                         ("q", "k", "v", "rp_d", "ci_d", "plan", "o", "lse"))
    # End to end on this rank's share: its q, k, v, CSR rows and work list up from pinned host
    # memory, the call, o and lse back, every step.
    host_in = [t.cpu().pin_memory() for t in (q, k, v, rp_d, ci_d, plan.tensor)]
    dev_in = [torch.empty_like(t) for t in (q, k, v, rp_d, ci_d, plan.tensor)]
    host_out = (torch.empty(o.shape, dtype=o.dtype).pin_memory(),
                torch.empty(lse.shape, dtype=lse.dtype).pin_memory())
    h2d = sum(t.numel() * t.element_size() for t in host_in)
    d2h = sum(t.numel() * t.element_size() for t in host_out)

    def e2e_step():
        for d_, h_ in zip(dev_in, host_in):
            d_.copy_(h_, non_blocking=True)
        pl = ub.Plan(dev_in[5], plan.grid, plan.B, plan.H, plan.T)
        ub.block_sparse_attn_fwd(dev_in[0], dev_in[1], dev_in[2], dev_in[3], dev_in[4], None,
                                 out=o, lse_out=lse, plan=pl)
        host_out[0].copy_(o, non_blocking=True)
        host_out[1].copy_(lse, non_blocking=True)

    e2e_step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    n_e2e = max(3, min(args.steps, 5))
    e0.record()
    for _ in range(n_e2e):
        e2e_step()
    e1.record()
    torch.cuda.synchronize()
    te = torch.tensor([e0.elapsed_time(e1) / n_e2e], device=device, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    e2e_ms = float(te.item())
    assert torch.equal(host_out[0].to(device), o)
    flops_total, flops_rank, rank_ms = x["flops_total"], x["flops_rank"], x["rank_ms"]
    line = {
        "metric": MIX_METRIC,
        "value": mix["value"],
        "unit": "TFLOP/s",
        "n_gpus": world,
        "steps": mix["timed_steps"],
        "warmup": 3,
        "ms_per_step": mix["ms"],
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "f16",
        "data": "synthetic (seeded N(0,1) fp16; mixed CSR pattern, seed 1)",
        "config": {
            "workload": mix["workload"] + "; one step = one call on each rank's share",
            "global_batch": MIX_B, "heads": MIX_H, "seq_len": MIX_T, "head_dim": D,
            "live_blocks": mix["live_blocks"],
            "parallelism": f"heads split contiguously x{world} ({x['n']} (batch, head) pairs per "
                           "rank), no collective in the kernel-only timing",
            "l2": "inputs (3 GiB at N=1) larger than L2, no flush",
            "schedule": "balanced work list (bsattn_plan) per rank",
        },
        "gpu_launches": mix["timed_steps"],
        "e2e": {"value": flops_total / (e2e_ms * 1e-3) / 1e12, "unit": "TFLOP/s",
                "ms_per_step": e2e_ms, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "path": "usagi_b200.block_sparse_attn_fwd from pinned host buffers, per rank"},
        "clocks": clk.summary(),
        "mix": mix,
        "roofline": {
            "bound": "tensor", "kernel": "bsattn_fwd_kernel",
            "achieved": flops_rank / (rank_ms * 1e-3) / 1e12, "peak": peaks["bf16_tflops"],
            "peak_source": peaks["source"] + " bf16 dense burst (fp16 runs at the same rate)",
            "unit": "TFLOP/s",
            "frac": flops_rank / (rank_ms * 1e-3) / 1e12 / peaks["bf16_tflops"],
            "algorithmic": "live tiles x 4*128^3 FLOP of this rank's share per launch",
            "traffic": None,
        },
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


# Window families whose rows also have the analytic form of bsattn_fwd_window: (window, global).
ANALYTIC = {"window8": (8, 0), "prefix4+window4": (4, 4)}


def measure_analytic(ub, inputs, outs, lses, flush, device, args):
    """The window families again, through bsattn_fwd_window (rows from closed forms, no CSR
    arrays), timed like the headline calls (L2 flushed before each), next to the CSR timing of the
    same calls; the outputs must equal the CSR outputs bit for bit."""
    fams = [f for f in FAMILIES if f in ANALYTIC]
    if not fams:
        return None
    plans = {f: ub.make_window_plan(B_PER_RANK, H, T, *ANALYTIC[f], device=device) for f in fams}
    res = {}
    for f in fams:
        q, k, v, rp, ci, plan = inputs[f]
        o_a = torch.empty_like(outs[f])
        l_a = torch.empty_like(lses[f])
        w, g = ANALYTIC[f]
        runs = {
            "csr": lambda: ub.block_sparse_attn_fwd(q, k, v, rp, ci, None, out=outs[f],
                                                    lse_out=lses[f], plan=plan),
            "analytic": lambda: ub.block_sparse_attn_fwd_window(
                q, k, v, None, window=w, global_blocks=g, out=o_a, lse_out=l_a, plan=plans[f]),
        }
        n = max(10, min(args.steps, 50))
        ms = {}
        for name, fn in runs.items():
            for _ in range(3):
                flush.zero_()
                fn()
            evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                   for _ in range(n)]
            for a, b in evs:
                flush.zero_()
                a.record()
                fn()
                b.record()
            torch.cuda.synchronize()
            ms[name] = statistics.median(a.elapsed_time(b) for a, b in evs)
        ub.check_errors(device)
        assert torch.equal(o_a, outs[f]) and torch.equal(l_a, lses[f])
        res[f] = {"ms_analytic": ms["analytic"], "ms_csr": ms["csr"], "window": w,
                  "global_blocks": g, "bitwise_equal_to_csr": True}
    return res


def measure_e2e(ub, inputs, outs, lses, flops_step, device, world, args):
    """Same metric through the public API with host buffers.  Per step: H2D of the step's inputs
    from pinned memory -- q, k, v once (the three families share them) and each family's
    row_ptr, col_idx and work list -- the three calls, and D2H of each family's o and lse, all
    inside the timed region.  Inputs go up on one copy stream, the calls run on the compute
    stream and results come down on a third stream, so one family's results travel to the host
    while the next family runs (PCIe is full duplex).  Inputs and outputs have two device buffer
    sets, used by alternate steps, so a step's upload starts as soon as the previous upload is
    done and a call does not wait for the previous step's download of its family.  Events keep
    every device buffer from being refilled before the work that reads it has finished."""
    import torch.distributed as dist
    q0, k0, v0 = inputs[FAMILIES[0]][:3]
    assert all(inputs[f][0] is q0 for f in FAMILIES), "families share q, k, v"
    host_qkv = [t.cpu().pin_memory() for t in (q0, k0, v0)]
    dev_qkv = [[torch.empty_like(t) for t in (q0, k0, v0)] for _ in range(2)]  # [buffer set]
    host_out, dev_out = {}, {}
    # Every family's int32 metadata (CSR rows and work list) packed into one buffer, so a step
    # moves it with a single copy; dev_in[f][b] are views into buffer set b.
    meta_src, spans = [], {}
    off = 0
    for f in FAMILIES:
        _, _, _, rp, ci, plan = inputs[f]
        srcs = [rp, ci] + ([plan.tensor] if plan is not None else [])
        spans[f] = []
        for t in srcs:
            assert t.dtype == torch.int32
            spans[f].append((off, tuple(t.shape)))
            meta_src.append(t.reshape(-1).cpu())
            off += t.numel()
    host_meta = torch.cat(meta_src).pin_memory()
    dev_meta = [torch.empty(off, dtype=torch.int32, device=device) for _ in range(2)]
    dev_in = {f: [[dev_meta[b][o:o + math.prod(shp)].view(shp) for o, shp in spans[f]]
                  for b in range(2)] for f in FAMILIES}
    for f in FAMILIES:
        host_out[f] = (torch.empty(outs[f].shape, dtype=torch.float16).pin_memory(),
                       torch.empty(lses[f].shape, dtype=torch.float32).pin_memory())
        dev_out[f] = [(torch.empty_like(outs[f]), torch.empty_like(lses[f])) for _ in range(2)]
    h2d = sum(t.numel() * t.element_size() for t in host_qkv) + \
        host_meta.numel() * host_meta.element_size()
    d2h = sum(t.numel() * t.element_size() for f in FAMILIES for t in host_out[f])
    comp = torch.cuda.current_stream(device)
    s_in, s_out = torch.cuda.Stream(device), torch.cuda.Stream(device)
    # last call that read buffer set b of q, k, v and of dev_in[f]
    done_call = {(f, b): None for f in FAMILIES for b in range(2)}
    done_out = {(f, b): None for f in FAMILIES for b in range(2)}  # last D2H of dev_out[f][b]
    step_no = [0]

    def e2e_step():
        b = step_no[0] & 1
        step_no[0] += 1
        qkv = dev_qkv[b]
        with torch.cuda.stream(s_in):
            for f in FAMILIES:  # set b is refilled only after every call that read it finished
                if done_call[(f, b)] is not None:
                    s_in.wait_event(done_call[(f, b)])
            for d, h in zip(qkv, host_qkv):
                d.copy_(h, non_blocking=True)
            dev_meta[b].copy_(host_meta, non_blocking=True)
            ev_in = torch.cuda.Event()
            ev_in.record(s_in)
        for f in FAMILIES:
            comp.wait_event(ev_in)
            if done_out[(f, b)] is not None:
                comp.wait_event(done_out[(f, b)])
            drp, dci = dev_in[f][b][:2]
            plan = None
            if len(dev_in[f][b]) > 2:
                p0 = inputs[f][5]
                plan = ub.Plan(dev_in[f][b][2], p0.grid, p0.B, p0.H, p0.T)
            ub.block_sparse_attn_fwd(qkv[0], qkv[1], qkv[2], drp, dci, None,
                                     out=dev_out[f][b][0], lse_out=dev_out[f][b][1], plan=plan)
            done_call[(f, b)] = torch.cuda.Event()
            done_call[(f, b)].record(comp)
            s_out.wait_event(done_call[(f, b)])
            with torch.cuda.stream(s_out):
                host_out[f][0].copy_(dev_out[f][b][0], non_blocking=True)
                host_out[f][1].copy_(dev_out[f][b][1], non_blocking=True)
                done_out[(f, b)] = torch.cuda.Event()
                done_out[(f, b)].record(s_out)

    e2e_steps = max(3, min(args.steps, 20))
    for _ in range(2):
        e2e_step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(comp)
    s_in.wait_event(e0)
    s_out.wait_event(e0)
    for _ in range(e2e_steps):
        e2e_step()
    for key in done_out:
        if done_out[key] is not None:
            comp.wait_event(done_out[key])
    e1.record(comp)
    torch.cuda.synchronize()
    t_e2e = torch.tensor([e0.elapsed_time(e1) / e2e_steps], device=device, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t_e2e, op=dist.ReduceOp.MAX)
    e2e_ms = float(t_e2e.item())
    e2e_value = world * flops_step / (e2e_ms * 1e-3) / 1e12
    last = (step_no[0] - 1) & 1
    for f in FAMILIES:  # the results that came back are the ones the device computed
        assert torch.equal(host_out[f][0].to(device), dev_out[f][last][0])
        assert torch.equal(host_out[f][0].to(device), outs[f])
    per_rank_s = e2e_ms * 1e-3
    return {"value": e2e_value, "unit": "TFLOP/s", "ms_per_step": e2e_ms,
            "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
            "h2d_GBps_per_rank": h2d / per_rank_s / 1e9,
            "d2h_GBps_per_rank": d2h / per_rank_s / 1e9,
            "host_copy_GBps_all_ranks": world * (h2d + d2h) / per_rank_s / 1e9,
            "numa": numa_info(device.index),
            "path": "usagi_b200.block_sparse_attn_fwd from pinned host buffers: q, k, v up once "
                    "per step (shared by the three families), each family's CSR rows and work "
                    "list, the calls, each family's o and lse down; H2D, calls and D2H on three "
                    "streams (one family's results travel while the next family runs); two "
                    "device buffer sets for inputs and outputs, used by alternate steps"}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--cpu-budget", type=float, default=12.0,
                    help="seconds of CPU work for the cpu_baseline sample")
    ap.add_argument("--ref-budget", type=float, default=4.0,
                    help="seconds of CPU work per reference-arm step")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-gather", action="store_true")
    ap.add_argument("--mix-transport", choices=["fused", "copy", "nccl"], default="fused",
                    help="how the scaling mix's output reaches rank 0: fused (default; each "
                         "rank's kernel stores its tiles straight into rank 0's buffer), copy "
                         "(copy-engine peer copies of finished chunks) or nccl (send/recv of "
                         "chunks)")
    ap.add_argument("--no-mix", action="store_true",
                    help="skip the scaling-mix leg (B=4,H=32,T=32768, strong scaling) of the line")
    ap.add_argument("--no-plan", action="store_true",
                    help="round-robin item order instead of the balanced work list")
    ap.add_argument("--family", choices=FAMILIES, default=None,
                    help="run one family only (profiling); the JSON line then covers that family")
    ap.add_argument("--workload", choices=["families", "mix", "dense"], default="families",
                    help="families: the headline 3-family workload (weak scaling); mix: the "
                         "head-sharded scaling configuration (strong scaling); dense: this "
                         "kernel on dense causal attention next to library kernels (comparison)")
    ap.add_argument("--quick", action="store_true",
                    help="device-timed region only: no e2e, cpu_baseline or gather (profiling)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.family:
        FAMILIES[:] = [args.family]
    if args.quick:
        args.no_cpu_baseline = True
        args.no_gather = True
        args.no_mix = True

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        return run_reference(args, rank, world)
    if args.workload == "mix":
        return run_mix(args, rank, world, local_rank)
    if args.workload == "dense":
        return run_dense(args, rank, world, local_rank)

    import torch.distributed as dist
    import usagi_b200 as ub
    from usagi_b200 import patterns as P
    from usagi_b200 import shard

    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    if os.environ.get("NCCL_DEBUG", "").upper() == "VERSION":
        os.environ["NCCL_DEBUG"] = "WARN"  # keep stdout to the single JSON line
    init_distributed(world, device)
    ub.setup(device=str(device))

    peaks = load_peaks()
    # Per-rank inputs resident in HBM; CSR metadata on device.
    inputs = {}
    q, k, v = make_inputs(device)  # shared by the three families
    for fam in FAMILIES:
        pat = P.family_pattern(fam, B_PER_RANK, H, T)
        # The balanced work list is built once per pattern on the host (bsattn_plan), like the
        # pattern itself; --no-plan keeps the round-robin item order.
        plan = None if args.no_plan else ub.make_plan(pat.row_ptr, pat.col_idx, B_PER_RANK, H, T,
                                                      device=device)
        inputs[fam] = (q, k, v, pat.row_ptr.to(device), pat.col_idx.to(device), plan)
    flops = {f: _pattern_flops(f) for f in FAMILIES}
    flops_step = sum(flops.values())
    outs = {f: torch.empty((B_PER_RANK, H, T, D), device=device, dtype=torch.float16)
            for f in FAMILIES}
    lses = {f: torch.empty((B_PER_RANK, H, T), device=device, dtype=torch.float32)
            for f in FAMILIES}
    flush = torch.empty(512 * 1024 * 1024 // 4, device=device, dtype=torch.float32)

    def call(f):
        q, k, v, rp, ci, plan = inputs[f]
        ub.block_sparse_attn_fwd(q, k, v, rp, ci, None, out=outs[f], lse_out=lses[f], plan=plan)

    for _ in range(args.warmup):
        for f in FAMILIES:
            flush.zero_()
            call(f)
    torch.cuda.synchronize()
    ub.check_errors(device)

    # ---------------- device-timed region: K steps, L2 flushed before every call
    n_calls = args.steps * len(FAMILIES)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(n_calls)]
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local_rank) as clk:
        i = 0
        for _ in range(args.steps):
            for f in FAMILIES:
                flush.zero_()
                ev[i][0].record()
                call(f)
                ev[i][1].record()
                i += 1
        torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ub.check_errors(device)
    per_call = [a.elapsed_time(b) for a, b in ev]
    fam_ms = {f: statistics.median(per_call[j::len(FAMILIES)]) for j, f in enumerate(FAMILIES)}
    total_ms = sum(per_call)
    t_kernel = torch.tensor([total_ms], device=device, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t_kernel, op=dist.ReduceOp.MAX)
    total_ms = float(t_kernel.item())
    ms_per_step = total_ms / args.steps
    value = world * flops_step / (ms_per_step * 1e-3) / 1e12
    geo_ms = math.exp(sum(math.log(fam_ms[f]) for f in FAMILIES) / len(FAMILIES))
    achieved = flops_step / (ms_per_step * 1e-3) / 1e12  # per launch-set on this GPU

    # ---------------- end-to-end through the public API with pinned host buffers
    e2e = None
    if not args.quick:
        e2e = measure_e2e(ub, inputs, outs, lses, flops_step, device, world, args)

    # ---------------- the window families through the analytic entry point (outside the timing)
    analytic = None
    if not args.quick and rank == 0:
        analytic = measure_analytic(ub, inputs, outs, lses, flush, device, args)

    # ---------------- optional gather of o to rank 0 (outside the data path)
    gather_ms = None
    if world > 1 and not args.no_gather:
        gather_ms = shard.timed_gather_to_root(outs[FAMILIES[0]], world, rank, device)

    clocks = clk.summary()

    # ---------------- the scaling configuration (strong scaling, pipelined gather to rank 0)
    mix = None
    if not args.no_mix:
        del flush
        torch.cuda.empty_cache()
        mix, _ = measure_mix(args, rank, world, device, peaks)
    line = {
        "metric": METRIC,
        "value": value,
        "unit": "TFLOP/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms_per_step,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f16",
        "data": "synthetic: q, k, v ~ N(0,1) fp32 from CPU seed 0 cast to fp16, the same tensors "
                "for the three families (BASELINE configs 1-3); CSR patterns generated per family "
                "(retrieval rows from seed 1)",
        "config": {
            "workload": "3 families (window8, prefix4+window4, retrieval8) B=2,H=16,T=8192,D=128 "
                        "per GPU; one step = one call per family",
            "global_batch": B_PER_RANK * world, "heads": H, "seq_len": T, "head_dim": D,
            "parallelism": f"head-sharded x{world} (batch entries split across ranks, no collective)",
            "l2": "flushed (512 MB write) before every timed call",
            "schedule": "round robin" if args.no_plan else "balanced work list (bsattn_plan)",
        },
        "ms_per_call": fam_ms,
        "ms_per_call_geomean": geo_ms,
        "tflops_per_call": {f: flops[f] / (fam_ms[f] * 1e-3) / 1e12 for f in FAMILIES},
        "gpu_launches": n_calls,
        "e2e": e2e,
        "clocks": clocks,
    }
    traffic = load_traffic()
    line["roofline"] = {
        "bound": "tensor",
        "kernel": "bsattn_fwd_kernel",
        "achieved": achieved,
        "peak": peaks["bf16_tflops"],
        "peak_source": peaks["source"] + " bf16 dense burst (fp16 runs at the same rate)",
        "unit": "TFLOP/s",
        "frac": achieved / peaks["bf16_tflops"],
        "algorithmic": "live tiles x 4*128^3 FLOP (QK^T + PV, full 128x128 tiles) per launch",
        "traffic": float(traffic["traffic_bytes_per_launch"]) if traffic and
        "traffic_bytes_per_launch" in traffic else None,
        "traffic_note": traffic.get("note") if traffic else None,
    }
    if analytic is not None:
        line["analytic_rows"] = analytic
    if mix is not None:
        line["mix"] = mix
    if gather_ms is not None:
        line["gather_ms"] = gather_ms
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        threads = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count()
        line["cpu_baseline"] = cpu_reference_throughput(args.cpu_budget, threads)
        line["cpu_baseline"]["config0"] = cpu_config0(threads)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
