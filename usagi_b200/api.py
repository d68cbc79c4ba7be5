"""Drop-in host API mirroring the reference submission module (Python side of the C ABI).

Reference interface (sissississi-013/usagi, kernels/v4_leaderboard_0740ms.py):

* ``VARIANT_MANIFEST`` (:25)                       -> same constant
* ``setup(suite_specs, device, variants)`` (:189)  -> loads the prebuilt sm_100a library and
  configures the device; nothing is JIT-compiled, so there is nothing else to warm up
* ``block_sparse_attn_fwd(q, k, v, row_ptr, col_idx, seq_lens) -> (o, lse)`` (:242) -> same
  call, same argument meaning; runs the CUDA kernel through ``bsattn_fwd``.

Differences a caller can see, all deliberate:

* ``o`` has the dtype of ``q`` by default: bf16 for the reference's bf16 inputs (v4 :152), fp16
  for fp16 inputs (the reference always stored bf16); ``out_dtype`` overrides it.
* bf16 inputs follow the reference's mixed recipe: Q K^T on bf16 operands, then fp16(P) times
  fp16(V) (v4 :103, :123).  A bf16 ``v`` is converted to fp16 once per call, by the library.
* No metadata cache keyed on ``data_ptr()`` (the reference's v4 :155-164 cache returns stale
  metadata when a freed buffer is reused with new content); int32 conversions happen per call and
  are no-ops for int32 inputs.
* Errors raise :class:`BsattnError` with the C ABI's message instead of a Triton error.
"""
from __future__ import annotations

import math
import os
import threading
from typing import Optional, Tuple

import torch

from . import _lib

__all__ = [
    "VARIANT_MANIFEST",
    "BsattnError",
    "setup",
    "block_sparse_attn_fwd",
    "check_errors",
    "set_timeout_ns",
    "Plan",
    "make_plan",
    "block_sparse_attn_fwd_window",
    "make_window_plan",
]

BLOCK_SIZE = 128
HEAD_DIM = 128
VARIANT_MANIFEST = [{"name": "default"}]


class BsattnError(RuntimeError):
    """Raised for any non-zero status of the C ABI."""

    def __init__(self, code: int, where: str = ""):
        self.code = int(code)
        msg = _lib.strerror(code)
        super().__init__(f"{where}: {msg} (code {code})" if where else f"{msg} (code {code})")


_ws_lock = threading.Lock()
_workspaces: dict = {}


def _workspace(device: torch.device, stream: int) -> torch.Tensor:
    """The error-word workspace of one (device, CUDA stream handle), created and zeroed on first
    use.  The zero fill must run eagerly: inside stream capture it would only be recorded (and
    run at replay), leaving the word uninitialised for eager calls, so a first use during capture
    is refused -- call once on the stream before capturing it, as a warm-up."""
    key = (device.index, stream)
    with _ws_lock:
        ws = _workspaces.get(key)
        if ws is None:
            if torch.cuda.is_current_stream_capturing():
                raise RuntimeError(
                    "usagi_b200: the first call on a CUDA stream must run outside graph capture "
                    "(it creates and zeroes the stream's error word); make one eager call on this "
                    "stream before capturing it")
            n = _lib.load().bsattn_workspace_bytes()
            ws = torch.zeros((n + 3) // 4, dtype=torch.int32, device=device)
            _workspaces[key] = ws
        return ws


def set_timeout_ns(ns: int) -> None:
    """Upper bound for any pipeline wait inside the kernel (see bsattn_set_timeout_ns)."""
    _lib.load().bsattn_set_timeout_ns(int(ns))


def setup(suite_specs=None, device="cuda", variants=None) -> None:
    """Counterpart of the reference ``setup`` (v4 :189-238): load the library, check the GPU."""
    lib = _lib.load()
    if str(device).startswith("cuda") and torch.cuda.is_available():
        dev = torch.device(device)
        with torch.cuda.device(dev if dev.index is not None else torch.cuda.current_device()):
            rc = lib.bsattn_setup()
        if rc != 0:
            raise BsattnError(rc, "setup")
    env = os.environ.get("BSATTN_TIMEOUT_NS")
    if env:
        set_timeout_ns(int(env))


def _bh_view(t: torch.Tensor, B: int, H: int, name: str) -> Tuple[torch.Tensor, int]:
    """Return (int32 tensor, per-head stride in elements) for CSR metadata.

    Accepts [B, H, n], [B*H, n] or [n] (one pattern for all heads); stride-0 expanded views
    (one pattern broadcast to every head) are passed through without a copy.
    """
    if t.dtype != torch.int32:
        t = t.to(torch.int32)  # v4 :161-162 ``.to(torch.int32)``
    if t.dim() == 1:
        t = t.contiguous()
        return t, 0
    if t.dim() == 2:
        if t.shape[0] != B * H:
            raise ValueError(f"{name}: expected {B * H} rows, got {tuple(t.shape)}")
        if t.stride(1) != 1:
            t = t.contiguous()
        return t, t.stride(0)
    if t.dim() == 3:
        if t.shape[0] != B or t.shape[1] != H:
            raise ValueError(f"{name}: expected leading dims ({B}, {H}), got {tuple(t.shape)}")
        if t.stride(2) != 1:
            t = t.contiguous()
        s0, s1 = t.stride(0), t.stride(1)
        if s0 == H * s1 or B == 1:
            return t, s1
        if H == 1:
            return t, s0
        t = t.contiguous()
        return t, t.stride(1)
    raise ValueError(f"{name}: expected 1-3 dims, got {t.dim()}")


class Plan:
    """Balanced work list for one problem shape and pattern (``bsattn_plan``), on the device.

    Items (query blocks of a head) are sorted by tile count, largest first, and dealt to the
    persistent CTAs in snake order, so every CTA ends within one item of the mean; without a plan
    CTA b takes items b, b + grid, ...  Valid for the B, H, T, row_ptr, max_nnz and seq_lens it
    was built from.
    """

    def __init__(self, tensor: torch.Tensor, grid: int, B: int, H: int, T: int):
        self.tensor, self.grid, self.B, self.H, self.T = tensor, grid, B, H, T


def make_plan(row_ptr: torch.Tensor, col_idx: torch.Tensor, B: int, H: int, T: int,
              seq_lens: Optional[torch.Tensor] = None, device="cuda",
              grid: Optional[int] = None) -> Plan:
    """Build a :class:`Plan` on the host from the pattern (copied to the host once) and move it
    to ``device``.  ``grid`` defaults to the persistent grid of the call: one CTA per SM."""
    lib = _lib.load()
    rp, rp_stride = _bh_view(row_ptr.detach().cpu(), B, H, "row_ptr")
    max_nnz = int(col_idx.shape[-1])
    return _build_plan(B, H, T, seq_lens, device, grid, "bsattn_plan",
                       lambda sl, g, buf, n: lib.bsattn_plan(rp.data_ptr(), rp_stride, sl, B, H, T,
                                                             max_nnz, g, buf, n))


def make_window_plan(B: int, H: int, T: int, window: int, global_blocks: int = 0,
                     seq_lens: Optional[torch.Tensor] = None, device="cuda",
                     grid: Optional[int] = None) -> Plan:
    """:class:`Plan` for :func:`block_sparse_attn_fwd_window` (``bsattn_plan_window``)."""
    lib = _lib.load()
    return _build_plan(B, H, T, seq_lens, device, grid, "bsattn_plan_window",
                       lambda sl, g, buf, n: lib.bsattn_plan_window(sl, B, H, T, int(window),
                                                                    int(global_blocks), g, buf, n))


def _build_plan(B, H, T, seq_lens, device, grid, name, fill) -> Plan:
    import ctypes
    lib = _lib.load()
    nqb = T // BLOCK_SIZE
    sl = None
    if seq_lens is not None:
        sl = seq_lens.detach().cpu().to(torch.int32).contiguous()
    dev = torch.device(device)
    if grid is None:
        grid = min(torch.cuda.get_device_properties(dev).multi_processor_count, B * H * nqb)
    nbytes = ctypes.c_size_t(0)
    rc = lib.bsattn_plan_bytes(B, H, T, grid, ctypes.byref(nbytes))
    if rc != 0:
        raise BsattnError(rc, "bsattn_plan_bytes")
    host = torch.empty(nbytes.value // 4, dtype=torch.int32)
    rc = fill(sl.data_ptr() if sl is not None else None, grid, host.data_ptr(), nbytes.value)
    if rc != 0:
        raise BsattnError(rc, name)
    return Plan(host.to(dev), grid, B, H, T)


def _prepare(q, k, v, seq_lens, out_dtype, out, lse_out, return_lse, alloc_out=True):
    """Shared checks and buffers of the entry points: (q, k, v, flags, seq_lens, o, lse).
    With ``alloc_out=False`` no o is checked or allocated (o is None): the caller supplies its
    device address."""
    lib = _lib.load()
    if q.dim() != 4:
        raise ValueError(f"q must be [B, H, T, D], got {tuple(q.shape)}")
    B, H, T, D = q.shape
    if k.shape != q.shape or v.shape != q.shape:
        raise ValueError("q, k, v must have the same shape")
    if q.dtype not in (torch.float16, torch.bfloat16) or k.dtype != q.dtype \
            or v.dtype not in (torch.float16, q.dtype):
        raise TypeError("q and k must both be float16 or both bfloat16, and v float16 or the "
                        f"dtype of q (got {q.dtype}, {k.dtype}, {v.dtype})")
    if not q.is_cuda:
        raise ValueError("block_sparse_attn_fwd needs CUDA tensors (there is no CPU path)")
    if out_dtype is None:
        out_dtype = q.dtype
    if out_dtype not in (torch.float16, torch.bfloat16):
        raise TypeError(f"out_dtype must be float16 or bfloat16, got {out_dtype}")
    dev = q.device
    q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
    flags = _lib.OUT_BF16 if out_dtype == torch.bfloat16 else _lib.OUT_F16
    if q.dtype == torch.bfloat16:
        flags |= _lib.IN_BF16
    if v.dtype == torch.bfloat16:
        v16 = torch.empty(v.shape, device=dev, dtype=torch.float16)
        with torch.cuda.device(dev):
            rc = lib.bsattn_bf16_to_f16(v.data_ptr(), v16.data_ptr(), v.numel(),
                                        torch.cuda.current_stream(dev).cuda_stream)
        if rc != 0:
            raise BsattnError(rc, "bsattn_bf16_to_f16")
        v = v16
    sl = None
    if seq_lens is not None:
        sl = seq_lens.to(device=dev, dtype=torch.int32).contiguous()
        if sl.numel() != B:
            raise ValueError(f"seq_lens: expected {B} entries, got {sl.numel()}")
    if not alloc_out:
        out = None
    elif out is None:
        out = torch.empty((B, H, T, D), device=dev, dtype=out_dtype)
    elif out.shape != (B, H, T, D) or out.dtype != out_dtype or not out.is_contiguous():
        raise ValueError("out has the wrong shape, dtype or layout")
    lse = None
    if return_lse:
        if lse_out is None:
            lse = torch.empty((B, H, T), device=dev, dtype=torch.float32)
        else:
            if lse_out.shape != (B, H, T) or lse_out.dtype != torch.float32 \
                    or not lse_out.is_contiguous():
                raise ValueError("lse_out has the wrong shape, dtype or layout")
            lse = lse_out
    return q, k, v, flags, sl, out, lse


def _plan_args(plan, B, H, T, dev):
    if plan is None:
        return None, 0
    if (plan.B, plan.H, plan.T) != (B, H, T) or plan.tensor.device != dev:
        raise ValueError("plan was built for another shape or device")
    return plan.tensor.data_ptr(), plan.grid


def block_sparse_attn_fwd(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                          row_ptr: torch.Tensor, col_idx: torch.Tensor,
                          seq_lens: Optional[torch.Tensor] = None, *,
                          scale: Optional[float] = None,
                          out_dtype: Optional[torch.dtype] = None,
                          out: Optional[torch.Tensor] = None,
                          lse_out: Optional[torch.Tensor] = None,
                          return_lse: bool = True,
                          plan: Optional[Plan] = None):
    """Block-sparse causal attention forward on a B200.

    q, k: fp16 or bf16 [B, H, T, 128] CUDA tensors of one dtype, T % 128 == 0; v: the same shape,
    fp16 or the dtype of q.  row_ptr: int [B, H, T/128 + 1]; col_idx: int [B, H, max_nnz] (or
    [B*H, .], or one shared [.] row); seq_lens: int [B] or None.  Returns ``(o, lse)`` like the
    reference (v4 :179): o [B, H, T, 128] in ``out_dtype`` (default: q's dtype), lse fp32
    [B, H, T] (None if ``return_lse=False``).  ``plan`` (from :func:`make_plan` for this pattern)
    balances the work across the persistent CTAs; results are identical with or without it.
    """
    return _fwd_csr(q, k, v, row_ptr, col_idx, seq_lens, scale, out_dtype, out, lse_out,
                    return_lse, plan, None)


def _fwd_csr(q, k, v, row_ptr, col_idx, seq_lens, scale, out_dtype, out, lse_out, return_lse,
             plan, out_ptr):
    """The CSR call (``bsattn_fwd_plan``); o goes to ``out`` or, when ``out_ptr`` is given, to
    that device address."""
    lib = _lib.load()
    q, k, v, flags, sl, out, lse = _prepare(q, k, v, seq_lens, out_dtype, out, lse_out,
                                            return_lse, alloc_out=out_ptr is None)
    B, H, T, D = q.shape
    dev = q.device
    nqb = T // BLOCK_SIZE
    rp, rp_stride = _bh_view(row_ptr.to(dev), B, H, "row_ptr")
    ci, ci_stride = _bh_view(col_idx.to(dev), B, H, "col_idx")
    if rp.shape[-1] != nqb + 1:
        raise ValueError(f"row_ptr: expected last dim {nqb + 1}, got {rp.shape[-1]}")
    max_nnz = int(ci.shape[-1])
    with torch.cuda.device(dev):
        stream = torch.cuda.current_stream(dev).cuda_stream
        ws = _workspace(dev, stream)
        plan_ptr, plan_grid = _plan_args(plan, B, H, T, dev)
        rc = lib.bsattn_fwd_plan(
            q.data_ptr(), k.data_ptr(), v.data_ptr(),
            out.data_ptr() if out is not None else out_ptr,
            lse.data_ptr() if lse is not None else None,
            rp.data_ptr(), ci.data_ptr(), sl.data_ptr() if sl is not None else None,
            B, H, T, D, rp_stride, ci_stride, max_nnz,
            float(scale) if scale is not None else 0.0, flags, plan_ptr, plan_grid,
            ws.data_ptr(), ws.numel() * 4, stream)
    if rc != 0:
        raise BsattnError(rc, "bsattn_fwd")
    return out, lse


def block_sparse_attn_fwd_into(o_ptr: int, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                               row_ptr: torch.Tensor, col_idx: torch.Tensor,
                               seq_lens: Optional[torch.Tensor] = None, *,
                               scale: Optional[float] = None,
                               out_dtype: Optional[torch.dtype] = None,
                               lse_out: Optional[torch.Tensor] = None,
                               return_lse: bool = True,
                               plan: Optional[Plan] = None):
    """:func:`block_sparse_attn_fwd` writing o to the device address ``o_ptr`` instead of a
    tensor: contiguous [B, H, T, 128] in ``out_dtype``, 16-byte aligned, reachable from q's GPU.
    That may be another GPU's buffer mapped into this process (CUDA IPC with peer access, as
    :class:`usagi_b200.shard.PeerGather` sets up): the kernel's tile stores then cross NVLink as
    each tile is finished, with no copy afterwards.  Returns lse (None if ``return_lse=False``).
    The call is ordered on the current stream like the tensor entry point; making the written
    memory visible to another process is the caller's synchronisation (an interprocess event)."""
    if not o_ptr:
        raise ValueError("o_ptr must be a device address")
    _, lse = _fwd_csr(q, k, v, row_ptr, col_idx, seq_lens, scale, out_dtype, None, lse_out,
                      return_lse, plan, int(o_ptr))
    return lse


def block_sparse_attn_fwd_window(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                                 seq_lens: Optional[torch.Tensor] = None, *, window: int,
                                 global_blocks: int = 0, scale: Optional[float] = None,
                                 out_dtype: Optional[torch.dtype] = None,
                                 out: Optional[torch.Tensor] = None,
                                 lse_out: Optional[torch.Tensor] = None,
                                 return_lse: bool = True, plan: Optional[Plan] = None):
    """Attention over analytic rows, with no CSR tensors (``bsattn_fwd_window``).

    Row i of every head lists the first ``global_blocks`` blocks not covered by the window, then
    blocks max(0, i - window + 1) .. i: the reference's analytic kernels ``_fwd_window`` and
    ``_fwd_window_global`` (kernels/v1_baseline.py:144, :227).  Same result, bit for bit, as
    :func:`block_sparse_attn_fwd` given those rows as CSR; the other arguments are the same.
    """
    lib = _lib.load()
    q, k, v, flags, sl, out, lse = _prepare(q, k, v, seq_lens, out_dtype, out, lse_out,
                                            return_lse)
    B, H, T, D = q.shape
    dev = q.device
    with torch.cuda.device(dev):
        stream = torch.cuda.current_stream(dev).cuda_stream
        ws = _workspace(dev, stream)
        plan_ptr, plan_grid = _plan_args(plan, B, H, T, dev)
        rc = lib.bsattn_fwd_window(
            q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(),
            lse.data_ptr() if lse is not None else None, sl.data_ptr() if sl is not None else None,
            B, H, T, D, int(window), int(global_blocks),
            float(scale) if scale is not None else 0.0, flags, plan_ptr, plan_grid,
            ws.data_ptr(), ws.numel() * 4, stream)
    if rc != 0:
        raise BsattnError(rc, "bsattn_fwd_window")
    return out, lse


def check_errors(device=None) -> None:
    """Synchronise and raise if a kernel on this device/stream reported a CSR or timeout error.

    The error word belongs to the CUDA stream handle, not to a ``torch.cuda.Stream`` object:
    torch hands out pooled stream handles again to later Stream objects, so an error that no
    check collected is reported by the next check on the same handle.  Checking clears it; call
    this before handing a pooled stream to unrelated work if errors must not carry over."""
    lib = _lib.load()
    dev = torch.device(device) if device is not None else torch.device("cuda",
                                                                         torch.cuda.current_device())
    with torch.cuda.device(dev):
        stream = torch.cuda.current_stream(dev).cuda_stream
        ws = _workspace(dev, stream)
        import ctypes
        st = ctypes.c_int(0)
        rc = lib.bsattn_check_error(ws.data_ptr(), stream, ctypes.byref(st))
    if rc != 0:
        raise BsattnError(rc, "bsattn_check_error")
    if st.value != 0:
        raise BsattnError(st.value, "kernel")


def default_scale(D: int = HEAD_DIM) -> float:
    return 1.0 / math.sqrt(D)
