"""GPU test of bsattn_fwd_noalloc, the entry point for callers that cannot allocate device memory
(for example code running inside a memory arena it does not own): it runs the same kernel with
the same grid as bsattn_fwd, which takes a caller-allocated workspace, so its output must equal
that entry point's bit for bit, and it must do so on consecutive calls, since every call on a GPU
reuses the same fixed scratch array compiled into the library.  One head is also checked against
the fp32 oracle under the parity tolerance of the other GPU tests.

This file is named to be collected last, so that a run stopping at the first failure has already
run every other test.  It does not depend on state left by other tests.
"""
import ctypes

import pytest
import torch

import usagi_b200 as ub
from usagi_b200 import _lib, api
from usagi_b200 import patterns as P
from oracle.bsattn_oracle import attn_blockwise

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)
MAX_TOL, MEAN_TOL = 1e-2, 1e-3  # the parity contract the other GPU tests use
REG_MAX, REG_MEAN = 4e-3, 2e-4  # their regression bound against the fp32 oracle


def _noalloc(q, k, v, row_ptr, col_idx, seq_lens, status):
    """One call through the C ABI; returns (rc, o, lse)."""
    lib = _lib.load()
    B, H, T, D = q.shape
    rp, rps = api._bh_view(row_ptr, B, H, "row_ptr")
    ci, cis = api._bh_view(col_idx, B, H, "col_idx")
    o = torch.empty_like(q)
    lse = torch.empty((B, H, T), device=DEV, dtype=torch.float32)
    stream = torch.cuda.current_stream(DEV).cuda_stream
    rc = lib.bsattn_fwd_noalloc(
        q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), lse.data_ptr(),
        rp.data_ptr(), ci.data_ptr(), seq_lens.data_ptr() if seq_lens is not None else None,
        B, H, T, D, rps, cis, int(ci.shape[-1]), 0.0, _lib.OUT_F16,
        status.data_ptr(), stream)
    return rc, o, lse


def _inputs(seed):
    B, H, T = 2, 4, 2048
    g = torch.Generator(device=DEV).manual_seed(seed)
    q, k, v = [torch.randn(B, H, T, 128, generator=g, device=DEV).half() for _ in range(3)]
    pat = P.retrieval_pattern(B, H, T, 8, seed=1)
    sl = torch.tensor([T, 1500], dtype=torch.int32, device=DEV)
    return q, k, v, pat.row_ptr.to(DEV), pat.col_idx.to(DEV), sl


def test_noalloc_matches_workspace_entry_point_on_consecutive_calls():
    ub.setup(device="cuda:0")
    q, k, v, rp, ci, sl = _inputs(seed=31)
    ref_o, ref_lse = ub.block_sparse_attn_fwd(q, k, v, rp, ci, sl)
    torch.cuda.synchronize()
    ub.check_errors(DEV)
    for call in range(2):
        status = torch.full((1,), 12345, dtype=torch.int32, device=DEV)
        rc, o, lse = _noalloc(q, k, v, rp, ci, sl, status)
        assert rc == 0, _lib.strerror(rc)
        torch.cuda.synchronize()
        assert int(status.item()) == 0, f"call {call}: device status {int(status.item())}"
        # same kernel, same grid, no work list: identical bits, not merely close values
        assert torch.equal(o, ref_o), (call, (o.float() - ref_o.float()).abs().max().item())
        assert torch.equal(lse, ref_lse), call
    # one head (b=1: seq_len 1500 < T) against the fp32 oracle
    H = q.shape[1]
    bh = H + 2
    sub = lambda t: t.reshape(-1, *t.shape[2:])[bh:bh + 1].unsqueeze(0).cpu()  # noqa: E731
    rps = rp.reshape(-1, rp.shape[-1])[bh:bh + 1].reshape(1, 1, -1).cpu()
    cis = ci.reshape(-1, ci.shape[-1])[bh:bh + 1].reshape(1, 1, -1).cpu()
    ro, rl = attn_blockwise(sub(q), sub(k), sub(v), rps, cis, sl[1:2].cpu())
    d = (sub(o).float() - ro).abs()
    assert d.max().item() <= REG_MAX and d.mean().item() <= REG_MEAN, d.max().item()
    assert d.max().item() <= MAX_TOL and d.mean().item() <= MEAN_TOL
    fin = torch.isfinite(rl)
    assert torch.equal(fin, torch.isfinite(sub(lse)))
    assert (sub(lse)[fin] - rl[fin]).abs().max().item() <= 2e-4


def test_noalloc_status_is_per_call():
    """An out-of-range CSR entry is reported in that call's status; the next valid call starts
    from a cleared error word and reports 0."""
    ub.setup(device="cuda:0")
    q, k, v, rp, ci, sl = _inputs(seed=32)
    bad = ci.clone()
    bad[0, 0, 1] = 10_000  # a key block past T/128
    status = torch.full((1,), 0, dtype=torch.int32, device=DEV)
    rc, o, _ = _noalloc(q, k, v, rp, bad, sl, status)
    assert rc == 0
    torch.cuda.synchronize()
    assert int(status.item()) == _lib.E_CSR
    assert torch.isfinite(o.float()).all()
    rc, o, _ = _noalloc(q, k, v, rp, ci, sl, status)
    assert rc == 0
    torch.cuda.synchronize()
    assert int(status.item()) == 0
