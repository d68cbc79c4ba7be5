"""Dense causal rows on the GPU: when every block at or below the diagonal is live (the window
family with a window as long as the sequence), block-sparse attention is plain causal attention.
That gives an independent check at full size, over every head: torch's SDPA (its own causal
kernel, fp16 in and out) for o, and an fp32 logsumexp of the causal scores for lse.  Rows of up to
256 tiles (T=32768) exercise long items, which the benchmark families (8-16 tiles per row) do not.
The reference's kernel semantics are those of kernels/v4_leaderboard_0740ms.py:31-136 with every
block listed; tolerances are the fp16 regression bound used by the other GPU tests (o: max 4e-3,
mean 2e-4 against another fp16 result; lse: 2e-4).
"""
import math

import pytest
import torch
import torch.nn.functional as F

import usagi_b200 as ub
from usagi_b200 import patterns as P

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)


@pytest.fixture(scope="module", autouse=True)
def _setup():
    ub.setup(device="cuda:0")
    yield
    ub.check_errors(DEV)


def _causal_lse(q, k, scale, rows=4096):
    """Natural-log logsumexp over keys <= query of the fp32 scores, per (b, h), in row chunks."""
    B, H, T, _ = q.shape
    out = torch.empty(B, H, T, device=q.device, dtype=torch.float32)
    key = torch.arange(T, device=q.device)
    for b in range(B):
        for h in range(H):
            kf = k[b, h].float()
            for r0 in range(0, T, rows):
                s = (q[b, h, r0:r0 + rows].float() @ kf.T) * scale
                qi = torch.arange(r0, min(r0 + rows, T), device=q.device)
                s.masked_fill_(key[None, :] > qi[:, None], float("-inf"))
                out[b, h, r0:r0 + rows] = torch.logsumexp(s, dim=-1)
    return out


@pytest.mark.parametrize("B,H,T", [(2, 16, 8192), (1, 2, 32768)])
def test_dense_causal_rows_match_sdpa(B, H, T):
    g = torch.Generator(device=DEV).manual_seed(7)
    q, k, v = [torch.randn(B, H, T, 128, generator=g, device=DEV).half() for _ in range(3)]
    nqb = T // 128
    pat = P.window_pattern(B, H, T, window=nqb)
    rp, ci = pat.row_ptr.to(DEV), pat.col_idx.to(DEV)
    plan = ub.make_plan(pat.row_ptr, pat.col_idx, B, H, T, device=DEV)
    o, lse = ub.block_sparse_attn_fwd(q, k, v, rp, ci, None, plan=plan)
    torch.cuda.synchronize()
    ub.check_errors(DEV)

    ref = F.scaled_dot_product_attention(q, k, v, is_causal=True)
    d = (o.float() - ref.float()).abs()
    assert d.max().item() <= 4e-3, d.max().item()
    assert d.mean().item() <= 2e-4, d.mean().item()

    ref_lse = _causal_lse(q, k, 1.0 / math.sqrt(128))
    dl = (lse - ref_lse).abs().max().item()
    assert dl <= 2e-4, dl

    # The same rows from closed forms, with no CSR arrays: bit for bit the CSR result.
    o_w, lse_w = ub.block_sparse_attn_fwd_window(q, k, v, None, window=nqb)
    torch.cuda.synchronize()
    ub.check_errors(DEV)
    assert torch.equal(o_w, o) and torch.equal(lse_w, lse)
