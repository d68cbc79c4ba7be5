"""bf16 inputs in the CPU oracle (the reference's original input dtype).

With bf16 q, k, v the reference computes Q K^T on bf16 operands in fp32 and P V as
fp16(P) . fp16(V) (kernels/v4_leaderboard_0740ms.py:103, :123).  The literal transcription follows
that recipe; the exact restatement uses fp32 P.  The two must agree within the fp16 rounding of P,
and converting V to fp16 before the call must not change the literal result (bf16 values inside
the fp16 range convert exactly).
"""
import torch

from oracle.bsattn_oracle import attn_blockwise, attn_online_literal
from usagi_b200 import patterns as P


def _inputs(seed=3):
    g = torch.Generator().manual_seed(seed)
    B, H, T = 1, 2, 512
    q, k, v = [torch.randn(B, H, T, 128, generator=g).bfloat16() for _ in range(3)]
    return q, k, v, P.retrieval_pattern(B, H, T, 3, seed=2)


def test_literal_matches_exact_for_bf16_inputs():
    q, k, v, pat = _inputs()
    lo, ll = attn_online_literal(q, k, v, pat.row_ptr, pat.col_idx)
    eo, el = attn_blockwise(q, k, v, pat.row_ptr, pat.col_idx)
    d = (lo - eo).abs()
    assert d.max().item() <= 4e-3 and d.mean().item() <= 2e-4, d.max().item()
    fin = torch.isfinite(el)
    assert torch.equal(fin, torch.isfinite(ll))
    assert (ll[fin] - el[fin]).abs().max().item() <= 1e-4


def test_literal_same_with_fp16_v():
    q, k, v, pat = _inputs(seed=4)
    a, la = attn_online_literal(q, k, v, pat.row_ptr, pat.col_idx)
    b, lb = attn_online_literal(q, k, v.half(), pat.row_ptr, pat.col_idx)
    assert torch.equal(a, b) and torch.equal(la, lb)
