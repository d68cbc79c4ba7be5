"""Numerics stress cases on the GPU, against the fp32 oracle (oracle/bsattn_oracle.attn_blockwise),
with the regression bound of the parity tests: max |do| <= 4e-3, mean <= 2e-4, lse within 2e-4
(relative 2e-6 where scores are large).

* Dense causal rows (every block 0..i): items of up to 32 tiles, the longest a CTA walks.
* Growing key magnitudes: each key block's scores are larger than the previous block's, so the
  running row max is raised on almost every tile.  The kernel raises it lazily (only when a
  block's max exceeds it by more than 2^8 in the exp2 domain) and rescales O and l in tensor
  memory; the result must still match the exact softmax (v4 :95-99 rescales on every block).
* A softmax scale other than 1/sqrt(D) (the entry point's `scale` argument).
"""
import pytest
import torch

import usagi_b200 as ub
from usagi_b200 import patterns as P
from oracle.bsattn_oracle import attn_blockwise

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)


@pytest.fixture(scope="module", autouse=True)
def _setup():
    ub.setup(device="cuda:0")
    yield
    ub.check_errors(DEV)


def _dense_causal(B, H, T):
    nqb = T // 128
    return P.shared_pattern([list(range(i + 1)) for i in range(nqb)], B, H, nqb, "causal")


def _check(o, lse, ro, rl, lse_rel=0.0):
    of = o.float().cpu()
    assert torch.isfinite(of).all()
    d = (of - ro).abs()
    assert d.max().item() <= 4e-3 and d.mean().item() <= 2e-4, (d.max().item(), d.mean().item())
    fin = torch.isfinite(rl)
    assert torch.equal(fin, torch.isfinite(lse.cpu()))
    dl = (lse.cpu()[fin] - rl[fin]).abs()
    assert (dl <= 2e-4 + lse_rel * rl[fin].abs()).all(), dl.max().item()


def test_dense_causal_long_rows():
    B, H, T = 1, 2, 4096
    g = torch.Generator().manual_seed(90)
    q, k, v = [torch.randn(B, H, T, 128, generator=g).half() for _ in range(3)]
    pat = _dense_causal(B, H, T)
    o, lse = ub.block_sparse_attn_fwd(q.to(DEV), k.to(DEV), v.to(DEV), pat.row_ptr.to(DEV),
                                      pat.col_idx.to(DEV))
    torch.cuda.synchronize()
    ub.check_errors(DEV)
    ro, rl = attn_blockwise(q, k, v, pat.row_ptr, pat.col_idx)
    _check(o, lse, ro, rl)


@pytest.mark.parametrize("fam", ["causal", "window16"])
def test_growing_scores_force_rescales(fam):
    B, H, T = 1, 2, 2048
    g = torch.Generator().manual_seed(91)
    q = torch.randn(B, H, T, 128, generator=g)
    k = torch.randn(B, H, T, 128, generator=g)
    v = torch.randn(B, H, T, 128, generator=g)
    # Key block j is scaled by 1 + 2.5 j: its largest scores exceed those of block j-1 by well
    # over 8 in log2 units, so the running max moves up tile after tile.
    grow = 1.0 + 2.5 * (torch.arange(T) // 128).float()
    k = k * grow.view(1, 1, T, 1)
    q, k, v = q.half(), k.half(), v.half()
    pat = _dense_causal(B, H, T) if fam == "causal" else P.window_pattern(B, H, T, 16)
    o, lse = ub.block_sparse_attn_fwd(q.to(DEV), k.to(DEV), v.to(DEV), pat.row_ptr.to(DEV),
                                      pat.col_idx.to(DEV))
    torch.cuda.synchronize()
    ub.check_errors(DEV)
    ro, rl = attn_blockwise(q, k, v, pat.row_ptr, pat.col_idx)
    # Sanity of the construction: the largest scaled score of the last row block is far above
    # what the first block of that row reaches.
    assert rl[0, 0, -1].item() > 50.0
    _check(o, lse, ro, rl, lse_rel=2e-6)


def test_custom_scale():
    B, H, T = 2, 2, 1024
    g = torch.Generator().manual_seed(92)
    q, k, v = [torch.randn(B, H, T, 128, generator=g).half() for _ in range(3)]
    pat = P.retrieval_pattern(B, H, T, 4, seed=3)
    for scale in (0.02, 0.3):
        o, lse = ub.block_sparse_attn_fwd(q.to(DEV), k.to(DEV), v.to(DEV), pat.row_ptr.to(DEV),
                                          pat.col_idx.to(DEV), scale=scale)
        torch.cuda.synchronize()
        ub.check_errors(DEV)
        ro, rl = attn_blockwise(q, k, v, pat.row_ptr, pat.col_idx, scale=scale)
        _check(o, lse, ro, rl, lse_rel=2e-6)
