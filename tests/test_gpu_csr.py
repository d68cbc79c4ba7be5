"""CSR patterns built on the GPU (bsattn_build_csr) against the host builders and the contract the
attention kernel relies on: every row ascending, distinct, ending with its own diagonal
(kernels/v4_leaderboard_0740ms.py:78-86, :107).
"""
import pytest
import torch

import usagi_b200 as ub
from usagi_b200 import patterns as P
from oracle.bsattn_oracle import attn_blockwise

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)


def _rows(pat, bh):
    rp = pat.row_ptr.reshape(-1, pat.nqb + 1)[bh].cpu().tolist()
    ci = pat.col_idx.reshape(-1, pat.col_idx.shape[-1])[bh].cpu().tolist()
    return [ci[rp[i]:rp[i + 1]] for i in range(pat.nqb)]


@pytest.mark.parametrize("T", [128, 1024, 8192, 32768])
def test_window_families_bit_identical(T):
    for dev_pat, host_pat in (
            (P.device_window_pattern(2, 3, T, 8), P.window_pattern(2, 3, T, 8)),
            (P.device_window_pattern(1, 1, T, 16), P.window_pattern(1, 1, T, 16)),
            (P.device_prefix_window_pattern(2, 3, T, 4, 4), P.prefix_window_pattern(2, 3, T, 4, 4)),
            (P.device_prefix_window_pattern(1, 2, T, 8, 8), P.prefix_window_pattern(1, 2, T, 8, 8))):
        torch.cuda.synchronize()
        assert torch.equal(dev_pat.row_ptr.cpu(), host_pat.row_ptr)
        assert dev_pat.col_idx.shape == host_pat.col_idx.shape
        assert torch.equal(dev_pat.col_idx.cpu(), host_pat.col_idx)
        assert dev_pat.live_blocks() == host_pat.live_blocks()


@pytest.mark.parametrize("n_random", [0, 1, 8, 16, 64])
def test_retrieval_rows_contract(n_random):
    B, H, T = 2, 3, 16384
    pat = P.device_retrieval_pattern(B, H, T, n_random, seed=7)
    host = P.retrieval_pattern(B, H, T, n_random, seed=7)
    torch.cuda.synchronize()
    # Same row lengths (hence row_ptr) as the host builder; the draws themselves differ.
    assert torch.equal(pat.row_ptr.cpu(), host.row_ptr)
    for bh in range(B * H):
        for i, row in enumerate(_rows(pat, bh)):
            assert row[-1] == i
            if i >= 1:
                assert row[-2] == i - 1
            assert all(a < b for a, b in zip(row, row[1:]))  # ascending, distinct
            assert all(0 <= c <= i for c in row)
            assert len(row) == (i + 1 if i < 2 else 2 + min(n_random, i - 1))


def test_retrieval_seeded_and_spread():
    B, H, T = 1, 4, 32768
    a = P.device_retrieval_pattern(B, H, T, 8, seed=11)
    b = P.device_retrieval_pattern(B, H, T, 8, seed=11)
    c = P.device_retrieval_pattern(B, H, T, 8, seed=12)
    torch.cuda.synchronize()
    assert torch.equal(a.col_idx, b.col_idx)
    assert not torch.equal(a.col_idx, c.col_idx)
    assert not torch.equal(a.col_idx[0, 0], a.col_idx[0, 1])  # heads draw independently
    # Uniform over 0 .. i-2: the random picks of the last row cover the range roughly evenly.
    nqb = T // 128
    picks = torch.tensor([r[:-2] for r in
                          (_rows(a, h)[nqb - 1] for h in range(H))]).reshape(-1).float()
    assert 0.3 * nqb < picks.mean().item() < 0.7 * nqb


def test_attention_on_device_built_patterns():
    B, H, T = 1, 2, 2048
    g = torch.Generator().manual_seed(31)
    q, k, v = [torch.randn(B, H, T, 128, generator=g).half() for _ in range(3)]
    ub.setup(device="cuda:0")
    for pat in (P.device_window_pattern(B, H, T, 8), P.device_prefix_window_pattern(B, H, T),
                P.device_retrieval_pattern(B, H, T, 8, seed=3)):
        o, lse = ub.block_sparse_attn_fwd(q.to(DEV), k.to(DEV), v.to(DEV), pat.row_ptr,
                                          pat.col_idx)
        torch.cuda.synchronize()
        ro, rl = attn_blockwise(q, k, v, pat.row_ptr.cpu(), pat.col_idx.cpu())
        d = (o.float().cpu() - ro).abs()
        assert d.max().item() <= 4e-3 and d.mean().item() <= 2e-4, (pat.name, d.max().item())
        assert (lse.cpu() - rl).abs().max().item() <= 2e-4
    ub.check_errors(DEV)
