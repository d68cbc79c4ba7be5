"""Analytic window rows on the GPU (bsattn_fwd_window): the reference's _fwd_window and
_fwd_window_global (kernels/v1_baseline.py:144-224, :227-322) walk prefix and window blocks
from closed forms instead of col_idx.  The same rows given as CSR run the same tiles in the same
order, so o and lse must equal the CSR path's bit for bit; the CSR path itself is checked against
the oracle elsewhere, and a few cases here go to the oracle directly (tolerances of the fp16
regression bound: max 4e-3, mean 2e-4, lse 2e-4).
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


def _inputs(B, H, T, seed, dtype=torch.float16):
    g = torch.Generator(device=DEV).manual_seed(seed)
    return [torch.randn(B, H, T, 128, generator=g, device=DEV).to(dtype) for _ in range(3)]


def _csr(B, H, T, window, global_blocks):
    if global_blocks:
        return P.prefix_window_pattern(B, H, T, global_blocks, window)
    return P.window_pattern(B, H, T, window)


def _both(q, k, v, window, global_blocks, seq_lens=None, **kw):
    B, H, T, _ = q.shape
    pat = _csr(B, H, T, window, global_blocks)
    a = ub.block_sparse_attn_fwd(q, k, v, pat.row_ptr.to(DEV), pat.col_idx.to(DEV), seq_lens, **kw)
    b = ub.block_sparse_attn_fwd_window(q, k, v, seq_lens, window=window,
                                        global_blocks=global_blocks, **kw)
    torch.cuda.synchronize()
    ub.check_errors(DEV)
    return pat, a, b


@pytest.mark.parametrize("window,global_blocks", [(8, 0), (4, 4)])
def test_benchmark_families_bitwise(window, global_blocks):
    B, H, T = 2, 16, 8192
    q, k, v = _inputs(B, H, T, 51)
    _, (o1, l1), (o2, l2) = _both(q, k, v, window, global_blocks)
    assert torch.equal(o1, o2) and torch.equal(l1, l2)
    plan = ub.make_window_plan(B, H, T, window, global_blocks, device=DEV)
    o3, l3 = ub.block_sparse_attn_fwd_window(q, k, v, window=window, global_blocks=global_blocks,
                                             plan=plan)
    torch.cuda.synchronize()
    ub.check_errors(DEV)
    assert torch.equal(o1, o3) and torch.equal(l1, l3)


@pytest.mark.parametrize("window,global_blocks", [(1, 0), (2, 0), (16, 0), (64, 0), (8, 8),
                                                  (1, 3), (3, 1), (2, 40)])
def test_shapes_and_seq_lens_bitwise(window, global_blocks):
    B, H, T = 2, 3, 2048
    q, k, v = _inputs(B, H, T, 52)
    sl = torch.tensor([700, 2048], dtype=torch.int32, device=DEV)
    for seq_lens in (None, sl):
        _, (o1, l1), (o2, l2) = _both(q, k, v, window, global_blocks, seq_lens)
        assert torch.equal(o1, o2) and torch.equal(l1, l2), (window, global_blocks, seq_lens)


def test_bf16_and_plan_grids_bitwise():
    B, H, T = 1, 4, 4096
    q, k, v = _inputs(B, H, T, 53, torch.bfloat16)
    sl = torch.tensor([3000], dtype=torch.int32, device=DEV)
    _, (o1, l1), (o2, l2) = _both(q, k, v, 4, 4, sl)
    assert o1.dtype == torch.bfloat16
    assert torch.equal(o1, o2) and torch.equal(l1, l2)
    for grid in (1, 13, 128):  # 128 = every item its own CTA
        plan = ub.make_window_plan(B, H, T, 4, 4, sl, device=DEV, grid=grid)
        o3, l3 = ub.block_sparse_attn_fwd_window(q, k, v, sl, window=4, global_blocks=4, plan=plan)
        torch.cuda.synchronize()
        ub.check_errors(DEV)
        assert torch.equal(o1, o3) and torch.equal(l1, l3), grid


@pytest.mark.parametrize("window,global_blocks", [(4, 0), (2, 3)])
def test_against_oracle(window, global_blocks):
    B, H, T = 1, 2, 1024
    g = torch.Generator().manual_seed(54)
    q, k, v = [torch.randn(B, H, T, 128, generator=g).half() for _ in range(3)]
    sl = torch.tensor([900], dtype=torch.int32)
    o, lse = ub.block_sparse_attn_fwd_window(q.to(DEV), k.to(DEV), v.to(DEV), sl.to(DEV),
                                             window=window, global_blocks=global_blocks)
    torch.cuda.synchronize()
    ub.check_errors(DEV)
    pat = _csr(B, H, T, window, global_blocks)
    ro, rl = attn_blockwise(q, k, v, pat.row_ptr, pat.col_idx, sl)
    d = (o.float().cpu() - ro).abs()
    assert d.max().item() <= 4e-3 and d.mean().item() <= 2e-4, d.max().item()
    fin = torch.isfinite(rl)
    assert torch.equal(fin, torch.isfinite(lse.cpu()))
    assert (lse.cpu()[fin] - rl[fin]).abs().max().item() <= 2e-4


def test_bad_window_raises():
    q, k, v = _inputs(1, 1, 256, 55)
    with pytest.raises(ub.BsattnError):
        ub.block_sparse_attn_fwd_window(q, k, v, window=0)
