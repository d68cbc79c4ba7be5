"""Work lists on the GPU: which CTA computes an item does not change the item's arithmetic, so the
outputs with a plan are bit-identical to the round-robin ones; a plan that does not match the call
is reported (BSATTN_E_PLAN) and the kernel does no work."""
import pytest
import torch

import usagi_b200 as ub
from usagi_b200 import _lib, api
from usagi_b200 import patterns as P

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)


def _inputs(B, H, T, seed):
    g = torch.Generator(device=DEV).manual_seed(seed)
    return [torch.randn(B, H, T, 128, generator=g, device=DEV).half() for _ in range(3)]


@pytest.mark.parametrize("fam", ["window8", "prefix4+window4", "retrieval8"])
def test_plan_bitwise_equal_full_size(fam):
    ub.setup(device="cuda:0")
    B, H, T = 2, 16, 8192
    q, k, v = _inputs(B, H, T, 41)
    pat = P.family_pattern(fam, B, H, T)
    rp, ci = pat.row_ptr.to(DEV), pat.col_idx.to(DEV)
    plan = ub.make_plan(pat.row_ptr, pat.col_idx, B, H, T, device=DEV)
    o1, l1 = ub.block_sparse_attn_fwd(q, k, v, rp, ci)
    o2, l2 = ub.block_sparse_attn_fwd(q, k, v, rp, ci, plan=plan)
    torch.cuda.synchronize()
    ub.check_errors(DEV)
    assert torch.equal(o1, o2) and torch.equal(l1, l2)


def test_plan_with_seq_lens_and_other_grids():
    ub.setup(device="cuda:0")
    B, H, T = 2, 3, 4096
    q, k, v = _inputs(B, H, T, 42)
    pat = P.retrieval_pattern(B, H, T, 8)
    sl = torch.tensor([1000, 4096], dtype=torch.int32)
    rp, ci, sld = pat.row_ptr.to(DEV), pat.col_idx.to(DEV), sl.to(DEV)
    o1, l1 = ub.block_sparse_attn_fwd(q, k, v, rp, ci, sld)
    for grid in (1, 7, 96):
        plan = ub.make_plan(pat.row_ptr, pat.col_idx, B, H, T, sl, device=DEV, grid=grid)
        o2, l2 = ub.block_sparse_attn_fwd(q, k, v, rp, ci, sld, plan=plan)
        torch.cuda.synchronize()
        ub.check_errors(DEV)
        assert torch.equal(o1, o2) and torch.equal(l1, l2), grid


def test_mismatched_plan_is_reported_and_does_no_work():
    ub.setup(device="cuda:0")
    B, H, T = 1, 2, 2048
    q, k, v = _inputs(B, H, T, 43)
    pat = P.window_pattern(B, H, T, 8)
    plan = ub.make_plan(pat.row_ptr, pat.col_idx, B, H, T, device=DEV, grid=8)
    rp, rps = api._bh_view(pat.row_ptr.to(DEV), B, H, "row_ptr")
    ci, cis = api._bh_view(pat.col_idx.to(DEV), B, H, "col_idx")
    o = torch.full_like(q, 3.0)
    lse = torch.full((B, H, T), 5.0, device=DEV)
    ws = api._workspace(DEV, torch.cuda.current_stream(DEV).cuda_stream)
    lib = _lib.load()
    rc = lib.bsattn_fwd_plan(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(),
                             lse.data_ptr(), rp.data_ptr(), ci.data_ptr(), None, B, H, T, 128,
                             rps, cis, int(ci.shape[-1]), 0.0, 0, plan.tensor.data_ptr(), 7,
                             ws.data_ptr(), ws.numel() * 4,
                             torch.cuda.current_stream(DEV).cuda_stream)
    assert rc == 0
    with pytest.raises(ub.BsattnError) as err:
        ub.check_errors(DEV)
    assert err.value.code == _lib.E_PLAN
    assert (o == 3.0).all() and (lse == 5.0).all()
    with pytest.raises(ValueError):
        ub.block_sparse_attn_fwd(q, k, v, pat.row_ptr.to(DEV), pat.col_idx.to(DEV),
                                 plan=ub.make_plan(pat.row_ptr, pat.col_idx, B, H, 1024,
                                                   device=DEV))
